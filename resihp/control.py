"""Control plane: fail-stop detection, world re-formation, consistent stop.

Semantics of the reference (``resihp/control.py:55-485``):

* A fail-stop is a real ``SIGKILL``. Detection is out of band: :meth:`ControlPlane.observe`
  rendezvouses at each iteration boundary on the launcher's store and reads the
  membership the supervisor published from its process table.
* A rank has a stable **plan rank** (its launch identity, the only rank the planner,
  plan and checkpoint speak) and a **torch rank** (its index in the current membership,
  re-assigned every time the world is re-formed); this class owns the translation.
* The **world group** is a Gloo group over the current membership, re-formed under a
  fresh store prefix after every fail-stop; control collectives ride it. On GPUs it also
  carries an NCCL communicator bound to the rank's device, created with the world. The
  **training groups** come from the current plan (NCCL on GPU -- each an
  ``ncclCommSplit`` of the world's communicator -- Gloo on CPU), built in one
  plan-derived order by every rank: one TP group per stage of degree > 1, one union
  group per pipeline hop, the executor group over every placed rank, the
  gradient-reduction groups (DP position groups and tied-embedding pairs) and, where
  state moves are collectives (CPU / FP32), the live group over every surviving rank.
* Six consistent-stop codes; :meth:`agree` raises the *same* :class:`ConsistentStop` on
  every rank, derived from the gathered reports rather than the local view.
* :meth:`safe_point` runs steps 4-9: mark failed, replan, dissolve and re-form the world,
  agree on the plan, build the new groups, recover along the single path, agree on plan
  and state digests. A stop leaves no training group behind.
"""

from __future__ import annotations

from dataclasses import dataclass
from datetime import timedelta
import os
import time

from . import membership
from .config import TrainConfig
from .parallel.dp import reduction_topology
from .plan import ExecutionPlan, InfeasiblePlan, boundary_hops, build_plan
from .recovery import TrainingGroups
from .utils.trace import nvtx_range

STOP_CODES = (
    "no_feasible_tp",
    "no_executable_pp",
    "no_feasible_dp_target",
    "checkpoint_unusable",
    "plan_disagreement",
    "state_mismatch",
)
_DIGEST_STOP = {"plan": "plan_disagreement", "state": "state_mismatch"}
GROUP_TIMEOUT = timedelta(seconds=int(os.environ.get("RESIHP_GROUP_TIMEOUT", "300")))
# On GPUs the world group also carries an NCCL communicator bound to this rank's device,
# created eagerly when the world forms; every NCCL training group is then split from it
# (ncclCommSplit) inside the safe point instead of being initialised from scratch on its
# first collective.
NCCL_SPLIT = os.environ.get("RESIHP_NCCL_SPLIT", "1") != "0"
# The checkpoint writer rank serialises and writes the file on a background thread.
ASYNC_CHECKPOINT = os.environ.get("RESIHP_ASYNC_CHECKPOINT", "1") != "0"


@dataclass(frozen=True)
class StopReason:
    code: str
    message: str


class ConsistentStop(RuntimeError):
    def __init__(self, reason: StopReason):
        super().__init__(f"{reason.code}: {reason.message}")
        self.reason = reason


class ControlPlane:
    """This rank's place in the world; rebuilds it after a real fail-stop."""

    def __init__(self, rank, members, store, training_backend, *, memory_budget=None, device=None,
                 vocab_size=None, sequence_length=None):
        # ``vocab_size`` / ``sequence_length``: the reference passes its run constants
        # here; the config carries them in this package, and any value given must agree
        self.vocab_size = vocab_size
        self.sequence_length = sequence_length
        self.rank = int(rank)
        self.members = tuple(sorted(members))
        self.store = store
        self.training_backend = training_backend
        self.epoch = 0
        self.boundary = 0
        self.world_group = None
        self.groups = TrainingGroups()
        self.memory_budget = memory_budget
        self.training_run = None
        self.checkpoint_path = None
        self.device = device
        self.state_digest = ""
        self.pin = False
        self.last_recovery: dict = {}
        self.resume_cursor = 0  # completed iterations training continues from after a safe point
        self.checkpoint_writer = None
        if ASYNC_CHECKPOINT:
            from .checkpoint import CheckpointWriter

            self.checkpoint_writer = CheckpointWriter()

    @classmethod
    def initialize(cls, *, training_backend=None, memory_budget=None, device=None) -> "ControlPlane":
        import torch

        rank = int(os.environ["RANK"])
        world = int(os.environ["WORLD_SIZE"])
        store = membership.connect(os.environ[membership.HOST_ENV], os.environ[membership.PORT_ENV])
        if training_backend is None:
            training_backend = "nccl" if torch.cuda.is_available() else "gloo"
        cp = cls(rank, range(world), store, training_backend, memory_budget=memory_budget, device=device)
        cp.form_world(cp.members, epoch=0)
        return cp

    # --- ranks ---------------------------------------------------------------------

    @property
    def world_size(self) -> int:
        return len(self.members)

    # the reference's names for this rank's training groups
    @property
    def tp_group(self):
        return self.groups.tp

    @property
    def executor_group(self):
        return self.groups.executor

    @property
    def boundary_groups(self) -> dict:
        return dict(self.groups.hops)

    def torch_rank(self, plan_rank: int) -> int:
        return self.members.index(plan_rank)

    # --- detection / world ---------------------------------------------------------

    def quiesce(self) -> None:
        """Wait until this rank's GPU has finished everything it was given.

        CUDA work -- NCCL collectives included -- is asynchronous, so a rank can reach the
        end of an iteration on the host while its last collective is still queued on the
        device. A fail-stop must find nothing in flight (a rank killed with a collective
        half issued would leave its peers' streams waiting for it), so the iteration ends
        here, on every rank, before the kill point and before the boundary rendezvous.
        A completed collective on this rank implies every peer has joined it as well.
        """
        import torch

        if self.device is not None and torch.device(self.device).type == "cuda":
            torch.cuda.synchronize(self.device)

    def observe(self) -> tuple[int, ...]:
        """Safe-point steps 3-4: arrive at the next boundary; the ranks that did not."""
        self.quiesce()
        self.boundary += 1
        published = membership.boundary(self.store, self.boundary, timeout=GROUP_TIMEOUT)
        return tuple(r for r in self.members if r not in published)

    def form_world(self, members, *, epoch: int) -> None:
        import torch.distributed as dist

        import torch

        self.members = tuple(sorted(members))
        self.epoch = int(epoch)
        backend, bound = "gloo", None
        if (NCCL_SPLIT and self.training_backend == "nccl" and self.device is not None
                and torch.device(self.device).type == "cuda"):
            backend, bound = "cpu:gloo,cuda:nccl", torch.device(self.device)
        dist.init_process_group(
            backend=backend,
            store=dist.PrefixStore(membership.PG_PREFIX.format(epoch=self.epoch), self.store),
            rank=self.torch_rank(self.rank),
            world_size=self.world_size,
            timeout=GROUP_TIMEOUT,
            device_id=bound,
        )
        self.world_group = dist.group.WORLD
        self.groups.world = self.world_group

    def dissolve_world(self) -> None:
        import torch.distributed as dist

        # No kernel is in flight at a safe point; a dead peer cannot join a barrier.
        if self.training_run is not None:
            self.training_run.stage.close_comm(barrier=False)
        self.destroy_training_groups()
        dist.destroy_process_group()
        self.world_group = None
        self.groups.world = None

    # --- training groups -----------------------------------------------------------

    def attach_run(self, run, *, checkpoint_path, device=None, pin=False) -> None:
        self.training_run = run
        self.checkpoint_path = checkpoint_path
        if device is not None:
            self.device = device
        self.pin = pin

    def is_training_rank(self, plan: ExecutionPlan) -> bool:
        return self.rank in set(plan.active_ranks)

    def _new_group(self, plan_ranks):
        import torch.distributed as dist

        return dist.new_group(
            ranks=[self.torch_rank(r) for r in plan_ranks], backend=self.training_backend, timeout=GROUP_TIMEOUT
        )

    def build_training_groups(self, plan: ExecutionPlan) -> TrainingGroups:
        """Safe-point step 6c: every rank creates every group in the same plan order."""
        g = TrainingGroups(world=self.world_group)
        for stage in sorted(plan.stages, key=lambda s: (s.replica_id, s.stage_id)):
            if len(stage.tp_members) == 1:
                continue  # a TP degree of 1 needs no communicator (the stage treats None as size 1)
            handle = self._new_group(stage.tp_members)
            if self.rank in stage.tp_members:
                g.tp = handle
        for hop in boundary_hops(plan):
            handle = self._new_group(hop)
            if self.rank in hop:
                g.hops[hop] = handle
        executors = self._world_or_new_group(plan.active_ranks)
        g.executor = executors if self.is_training_rank(plan) else None
        topo = reduction_topology(plan)
        for members in topo.tied_groups + topo.dp_groups:
            handle = self._new_group(members)
            if self.rank in members:
                g.reduce[members] = handle
        if self._needs_live_group(plan):
            g.live = self._world_or_new_group(self.members)
        self.groups = g
        return g

    def _world_carries_training(self) -> bool:
        """The world group can run the training collectives itself: it is Gloo and so is
        training, or it carries the device-bound NCCL communicator."""
        import torch

        if self.training_backend == "gloo":
            return True
        return (NCCL_SPLIT and self.training_backend == "nccl" and self.device is not None
                and torch.device(self.device).type == "cuda")

    def _world_or_new_group(self, plan_ranks):
        """The world group itself when ``plan_ranks`` are all its members (one communicator
        fewer to create at a safe point), else a new group. Every rank decides alike."""
        if tuple(sorted(plan_ranks)) == self.members and self._world_carries_training():
            return self.world_group
        return self._new_group(plan_ranks)

    def _needs_live_group(self, plan: ExecutionPlan) -> bool:
        """The live group carries collective state moves; the CUDA bf16 path moves state
        peer to peer instead (:func:`resihp.recovery.recover`) and does not need it."""
        from .parallel import peer

        return not (self.training_backend == "nccl" and plan.config.dtype == "bf16" and peer.ENABLED)

    def destroy_training_groups(self) -> None:
        import torch.distributed as dist

        g = self.groups
        handles = [g.tp, *g.hops.values(), g.executor, *g.reduce.values(), g.live]
        seen = {id(self.world_group)}  # a training group may be the world itself: dissolve_world ends it
        for h in handles:
            if h is not None and id(h) not in seen:
                seen.add(id(h))
                dist.destroy_process_group(h)
        self.groups = TrainingGroups(world=self.world_group)

    # --- the iteration -------------------------------------------------------------

    def training_step(self):
        if self.training_run is None:
            return None
        return self.training_run.step()

    def commit_checkpoint(self, plan: ExecutionPlan, *, cursor: int) -> None:
        from .recovery import commit_checkpoint

        if not self.is_training_rank(plan):
            return
        with nvtx_range("checkpoint_commit"):
            commit_checkpoint(
                self.training_run, self.checkpoint_path, plan=plan, groups=self.groups,
                writer=self.rank == plan.active_ranks[0], cursor=cursor, device=self.device,
                background=self.checkpoint_writer,
            )

    def flush_checkpoint(self) -> None:
        """Wait for this rank's checkpoint write in flight (a no-op on non-writers)."""
        if self.checkpoint_writer is not None:
            self.checkpoint_writer.flush()

    def _recover_state(self, plan, previous, cursor) -> None:
        from .recovery import recover

        self.training_run, self.state_digest, self.resume_cursor = recover(
            self.training_run, plan=plan, previous=previous, rank=self.rank, cursor=cursor,
            checkpoint_path=self.checkpoint_path, groups=self.groups, device=self.device, pin=self.pin,
        )

    def agree(self, reason: StopReason | None = None, **digests: str) -> None:
        """Unanimous decision over the world group (same ConsistentStop everywhere)."""
        import torch.distributed as dist

        local = (None if reason is None else (reason.code, reason.message), tuple(sorted(digests.items())))
        gathered: list = [None] * self.world_size
        dist.all_gather_object(gathered, local, group=self.world_group)
        for index, (reported, _) in enumerate(gathered):
            if reported is not None:
                raise ConsistentStop(StopReason(reported[0], f"rank {self.members[index]}: {reported[1]}"))
        for label in sorted(digests):
            values = {dict(entry)[label] for _, entry in gathered}
            if len(values) > 1:
                raise ConsistentStop(StopReason(_DIGEST_STOP[label], f"ranks disagree on the {label} digest: {sorted(values)}"))

    def safe_point(self, config: TrainConfig, plan: ExecutionPlan, failed_ranks, lost, *, next_step: int):
        """Steps 4-9 of the fail-stop safe point; returns ``(new plan, failed ranks)``.

        Afterwards :attr:`resume_cursor` holds the completed-iteration count training
        continues from (``next_step``, or an older checkpoint's count after a rollback),
        the same on every rank.
        """
        t0 = time.perf_counter()
        phases = {}
        # the checkpoint file must be complete before the first agreement: every rank
        # may read it during recovery
        self.flush_checkpoint()
        for name, given, have in (("vocab_size", self.vocab_size, config.vocab_size),
                                  ("sequence_length", self.sequence_length, config.seq_len)):
            if given is not None and given != have:
                raise ValueError(f"{name}={given} does not match the config ({have})")
        failed = tuple(sorted(set(failed_ranks) | set(lost)))
        survivors = tuple(r for r in self.members if r not in set(lost))
        new_plan, reason = None, None
        try:
            new_plan = build_plan(
                config, step=next_step, version=plan.version + 1, failed_ranks=failed, previous=plan,
                memory_budget=self.memory_budget, vocab_size=config.vocab_size, sequence_length=config.seq_len,
            )
        except InfeasiblePlan as error:
            reason = StopReason(error.reason.code, error.reason.message)
        phases["replan_s"] = time.perf_counter() - t0
        t = time.perf_counter()
        with nvtx_range("dissolve_world"):
            self.dissolve_world()
        phases["dissolve_world_s"] = time.perf_counter() - t
        t1 = time.perf_counter()
        with nvtx_range("form_world"):
            self.form_world(survivors, epoch=self.epoch + 1)
        phases["form_world_s"] = time.perf_counter() - t1
        phases["reform_world_s"] = time.perf_counter() - t
        self.agree(reason, plan="" if new_plan is None else new_plan.digest)
        try:
            t = time.perf_counter()
            with nvtx_range("build_groups"):
                self.build_training_groups(new_plan)
            phases["build_groups_s"] = time.perf_counter() - t
            t = time.perf_counter()
            reason = None
            try:
                with nvtx_range("recover_state"):
                    self._recover_state(new_plan, plan, next_step)
            except Exception as error:  # classified below; anything else is a bug
                from .recovery import recovery_stop_code

                code = recovery_stop_code(error)
                if code is None:
                    raise
                reason = StopReason(code, str(error))
            phases["recover_state_s"] = time.perf_counter() - t
            self.agree(reason)
            self.agree(plan=new_plan.digest, state=self.state_digest)
        except ConsistentStop:
            self.destroy_training_groups()
            raise
        phases["total_s"] = time.perf_counter() - t0
        self.last_recovery = phases
        return new_plan, failed

    def shutdown(self) -> None:
        import torch.distributed as dist

        self.flush_checkpoint()
        if self.training_run is not None:
            self.training_run.stage.close_comm(barrier=True)
        self.destroy_training_groups()
        dist.barrier(group=self.world_group)
        dist.destroy_process_group()
        self.world_group = None
