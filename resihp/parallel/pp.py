"""The pipeline runtime: assignment-driven 1F1B over scatter/gather stage boundaries.

Same execution contract as the reference (``resihp/parallel/pp.py:73-451``):

* the 1F1B order comes from :func:`resihp.planner.pp.pipeline_phases`, which also sizes
  the planner's activation budget, and :attr:`PipelineRuntime.schedule` records what
  ran (``F<mb>`` / ``B<mb>`` / ``W``);
* a stage boundary moves one authoritative copy of the activation, cut into
  ``N = max(TP_up, TP_down)`` contiguous chunks, chunk ``k`` travelling between
  ``up[k*U//N]`` and ``down[k*D//N]`` (:func:`scatter_routing`); the steady-state
  send-forward/recv-backward pairs are one fused ``batch_isend_irecv`` on the hop's
  union group (issuing them separately deadlocks);
* every micro-batch loss is scaled by the global micro-batch count, gradients of all
  holders are summed (:class:`resihp.parallel.dp.GradientReducer`) and one AdamW step
  is applied.

With sequence parallelism a rank holds only its token shard of the boundary tensor,
which is exactly its run of chunks: it sends its own chunks and the receiver keeps
the chunks it receives as its shard, so no all-gather is needed on either side.
Without it the boundary tensor is replicated in the TP group and the receiver
rebuilds it with an all-gather, as in the reference.
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..planner.pp import pipeline_phases
from ..utils.trace import nvtx_range
from .dp import ActivationLog, executor_route, global_micro_count, stage_pipeline


def scatter_routing(up_members, down_members):
    """``(sender, receiver)`` of each of the ``max(U, D)`` chunks of one hop."""
    up, down = tuple(up_members), tuple(down_members)
    n = max(len(up), len(down))
    return tuple((up[k * len(up) // n], down[k * len(down) // n]) for k in range(n))


class PipelineRuntime:
    """One rank's 1F1B execution of an iteration, driven by the plan's assignment.

    ``reducer`` sums gradients across holders before the optimizer step (``None``: a
    single holder, nothing to reduce).
    """

    def __init__(self, stage, *, rank, replica_id, assignment, boundary_groups=None, reducer=None):
        self.stage = stage
        self.rank = int(rank)
        self.replica_id = int(replica_id)
        self.assignment = assignment
        self.boundary_groups = dict(boundary_groups or {})
        self.reducer = reducer
        self.routes = executor_route(assignment, self.rank)
        self.micro_batches = [r["micro_batch"] for r in self.routes]
        self.micro_total = global_micro_count(assignment)
        self.schedule: list[str] = []
        self.activation_log = ActivationLog()
        self.stage_index, self.num_stages = self._position()
        self.executors, self.upstream, self.downstream = self._neighbours()
        if self.routes and ((self.upstream is None) != stage.is_first or (self.downstream is None) != stage.is_last):
            raise ValueError("the stage's pipeline ends disagree with the assignment")
        if self.routes and len(self.executors) != stage.tp_size:
            raise ValueError("the stage's TP group disagrees with the assignment's executors")

    def _position(self):
        seen = set()
        for mb in self.micro_batches:
            chain = stage_pipeline(self.assignment, mb)
            idx = next(i for i, p in enumerate(chain) if self.rank in p.executor_ranks)
            seen.add((idx, len(chain)))
        if len(seen) > 1:
            raise ValueError("assignment puts this rank at differing pipeline positions")
        return seen.pop() if seen else (0, 1)

    def _neighbours(self):
        seen = {(r["executors"], r["upstream"], r["downstream"]) for r in self.routes}
        if len(seen) > 1:
            raise ValueError("assignment gives this rank differing neighbours across micro-batches")
        return seen.pop() if seen else ((self.rank,), None, None)

    # --- boundary transfers ---------------------------------------------------------

    def _hop(self, up, down):
        key = tuple(sorted(set(up) | set(down)))
        return key, self.boundary_groups[key]

    def _peer(self, hop, group, peer):
        return dist.get_global_rank(group, hop.index(peer))

    def _my_chunks(self, up, down):
        sending = self.rank in up
        return tuple(
            (k, recv if sending else send)
            for k, (send, recv) in enumerate(scatter_routing(up, down))
            if (send if sending else recv) == self.rank
        )

    def _first_chunk(self, members, n):
        """Index of the first of this rank's chunks when it holds its own token shard."""
        return members.index(self.rank) * (n // len(members))

    def _send_ops(self, tensor, up, down):
        hop, group = self._hop(up, down)
        n = max(len(up), len(down))
        flat = tensor.detach().reshape(-1)
        mine = up if self.rank in up else down
        if self.stage.sp:
            width = flat.numel() // (n // len(mine))
            base = self._first_chunk(mine, n)
        else:
            width = flat.numel() // n
            base = 0
        return [
            dist.P2POp(dist.isend, flat[(k - base) * width: (k - base + 1) * width].contiguous(), self._peer(hop, group, peer), group)
            for k, peer in self._my_chunks(up, down)
        ]

    def _recv_ops(self, shape, up, down):
        hop, group = self._hop(up, down)
        n = max(len(up), len(down))
        mine = self._my_chunks(up, down)
        full = math.prod(shape) * (self.stage.tp_size if self.stage.sp else 1)
        width = full // n
        slab = torch.empty(len(mine) * width, dtype=self.stage.act_dtype, device=self.stage.device)
        ops = [
            dist.P2POp(dist.irecv, slab[i * width: (i + 1) * width], self._peer(hop, group, peer), group)
            for i, (_k, peer) in enumerate(mine)
        ]
        return slab, ops

    def _reconstruct(self, slab, shape):
        if self.stage.sp or self.stage.tp_size == 1:
            return slab.view(shape)
        out = torch.empty(slab.numel() * self.stage.tp_size, dtype=slab.dtype, device=slab.device)
        dist.all_gather_into_tensor(out, slab, group=self.stage.group)
        return out.view(shape)

    @staticmethod
    def _exchange(ops):
        ops = list(ops)
        if ops:
            with nvtx_range("p2p"):
                for work in dist.batch_isend_irecv(ops):
                    work.wait()

    def _recv_forward(self, shape):
        if self.upstream is None:
            return None
        slab, ops = self._recv_ops(shape, self.upstream, self.executors)
        self._exchange(ops)
        return self._reconstruct(slab, shape).requires_grad_(True)

    def _send_forward(self, out):
        if self.downstream is not None:
            self._exchange(self._send_ops(out, self.executors, self.downstream))

    def _send_forward_recv_backward(self, out, shape):
        if self.downstream is None:
            return None
        slab, recvs = self._recv_ops(shape, self.executors, self.downstream)
        self._exchange(self._send_ops(out, self.executors, self.downstream) + recvs)
        return self._reconstruct(slab, shape)

    def _recv_backward(self, shape):
        if self.downstream is None:
            return None
        slab, ops = self._recv_ops(shape, self.executors, self.downstream)
        self._exchange(ops)
        return self._reconstruct(slab, shape)

    def _send_backward(self, grad):
        if self.upstream is not None:
            self._exchange(self._send_ops(grad, self.upstream, self.executors))

    def _send_backward_recv_forward(self, grad, shape):
        if self.upstream is None:
            return None
        slab, recvs = self._recv_ops(shape, self.upstream, self.executors)
        self._exchange(self._send_ops(grad, self.upstream, self.executors) + recvs)
        return self._reconstruct(slab, shape).requires_grad_(True)

    # --- the iteration --------------------------------------------------------------

    def train_step(self, tokens, *, return_tensor: bool = False):
        """Run this rank's 1F1B schedule over the global batch ``tokens``.

        Returns the summed scaled loss on the last stage (a float, or the device tensor
        with ``return_tensor``), ``None`` elsewhere.
        """
        if tokens.shape[0] % self.micro_total:
            raise ValueError("batch size must be divisible by the micro-batch count")
        stage = self.stage
        device = stage.device
        chunks = tokens.chunk(self.micro_total, dim=0)
        mb = chunks[0].shape[0]
        shape = stage.boundary_shape(mb)
        loss_scale = 1.0 / (mb * (stage.sequence_length - 1) * self.micro_total)
        stage.zero_grad()
        self.schedule = []
        self.activation_log = ActivationLog()
        inputs, outputs, held = [], [], []
        total = torch.zeros((), dtype=torch.float32, device=device)
        count = 0

        def forward(received):
            nonlocal count
            index = self.micro_batches[count]
            count += 1
            self.schedule.append(f"F{index}")
            data = chunks[index].to(device, non_blocking=True)
            with nvtx_range(f"F{index}"):
                out = stage.forward(
                    tokens=data if (stage.is_first or stage.is_last) else None,
                    hidden=received,
                    loss_scale=loss_scale,
                )
            if stage.is_last:
                total.add_(out.detach())
            self.activation_log.retain(index)
            inputs.append(received)
            outputs.append(out)
            held.append(index)
            return out

        def backward(grad_output):
            index = held.pop(0)
            self.schedule.append(f"B{index}")
            received = inputs.pop(0)
            out = outputs.pop(0)
            with nvtx_range(f"B{index}"):
                if stage.is_last:
                    out.backward()
                else:
                    out.backward(grad_output)
            self.activation_log.release(index)
            return None if stage.is_first else received.grad

        warmup, steady = pipeline_phases(len(self.micro_batches), stage_index=self.stage_index, num_stages=self.num_stages)
        for _ in range(warmup):
            self._send_forward(forward(self._recv_forward(shape)))
        received = self._recv_forward(shape) if steady else None
        for i in range(steady):
            grad_out = self._send_forward_recv_backward(forward(received), shape)
            grad_in = backward(grad_out)
            if i == steady - 1:
                self._send_backward(grad_in)
            else:
                received = self._send_backward_recv_forward(grad_in, shape)
        for _ in range(warmup):
            self._send_backward(backward(self._recv_backward(shape)))

        self.schedule.append("W")
        with nvtx_range("W"):
            if self.reducer is None or not self.reducer.reduce_and_step(stage):
                stage.optimizer_step()
        if not stage.is_last:
            return None
        return total if return_tensor else float(total)
