"""A model of the fused kernels' cross-GPU protocols, for race and deadlock checks.

Mirrors ``resihp/csrc/fused_gemm.cu`` (and the DP step of ``peer_state.cu``) at the level
of what synchronises. Every tile producer, epilogue and copy-warp group of every CTA of
every rank is an agent; counter words and claim counters are shared integers; data
buffers hold, per row block or tile, the epoch whose values they contain. A random
scheduler interleaves the agents (each rank's calls run in stream order; a rank starts
call e+1 once every agent of call e finished), every wait blocks until its condition
holds, and every read checks that the data is the epoch being computed -- a stale or
already overwritten block is a race. If no agent can move while some are unfinished,
the protocol deadlocked (the kernels' bounded waits would report error code 4). Work is
claimed from per-rank counters as in the kernels, and the host side -- the bases
advanced per call -- comes from the extension's own host functions, so a host that
advances by a different count than the kernel claims shows up here (as a missed or
repeated tile, a race or a deadlock).
"""

from __future__ import annotations

import random

from resihp.ops import _ext

FBM = 128
RING = 4  # tile ring depth between a CTA's producer and its epilogue
COPY_BATCH = 8  # copy items claimed at once (fused_gemm.cu: kCopyBatch)
MODES = {"ag": 1, "rs": 2, "ar": 3}


class ProtocolError(AssertionError):
    pass


def fused_tile(t, tiles_m_chunk, tiles_n, rank, tp, first, rows_per_rank):
    """Tile t -> (chunk, m0, tn), the kernel's order (chunks from rank + first, groups of 8 along M)."""
    per_chunk = tiles_m_chunk * tiles_n
    pos, local = divmod(t, per_chunk)
    chunk = (rank + first + pos) % tp
    group_rows = 8
    per_group = group_rows * tiles_n
    group, in_group = divmod(local, per_group)
    g0 = group * group_rows
    size = min(tiles_m_chunk - g0, group_rows)
    m0 = chunk * rows_per_rank + (g0 + in_group % size) * FBM
    return chunk, m0, in_group // size


class _Rank:
    def __init__(self, tp, blocks, per_chunk):
        self.ag_cnt = [[0] * blocks for _ in range(tp)]         # [src][row block] push units landed
        self.land = [dict(), dict()]                            # parity -> {(chunk, row block): epoch}
        self.rs_cnt = [[0] * per_chunk, [0] * per_chunk]        # [call parity][own tile] -> partial tiles landed
        self.recv = [dict(), dict()]                            # parity -> {(src, tile): epoch}
        self.send = dict()                                      # local send buffer: {global tile: epoch}
        self.send_cnt = [0] * (per_chunk * tp)                  # global tile -> partial warps in the send buffer
        self.own_cnt = [0] * per_chunk                          # own tile -> own-partial warps in y
        self.own_y = dict()                                     # own tile -> epoch of the own partial in y
        self.ar_cnt = [0] * (per_chunk * tp)                    # global tile -> reduced tiles landed
        self.out = [dict(), dict()]                             # parity -> {global tile: ar epoch}
        self.ctr = {"tile": 0, "copy": 0}                       # claim counters (device)
        self.base = {"tile": 0, "copy": 0}                      # what the host believes they hold
        self.seen_tiles: list[int] = []
        self.seen_items: list[int] = []


class Simulation:
    """``tp`` ranks running ``epochs`` calls of one op (``"ag"``, ``"rs"`` or ``"ar"``)."""

    def __init__(self, op, *, tp, rows_per_rank, n, grid, epochs, seed, slices=4, keep_gathered=True,
                 copy_claims=None, push_depth=1, flush_before_wait=True):
        self.k = _ext.require()
        self.op, self.mode = op, MODES[op]
        self.tp, self.rows, self.n, self.grid, self.epochs = tp, rows_per_rank, n, grid, epochs
        self.slices, self.keep = slices, keep_gathered
        # RS / AR partial-tile pushes whose counter release a copy agent may still owe
        # (1: each push is released as soon as its data is complete, as the kernels do;
        # 2+: the release of push i waits until push i+depth-1 is issued). With
        # ``flush_before_wait`` every owed release is paid before the agent waits on a peer.
        self.push_depth, self.flush_before_wait = push_depth, flush_before_wait
        self.rng = random.Random(seed)
        self.blocks = rows_per_rank // FBM
        self.tiles_n = (n + 255) // 256
        self.per_chunk = self.blocks * self.tiles_n
        self.tiles = self.per_chunk * tp
        self.t_rows = rows_per_rank * tp
        self.copy_claims = copy_claims or (lambda: self.k.fused_copy_claims(
            self.mode, self.t_rows, self.n, self.tp, self.slices, self.tp if self.keep else 0, self.grid))
        self.ranks = [_Rank(tp, self.blocks, self.per_chunk) for _ in range(tp)]
        self.slices_red = self.k.fused_red_slices(self.t_rows, n, tp, grid)  # row slices per own-tile reduction

    def _read(self, version, e, what):
        if version != e:
            raise ProtocolError(f"race: {what} holds epoch {version}, expected {e}")

    def _claim(self, me, kind, limit, batch=1):
        got = me.ctr[kind] - me.base[kind]
        me.ctr[kind] += batch
        return got if 0 <= got < limit else -1

    # --- agents (generators yielding wait predicates) ----------------------------------

    def _producer(self, r, e, queue):
        """Claims tiles (at most RING ahead of the epilogue) and loads their inputs."""
        me = self.ranks[r]
        par = e % 2
        first = 0 if self.op == "ag" else 1
        while True:
            yield lambda: queue["claimed"] - queue["done"] < RING
            t = self._claim(me, "tile", self.tiles)
            if t < 0:
                queue["items"].append(None)
                queue["claimed"] += 1
                return
            me.seen_tiles.append(t)
            c, m0, tn = fused_tile(t, self.blocks, self.tiles_n, r, self.tp, first, self.rows)
            rb = (m0 - c * self.rows) // FBM
            if self.op == "ag" and c != r:
                yield lambda c=c, rb=rb: me.ag_cnt[c][rb] >= self.slices * e
                self._read(me.land[par].get((c, rb)), e, f"AG landing of rank {c} block {rb} on rank {r}")
            queue["items"].append((c, rb, tn))
            queue["claimed"] += 1

    def _epilogue(self, r, e, queue, ar_e):
        me = self.ranks[r]
        par = e % 2
        i = 0
        while True:
            yield lambda i=i: len(queue["items"]) > i
            item = queue["items"][i]
            i += 1
            queue["done"] += 1
            if item is None:
                return
            c, rb, tn = item
            local = rb * self.tiles_n + tn
            if self.op == "ag":
                continue
            gtile = (c * self.blocks + rb) * self.tiles_n + tn
            if c != r:
                me.send[gtile] = e                                  # partial into the local send buffer
                yield lambda: True
                me.send_cnt[gtile] += 4                             # four epilogue warps count it
                continue
            me.own_y[local] = e                                     # the own partial into y
            yield lambda: True
            me.own_cnt[local] += 4                                  # for the copy warps' reduction

    def _copy(self, r, e, ar_e, xg):
        """One CTA's copy warps: claim COPY_BATCH items at a time; a batch's pushes land,
        then (one fence) their counts; then its gathered-copy and AR items."""
        me = self.ranks[r]
        par = e % 2
        units = self.blocks * self.slices
        n_push = (self.tp - 1) * units if self.op == "ag" else 0
        n_xg = self.tp * units if (self.op == "ag" and self.keep) else 0
        n_rsp = (self.tp - 1) * self.per_chunk if self.op != "ag" else 0
        n_own = self.per_chunk * self.slices_red if self.op != "ag" else 0
        n_ar = (self.tp - 1) * self.per_chunk if self.op == "ar" else 0
        items = n_push + n_xg if self.op == "ag" else n_rsp + n_own + n_ar
        if items == 0:
            return
        # an RS / AR item is a whole tile (or a slice); AG items come in batches small
        # enough to spread over the grid (fused_gemm.cu ag_copy_batch)
        size = 1 if self.op != "ag" else max(1, min(COPY_BATCH, items // (2 * self.grid)))
        owed = []  # (owner, own tile, parity) of pushed partials whose count is not yet released
        while True:
            first = self._claim(me, "copy", items, size)
            yield lambda: True
            if first < 0:
                self._release(owed, 0)  # a CTA leaves only after every push is counted
                return
            batch = range(first, min(first + size, items))
            me.seen_items.extend(batch)
            pushed = []
            for it in batch:
                if it < n_push:
                    j, u = divmod(it, units)
                    dest = (r - j - 1) % self.tp
                    self.ranks[dest].land[par][(r, u // self.slices)] = e
                    pushed.append((dest, u // self.slices))
            if pushed:
                yield lambda: True
                for dest, rb in pushed:
                    self.ranks[dest].ag_cnt[r][rb] += 1
            for it in batch:
                if self.op != "ag":
                    yield from self._rs_item(r, e, ar_e, it, n_rsp, n_own, owed)
                    continue
                if it < n_push:
                    continue
                if it < n_push + n_xg:
                    i2 = it - n_push
                    c = (r + i2 // units) % self.tp
                    rb = (i2 % units) // self.slices
                    if c != r:
                        yield lambda c=c, rb=rb: me.ag_cnt[c][rb] >= self.slices * e
                        self._read(me.land[par].get((c, rb)), e, f"AG landing of rank {c} block {rb} (xg) on {r}")
                    xg[(c, rb)] = xg.get((c, rb), 0) + 1

    def _release(self, owed, keep):
        """Count the oldest owed pushes in their owners' tile counters until ``keep`` remain."""
        while len(owed) > keep:
            owner, local, par = owed.pop(0)
            self.ranks[owner].rs_cnt[par][local] += 1

    def _rs_item(self, r, e, ar_e, it, n_rsp, n_own, owed):
        """One RS / AR copy item: push a peer-chunk partial tile to its owner, reduce a
        16-row slice of an own tile (and, AR, push it to every peer), or take another
        owner's reduced tile (AR)."""
        me = self.ranks[r]
        par = e % 2
        if it < n_rsp:
            c, m0, tn = fused_tile(it, self.blocks, self.tiles_n, r, self.tp, 1, self.rows)
            rb = (m0 - c * self.rows) // FBM
        elif it < n_rsp + n_own:
            t = n_rsp + (it - n_rsp) // self.slices_red
            c, m0, tn = fused_tile(t, self.blocks, self.tiles_n, r, self.tp, 1, self.rows)
            rb = (m0 - c * self.rows) // FBM
        else:
            i3 = it - n_rsp - n_own
            c = (r + 1 + i3 // self.per_chunk) % self.tp
            rb, tn = divmod(i3 % self.per_chunk, self.tiles_n)
        local = rb * self.tiles_n + tn
        gtile = (c * self.blocks + rb) * self.tiles_n + tn
        if it < n_rsp:
            yield lambda: me.send_cnt[gtile] >= 4 * e
            self._read(me.send.get(gtile), e, f"send buffer tile {gtile} on {r}")
            self.ranks[c].recv[par][(r, local)] = e                 # the partial into the owner
            yield lambda: True
            owed.append((c, local, par))
            self._release(owed, self.push_depth - 1)
            return
        if self.flush_before_wait:
            self._release(owed, 0)  # the items below wait on peers
        if it < n_rsp + n_own:
            if c != r:
                raise ProtocolError(f"own reduction item {it} on rank {r} maps to chunk {c}")
            yield lambda: me.own_cnt[local] >= 4 * e
            yield lambda: me.rs_cnt[par][local] >= (self.tp - 1) * ((e + 1) // 2)
            self._read(me.own_y.get(local), e, f"own partial of tile {local} on {r}")
            for src in range(self.tp):
                if src != r:
                    self._read(me.recv[par].get((src, local)), e, f"RS receive of tile {local} from {src} on {r}")
            if self.op == "ar":
                for p in range(self.tp):
                    if p != r:
                        self.ranks[p].out[ar_e % 2][gtile] = ar_e
                yield lambda: True
                for p in range(self.tp):
                    if p != r:
                        self.ranks[p].ar_cnt[gtile] += 1
        else:
            yield lambda: me.ar_cnt[gtile] >= self.slices_red * ar_e
            self._read(me.out[ar_e % 2].get(gtile), ar_e, f"AR output tile {gtile} on {r}")

    # --- the scheduler -------------------------------------------------------------------

    def _call_agents(self, r, e):
        me = self.ranks[r]
        me.seen_tiles, me.seen_items = [], []
        self._xg = getattr(self, "_xg", {})
        self._xg[r] = {}
        agents = []
        for _ in range(self.grid):
            queue = {"items": [], "claimed": 0, "done": 0}
            agents.append(self._producer(r, e, queue))
            agents.append(self._epilogue(r, e, queue, e))
            agents.append(self._copy(r, e, e, self._xg[r]))
        return agents

    def _finish_call(self, r, e):
        me = self.ranks[r]
        if sorted(me.seen_tiles) != list(range(self.tiles)):
            raise ProtocolError(f"call {e} on rank {r} computed tiles {sorted(me.seen_tiles)}, not each tile once")
        if self.op == "ag" and self.keep:
            units = self.blocks * self.slices
            full = {(c, rb): self.slices for c in range(self.tp) for rb in range(self.blocks)}
            if self._xg[r] != full or len(me.seen_items) != (2 * self.tp - 1) * units:
                raise ProtocolError(f"call {e} on rank {r}: gathered copy incomplete")
        # the host advances its bases by what the extension says a launch claims
        me.base["tile"] += self.k.fused_tile_claims(self.t_rows, self.n, self.grid)
        me.base["copy"] += self.copy_claims()
        if me.base["tile"] != me.ctr["tile"] or me.base["copy"] != me.ctr["copy"]:
            raise ProtocolError(f"race: host bases {me.base} disagree with the claim counters {me.ctr} on rank {r}")

    def run(self) -> int:
        """Interleave every call of every rank; return the number of scheduling steps."""
        epoch = [1] * self.tp
        live = {r: [[a, None] for a in self._call_agents(r, 1)] for r in range(self.tp)}
        steps = 0
        while live:
            ready = []
            for r, agents in live.items():
                for slot in agents:
                    cond = slot[1]
                    if cond is None or cond():
                        ready.append((r, slot))
            if not ready:
                raise ProtocolError(f"deadlock at epochs {epoch}: every agent waits")
            r, slot = self.rng.choice(ready)
            try:
                slot[1] = next(slot[0])
            except StopIteration:
                live[r].remove(slot)
                if not live[r]:
                    self._finish_call(r, epoch[r])
                    epoch[r] += 1
                    if epoch[r] > self.epochs:
                        del live[r]
                    else:
                        live[r] = [[a, None] for a in self._call_agents(r, epoch[r])]
            steps += 1
        return steps


class DpSimulation:
    """``dp`` replicas running ``epochs`` training steps, each: backward accumulates into
    the current gradient buffer, then the fused DP kernel (``peer_state.cu``) -- per CTA:
    announce the epoch in every peer's flag array and wait for every peer's; then either
    (one-phase) read every replica's current buffer for the CTA's slice and write the sum
    into the local other buffer, or (``push``) reduce this replica's part of the slice
    from every replica's current buffer, push the sum into every replica's other buffer,
    flag it in a second flag array, wait for every peer's part, and read the whole slice
    from the local other buffer -- after which the buffers swap roles (the next backward
    zeroes and fills the summed one)."""

    def __init__(self, *, dp, grid, epochs, seed, push=False):
        self.dp, self.grid, self.epochs, self.push = dp, grid, epochs, push
        self.rng = random.Random(seed)
        # per replica: flag words [grid][dp] (two arrays), two gradient buffers of
        # per-(slice, part) versions
        self.flags = [[[0] * dp for _ in range(grid)] for _ in range(dp)]
        self.flags2 = [[[0] * dp for _ in range(grid)] for _ in range(dp)]
        self.grads = [[dict(), dict()] for _ in range(dp)]
        self.parity = [0] * dp

    def _backward(self, r, e):
        cur = self.parity[r]
        for b in range(self.grid):
            for q in range(self.dp):
                self.grads[r][cur][(b, q)] = ("acc", e)                 # zeroed, then accumulated
            yield lambda: True

    def _check(self, got, want, what):
        if got != want:
            raise ProtocolError(f"race: {what} holds {got}, expected {want}")

    def _cta(self, r, b, e):
        cur = self.parity[r]
        for q in range(self.dp):
            if q != r:
                self.flags[q][b][r] = max(self.flags[q][b][r], e)       # release store of the epoch
        yield lambda: all(self.flags[r][b][q] >= e for q in range(self.dp) if q != r)
        if not self.push:
            for q in range(self.dp):
                for part in range(self.dp):
                    self._check(self.grads[q][cur].get((b, part)), ("acc", e), f"replica {q} slice {b}")
                yield lambda: True
            for part in range(self.dp):
                self.grads[r][1 - cur][(b, part)] = ("sum", e)
            return
        for q in range(self.dp):
            self._check(self.grads[q][cur].get((b, r)), ("acc", e), f"replica {q} slice {b} part {r}")
            yield lambda: True
        for q in range(self.dp):
            # the same buffer index in every replica's region (the layouts are identical)
            self.grads[q][1 - cur][(b, r)] = ("sum", e)
            yield lambda: True
        for q in range(self.dp):
            if q != r:
                self.flags2[q][b][r] = max(self.flags2[q][b][r], e)
        yield lambda: all(self.flags2[r][b][q] >= e for q in range(self.dp) if q != r)
        for part in range(self.dp):
            self._check(self.grads[r][1 - cur].get((b, part)), ("sum", e), f"replica {r} sum slice {b} part {part}")

    def run(self) -> int:
        phase = {r: ("backward", 1) for r in range(self.dp)}
        live = {r: [[self._backward(r, 1), None]] for r in range(self.dp)}
        steps = 0
        while live:
            ready = [(r, s) for r, agents in live.items() for s in agents if s[1] is None or s[1]()]
            if not ready:
                raise ProtocolError(f"deadlock in phases {phase}")
            r, slot = self.rng.choice(ready)
            try:
                slot[1] = next(slot[0])
            except StopIteration:
                live[r].remove(slot)
                if not live[r]:
                    kind, e = phase[r]
                    if kind == "backward":
                        phase[r] = ("kernel", e)
                        live[r] = [[self._cta(r, b, e), None] for b in range(self.grid)]
                    else:
                        self.parity[r] = 1 - self.parity[r]              # the summed buffer is now current
                        if e == self.epochs:
                            del live[r]
                        else:
                            phase[r] = ("backward", e + 1)
                            live[r] = [[self._backward(r, e + 1), None]]
            steps += 1
        return steps
