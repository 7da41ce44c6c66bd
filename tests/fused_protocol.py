"""A model of the fused TP kernels' cross-GPU protocol, for race and deadlock checks.

Mirrors ``resihp/csrc/fused_gemm.cu`` at the level of what synchronises: every copy
warp, TMA producer and epilogue of every CTA of every rank is an agent; flag words and
counters are shared integers; data buffers hold, per row or tile, the epoch whose values
they contain. A random scheduler interleaves the agents (each rank's calls run in stream
order), every wait blocks until its condition holds, and every read of data checks that
the data is the epoch being computed -- a stale or overwritten row is a race. If no agent
can move while some are unfinished, the protocol deadlocked (the kernels' bounded waits
would report error code 4). The host side -- the counter bases advanced per call and
the per-call targets -- comes from the extension's own host functions, so a mismatch
between what the host expects and what the kernel's warps add (the bug class met on a
GPU once) shows up here as a deadlock.
"""

from __future__ import annotations

import random

from resihp.ops import _ext

FBM = 128


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
    def __init__(self, tp, rows_per_rank, tiles):
        t = rows_per_rank * tp
        self.sig = [0] * 8
        self.pub = 0
        self.ready = [0] * tp
        self.rb_ready = [0] * (t // FBM)
        self.slot = [[None] * rows_per_rank, [None] * rows_per_rank]
        self.xg = [None] * t
        self.part = [dict(), dict()]
        self.flags = [0] * tiles
        self.recv = {}
        self.pulled = {}
        # host bookkeeping of the workspace
        self.pub_base = self.ready_base = self.rb_base = 0


class Simulation:
    """``tp`` ranks running ``epochs`` calls of one op (``"ag"`` or ``"rs"``)."""

    def __init__(self, op, *, tp, rows_per_rank, n, grid, variant, epochs, seed, host_step=None):
        self.k = _ext.require()
        self.op, self.tp, self.rows, self.n, self.grid, self.variant = op, tp, rows_per_rank, n, grid, variant
        self.epochs = epochs
        self.rng = random.Random(seed)
        self.cw = self.k.fused_counter_step(1, variant)            # copy warps per CTA
        self.host_step = host_step or (lambda g: self.k.fused_counter_step(g, variant))
        self.tiles_m_chunk = rows_per_rank // FBM
        self.tiles_n = (n + 255) // 256
        self.tiles = self.tiles_m_chunk * self.tiles_n * tp
        self.ranks = [_Rank(tp, rows_per_rank, self.tiles) for _ in range(tp)]
        t_rows = rows_per_rank * tp
        self.slices = self.k.fused_block_step(t_rows, n, tp, grid) // self.k.fused_counter_step(1, 1)

    # --- agents (generators yielding wait predicates) ----------------------------------

    def _rows_of(self, b, w):
        lo = self.rows * b // self.grid
        hi = self.rows * (b + 1) // self.grid
        return list(range(lo + w, hi, self.cw))

    def _ag_copy(self, r, b, w, e, pub_target):
        me = self.ranks[r]
        par = e % 2
        for row in self._rows_of(b, w):                                 # publish
            me.slot[par][row] = e
            me.xg[r * self.rows + row] = e
        yield lambda: True
        me.pub += 1
        if me.pub == pub_target:
            for p in range(self.tp):
                if p != r:
                    self.ranks[p].sig[r] = e                            # announce to every peer
        if self.variant == 0:
            for step in range(1, self.tp):
                c = (r + step) % self.tp
                yield lambda c=c: me.sig[c] >= e
                for row in self._rows_of(b, w):
                    self._read(self.ranks[c].slot[par][row], e, f"AG slot of rank {c} row {row}")
                    me.xg[c * self.rows + row] = e
                yield lambda: True
                me.ready[c] += 1
        else:
            blocks, s = self.tiles_m_chunk, self.slices
            srows = FBM // s
            units = (self.tp - 1) * blocks * s
            for u in range(b, units, self.grid):
                c = (r + 1 + u // (blocks * s)) % self.tp
                rb = (u // s) % blocks
                r0 = rb * FBM + (u % s) * srows
                yield lambda c=c: me.sig[c] >= e
                for row in range(r0 + w, r0 + srows, self.cw):
                    self._read(self.ranks[c].slot[par][row], e, f"AG slot of rank {c} row {row}")
                    me.xg[c * self.rows + row] = e
                me.rb_ready[c * blocks + rb] += 1

    def _ag_producer(self, r, b, e, ready_target, rb_target):
        me = self.ranks[r]
        for t in range(b, self.tiles, self.grid):
            c, m0, _tn = fused_tile(t, self.tiles_m_chunk, self.tiles_n, r, self.tp, 0, self.rows)
            if c == r:
                continue
            if self.variant == 0:
                yield lambda c=c: me.ready[c] >= ready_target
            else:
                key = c * self.tiles_m_chunk + (m0 - c * self.rows) // FBM
                yield lambda key=key: me.rb_ready[key] >= rb_target
            for row in range(m0, m0 + FBM):
                self._read(me.xg[row], e, f"AG gathered row {row} on rank {r}")

    def _rs_tiles(self, r, b):
        out = []
        for t in range(b, self.tiles, self.grid):
            c, m0, tn = fused_tile(t, self.tiles_m_chunk, self.tiles_n, r, self.tp, 1, self.rows)
            out.append((c, (m0 // FBM) * self.tiles_n + tn))
        return out

    def _rs_epilogue(self, r, b, e):
        me = self.ranks[r]
        par = e % 2
        j = 0
        for c, flag in self._rs_tiles(r, b):
            if c != r:
                me.part[par][flag] = e                                  # partial tile of a peer's rows
                me.flags[flag] += 4                                     # four epilogue warps
                yield lambda: True
            else:
                yield lambda j=j: me.pulled.get((e, b, j), 0) >= self.cw
                for src in range(self.tp):
                    if src != r:
                        self._read(me.recv.get((src, flag)), e, f"RS receive of tile {flag} from {src}")
                j += 1

    def _rs_copy(self, r, b, w, e):
        me = self.ranks[r]
        par = e % 2
        j = 0
        for c, flag in self._rs_tiles(r, b):
            if c != r:
                continue
            peers = [s for s in range(self.tp) if s != r]
            mine = peers if self.variant == 0 else [s for i, s in enumerate(peers) if i % self.cw == w]
            pending = list(mine)
            while pending:
                if self.variant == 0:
                    src = pending[0]
                    yield lambda src=src: self.ranks[src].flags[flag] >= 4 * e
                else:
                    yield lambda: any(self.ranks[s].flags[flag] >= 4 * e for s in pending)
                    src = next(s for s in pending if self.ranks[s].flags[flag] >= 4 * e)
                self._read(self.ranks[src].part[par].get(flag), e, f"RS partial tile {flag} of rank {src}")
                me.recv[(src, flag)] = e
                pending.remove(src)
            me.pulled[(e, b, j)] = me.pulled.get((e, b, j), 0) + 1
            j += 1

    def _read(self, version, e, what):
        if version != e:
            raise ProtocolError(f"race: {what} holds epoch {version}, expected {e}")

    # --- the scheduler -------------------------------------------------------------------

    def _call_agents(self, r, e):
        me = self.ranks[r]
        step = self.host_step(self.grid)
        agents = []
        if self.op == "ag":
            pub_target = me.pub_base + step
            ready_target = me.ready_base + step
            rb_target = me.rb_base + self.k.fused_block_step(self.rows * self.tp, self.n, self.tp, self.grid)
            for b in range(self.grid):
                agents.append(self._ag_producer(r, b, e, ready_target, rb_target))
                for w in range(self.cw):
                    agents.append(self._ag_copy(r, b, w, e, pub_target))
            me.pub_base += step
            if self.variant == 0:
                me.ready_base += step
            else:
                me.rb_base += self.k.fused_block_step(self.rows * self.tp, self.n, self.tp, self.grid)
        else:
            for b in range(self.grid):
                agents.append(self._rs_epilogue(r, b, e))
                for w in range(self.cw):
                    agents.append(self._rs_copy(r, b, w, e))
        return agents

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
    announce the epoch in every peer's flag array, wait for every peer's announcement,
    read every replica's current buffer for the CTA's slice, write the sum into the other
    buffer -- after which the buffers swap roles (the next backward zeroes and fills the
    summed one)."""

    def __init__(self, *, dp, grid, epochs, seed):
        self.dp, self.grid, self.epochs = dp, grid, epochs
        self.rng = random.Random(seed)
        # per replica: flag words [grid][dp], two gradient buffers of per-slice versions
        self.flags = [[[0] * dp for _ in range(grid)] for _ in range(dp)]
        self.grads = [[[None] * grid, [None] * grid] for _ in range(dp)]
        self.parity = [0] * dp

    def _backward(self, r, e):
        cur = self.parity[r]
        for b in range(self.grid):
            self.grads[r][cur][b] = ("acc", e)                          # zeroed, then accumulated
            yield lambda: True

    def _cta(self, r, b, e):
        cur = self.parity[r]
        for q in range(self.dp):
            if q != r:
                self.flags[q][b][r] = max(self.flags[q][b][r], e)       # release store of the epoch
        yield lambda: all(self.flags[r][b][q] >= e for q in range(self.dp) if q != r)
        for q in range(self.dp):
            # every replica's buffer of this epoch holds this step's accumulation
            got = self.grads[q][cur][b]
            if got != ("acc", e):
                raise ProtocolError(f"race: replica {q} slice {b} holds {got}, expected the epoch-{e} gradients")
            yield lambda: True
        self.grads[r][1 - cur][b] = ("sum", e)

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
