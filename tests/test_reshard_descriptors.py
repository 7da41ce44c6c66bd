"""The state-move copy descriptors, executed on the host.

``GatherPlan`` turns shard pieces into raw-address copy descriptors for the GPU gather
kernel: byte offsets of the three state fields inside each rank's flat-state region, the
tensor's element offset in the donor's and in the target's layout, row strides, and the
target's bf16 compute copy. Here the regions are host buffers and a small interpreter
performs exactly what the kernel does for each descriptor row (a strided fp32 copy
plus, for the master field, the bf16 copy), so the address arithmetic is checked against
``local_slice`` on CPU.
"""

import ctypes

import torch

from resihp.models.layout import TensorSpec
from resihp.ops import _ext
from resihp.parallel import peer
from resihp.parallel.tp import FlatState, local_slice

LOGICAL = [("a", (40, 24), 0), ("b", (24, 40), 1), ("n", (24,), None), ("c", (30, 12), 1)]


class _HostRegions:
    """Stands in for the extension's region allocator: host buffers, no IPC."""

    def __init__(self):
        self.keep = []

    def symm_region(self, total, device):
        t = torch.zeros(total, dtype=torch.uint8)
        self.keep.append(t)
        return t, b"host"


def _flat(degree, index):
    entries = [(TensorSpec(n, s, d, "normal"), tuple(local_slice(torch.empty(s), d, index, degree).shape))
               for n, s, d in LOGICAL]
    return FlatState(entries, "cpu", torch.bfloat16, shared=True)


def _execute(rows):
    """The gather kernel's semantics, descriptor by descriptor (host memory)."""
    for src, dst, bf16, src_ld, dst_ld, nrows, cols, _base, _vec4 in rows:
        for r in range(nrows):
            s = src + 4 * r * src_ld
            d = dst + 4 * r * dst_ld
            ctypes.memmove(d, s, 4 * cols)
            if bf16:
                vals = torch.frombuffer(bytearray(ctypes.string_at(s, 4 * cols)), dtype=torch.float32)
                out = vals.bfloat16()
                ctypes.memmove(bf16 + 2 * r * dst_ld, out.data_ptr(), 2 * cols)


def test_gather_descriptors_rebuild_local_slices(monkeypatch):
    host = _HostRegions()
    monkeypatch.setattr(_ext, "require", lambda: host)
    g = torch.Generator().manual_seed(3)
    fulls = {n: {f: torch.randn(s, generator=g) for f in ("param", "exp_avg", "exp_avg_sq")} for n, s, _d in LOGICAL}
    for old, new in ((2, 1), (1, 2), (2, 2), (1, 1)):
        donors = []
        for i in range(old):
            f = _flat(old, i)
            for name, s, d in LOGICAL:
                f.view(f.master, name).copy_(local_slice(fulls[name]["param"], d, i, old))
                f.view(f.exp_avg, name).copy_(local_slice(fulls[name]["exp_avg"], d, i, old))
                f.view(f.exp_avg_sq, name).copy_(local_slice(fulls[name]["exp_avg_sq"], d, i, old))
            donors.append(f)
        for t in range(new):
            target = _flat(new, t)
            plan = peer.GatherPlan()
            for name, s, d in LOGICAL:
                for piece in peer.shard_pieces(s, d, old, new, t):
                    src = donors[piece.donor]
                    plan.add([piece], src_region=src.region_ptr, src_fields=src.field_offsets,
                             src_tensor_off=src.offsets[name][0], dst_flat=target,
                             dst_tensor_off=target.offsets[name][0])
            assert plan.items == sum(row[5] for row in plan.rows)
            _execute(plan.rows)
            for name, s, d in LOGICAL:
                for f, buf in (("param", target.master), ("exp_avg", target.exp_avg), ("exp_avg_sq", target.exp_avg_sq)):
                    assert torch.equal(target.view(buf, name), local_slice(fulls[name][f], d, t, new)), (old, new, name, f)
                assert torch.equal(target.view(target.work, name), local_slice(fulls[name]["param"], d, t, new).bfloat16())


def test_split_rows_descriptors_keep_item_order(monkeypatch):
    host = _HostRegions()
    monkeypatch.setattr(_ext, "require", lambda: host)
    a, b = _flat(1, 0), _flat(1, 0)
    plan = peer.GatherPlan()
    n = 40 * 24
    plan.add([peer.Piece(0, 0, n, 0, n, 1, n)], src_region=a.region_ptr, src_fields=a.field_offsets,
             src_tensor_off=a.offsets["a"][0], dst_flat=b, dst_tensor_off=b.offsets["a"][0])
    bases = [row[7] for row in plan.rows]
    assert bases == sorted(bases) and bases[0] == 0  # the kernel binary-searches item_base
    assert all(row[6] <= peer.COPY_ROW for row in plan.rows)
