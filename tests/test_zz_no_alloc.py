"""b2g_enqueue_static: the no-allocation entry point (library's static scratch).

Collected last (file name) so that it also runs after every other GPU test
has used the device; each test passes alone as well.  Results must be
bit-identical to b2g_enqueue_ex with a caller-allocated workspace -- the
kernel and its summation order are the same, only the scratch differs -- on
two calls in a row, so the second call sees the scratch the first one left.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _op_and_weights(b2g, orc, syn, K, N, wd, mode, fuse=0, seed=51):
    op = b2g.GemvOp(K, N, weight_dtype=wd, scale_mode=mode, max_m=8, fuse=fuse)
    planes = []
    scales = []
    for j in range(2 if fuse & b2g.FUSE_GATE_UP_SILU else 1):
        W = syn.weights(seed + j, K, N)
        if wd == 0:
            planes.append(dev(W))
        else:
            q, s = orc.quantize_e4m3(W, mode)
            planes.append(dev(q))
            if s is not None:
                scales.append(s)
    packed = op.prepack(*planes)
    s = None if not scales else dev(np.concatenate(scales))
    return op, packed, s


# (K, N, weight dtype, scale mode, fusion): split-K down projection, fused
# gate||up with RMSNorm, an FP16 op, and a small ragged shape.
CASES = [
    (8192, 3072, 1, 3, 0),
    (3072, 8192, 1, 3, 1 | 2),
    (3072, 8192, 0, 0, 0),
    (200, 120, 1, 2, 0),
]


@pytest.mark.parametrize("K,N,wd,mode,fuse", CASES)
def test_static_matches_enqueue_ex_twice(b2g, orc, syn, cuda, K, N, wd, mode, fuse):
    op, packed, s = _op_and_weights(b2g, orc, syn, K, N, wd, mode, fuse)
    assert op.workspace_bytes() <= b2g.STATIC_SCRATCH_BYTES
    for M in (1, 8):
        x = dev(syn.activations(300 + M, M, K))
        want = op.enqueue(x, packed, s)
        ys = [torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda") for _ in range(2)]
        for y in ys:
            op.enqueue_static(x, packed, y, s)
        torch.cuda.synchronize()
        for y in ys:
            assert torch.equal(y, want), (K, N, M)
    assert b2g.device_error() == 0


def test_static_residual_add(b2g, orc, syn, cuda):
    K, N = 8192, 3072
    op, packed, s = _op_and_weights(b2g, orc, syn, K, N, 1, 3, b2g.FUSE_RESIDUAL_ADD)
    x = dev(syn.activations(311, 4, K))
    r = dev(syn.activations(312, 4, N))
    want = op.enqueue(x, packed, s, residual=r)
    for _ in range(2):
        y = torch.empty((4, N), dtype=torch.float16, device="cuda")
        op.enqueue_static(x, packed, y, s, residual=r)
        torch.cuda.synchronize()
        assert torch.equal(y, want)


def test_static_ops_interleaved_in_one_stream(b2g, orc, syn, cuda):
    """Ops with different tile counts take turns on the one scratch."""
    a = _op_and_weights(b2g, orc, syn, 8192, 3072, 1, 3)
    b = _op_and_weights(b2g, orc, syn, 3072, 8192, 1, 3, seed=61)
    xa = dev(syn.activations(321, 8, 8192))
    xb = dev(syn.activations(322, 8, 3072))
    want_a = a[0].enqueue(xa, a[1], a[2])
    want_b = b[0].enqueue(xb, b[1], b[2])
    outs = []
    for op, packed, s, x, n in ((*a, xa, 3072), (*b, xb, 8192), (*a, xa, 3072), (*b, xb, 8192)):
        y = torch.empty((8, n), dtype=torch.float16, device="cuda")
        outs.append(op.enqueue_static(x, packed, y, s))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], want_a) and torch.equal(outs[2], want_a)
    assert torch.equal(outs[1], want_b) and torch.equal(outs[3], want_b)


def test_static_makes_no_torch_allocation(b2g, orc, syn, cuda):
    op, packed, s = _op_and_weights(b2g, orc, syn, 8192, 3072, 1, 3)
    x = dev(syn.activations(331, 2, 8192))
    y = torch.empty((2, 3072), dtype=torch.float16, device="cuda")
    op.enqueue_static(x, packed, y, s)
    torch.cuda.synchronize()
    before = torch.cuda.memory_stats()["allocation.all.allocated"]
    op.enqueue_static(x, packed, y, s)
    op.enqueue_static(x, packed, y, s)
    torch.cuda.synchronize()
    assert torch.cuda.memory_stats()["allocation.all.allocated"] == before


def test_static_rejects_oversize_and_workspace(b2g, cuda):
    """A call needing more than the static scratch fails with
    ERR_SCRATCH_LIMIT before anything is launched; a caller workspace is
    refused (that is b2g_enqueue_ex's job)."""
    import ctypes
    # 4096 CTAs on gate||up cut into equal byte ranges: up to 8 CTAs share a
    # tile, 4.1 MiB of partials.
    big = b2g.GemvOp(3072, 8192, weight_dtype="fp8_e4m3", scale_mode="none", max_m=8,
                     fuse=b2g.FUSE_GATE_UP_SILU)
    big.set_option(b2g.OPT_PARTITION, b2g.PARTITION_UNITS)
    big.set_option(b2g.OPT_GRID, 4096)
    assert big.workspace_bytes() > b2g.STATIC_SCRATCH_BYTES
    x = torch.zeros((1, 3072), dtype=torch.float16, device="cuda")
    y = torch.full((1, 8192), 7.0, dtype=torch.float16, device="cuda")
    packed = torch.zeros(16, dtype=torch.uint8, device="cuda")  # never read: the call is refused first
    with pytest.raises(b2g.B2GError) as e:
        big.enqueue_static(x, packed, y)
    assert e.value.status == b2g.ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())

    small = b2g.GemvOp(200, 120, weight_dtype="fp8_e4m3", scale_mode="none", max_m=8)
    ws = small.workspace()
    a = b2g.EnqueueArgs(1, x.data_ptr(), 200, packed.data_ptr(), 0, 0, 0, y.data_ptr(), 120,
                        ws.data_ptr(), 1e-5, 0, None, None)
    st = b2g.lib().b2g_enqueue_static(small.h, ctypes.byref(a), b2g._stream(None))
    assert st == b2g.ERR_INVALID
