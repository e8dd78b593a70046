"""GPU parity: the CUDA path (through the C ABI) against the CPU oracle.

Tolerances: rel-L2 <= 1e-3 for FP16 weights and <= 5e-3 for
E4M3 weights, measured against the fp64 oracle over the same quantised bytes
and scales; max-abs is asserted against a stated bound as well.  Quantisation
itself is bit-exact.  The reference's own acceptance gates are checked on its
own `check` inputs: cos >= 0.999 (FP8, kernels/gemv_fp8.cu:392) and
cos > 0.9999 with max_rel < 0.05 (FP16, kernels/gemv_fp16.cu:342).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN

pytestmark = pytest.mark.gpu

TOL = {0: 1e-3, 1: 5e-3}  # weight dtype -> rel-L2 bound
MAX_ABS = {0: 2e-2, 1: 5e-2}  # outputs here are O(1); fp16 ulp at 8 is 2^-7


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def make_weights(orc, syn, seed, K, N, wdtype, mode, layout=0):
    """(device W for prepack, host W, host scales) with W in `layout`."""
    W16 = syn.weights(seed, K, N)
    Wl = W16 if layout == 0 else np.ascontiguousarray(W16.T)
    if wdtype == 0:
        return dev(Wl), Wl, None
    q, s = orc.quantize_e4m3(Wl, mode, layout)
    return dev(q), q, s


def run_op(b2g, K, N, wd, mode, x, Wd, s, layout=0, fuse=0, w1=None, **kw):
    op = b2g.GemvOp(K, N, weight_dtype=wd, scale_mode=mode, layout=layout, max_m=8, fuse=fuse)
    for k, v in kw.pop("options", {}).items():
        op.set_option(k, v)
    packed = op.prepack(Wd, w1)
    y = op.enqueue(x, packed, None if s is None else dev(s), **kw)
    torch.cuda.synchronize()
    return op, packed, y


def check(orc, got, want, wd, what=""):
    r = orc.compare(host(got), want)
    assert r["rel_l2"] <= TOL[wd], (what, r)
    assert r["max_abs"] <= MAX_ABS[wd] * max(1.0, np.abs(want).max() / 4), (what, r)
    return r


# --------------------------------------------------------------------------
# Quantisation: bit-exact against the oracle
# --------------------------------------------------------------------------
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
@pytest.mark.parametrize("layout", [0, 1])
def test_quantize_bit_exact(b2g, orc, syn, cuda, mode, layout):
    W = syn.weights(21, 200, 120)
    W[3, :] *= 40  # a few large values (fp16 scale modes saturate differently)
    Wl = W if layout == 0 else np.ascontiguousarray(W.T)
    q, s = b2g.quantize_e4m3(dev(Wl), mode, layout)
    qo, so = orc.quantize_e4m3(Wl, mode, layout)
    assert np.array_equal(host(q), qo)
    if so is not None:
        assert np.array_equal(host(s).view(np.uint8), so.view(np.uint8))


def test_quantize_bit_exact_full_shape(b2g, orc, syn, cuda):
    W = syn.weights(1000, 3072, 8192)
    q, s = b2g.quantize_e4m3(dev(W), "channel_fp32")
    qo, so = orc.quantize_e4m3(W, orc.SCALE_CHANNEL_FP32)
    assert np.array_equal(host(s), so)
    assert np.array_equal(host(q), qo)


# --------------------------------------------------------------------------
# GEMV parity
# --------------------------------------------------------------------------
SHAPES = [(3072, 8192), (8192, 3072), (200, 120), (33, 17), (1000, 40), (64, 4096)]


@pytest.mark.parametrize("K,N", SHAPES)
@pytest.mark.parametrize("wd,mode", [(1, 3), (1, 0), (1, 2), (1, 1), (0, 0)])
def test_gemv_parity(b2g, orc, syn, cuda, K, N, wd, mode):
    Wd, Wh, s = make_weights(orc, syn, 31, K, N, wd, mode)
    for M in (1, 2, 4, 8):
        x = syn.activations(100 + M, M, K)
        _, _, y = run_op(b2g, K, N, wd, mode, dev(x), Wd, s)
        want = orc.gemv(Wh, orc.WTYPE_FP8 if wd else orc.WTYPE_FP16, x, mode, s)
        check(orc, y, want, wd, (K, N, M))


# The adjacent decode projections of the same model, on the same kernels:
# qkv_proj 3072 -> 5120 (320 tiles) and o_proj 3072 -> 3072 (192 tiles).
@pytest.mark.parametrize("K,N", [(3072, 5120), (3072, 3072)])
@pytest.mark.parametrize("wd,mode", [(1, 3), (0, 0)])
def test_adjacent_decode_projections(b2g, orc, syn, cuda, K, N, wd, mode):
    Wd, Wh, s = make_weights(orc, syn, 41, K, N, wd, mode)
    for M in (1, 8):
        x = syn.activations(500 + M, M, K)
        _, _, y = run_op(b2g, K, N, wd, mode, dev(x), Wd, s)
        want = orc.gemv(Wh, orc.WTYPE_FP8 if wd else orc.WTYPE_FP16, x, mode, s)
        check(orc, y, want, wd, (K, N, M))


def test_vocab_projection_in_waves(b2g, orc, cuda):
    """lm_head 3072 -> 128256 (8016 tiles): more tiles per CTA than its shared
    slots hold at one CTA per SM, so the planner launches more CTAs, run as
    successive waves.  Weights are drawn on the device (394 M of them) and
    quantised there (bit-exact against the oracle elsewhere); the output is
    checked against the oracle on column blocks at both ends and the middle."""
    K, N = 3072, 128256
    g = torch.Generator(device=cuda).manual_seed(55)
    W = (torch.randn(K, N, generator=g, device=cuda) * 0.02).half()
    q, s = b2g.quantize_e4m3(W, "channel_fp32")
    del W
    op = b2g.GemvOp(K, N, weight_dtype=1, scale_mode="channel_fp32", max_m=8)
    plan = op.plan(8)
    assert plan["n_slots"] <= 8 and plan["grid"] * plan["n_slots"] >= plan["n_tiles"], plan
    packed = op.prepack(q)
    qh, sh = host(q), host(s)
    rng = np.random.default_rng(56)
    for M in (1, 8):
        x = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
        y = host(op.enqueue(dev(x), packed, s))
        for lo in (0, N // 2 - 2048, N - 4096):
            cols = slice(lo, lo + 4096)
            want = orc.gemv(np.ascontiguousarray(qh[:, cols]), orc.WTYPE_FP8, x, orc.SCALE_CHANNEL_FP32,
                            np.ascontiguousarray(sh[cols]))
            r = orc.compare(y[:, cols], want)
            assert r["rel_l2"] <= TOL[1], (M, lo, r)
            assert r["max_abs"] <= MAX_ABS[1] * max(1.0, np.abs(want).max() / 4), (M, lo, r)
    assert b2g.device_error() == 0


@pytest.mark.parametrize("K,N", [(3072, 8192), (200, 120)])
def test_gemv_nk_layout(b2g, orc, syn, cuda, K, N):
    for wd in (0, 1):
        mode = 3 if wd else 0
        Wd, Wh, s = make_weights(orc, syn, 32, K, N, wd, mode, layout=1)
        x = syn.activations(7, 8, K)
        _, _, y = run_op(b2g, K, N, wd, mode, dev(x), Wd, s, layout=1)
        want = orc.gemv(Wh, orc.WTYPE_FP8 if wd else orc.WTYPE_FP16, x, mode, s, orc.LAYOUT_NK)
        check(orc, y, want, wd)


def test_reference_check_inputs_fp8_and_fp16(b2g, orc, cuda):
    """The reference's `check` inputs (srand(1234) uniform, no scale) at both
    shapes, against its own fp64 outputs (tests/golden/ref_gemv_full.npz)."""
    z = np.load(GOLDEN / "ref_gemv_full.npz")
    for name, K, N in (("up", 3072, 8192), ("down", 8192, 3072)):
        W, x = orc.fill_host_ref(K, N)
        q = orc.f16_to_e4m3(W)
        _, _, y8 = run_op(b2g, K, N, 1, 0, dev(x[None]), dev(q), None)
        r8 = orc.compare(host(y8)[0], z[f"{name}_y_e4m3"])
        assert r8["cos"] >= 0.999 and r8["rel_l2"] <= 5e-3, r8
        _, _, y16 = run_op(b2g, K, N, 0, 0, dev(x[None]), dev(W), None)
        r16 = orc.compare(host(y16)[0], z[f"{name}_y_fp16"])
        assert r16["cos"] > 0.9999 and r16["max_rel"] < 0.05 and r16["rel_l2"] <= 1e-3, r16


def test_cfg0_fp16_seed0(b2g, orc, syn, cuda):
    z = np.load(GOLDEN / "cfg0_fp16.npz")
    W, x = syn.cfg0_fp16_gemv()
    _, _, y = run_op(b2g, 3072, 8192, 0, 0, dev(x), dev(W), None)
    r = orc.compare(host(y)[0], z["y"])
    assert r["rel_l2"] <= 1e-3 and r["cos"] > 0.9999, r


def test_unaligned_rows_and_strides(b2g, orc, syn, cuda):
    K, N = 200, 120
    Wd, Wh, s = make_weights(orc, syn, 33, K, N, 1, 3)
    xbig = syn.activations(9, 5, K + 3)  # row stride K+3: no 16-byte row alignment
    x = dev(xbig)[:, :K]
    y = torch.zeros((5, N + 5), dtype=torch.float16, device="cuda")[:, :N]
    _, _, y = run_op(b2g, K, N, 1, 3, x, Wd, s, y=y)
    want = orc.gemv(Wh, orc.WTYPE_FP8, xbig[:, :K], 3, s)
    check(orc, y, want, 1)


# --------------------------------------------------------------------------
# Stream-K properties
# --------------------------------------------------------------------------
@pytest.mark.parametrize("K,N,grid", [(8192, 3072, 148), (8192, 3072, 160), (8192, 3072, 296),
                                      (8192, 3072, 500), (3072, 8192, 120), (3072, 8192, 296)])
def test_grid_partitions(b2g, orc, syn, cuda, K, N, grid):
    Wd, Wh, s = make_weights(orc, syn, 34, K, N, 1, 3)
    x = syn.activations(10, 8, K)
    _, _, y = run_op(b2g, K, N, 1, 3, dev(x), Wd, s, options={b2g.OPT_GRID: grid})
    check(orc, y, orc.gemv(Wh, orc.WTYPE_FP8, x, 3, s), 1, grid)


@pytest.mark.parametrize("part", ["units", "tiles"])
@pytest.mark.parametrize("K,N,fuse,grid", [(3072, 8192, 0, 0), (8192, 3072, 0, 0), (200, 120, 0, 0),
                                           (3072, 8192, 3, 0), (8192, 3072, 0, 120), (1000, 40, 0, 0)])
def test_partition_modes(b2g, orc, syn, cuda, part, K, N, fuse, grid):
    """Equal byte ranges (tiles split between CTAs) and whole tiles per CTA."""
    mode = {"units": b2g.PARTITION_UNITS, "tiles": b2g.PARTITION_TILES}[part]
    Wd, Wh, s = make_weights(orc, syn, 35, K, N, 1, 3)
    w1 = None
    if fuse & b2g.FUSE_GATE_UP_SILU:
        Wd1, Wh1, s1 = make_weights(orc, syn, 36, K, N, 1, 3)
        w1, s = Wd1, np.concatenate([s, s1])
    for M in (1, 8):
        x = syn.activations(11 + M, M, K)
        op, _, y = run_op(b2g, K, N, 1, 3, dev(x), Wd, s, fuse=fuse, w1=w1,
                          options={b2g.OPT_PARTITION: mode, b2g.OPT_GRID: grid})
        assert op.plan(M)["partition"] == mode
        if fuse & b2g.FUSE_GATE_UP_SILU:
            want = orc.gate_up_silu(orc.rmsnorm(x), Wh, Wh1, orc.WTYPE_FP8, 3, s[:N], s[N:])
        else:
            want = orc.gemv(Wh, orc.WTYPE_FP8, x, 3, s)
        check(orc, y, np.asarray(want, np.float64), 1, (part, M))
    assert b2g.device_error() == 0


@pytest.mark.parametrize("ks,part,grid", [(2, "units", 0), (2, "tiles", 0), (4, "units", 0), (4, "tiles", 0),
                                           (8, "units", 296)])
def test_ksplit_ranges(b2g, orc, syn, cuda, ks, part, grid):
    """K cut into several ranges: every tile's ranges are summed across CTAs
    (the residual op, so the finisher also adds the residual)."""
    K, N = 8192, 3072
    mode = {"units": b2g.PARTITION_UNITS, "tiles": b2g.PARTITION_TILES}[part]
    Wd, Wh, s = make_weights(orc, syn, 37, K, N, 1, 3)
    for M in (1, 8):
        x = syn.activations(40 + M, M, K)
        r = syn.activations(50 + M, M, N)
        op = b2g.GemvOp(K, N, weight_dtype=1, scale_mode=3, max_m=8, fuse=b2g.FUSE_RESIDUAL_ADD)
        op.set_option(b2g.OPT_GRID, grid)
        op.set_option(b2g.OPT_PARTITION, mode)
        op.set_option(b2g.OPT_KSPLIT, ks)
        assert op.plan(M)["ksplit"] == ks
        packed = op.prepack(Wd)
        y = op.enqueue(dev(x), packed, dev(s), residual=dev(r))
        torch.cuda.synchronize()
        want = orc.residual_add(r, orc.to_f16(orc.gemv(Wh, orc.WTYPE_FP8, x, 3, s))).astype(np.float64)
        check(orc, y, want, 1, (ks, part, M))
    assert b2g.device_error() == 0


def test_refused_option_keeps_plan(b2g, orc, syn, cuda):
    """A grid of one CTA would hand it all 192 tiles of 8192->3072, far more
    than its 8 shared slots: no valid plan, so the option is refused and the
    op keeps its previous, working plan.  A K split that does not divide the
    256 k-blocks (3) is refused as invalid."""
    K, N = 8192, 3072
    op = b2g.GemvOp(K, N, weight_dtype=1, scale_mode=3, max_m=8)
    before = op.plan(8)
    with pytest.raises(b2g.B2GError) as e:
        op.set_option(b2g.OPT_GRID, 1)
    assert e.value.status == b2g.ERR_UNSUPPORTED
    assert op.plan(8) == before
    with pytest.raises(b2g.B2GError) as e:
        op.set_option(b2g.OPT_KSPLIT, 3)
    assert e.value.status == b2g.ERR_INVALID
    assert op.plan(8) == before
    Wd, Wh, s = make_weights(orc, syn, 38, K, N, 1, 3)
    x = syn.activations(60, 8, K)
    y = op.enqueue(dev(x), op.prepack(Wd), dev(s))
    torch.cuda.synchronize()
    check(orc, y, orc.gemv(Wh, orc.WTYPE_FP8, x, 3, s), 1)


def test_ksplit_8_plans_in_waves(b2g, orc, syn, cuda):
    """K split into 8 ranges of 8192->3072 gives 1536 virtual tiles: one CTA
    per SM would touch more than its 8 slots, so the planner grows the grid
    into waves of CTAs with at most 7 whole tiles each; the result still
    matches the oracle."""
    K, N = 8192, 3072
    op = b2g.GemvOp(K, N, weight_dtype=1, scale_mode=3, max_m=8)
    op.set_option(b2g.OPT_KSPLIT, 8)
    plan = op.plan(8)
    assert plan["ksplit"] == 8
    assert plan["grid"] > torch.cuda.get_device_properties(0).multi_processor_count
    assert plan["n_slots"] <= 8
    Wd, Wh, s = make_weights(orc, syn, 39, K, N, 1, 3)
    packed = op.prepack(Wd)
    for M in (1, 8):
        x = syn.activations(61 + M, M, K)
        y = op.enqueue(dev(x), packed, dev(s))
        torch.cuda.synchronize()
        check(orc, y, orc.gemv(Wh, orc.WTYPE_FP8, x, 3, s), 1, ("ksplit8", M))
    assert b2g.device_error() == 0


def test_deterministic_and_rows_independent(b2g, orc, syn, cuda):
    K, N = 3072, 8192
    Wd, Wh, s = make_weights(orc, syn, 35, K, N, 1, 3)
    x = dev(syn.activations(11, 8, K))
    op = b2g.GemvOp(K, N, max_m=8)
    packed = op.prepack(Wd)
    ws = op.workspace()
    sd = dev(s)
    y1 = op.enqueue(x, packed, sd, workspace=ws)
    y2 = op.enqueue(x, packed, sd, workspace=ws)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    # each token column of the tensor-core tile is independent of the others
    for m in (0, 5):
        ym = op.enqueue(x[m:m + 1].contiguous(), packed, sd, workspace=ws)
        torch.cuda.synchronize()
        assert torch.equal(ym[0], y1[m])
    # the kernels leave the tile counters at zero
    counters = ws[:op.plan(8)["n_tiles"] * 4].view(torch.int32)
    assert int(counters.abs().sum()) == 0
    assert b2g.device_error() == 0


@pytest.mark.parametrize("wd", [0, 1])
def test_cuda_core_ffma_variant(b2g, orc, syn, cuda, wd):
    for K, N in ((3072, 8192), (8192, 3072), (200, 120)):
        Wd, Wh, s = make_weights(orc, syn, 36, K, N, wd, 3 if wd else 0)
        for M in (1, 8):
            x = syn.activations(12, M, K)
            _, _, y = run_op(b2g, K, N, wd, 3 if wd else 0, dev(x), Wd, s,
                             options={b2g.OPT_MATH: b2g.MATH_FFMA})
            want = orc.gemv(Wh, orc.WTYPE_FP8 if wd else orc.WTYPE_FP16, x, 3 if wd else 0, s)
            check(orc, y, want, wd, ("ffma", K, N, M))


def test_output_guard_bands(b2g, orc, syn, cuda):
    K, N, M = 3072, 8192, 8
    Wd, Wh, s = make_weights(orc, syn, 37, K, N, 1, 3)
    buf = torch.full((M * N + 2048,), 12345.0, dtype=torch.float16, device="cuda")
    y = buf[1024:1024 + M * N].view(M, N)
    run_op(b2g, K, N, 1, 3, dev(syn.activations(13, M, K)), Wd, s, y=y)
    assert torch.all(buf[:1024] == 12345.0) and torch.all(buf[1024 + M * N:] == 12345.0)


# --------------------------------------------------------------------------
# Fused ops
# --------------------------------------------------------------------------
@pytest.mark.parametrize("wd", [0, 1])
@pytest.mark.parametrize("K,N", [(3072, 8192), (200, 120)])
def test_fused_gate_up_silu_with_rmsnorm(b2g, orc, syn, cuda, wd, K, N):
    mode = 3 if wd else 0
    Wg_d, Wg, sg = make_weights(orc, syn, 40, K, N, wd, mode)
    Wu_d, Wu, su = make_weights(orc, syn, 41, K, N, wd, mode)
    scales = None if sg is None else np.concatenate([sg, su])
    for M in (1, 3, 8):
        h = syn.activations(50 + M, M, K)
        for rms in (False, True):
            fuse = b2g.FUSE_GATE_UP_SILU | (b2g.FUSE_RMSNORM_INPUT if rms else 0)
            _, _, a = run_op(b2g, K, N, wd, mode, dev(h), Wg_d, scales, fuse=fuse, w1=Wu_d)
            xin = orc.rmsnorm(h) if rms else h
            want = orc.gate_up_silu(xin, Wg, Wu, orc.WTYPE_FP8 if wd else orc.WTYPE_FP16, mode, sg, su)
            check(orc, a, want.astype(np.float64), wd, (K, N, M, rms))


def test_down_residual_in_place(b2g, orc, syn, cuda):
    K, N, M = 8192, 3072, 8
    Wd, Wh, s = make_weights(orc, syn, 42, K, N, 1, 3)
    a = syn.activations(60, M, K)
    h = syn.activations(61, M, N)
    hd = dev(h)
    run_op(b2g, K, N, 1, 3, dev(a), Wd, s, fuse=b2g.FUSE_RESIDUAL_ADD, y=hd, residual=hd)
    y = orc.to_f16(orc.gemv(Wh, orc.WTYPE_FP8, a, 3, s))
    want = orc.residual_add(h, y).astype(np.float64)
    check(orc, hd, want, 1)


# --------------------------------------------------------------------------
# Stack
# --------------------------------------------------------------------------
def build_stack(b2g, orc, syn, hidden, inter, n_layers, wd=1, mode=3, max_m=8):
    st = b2g.Stack(hidden, inter, n_layers, weight_dtype=wd, scale_mode=mode, max_m=max_m)
    layers = []
    for l in range(n_layers):
        sg_, su_, sd_ = 1000 + 3 * l, 1001 + 3 * l, 1002 + 3 * l
        Wg, Wu, Wdn = (syn.weights(sg_, hidden, inter), syn.weights(su_, hidden, inter),
                       syn.weights(sd_, inter, hidden))
        if wd:
            qg, sg = b2g.quantize_e4m3(dev(Wg), mode)
            qu, su = b2g.quantize_e4m3(dev(Wu), mode)
            qd, sd = b2g.quantize_e4m3(dev(Wdn), mode)
        else:
            qg, qu, qd, sg, su, sd = dev(Wg), dev(Wu), dev(Wdn), None, None, None
        pgu = st.gate_up.prepack(qg, qu)
        pd = st.down.prepack(qd)
        sgu = None if sg is None else torch.cat([sg, su])
        st.set_layer(l, pgu, sgu, pd, sd)
        layers.append({"wg": host(qg), "wu": host(qu), "wd": host(qd),
                       "sg": None if sg is None else host(sg), "su": None if su is None else host(su),
                       "sd": None if sd is None else host(sd)})
    return st, layers


@pytest.mark.parametrize("wd", [0, 1])
def test_stack_small(b2g, orc, syn, cuda, wd):
    mode = 3 if wd else 0
    st, layers = build_stack(b2g, orc, syn, 256, 512, 3, wd, mode)
    for M in (1, 8):
        h0 = syn.hidden_state(M, 256)
        h = dev(h0)
        act = torch.empty((M, 512), dtype=torch.float16, device="cuda")
        st.enqueue(h, act, st.workspace())
        torch.cuda.synchronize()
        want = orc.mlp_stack(h0, layers, wtype=orc.WTYPE_FP8 if wd else orc.WTYPE_FP16,
                             scale_mode=mode)
        check(orc, h, want.astype(np.float64), wd, M)


def test_stack_full_28_layers(b2g, orc, syn, cuda):
    """The full decode stack (hidden 3072, intermediate 8192, 28 layers,
    per-channel FP32 E4M3) at M=8 against the oracle."""
    st, layers = build_stack(b2g, orc, syn, 3072, 8192, 28)
    M = 8
    h0 = syn.hidden_state(M)
    h = dev(h0)
    act = torch.empty((M, 8192), dtype=torch.float16, device="cuda")
    st.enqueue(h, act, st.workspace())
    torch.cuda.synchronize()
    want = orc.mlp_stack(h0, layers)
    r = orc.compare(host(h), want.astype(np.float64))
    assert r["rel_l2"] <= 5e-3, r
    assert b2g.device_error() == 0


@pytest.mark.parametrize("wd", [0, 1])
@pytest.mark.parametrize("hidden,inter,n_layers", [(256, 512, 3), (3072, 8192, 2), (96, 160, 33)])
def test_stack_persistent_matches_per_layer(b2g, orc, syn, cuda, wd, hidden, inter, n_layers):
    """The one-launch stack kernel and the per-layer launches compute the same
    partition in the same order: bitwise-identical hidden states.  33 layers
    exercise the host's split into launches of at most 32 layers."""
    mode = 3 if wd else 0
    st, _ = build_stack(b2g, orc, syn, hidden, inter, n_layers, wd, mode)
    ws = st.workspace()
    for M in (1, 3, 8):
        h0 = dev(syn.hidden_state(M, hidden))
        out = {}
        for m in ("per_layer", "persistent", "per_layer", "persistent"):
            st.set_mode(m)
            h = h0.clone()
            act = torch.empty((M, inter), dtype=torch.float16, device="cuda")
            st.enqueue(h, act, ws)
            torch.cuda.synchronize()
            if m in out:
                assert torch.equal(out[m], h), (m, M)
            out[m] = h
        assert torch.equal(out["per_layer"], out["persistent"]), M
    assert b2g.device_error() == 0
    # Counters and the grid-barrier word are back to zero.
    assert int(ws[:65536].count_nonzero()) == 0


def test_stack_persistent_full_vs_oracle(b2g, orc, syn, cuda):
    st, layers = build_stack(b2g, orc, syn, 3072, 8192, 4)
    st.set_mode("persistent")
    for M in (1, 8):
        h0 = syn.hidden_state(M)
        h = dev(h0)
        act = torch.empty((M, 8192), dtype=torch.float16, device="cuda")
        st.enqueue(h, act, st.workspace())
        torch.cuda.synchronize()
        want = orc.mlp_stack(h0, layers)
        check(orc, h, want.astype(np.float64), 1, M)
