"""The TMA pipeline (B2G_OPT_PIPE = TMA: one warp streams each CTA's weight
range into a shared-memory ring with 1-D bulk copies, 16 warps compute from
it) against the register pipeline and the oracle.

Both pipelines give each warp the same units in the same order and combine
the warps' partials in the same order, so their outputs must be bitwise
equal; the oracle check applies the same tolerances as the other parity
tests (rel-L2 <= 1e-3 FP16, <= 5e-3 E4M3 against the fp64 restatement of the
reference's host loop, kernels/gemv_fp8.cu:313-335)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {0: 1e-3, 1: 5e-3}


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _weights(orc, syn, seed, K, N, wd, mode):
    W16 = syn.weights(seed, K, N)
    if wd == 0:
        return dev(W16), W16, None
    q, s = orc.quantize_e4m3(W16, mode)
    return dev(q), q, s


def _pair(b2g, K, N, wd, mode, fuse=0, options=()):
    """(register-pipeline op, TMA-pipeline op) with the same fields and options."""
    ops = []
    for pipe in (b2g.PIPE_REGISTERS, b2g.PIPE_TMA):
        op = b2g.GemvOp(K, N, weight_dtype=wd, scale_mode=mode, max_m=8, fuse=fuse)
        for k, v in options:
            op.set_option(k, v)
        op.set_option(b2g.OPT_PIPE, pipe)
        ops.append(op)
    return ops


SHAPES = [(3072, 8192, 1, 3), (8192, 3072, 1, 3), (3072, 8192, 0, 0), (8192, 3072, 0, 0),
          (200, 120, 1, 2), (33, 17, 1, 1), (3072, 5120, 1, 3)]


@pytest.mark.parametrize("K,N,wd,mode", SHAPES)
def test_tma_matches_register_pipeline(b2g, orc, syn, cuda, K, N, wd, mode):
    reg, tma = _pair(b2g, K, N, wd, mode)
    for M in (1, 8):
        assert tma.plan(M)["pipe"] == b2g.PIPE_TMA and tma.plan(M)["n_stages"] >= 2, tma.plan(M)
        assert reg.plan(M)["pipe"] == b2g.PIPE_REGISTERS
    Wd, Wh, s = _weights(orc, syn, 700 + K % 97, K, N, wd, mode)
    packed = reg.prepack(Wd)
    assert torch.equal(packed, tma.prepack(Wd))  # one packed layout for both pipelines
    sd = None if s is None else dev(s)
    for M in (1, 2, 4, 8):
        x = dev(syn.activations(710 + M, M, K))
        y_reg = reg.enqueue(x, packed, sd)
        y_tma = tma.enqueue(x, packed, sd)
        torch.cuda.synchronize()
        assert torch.equal(y_reg, y_tma), (K, N, wd, M)
        want = orc.gemv(Wh, orc.WTYPE_FP8 if wd else orc.WTYPE_FP16, syn.activations(710 + M, M, K), mode, s)
        r = orc.compare(y_tma.cpu().numpy(), want)
        assert r["rel_l2"] <= TOL[wd], (K, N, wd, M, r)
    assert b2g.device_error() == 0


@pytest.mark.parametrize("part", ["units", "tiles"])
@pytest.mark.parametrize("grid", [0, 37, 148, 300])
def test_tma_partitions_and_split_tiles(b2g, orc, syn, cuda, part, grid):
    """Equal byte ranges split tiles between CTAs (cross-CTA combine of the
    partials); a grid above one CTA per SM runs as waves."""
    K, N = 8192, 3072
    mode_v = {"units": b2g.PARTITION_UNITS, "tiles": b2g.PARTITION_TILES}[part]
    opts = [(b2g.OPT_PARTITION, mode_v)] + ([(b2g.OPT_GRID, grid)] if grid else [])
    reg, tma = _pair(b2g, K, N, 1, 3, options=opts)
    Wd, Wh, s = _weights(orc, syn, 720, K, N, 1, 3)
    packed = reg.prepack(Wd)
    sd = dev(s)
    for M in (1, 8):
        x = dev(syn.activations(721 + M, M, K))
        y_reg = reg.enqueue(x, packed, sd)
        y_tma = tma.enqueue(x, packed, sd)
        torch.cuda.synchronize()
        assert torch.equal(y_reg, y_tma), (part, grid, M)
    assert b2g.device_error() == 0


def test_tma_fused_gate_up_rmsnorm_and_residual(b2g, orc, syn, cuda):
    """The decode layer's two ops on the TMA pipeline: RMSNorm + gate||up +
    SiLU*up, then down + residual, against the oracle's layer."""
    H, I = 3072, 8192
    gu = b2g.GemvOp(H, I, weight_dtype=1, scale_mode=3, max_m=8,
                    fuse=b2g.FUSE_GATE_UP_SILU | b2g.FUSE_RMSNORM_INPUT)
    dn = b2g.GemvOp(I, H, weight_dtype=1, scale_mode=3, max_m=8, fuse=b2g.FUSE_RESIDUAL_ADD)
    for op in (gu, dn):
        op.set_option(b2g.OPT_PIPE, b2g.PIPE_TMA)
    wg, wgh, sg = _weights(orc, syn, 730, H, I, 1, 3)
    wu, wuh, su = _weights(orc, syn, 731, H, I, 1, 3)
    wd_, wdh, sd = _weights(orc, syn, 732, I, H, 1, 3)
    pgu, pd = gu.prepack(wg, wu), dn.prepack(wd_)
    sgu = dev(np.concatenate([sg, su]))
    layer = {"wg": wgh, "wu": wuh, "wd": wdh, "sg": sg, "su": su, "sd": sd}
    for M in (1, 8):
        h0 = syn.hidden_state(M, H, seed=733)
        h = dev(h0)
        act = gu.enqueue(h, pgu, sgu)
        dn.enqueue(act, pd, dev(sd), y=h, residual=h)
        torch.cuda.synchronize()
        want = orc.mlp_layer(h0, layer)
        r = orc.compare(h.cpu().numpy(), want.astype(np.float64))
        assert r["rel_l2"] <= 5e-3, (M, r)
    assert b2g.device_error() == 0


def test_tma_stack_bitwise_equal(b2g, orc, syn, cuda):
    """A 4-layer decode stack chained with programmatic dependent launch and
    the L2 prefetch: both pipelines give bitwise the same hidden state."""
    H, I, NL, M = 3072, 8192, 4, 8
    outs = []
    for pipe in (b2g.PIPE_REGISTERS, b2g.PIPE_TMA):
        st = b2g.Stack(H, I, NL, max_m=8)
        st.gate_up.set_option(b2g.OPT_PIPE, pipe)
        st.down.set_option(b2g.OPT_PIPE, pipe)
        for l in range(NL):
            seeds = syn.layer_seeds(l)
            qs = [b2g.quantize_e4m3(torch.from_numpy(syn.weights(sd, K, N)).cuda(), "channel_fp32")
                  for sd, (K, N) in zip(seeds, ((H, I), (H, I), (I, H)))]
            (qg, sg), (qu, su), (qd, sdd) = qs
            st.set_layer(l, st.gate_up.prepack(qg, qu), torch.cat([sg, su]), st.down.prepack(qd), sdd)
        h = dev(syn.hidden_state(M, H))
        act = torch.empty((M, I), dtype=torch.float16, device="cuda")
        st.enqueue(h, act, st.workspace("cuda"))
        torch.cuda.synchronize()
        outs.append(h)
    assert torch.equal(outs[0], outs[1])
    assert b2g.device_error() == 0


@pytest.mark.parametrize("wd,M,NL", [(1, 8, 4), (1, 1, 3), (0, 4, 2)])
def test_persistent_tma_stack_bitwise_equal(b2g, orc, syn, cuda, wd, M, NL):
    """The stack in one cooperative launch on the TMA pipeline (one ring
    through every phase of every layer, grid barriers among the computing
    warps only) gives bitwise the hidden state of the per-layer launches, and
    matches the oracle's stack."""
    H, I = 3072, 8192
    mode_name = "channel_fp32" if wd else "none"
    dtype = "fp8_e4m3" if wd else "fp16"
    st = b2g.Stack(H, I, NL, weight_dtype=dtype, scale_mode=mode_name, max_m=8)
    host_layers = []
    for l in range(NL):
        seeds = syn.layer_seeds(l)
        ws16 = [syn.weights(sd, K, N) for sd, (K, N) in zip(seeds, ((H, I), (H, I), (I, H)))]
        if wd:
            qs = [b2g.quantize_e4m3(torch.from_numpy(w).cuda(), "channel_fp32") for w in ws16]
        else:
            qs = [(torch.from_numpy(w).cuda(), None) for w in ws16]
        (qg, sg), (qu, su), (qd, sdd) = qs
        st.set_layer(l, st.gate_up.prepack(qg, qu), None if sg is None else torch.cat([sg, su]),
                     st.down.prepack(qd), sdd)
        host_layers.append({"wg": qg.cpu().numpy(), "wu": qu.cpu().numpy(), "wd": qd.cpu().numpy(),
                            "sg": None if sg is None else sg.cpu().numpy(),
                            "su": None if su is None else su.cpu().numpy(),
                            "sd": None if sdd is None else sdd.cpu().numpy()})
    h0 = syn.hidden_state(M, H)
    ws = st.workspace("cuda")
    outs = []
    for mode in ("per_layer", "persistent_tma", "persistent_tma"):
        st.set_mode(mode)
        h = dev(h0)
        act = torch.empty((M, I), dtype=torch.float16, device="cuda")
        st.enqueue(h, act, ws)
        torch.cuda.synchronize()
        outs.append(h)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    kw = {} if wd else {"wtype": orc.WTYPE_FP16, "scale_mode": orc.SCALE_NONE}
    want = orc.mlp_stack(h0, host_layers, **kw)
    r = orc.compare(outs[1].cpu().numpy(), want.astype(np.float64))
    assert r["rel_l2"] <= (5e-3 if wd else 1e-3), r
    # the grid-barrier counter is back at zero for the next launch
    assert b2g.device_error() == 0
