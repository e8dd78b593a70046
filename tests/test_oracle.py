"""The oracle, pinned against the reference's own code and golden vectors (CPU).

Fixtures in tests/golden/ were produced by tests/golden/make_golden.py from
the reference's sources: its E4M3 table tool, its numpy twin and its host
fill/pack/fp64-GEMV functions.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import GOLDEN


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# --------------------------------------------------------------------------
# E4M3 / fp16 element rules
# --------------------------------------------------------------------------
def test_e4m3_table_matches_reference_tool(orc):
    """Every finite fp16 -> E4M3 code equals the reference's __nv_fp8_e4m3(half)
    table (kernels/opt_loop/fp8_accuracy/e4m3_selftest.cu)."""
    z = np.load(GOLDEN / "e4m3_kat.npz")
    h = z["fp16_bits"]
    assert h.size == 63488
    got = orc.f16_to_e4m3(h.view(np.float16))
    assert np.array_equal(got, z["fp8_bits"])
    assert np.array_equal(orc.e4m3_to_f64(z["fp8_bits"]), z["fp8_value"])


def test_e4m3_matches_reference_numpy_twin(orc):
    """float32 -> E4M3 equals fp8_numpy_study.py:34-36 (clip, f32, e4m3fn)."""
    z = np.load(GOLDEN / "numpy_twin.npz")
    got = orc.e4m3_to_f64(orc.f32_to_e4m3(z["x"]))
    assert np.array_equal(got, z["y"])


def test_e4m3_decode_all_codes(orc):
    codes = np.arange(256, dtype=np.uint8)
    v = orc.e4m3_to_f64(codes)
    ref = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).to(torch.float64).numpy()
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(v), nan)
    assert np.array_equal(v[~nan], ref[~nan])
    assert v[0x7E] == 448.0 and v[0x01] == 2.0 ** -9


def test_f16_encoder_matches_numpy(orc):
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.normal(0, 1, 20000), rng.normal(0, 3e4, 2000),
                        rng.normal(0, 1e-6, 2000), [65504, 65519.99, 65520, 1e9, -0.0, 2 ** -25,
                                                    3 * 2 ** -26]])
    got = orc.to_f16(x)
    want = x.astype(np.float16)  # numpy: IEEE RNE, overflow -> inf
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


def test_e4m3_encoder_ties_and_saturation(orc):
    # exact midpoints round to the even code; >= 448 saturates
    assert orc.f32_to_e4m3(np.float32([1.0625]))[0] == 0x38  # 1.0 (even) vs 1.125
    assert orc.f32_to_e4m3(np.float32([1.1875]))[0] == 0x3A  # 1.25 (even) vs 1.125
    assert orc.f32_to_e4m3(np.float32([464.0, 1e30, -1e30]))[0] == 0x7E
    assert orc.f32_to_e4m3(np.float32([-1e30]))[0] == 0xFE
    assert orc.f32_to_e4m3(np.float32([2.0 ** -10]))[0] == 0x00  # tie to even (0)
    assert orc.f32_to_e4m3(np.float32([3 * 2.0 ** -10]))[0] == 0x02


# --------------------------------------------------------------------------
# Reference host functions
# --------------------------------------------------------------------------
def test_fill_pack_and_fp64_gemv_match_reference_small(orc):
    z = np.load(GOLDEN / "ref_gemv_small.npz")
    for i in range(int(z["n"])):
        K, N = int(z[f"s{i}_K"]), int(z[f"s{i}_N"])
        W, x = orc.fill_host_ref(K, N)
        assert np.array_equal(W.view(np.uint16).ravel(), z[f"s{i}_W"])
        assert np.array_equal(x.view(np.uint16), z[f"s{i}_x"])
        q = orc.f16_to_e4m3(W)
        assert np.array_equal(q.ravel(), z[f"s{i}_q"])
        # the oracle's loop is the reference's loop: bit-identical doubles
        y8 = orc.gemv_loop(q, orc.WTYPE_FP8, x[None])[0]
        assert np.array_equal(y8, z[f"s{i}_y_e4m3"])
        y16 = orc.gemv_loop(W, orc.WTYPE_FP16, x[None])[0]
        assert np.array_equal(y16, z[f"s{i}_y_fp16"])
        ys = orc.gemv_loop(z[f"s{i}_qc"].reshape(K, N), orc.WTYPE_FP8, x[None])
        s = z[f"s{i}_sc"].view(np.float16)
        ys = ys * s.astype(np.float64)[None, :]
        assert np.array_equal(ys[0], z[f"s{i}_y_scaled"])


@pytest.mark.parametrize("name,K,N", [("up", 3072, 8192), ("down", 8192, 3072)])
def test_full_shape_reference_check_case(orc, name, K, N):
    """The reference's own `check` inputs at both MLP shapes: identical draws,
    identical E4M3 bytes, and the oracle's fp64 GEMV equals the reference's."""
    z = np.load(GOLDEN / "ref_gemv_full.npz")
    W, x = orc.fill_host_ref(K, N)
    assert sha(W.view(np.uint16).ravel()) == str(z[f"{name}_W_sha"])
    assert sha(x.view(np.uint16)) == str(z[f"{name}_x_sha"])
    q = orc.f16_to_e4m3(W)
    assert sha(q.ravel()) == str(z[f"{name}_q_sha"])
    y8 = orc.gemv_loop(q, orc.WTYPE_FP8, x[None])[0]
    assert np.array_equal(y8, z[f"{name}_y_e4m3"])
    y16 = orc.gemv_loop(W, orc.WTYPE_FP16, x[None])[0]
    assert np.array_equal(y16, z[f"{name}_y_fp16"])


def test_cfg0_fp16_gemv_seed0(orc, syn):
    """FP16 GEMV K=3072 N=8192 M=1 seed 0: the synthetic draws are the ones the
    golden was made from, and the oracle equals the reference's fp64 loop."""
    z = np.load(GOLDEN / "cfg0_fp16.npz")
    W, x = syn.cfg0_fp16_gemv()
    assert sha(W) == str(z["W_sha"]) and sha(x) == str(z["x_sha"])
    y = orc.gemv_loop(W, orc.WTYPE_FP16, x)[0]
    assert np.array_equal(y, z["y"])
    # and the BLAS-order fp64 path agrees to rounding
    y2 = orc.gemv(W, orc.WTYPE_FP16, x)[0]
    assert np.max(np.abs(y2 - y)) < 1e-12


# --------------------------------------------------------------------------
# Scale rules (independent implementations through torch's float8 dtype)
# --------------------------------------------------------------------------
def _torch_e4m3(v32: np.ndarray) -> np.ndarray:
    t = torch.from_numpy(np.clip(v32, -448, 448).astype(np.float32))
    return t.to(torch.float8_e4m3fn).view(torch.uint8).numpy()


@pytest.mark.parametrize("layout", [0, 1])
def test_quantize_channel_fp32_rule(orc, syn, layout):
    W = syn.weights(11, 96, 80)
    Wl = W if layout == 0 else np.ascontiguousarray(W.T)
    q, s = orc.quantize_e4m3(Wl, orc.SCALE_CHANNEL_FP32, layout)
    amax = np.abs(W.astype(np.float32)).max(axis=0)
    s_ref = (np.maximum(amax, np.float32(1e-12)) / np.float32(448)).astype(np.float32)
    assert np.array_equal(s, s_ref)
    q_ref = _torch_e4m3(W.astype(np.float32) / s_ref[None, :])
    assert np.array_equal(q if layout == 0 else q.T, q_ref)


@pytest.mark.parametrize("mode", [1, 2])
def test_quantize_fp16_scale_rules(orc, syn, mode):
    """check_real's rule (kernels/gemv_fp8.cu:517-543): fp16 scale, fp16
    pre-divided weight, then E4M3."""
    W = syn.weights(12, 64, 48)
    q, s = orc.quantize_e4m3(W, mode)
    a = np.abs(W.astype(np.float32))
    amax = a.max() if mode == 1 else a.max(axis=0)
    s16 = (np.maximum(amax, np.float32(1e-12)) / np.float32(448)).astype(np.float16)
    assert np.array_equal(np.atleast_1d(s16)[:s.size], s)
    wdiv = (W.astype(np.float32) / s16.astype(np.float32)).astype(np.float16)
    assert np.array_equal(q, _torch_e4m3(wdiv.astype(np.float32)))


def test_quantize_zero_column(orc):
    W = np.zeros((8, 4), np.float16)
    W[:, 1] = 0.5
    q, s = orc.quantize_e4m3(W, orc.SCALE_CHANNEL_FP32)
    assert np.all(q[:, 0] == 0) and s[0] > 0
    # fp16 scale of an all-zero column underflows to 0 -> 0/0 -> NaN code,
    # exactly as check_real would produce
    q2, s2 = orc.quantize_e4m3(W, orc.SCALE_CHANNEL_FP16)
    assert s2[0] == 0 and np.all((q2[:, 0] & 0x7F) == 0x7F)


# --------------------------------------------------------------------------
# Composite oracle pieces
# --------------------------------------------------------------------------
def test_gemv_loop_vs_blas(orc, syn):
    W = syn.weights(3, 200, 120)
    x = syn.activations(4, 5, 200)
    q, s = orc.quantize_e4m3(W, orc.SCALE_CHANNEL_FP32)
    y1 = orc.gemv_loop(q, orc.WTYPE_FP8, x) * s.astype(np.float64)[None]
    y2 = orc.gemv(q, orc.WTYPE_FP8, x, orc.SCALE_CHANNEL_FP32, s)
    assert np.allclose(y1, y2, rtol=1e-12, atol=1e-12)
    # NK layout gives the same result
    qn, sn = orc.quantize_e4m3(np.ascontiguousarray(W.T), orc.SCALE_CHANNEL_FP32, orc.LAYOUT_NK)
    y3 = orc.gemv(qn, orc.WTYPE_FP8, x, orc.SCALE_CHANNEL_FP32, sn, orc.LAYOUT_NK)
    assert np.array_equal(y2, y3)


def test_rmsnorm_silu_and_tp_restatement(orc, syn):
    h = syn.activations(5, 3, 64)
    n = orc.rmsnorm(h).astype(np.float64)
    assert np.allclose((n ** 2).mean(axis=1), 1.0, atol=2e-3)
    g = np.array([[-20.0, -1.0, 0.0, 1.0, 20.0]], np.float16)
    a = orc.silu_mul(g, np.ones_like(g)).astype(np.float64)
    assert a[0, 2] == 0 and abs(a[0, 4] - 20.0) < 1e-2 and abs(a[0, 0]) < 1e-6
    # tensor-parallel restatement == unsharded layer within fp16 rounding
    layer = {}
    for key, (K, N, sd) in {"wg": (64, 96, 1), "wu": (64, 96, 2), "wd": (96, 64, 3)}.items():
        q, s = orc.quantize_e4m3(syn.weights(sd, K, N), orc.SCALE_CHANNEL_FP32)
        layer[key], layer["s" + key[1]] = q, s
    h1 = orc.mlp_layer(h, layer)
    h2 = orc.mlp_layer_tp(h, layer, tp=4)
    assert orc.compare(h2, h1.astype(np.float64))["rel_l2"] < 2e-3


def test_checkreal_x_matches_reference(orc):
    """checkreal's synthetic activations (kernels/gemv_fp8.cu:408-413) as the
    reference's own fill_x draws them."""
    z = np.load(GOLDEN / "checkreal_x.npz")
    for K in (3072, 8192):
        for seed in (1234, 7):
            assert np.array_equal(orc.fill_x_ref(K, seed).view(np.uint16), z[f"K{K}_s{seed}"]), (K, seed)
