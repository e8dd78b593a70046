"""The reference's `checkreal` replayed through this library's kernel.

kernels/gemv_fp8.cu:484-685 (`check_real`) reads a raw fp16 [K, N] weight
blob named L{ll}.{proj}.K{K}.N{N}.fp16.bin, draws x with fill_x (:408-413),
derives fp16 scales from the column (or tensor) absmax / 448, pre-divides and
packs to E4M3 (:515-543), runs the GPU GEMV with the scale folded into the
epilogue (:650-655) and gates on cos >= 0.999 against both fp64 references:
cpu_reference_scaled over the dequantised codes (:470-482) and
cpu_reference_fp16 over the original weights (:325-335), gate at :681-683.

Here the same chain runs through the library: blobs in the reference's file
format (synthetic N(0, 0.02) weights; the model's real weights are not
available) -> weight_file.import_reference_blobs -> the device quantiser with
the reference's fp16 scale rules -> b2g_enqueue.  The references are the
reference's own host functions (oracle/_ref, compiled from its sources) when
present, else the oracle's restatement of them.
"""
from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [("up_proj", 3072, 8192), ("down_proj", 8192, 3072)]
MODES = {"tensor_fp16": 1, "channel_fp16": 2}
FP8_TOL = 5e-3  # rel-L2 against the dequantised-weight reference (fp32 accumulation vs fp64)


def _references(orc, q, W16, x, s_full):
    """(y_e4m3_scaled, y_fp16) in fp64 for one activation row."""
    K, N = W16.shape
    R = orc.ref()
    if R is not None:
        ye, yf = np.empty(N), np.empty(N)
        R.ref_cpu_reference_scaled(np.ascontiguousarray(q).ravel(), x.view(np.uint16), s_full.view(np.uint16),
                                   ye, K, N)
        R.ref_cpu_reference_fp16(np.ascontiguousarray(W16).view(np.uint16).ravel(), x.view(np.uint16), yf, K, N)
        return ye, yf
    ye = orc.gemv_loop(q, orc.WTYPE_FP8, x[None])[0] * s_full.astype(np.float64)
    yf = orc.gemv_loop(W16, orc.WTYPE_FP16, x[None])[0]
    return ye, yf


def _cosine(orc, y16, want):
    R = orc.ref()
    if R is not None:
        out = np.empty(3)
        R.ref_cosine_stats(np.ascontiguousarray(y16).view(np.uint16), np.ascontiguousarray(want), want.size, out)
        return out[0]
    return orc.compare(y16[None], want[None])["cos"]


@pytest.mark.parametrize("proj,K,N", SHAPES)
def test_checkreal_replay(b2g, orc, syn, cuda, tmp_path, proj, K, N):
    wfm = importlib.import_module("b2g.weights_file")
    W16 = syn.weights(900 + K, K, N)
    (tmp_path / f"L00.{proj}.K{K}.N{N}.fp16.bin").write_bytes(W16.tobytes())
    wfm.import_reference_blobs(tmp_path, tmp_path / "real.b2gw")
    wf = wfm.WeightFile(tmp_path / "real.b2gw")
    rec = wf.find(0, proj)
    assert (rec.kind, rec.K, rec.N) == (wfm.KIND_FP16_KN, K, N)
    blob, _ = wf.read(rec)
    assert np.array_equal(blob.view(np.uint16), W16.view(np.uint16))  # the blob's bytes unchanged
    W_dev = torch.from_numpy(blob).to(cuda)

    # checkreal's x for M = 1 (its seed 1234), plus three more rows (seeds
    # 1235..1237) through the same launch: each row must pass on its own.
    rows = np.stack([orc.fill_x_ref(K, 1234 + m) for m in range(4)])
    for mode_name, mode in MODES.items():
        q, s = b2g.quantize_e4m3(W_dev, mode_name)
        q_h, s_h = q.cpu().numpy(), s.cpu().numpy()
        # the device quantiser is the reference's rule, bit for bit
        q_o, s_o = orc.quantize_e4m3(W16, mode)
        assert np.array_equal(q_h, q_o) and np.array_equal(s_h.view(np.uint16), s_o.view(np.uint16)), mode_name
        s_full = np.full(N, s_h[0], np.float16) if mode == 1 else s_h  # checkreal keeps N copies of the tensor scale
        op = b2g.GemvOp(K, N, weight_dtype="fp8_e4m3", scale_mode=mode_name, max_m=8)
        packed = op.prepack(q)
        for M in (1, 4):
            y = op.enqueue(torch.from_numpy(rows[:M]).to(cuda), packed, s)
            torch.cuda.synchronize()
            y_h = y.cpu().numpy()
            for m in range(M):
                ye, yf = _references(orc, q_h, W16, rows[m], s_full)
                cos_e4, cos_f16 = _cosine(orc, y_h[m], ye), _cosine(orc, y_h[m], yf)
                # the reference's gate (kernels/gemv_fp8.cu:681-683)
                assert cos_e4 >= 0.999 and cos_f16 >= 0.999, (mode_name, M, m, cos_e4, cos_f16)
                r = orc.compare(y_h[m:m + 1], ye[None])
                assert r["rel_l2"] <= FP8_TOL, (mode_name, M, m, r)
    assert b2g.device_error() == 0
