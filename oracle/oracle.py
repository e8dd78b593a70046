"""CPU oracle for the decode-GEMV path.  TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module.  The product library never calls it, and there is no CPU fallback
anywhere in the product: when the CUDA library is missing, the product raises.

Two layers:

* ``liboracle.so`` (``oracle/b2g_oracle.c``): the C restatement of the
  reference's E4M3 packing, scale rules and fp64 GEMV loop, each function
  citing the reference line it follows.
* numpy fp64 composites below for the parts the reference has no code for
  (fused gate/up + SiLU*up, RMSNorm, residual, the layer stack, tensor-parallel
  sharding).  Intermediate tensors are rounded to fp16 exactly where the
  library materialises them in fp16, so both sides compute the same function.

``ref()`` returns the reference's own host functions compiled from its sources
(``oracle/_ref/libref_host.so``), or None where they were not built.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_LIB_PATH = HERE / "_ref" / "libref_host.so"
KAT_TOOL = HERE / "_ref" / "e4m3_selftest"

LAYOUT_KN, LAYOUT_NK = 0, 1
SCALE_NONE, SCALE_TENSOR_FP16, SCALE_CHANNEL_FP16, SCALE_CHANNEL_FP32 = 0, 1, 2, 3
WTYPE_FP16, WTYPE_FP8 = 0, 1

_lib = None
_ref = None

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_sz = ctypes.c_size_t


def lib():
    """Load (building with gcc if needed) the C oracle."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "oracle"], check=True)
    L = ctypes.CDLL(str(LIB_PATH))
    L.orc_f16_to_e4m3_array.argtypes = [_u16p, _sz, _u8p]
    L.orc_f32_to_e4m3_array.argtypes = [_f32p, _sz, _u8p]
    L.orc_e4m3_to_f64_array.argtypes = [_u8p, _sz, _f64p]
    L.orc_f64_to_f16_array.argtypes = [_f64p, _sz, _u16p]
    L.orc_fill_host_ref.argtypes = [_u16p, _sz, _u16p, ctypes.c_int]
    L.orc_fill_x_ref.argtypes = [_u16p, ctypes.c_int, ctypes.c_uint]
    L.orc_quantize_e4m3.argtypes = [_u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int, _u8p, ctypes.c_void_p]
    L.orc_quantize_e4m3.restype = ctypes.c_int
    L.orc_gemv_f64.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                               ctypes.c_int, _u16p, ctypes.c_int, ctypes.c_long, _f64p]
    L.orc_apply_scale.argtypes = [_f64p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    L.orc_cosine_stats.argtypes = [_u16p, _f64p, _sz, _f64p]
    L.orc_num_threads.restype = ctypes.c_int
    _lib = L
    return L


def ref():
    """The reference's own host functions (compiled from its sources), or None."""
    global _ref
    if _ref is not None:
        return _ref
    if not REF_LIB_PATH.exists():
        return None
    R = ctypes.CDLL(str(REF_LIB_PATH))
    R.ref_fill_host.argtypes = [_u16p, _sz, _u16p, ctypes.c_int, ctypes.c_int]
    R.ref_pack_e4m3.argtypes = [_u16p, _sz, _u8p]
    R.ref_fill_x.argtypes = [_u16p, ctypes.c_int, ctypes.c_uint]
    R.ref_e4m3_to_double.argtypes = [ctypes.c_uint8]
    R.ref_e4m3_to_double.restype = ctypes.c_double
    R.ref_cpu_reference_e4m3.argtypes = [_u8p, _u16p, _f64p, ctypes.c_int, ctypes.c_int]
    R.ref_cpu_reference_fp16.argtypes = [_u16p, _u16p, _f64p, ctypes.c_int, ctypes.c_int]
    R.ref16_cpu_reference.argtypes = [_u16p, _u16p, _f64p, ctypes.c_int, ctypes.c_int]
    R.ref_cpu_reference_scaled.argtypes = [_u8p, _u16p, _u16p, _f64p, ctypes.c_int, ctypes.c_int]
    R.ref_cosine_stats.argtypes = [_u16p, _f64p, ctypes.c_int, _f64p]
    R.ref_cpu_plan_create.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int]
    R.ref_cpu_plan_create.restype = ctypes.c_void_p
    R.ref_cpu_plan_run.argtypes = [ctypes.c_void_p, _u16p, ctypes.c_int, _f64p]
    R.ref_cpu_plan_destroy.argtypes = [ctypes.c_void_p]
    _ref = R
    return R


# --------------------------------------------------------------------------
# Element conversions
# --------------------------------------------------------------------------
def f16_bits(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float16)).view(np.uint16)


def f16_to_e4m3(h16: np.ndarray) -> np.ndarray:
    """E4M3 codes of fp16 values (pack_e4m3, kernels/gemv_fp8.cu:297-304)."""
    h = f16_bits(h16).ravel()
    out = np.empty(h.size, np.uint8)
    lib().orc_f16_to_e4m3_array(h, h.size, out)
    return out.reshape(np.shape(h16))


def f32_to_e4m3(f32: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(f32, dtype=np.float32).ravel()
    out = np.empty(f.size, np.uint8)
    lib().orc_f32_to_e4m3_array(f, f.size, out)
    return out.reshape(np.shape(f32))


def e4m3_to_f64(q: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(q, dtype=np.uint8).ravel()
    out = np.empty(b.size, np.float64)
    lib().orc_e4m3_to_f64_array(b, b.size, out)
    return out.reshape(np.shape(q))


def to_f16(v: np.ndarray) -> np.ndarray:
    """Round fp64 values to fp16 (RNE) with the oracle's own encoder."""
    d = np.ascontiguousarray(v, dtype=np.float64).ravel()
    out = np.empty(d.size, np.uint16)
    lib().orc_f64_to_f16_array(d, d.size, out)
    return out.view(np.float16).reshape(np.shape(v))


# --------------------------------------------------------------------------
# Reference generators and quantisers
# --------------------------------------------------------------------------
def fill_host_ref(K: int, N: int):
    """The reference's check-mode draws (kernels/gemv_fp8.cu:285-295): W [K,N], x [K] fp16."""
    W = np.empty(K * N, np.uint16)
    x = np.empty(K, np.uint16)
    lib().orc_fill_host_ref(W, W.size, x, K)
    return W.view(np.float16).reshape(K, N), x.view(np.float16)


def fill_x_ref(K: int, seed: int) -> np.ndarray:
    """checkreal's synthetic activations (kernels/gemv_fp8.cu:408-413): srand(seed),
    then x[i] = fp16(((rand() % 2001) - 1000) / 4000), i.e. Uniform[-0.25, 0.25]."""
    x = np.empty(K, np.uint16)
    lib().orc_fill_x_ref(x, K, seed)
    return x.view(np.float16)


def quantize_e4m3(w16: np.ndarray, scale_mode: int, layout: int = LAYOUT_KN):
    """Quantise fp16 W (layout KN: [K,N]; NK: [N,K]) -> (codes, scales).

    scales: None (NONE), fp16[1] (TENSOR_FP16), fp16[N] (CHANNEL_FP16),
    fp32[N] (CHANNEL_FP32).  Rules in oracle/b2g_oracle.c:orc_quantize_e4m3.
    """
    w = f16_bits(w16)
    if layout == LAYOUT_KN:
        K, N = w.shape
    else:
        N, K = w.shape
    q = np.empty(w.shape, np.uint8)
    if scale_mode == SCALE_NONE:
        s = None
        sp = None
    elif scale_mode == SCALE_CHANNEL_FP32:
        s = np.empty(N, np.float32)
        sp = s.ctypes.data
    elif scale_mode == SCALE_CHANNEL_FP16:
        s = np.empty(N, np.float16)
        sp = s.ctypes.data
    elif scale_mode == SCALE_TENSOR_FP16:
        s = np.empty(1, np.float16)
        sp = s.ctypes.data
    else:
        raise ValueError(scale_mode)
    rc = lib().orc_quantize_e4m3(np.ascontiguousarray(w), K, N, layout, scale_mode, q, sp)
    if rc != 0:
        raise ValueError("orc_quantize_e4m3 rejected its arguments")
    return q, s


def scale_vector(scale_mode: int, scales, N: int) -> np.ndarray:
    """Per-channel scale as fp64 [N] (ones for NONE)."""
    if scale_mode == SCALE_NONE:
        return np.ones(N)
    s = np.asarray(scales).astype(np.float64)
    if scale_mode == SCALE_TENSOR_FP16:
        return np.full(N, s[0])
    return s


# --------------------------------------------------------------------------
# GEMV
# --------------------------------------------------------------------------
def gemv_loop(w, wtype: int, x16: np.ndarray, layout: int = LAYOUT_KN, K=None, N=None):
    """fp64 GEMV by the reference's loop (cpu_reference_e4m3/fp16 generalised
    to M rows), C implementation.  Returns unscaled y [M, N] fp64."""
    x = f16_bits(np.atleast_2d(x16))
    M = x.shape[0]
    if K is None or N is None:
        K, N = (w.shape if layout == LAYOUT_KN else w.shape[::-1])
    wa = np.ascontiguousarray(w if wtype == WTYPE_FP8 else f16_bits(w))
    y = np.empty((M, N), np.float64)
    lib().orc_gemv_f64(wa.ctypes.data, wtype, layout, K, N, np.ascontiguousarray(x), M,
                       x.shape[1], y)
    return y


def dequant(w, wtype: int, layout: int = LAYOUT_KN) -> np.ndarray:
    """Weights as fp64 [K, N] (layout normalised)."""
    d = e4m3_to_f64(w) if wtype == WTYPE_FP8 else np.asarray(w, np.float16).astype(np.float64)
    return d if layout == LAYOUT_KN else d.T


def gemv(w, wtype: int, x16, scale_mode=SCALE_NONE, scales=None, layout=LAYOUT_KN):
    """y = s * (x @ deq(W)) in fp64 (BLAS order), shape [M, N]."""
    d = dequant(w, wtype, layout)
    x = np.atleast_2d(np.asarray(x16, np.float16)).astype(np.float64)
    y = x @ d
    return y * scale_vector(scale_mode, scales, d.shape[1])[None, :]


# --------------------------------------------------------------------------
# Fused ops and the stack (no reference code exists for these; the dataflow is
# the ONNX graph's: post_attention_layernorm -> gate/up -> SiLU(gate)*up ->
# down, kernels/opt_loop/fp8_accuracy/capture_real_activations.py:39-42)
# --------------------------------------------------------------------------
def silu_mul(g16, u16) -> np.ndarray:
    """a = fp16(SiLU(g) * u) with SiLU(g) = g / (1 + exp(-g)), fp64 math."""
    g = np.asarray(g16, np.float16).astype(np.float64)
    u = np.asarray(u16, np.float16).astype(np.float64)
    return to_f16(g / (1.0 + np.exp(-g)) * u)


def rmsnorm(h16, eps: float = 1e-5) -> np.ndarray:
    """n = fp16(h / sqrt(mean(h^2) + eps)) per row, gamma = 1."""
    h = np.atleast_2d(np.asarray(h16, np.float16)).astype(np.float64)
    r = 1.0 / np.sqrt((h * h).mean(axis=1, keepdims=True) + eps)
    return to_f16(h * r)


def residual_add(h16, y16) -> np.ndarray:
    return to_f16(np.asarray(h16, np.float16).astype(np.float64)
                  + np.asarray(y16, np.float16).astype(np.float64))


def gate_up_silu(x16, wg, wu, wtype, scale_mode=SCALE_NONE, sg=None, su=None, layout=LAYOUT_KN):
    g = to_f16(gemv(wg, wtype, x16, scale_mode, sg, layout))
    u = to_f16(gemv(wu, wtype, x16, scale_mode, su, layout))
    return silu_mul(g, u)


def mlp_layer(h16, layer: dict, wtype=WTYPE_FP8, scale_mode=SCALE_CHANNEL_FP32,
              eps: float = 1e-5, layout=LAYOUT_KN) -> np.ndarray:
    """h' = h + down(SiLU(gate(n)) * up(n)), n = RMSNorm(h); every stage fp16."""
    n = rmsnorm(h16, eps)
    a = gate_up_silu(n, layer["wg"], layer["wu"], wtype, scale_mode,
                     layer.get("sg"), layer.get("su"), layout)
    y = to_f16(gemv(layer["wd"], wtype, a, scale_mode, layer.get("sd"), layout))
    return residual_add(h16, y)


def mlp_stack(h16, layers, **kw) -> np.ndarray:
    h = np.atleast_2d(np.asarray(h16, np.float16))
    for layer in layers:
        h = mlp_layer(h, layer, **kw)
    return h


def mlp_layer_tp(h16, layer: dict, tp: int, wtype=WTYPE_FP8, scale_mode=SCALE_CHANNEL_FP32,
                 eps: float = 1e-5) -> np.ndarray:
    """Tensor-parallel restatement: gate/up column shards, down K shards, each
    rank's down partial rounded to fp16, partials summed in rank order in fp32
    then rounded once to fp16, residual added in fp16."""
    n = rmsnorm(h16, eps)
    N = layer["wg"].shape[1]
    sh = N // tp
    parts = []
    for r in range(tp):
        cs = slice(r * sh, (r + 1) * sh)

        def sl(s):
            return None if s is None else (s if np.size(s) == 1 else np.asarray(s)[cs])
        a = gate_up_silu(n, layer["wg"][:, cs], layer["wu"][:, cs], wtype, scale_mode,
                         sl(layer.get("sg")), sl(layer.get("su")))
        parts.append(to_f16(gemv(layer["wd"][cs, :], wtype, a, scale_mode, layer.get("sd"))))
    acc = np.zeros(parts[0].shape, np.float32)
    for p in parts:
        acc = acc + p.astype(np.float32)
    y = to_f16(acc.astype(np.float64))
    return residual_add(h16, y)


# --------------------------------------------------------------------------
# Metrics (kernels/gemv_fp8.cu:337-355 plus rel-L2)
# --------------------------------------------------------------------------
def compare(got16, want: np.ndarray) -> dict:
    g = np.asarray(got16, np.float16).astype(np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    err = g - w
    den = np.maximum(np.abs(w), 1e-3)
    nw = np.linalg.norm(w)
    return {
        "rel_l2": float(np.linalg.norm(err) / nw) if nw > 0 else float(np.linalg.norm(err)),
        "max_abs": float(np.abs(err).max()) if err.size else 0.0,
        "max_rel": float((np.abs(err) / den).max()) if err.size else 0.0,
        "cos": float(g @ w / (np.linalg.norm(g) * nw)) if nw > 0 and np.linalg.norm(g) > 0 else 1.0,
    }


def num_threads() -> int:
    return int(lib().orc_num_threads())


def cpu_count() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
