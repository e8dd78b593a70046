"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Run in a container that has the reference checkout, after
``make -C oracle REF=<checkout>`` has built oracle/_ref/ from the reference
sources:

    python tests/golden/make_golden.py --ref <checkout>

Fixtures written (all small, committed):

* ``e4m3_kat.npz``      -- the reference's E4M3 table: every finite fp16 bit
  pattern and the code/value that ``__nv_fp8_e4m3(__half)`` gives, printed by
  kernels/opt_loop/fp8_accuracy/e4m3_selftest.cu (built from the reference
  sources into oracle/_ref/e4m3_selftest).
* ``numpy_twin.npz``    -- inputs and outputs of the reference's numpy twin
  ``quant_e4m3`` (kernels/opt_loop/fp8_accuracy/fp8_numpy_study.py:34-36),
  imported from the reference checkout.
* ``ref_gemv_small.npz`` -- for a few small shapes: the reference's
  fill_host() draws (kernels/gemv_fp8.cu:285-295), pack_e4m3() codes
  (:297-304), cpu_reference_e4m3() / cpu_reference_fp16() outputs
  (:313-335) and cpu_reference_scaled() (:470-482) on oracle-made fp16 scales.
* ``ref_gemv_full.npz`` -- for the two MLP shapes (3072x8192, 8192x3072): the
  sha256 of the reference's fill_host() W and x, and the fp64 outputs of
  cpu_reference_e4m3() and cpu_reference_fp16() on them.
* ``cfg0_fp16.npz``     -- FP16 GEMV K=3072 N=8192 M=1 on W ~ N(0,0.02),
  x ~ N(0,1) from numpy seed 0: sha256 of W and x, and the fp64 output of the
  reference's gemv_fp16.cu cpu_reference() (kernels/gemv_fp16.cu:287-297).
* ``checkreal_x.npz``   -- checkreal's synthetic activations (fill_x,
  kernels/gemv_fp8.cu:408-413) for K = 3072 and 8192 at seeds 1234 and 7.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle as orc  # noqa: E402

OUT = Path(__file__).resolve().parent


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def kat():
    txt = subprocess.run([str(orc.KAT_TOOL)], check=True, capture_output=True, text=True).stdout
    rows = np.loadtxt(txt.splitlines()[1:], delimiter=",", dtype=np.float64)
    np.savez_compressed(OUT / "e4m3_kat.npz",
                        fp16_bits=rows[:, 0].astype(np.uint16),
                        fp8_bits=rows[:, 1].astype(np.uint8),
                        fp8_value=rows[:, 2])
    print("e4m3_kat:", rows.shape[0], "rows")


def numpy_twin(ref_root: Path):
    path = ref_root / "kernels/opt_loop/fp8_accuracy/fp8_numpy_study.py"
    spec = importlib.util.spec_from_file_location("ref_fp8_numpy_study", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = np.random.default_rng(20240611)
    parts = [
        rng.normal(0, 1, 20000).astype(np.float32),
        rng.normal(0, 100, 20000).astype(np.float32),
        rng.uniform(-600, 600, 5000).astype(np.float32),
        (rng.normal(0, 1e-2, 5000)).astype(np.float32),
    ]
    # exact E4M3 midpoints (ties) and their neighbours, both signs
    codes = np.arange(0, 0x7E, dtype=np.uint8)
    v = orc.e4m3_to_f64(codes)
    mids = ((v[:-1] + v[1:]) / 2).astype(np.float32)
    ties = np.concatenate([mids, np.nextafter(mids, 0), np.nextafter(mids, 1e9)])
    parts += [ties, -ties, np.array([0.0, -0.0, 448, 449, 464, 480, 1e6, -1e6, 2**-10, 2**-9],
                                    np.float32)]
    x = np.concatenate(parts).astype(np.float32)
    y = mod.quant_e4m3(x.astype(np.float64))
    np.savez_compressed(OUT / "numpy_twin.npz", x=x, y=y)
    print("numpy_twin:", x.size, "values")


def ref_small():
    R = orc.ref()
    shapes = [(96, 80), (64, 48), (33, 17), (256, 40)]
    out = {}
    for i, (K, N) in enumerate(shapes):
        W = np.empty(K * N, np.uint16)
        x = np.empty(K, np.uint16)
        R.ref_fill_host(W, W.size, x, K, N)
        q = np.empty(K * N, np.uint8)
        R.ref_pack_e4m3(W, W.size, q)
        y8 = np.empty(N, np.float64)
        y16 = np.empty(N, np.float64)
        R.ref_cpu_reference_e4m3(q, x, y8, K, N)
        R.ref_cpu_reference_fp16(W, x, y16, K, N)
        wq, s = orc.quantize_e4m3(W.view(np.float16).reshape(K, N), orc.SCALE_CHANNEL_FP16)
        ys = np.empty(N, np.float64)
        R.ref_cpu_reference_scaled(np.ascontiguousarray(wq.ravel()), x,
                                   np.ascontiguousarray(s).view(np.uint16), ys, K, N)
        out.update({f"s{i}_K": K, f"s{i}_N": N, f"s{i}_W": W, f"s{i}_x": x, f"s{i}_q": q,
                    f"s{i}_y_e4m3": y8, f"s{i}_y_fp16": y16, f"s{i}_qc": wq.ravel(),
                    f"s{i}_sc": np.asarray(s).view(np.uint16), f"s{i}_y_scaled": ys})
    out["n"] = len(shapes)
    np.savez_compressed(OUT / "ref_gemv_small.npz", **out)
    print("ref_gemv_small:", shapes)


def ref_full():
    R = orc.ref()
    out = {}
    for name, K, N in (("up", 3072, 8192), ("down", 8192, 3072)):
        W = np.empty(K * N, np.uint16)
        x = np.empty(K, np.uint16)
        R.ref_fill_host(W, W.size, x, K, N)
        q = np.empty(K * N, np.uint8)
        R.ref_pack_e4m3(W, W.size, q)
        y8 = np.empty(N, np.float64)
        y16 = np.empty(N, np.float64)
        R.ref_cpu_reference_e4m3(q, x, y8, K, N)
        R.ref_cpu_reference_fp16(W, x, y16, K, N)
        out.update({f"{name}_W_sha": sha(W), f"{name}_x_sha": sha(x), f"{name}_q_sha": sha(q),
                    f"{name}_y_e4m3": y8, f"{name}_y_fp16": y16})
    np.savez_compressed(OUT / "ref_gemv_full.npz", **out)
    print("ref_gemv_full: up, down")


def cfg0():
    sys.path.insert(0, str(ROOT))
    from importlib import util
    pkg = ROOT / "llama-3.2-3b-instruct-gemm-optimization_b200" / "synthetic.py"
    spec = util.spec_from_file_location("b2g_synthetic", pkg)
    syn = util.module_from_spec(spec)
    spec.loader.exec_module(syn)
    W, x = syn.cfg0_fp16_gemv()
    R = orc.ref()
    y = np.empty(W.shape[1], np.float64)
    R.ref16_cpu_reference(np.ascontiguousarray(W).view(np.uint16).ravel(),
                          np.ascontiguousarray(x.ravel()).view(np.uint16), y, *W.shape)
    np.savez_compressed(OUT / "cfg0_fp16.npz", W_sha=sha(W), x_sha=sha(x), y=y)
    print("cfg0_fp16: y", y.shape)


def checkreal_x():
    R = orc.ref()
    out = {}
    for K in (3072, 8192):
        for seed in (1234, 7):
            x = np.empty(K, np.uint16)
            R.ref_fill_x(x, K, seed)
            out[f"K{K}_s{seed}"] = x
    np.savez_compressed(OUT / "checkreal_x.npz", **out)
    print("checkreal_x:", sorted(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the reference checkout")
    a = ap.parse_args()
    if orc.ref() is None or not orc.KAT_TOOL.exists():
        sys.exit("oracle/_ref is not built: run `make -C oracle` with the reference present")
    kat()
    numpy_twin(Path(a.ref))
    ref_small()
    ref_full()
    cfg0()
    checkreal_x()


if __name__ == "__main__":
    main()
