"""E4M3 accuracy of the MLP projections under each scale rule.  TEST INFRASTRUCTURE.

Restates the reference's two accuracy studies on this build's oracle (the
scale rules and E4M3 codes are the oracle's, which the device quantiser
matches bit for bit):

* kernels/opt_loop/fp8_accuracy/fp8_real_activation_study.py:80-118: per
  projection, cosine / relative L2 / SNR of y = x . deq(Q(W)) against
  y = x . W, both in fp64; weight statistics (absmax, std, fraction below
  E4M3's smallest normal 2^-6, count above 448) and activation statistics
  (rms, kurtosis); a summary per scale rule (min / median / max cosine and
  whether all reach 0.999);
* kernels/gemv_fp8.cu:484-685 (checkreal): the same for one blob, with the
  reference's gate cos >= 0.999 (gemv_fp8.cu:681-683).

Scale rules: none, tensor_fp16, channel_fp16 (checkreal's rule,
gemv_fp8.cu:515-540) and channel_fp32 (this build's default).

Inputs are the reference's files: weight blobs ``L{ll}.{proj}.K{K}.N{N}.fp16.bin``
(extract_real_weights.py:65) and captured activations
``L{ll}.{proj}.K{K}.x.fp16.bin`` (fp8_real_activation_study.py:82).  Real
weights and captures are not in this container; without captures, x is
synthetic -- ``uniform``: Uniform(-0.25, 0.25), the reference's synthetic
draw (gemv_fp8.cu:285-295; seeded numpy here, not C rand); ``dataflow``: the
layer's own dataflow from a seeded N(0, 1) hidden state: gate/up take
RMSNorm(h), down takes SiLU(x.Wg) * (x.Wu) over the fp16 weights.

    python oracle/accuracy_study.py --weights DIR [--acts DIR | --x uniform|dataflow] [--out rows.json]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_spec = importlib.util.spec_from_file_location("oracle_for_study", HERE / "oracle.py")
orc = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(orc)

MODES = {"none": orc.SCALE_NONE, "tensor_fp16": orc.SCALE_TENSOR_FP16,
         "channel_fp16": orc.SCALE_CHANNEL_FP16, "channel_fp32": orc.SCALE_CHANNEL_FP32}
GATE = 0.999
E4M3_MIN_NORMAL, E4M3_MAX = 2.0 ** -6, 448.0
BLOB = re.compile(r"^L(\d+)\.(gate_proj|up_proj|down_proj)\.K(\d+)\.N(\d+)\.fp16\.bin$")


def weight_stats(w16) -> dict:
    a = np.abs(np.asarray(w16, np.float16).astype(np.float64))
    return {"w_absmax": float(a.max()), "w_std": float(np.asarray(w16, np.float64).std()),
            "w_frac_below_min_normal": float((a < E4M3_MIN_NORMAL).mean()),
            "w_n_saturating": int((a > E4M3_MAX).sum())}


def x_stats(x16) -> dict:
    x = np.asarray(x16, np.float16).astype(np.float64).ravel()
    v = x.var()
    return {"x_rms": float(np.sqrt((x * x).mean())),
            "x_kurtosis": float(((x - x.mean()) ** 4).mean() / (v * v)) if v > 0 else 0.0}


def score(y, ref) -> dict:
    y, ref = np.ravel(y), np.ravel(ref)
    err = y - ref
    return {"cos": float(y @ ref / (np.linalg.norm(y) * np.linalg.norm(ref))),
            "rel_l2": float(np.linalg.norm(err) / np.linalg.norm(ref)),
            "snr_db": float(10.0 * np.log10((ref @ ref) / (err @ err))) if err.any() else float("inf")}


def study_tensor(w16, x16, modes=tuple(MODES)) -> dict:
    """Scores of each scale rule for one projection: y = x . W (x [K] or [M, K])."""
    ref = np.atleast_2d(np.asarray(x16, np.float16)).astype(np.float64) @ np.asarray(w16, np.float64)
    out = {"K": int(w16.shape[0]), "N": int(w16.shape[1]), **weight_stats(w16), **x_stats(x16)}
    for name in modes:
        q, s = orc.quantize_e4m3(w16, MODES[name])
        y = orc.gemv(q, orc.WTYPE_FP8, x16, MODES[name], s)
        for k, v in score(y, ref).items():
            out[f"{k}_{name}"] = v
    return out


def find_blobs(src: Path) -> dict:
    """(layer, proj) -> (K, N, path) from a reference weight directory."""
    out = {}
    man = src / "manifest.json"
    entries = ([Path(r["path"]).name for r in json.loads(man.read_text())] if man.exists()
               else [p.name for p in src.iterdir()])
    for name in entries:
        m = BLOB.match(name)
        if m:
            out[(int(m.group(1)), m.group(2))] = (int(m.group(3)), int(m.group(4)), src / name)
    return out


def load_blob(K: int, N: int, path: Path) -> np.ndarray:
    w = np.fromfile(path, dtype=np.float16)
    if w.size != K * N:
        raise ValueError(f"{path}: {w.size * 2} B, expected K*N*2 = {K * N * 2}")
    return w.reshape(K, N)


def synthetic_x(kind: str, layer: int, proj: str, K: int, blobs: dict, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed + 101 * layer)
    if kind == "uniform":
        return rng.uniform(-0.25, 0.25, K).astype(np.float16)
    if kind != "dataflow":
        raise ValueError(f"unknown synthetic x {kind!r}")
    (Kg, Ng, pg), (Ku, Nu, pu) = blobs[(layer, "gate_proj")], blobs[(layer, "up_proj")]
    h = rng.standard_normal(Kg).astype(np.float16)
    xn = orc.rmsnorm(h)[0]
    if proj in ("gate_proj", "up_proj"):
        return xn
    g = orc.to_f16(xn.astype(np.float64) @ load_blob(Kg, Ng, pg).astype(np.float64))
    u = orc.to_f16(xn.astype(np.float64) @ load_blob(Ku, Nu, pu).astype(np.float64))
    return orc.silu_mul(g, u)


def run(weights: Path, acts: Path | None = None, x_kind: str = "dataflow", layers=None,
        modes=tuple(MODES), log=None) -> list:
    blobs = find_blobs(Path(weights))
    rows = []
    for (layer, proj), (K, N, path) in sorted(blobs.items()):
        if layers is not None and layer not in layers:
            continue
        if acts is not None:
            x = np.fromfile(Path(acts) / f"L{layer:02d}.{proj}.K{K}.x.fp16.bin", dtype=np.float16)
            if x.size != K:
                raise ValueError(f"activation for L{layer:02d}.{proj}: {x.size} values, want {K}")
            src = "captured"
        else:
            x = synthetic_x(x_kind, layer, proj, K, blobs)
            src = x_kind
        row = {"layer": layer, "proj": proj, "x_source": src, **study_tensor(load_blob(K, N, path), x, modes)}
        rows.append(row)
        if log:
            log(f"L{layer:02d} {proj:<10} K={K:<5} N={N:<5} "
                + " ".join(f"cos_{m}={row[f'cos_{m}']:.8f}" for m in modes)
                + f" x_kurt={row['x_kurtosis']:.1f}")
    return rows


def summary(rows, modes=tuple(MODES)) -> dict:
    out = {}
    for m in modes:
        c = np.array([r[f"cos_{m}"] for r in rows])
        out[m] = {"cos_min": float(c.min()), "cos_median": float(np.median(c)), "cos_max": float(c.max()),
                  "all_pass": bool((c >= GATE).all()), "rel_l2_max": float(max(r[f"rel_l2_{m}"] for r in rows))}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--weights", type=Path, required=True, help="directory of L<l>.<proj>.K<k>.N<n>.fp16.bin blobs")
    ap.add_argument("--acts", type=Path, help="directory of captured L<l>.<proj>.K<k>.x.fp16.bin activations")
    ap.add_argument("--x", default="dataflow", choices=["dataflow", "uniform"], help="synthetic x without --acts")
    ap.add_argument("--layers", type=int, nargs="*")
    ap.add_argument("--out", type=Path)
    a = ap.parse_args(argv)
    rows = run(a.weights, a.acts, a.x, a.layers, log=print)
    s = summary(rows)
    print(f"\n=== {len(rows)} projections ===")
    for m, v in s.items():
        print(f"  scale={m:<13} cos min={v['cos_min']:.8f} median={v['cos_median']:.8f} "
              f"max={v['cos_max']:.8f}  all>={GATE}: {v['all_pass']}")
    if a.out:
        a.out.write_text(json.dumps({"rows": rows, "summary": s}, indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
