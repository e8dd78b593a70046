"""The E4M3 accuracy study (oracle/accuracy_study.py) on CPU.

* Pinned to the reference's own study: its no-scale rule (clip, fp32, E4M3 via
  ml_dtypes; kernels/opt_loop/fp8_accuracy/fp8_real_activation_study.py:36-38,
  87) gives the same codes as the oracle's, so the same scores.
* On synthetic blobs in the reference's file layout: every projection scored
  under every scale rule, with captured or synthetic activations.
"""
from __future__ import annotations

import importlib.util
import json

import numpy as np
import pytest

from conftest import ROOT


@pytest.fixture(scope="module")
def study():
    spec = importlib.util.spec_from_file_location("accuracy_study", ROOT / "oracle" / "accuracy_study.py")
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _blobs(d, layers, hidden, inter, seed=0):
    rng = np.random.default_rng(seed)
    for layer in layers:
        for proj, (K, N) in (("gate_proj", (hidden, inter)), ("up_proj", (hidden, inter)),
                             ("down_proj", (inter, hidden))):
            w = (rng.standard_normal((K, N), dtype=np.float32) * 0.02).astype(np.float16)
            w.tofile(d / f"L{layer:02d}.{proj}.K{K}.N{N}.fp16.bin")


def test_no_scale_rule_matches_reference_study(study):
    ml_dtypes = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(11)
    w16 = (rng.standard_normal((256, 384), dtype=np.float32) * 0.05).astype(np.float16)
    w16[0, :8] = [500, -500, 448, 1e-4, -3e-3, 0.0, 240, -0.0156]  # saturating, subnormal and exact edges
    x16 = rng.uniform(-0.25, 0.25, 256).astype(np.float16)
    # the reference study's rule and scores, restated
    w = w16.astype(np.float64)
    deq = np.clip(w, -448.0, 448.0).astype(np.float32).astype(ml_dtypes.float8_e4m3fn).astype(np.float64)
    x = x16.astype(np.float64)
    ref, y = x @ w, x @ deq
    want_cos = float(y @ ref / (np.linalg.norm(y) * np.linalg.norm(ref)))
    row = study.study_tensor(w16, x16, modes=("none",))
    assert abs(row["cos_none"] - want_cos) < 1e-12
    assert abs(row["rel_l2_none"] - np.linalg.norm(y - ref) / np.linalg.norm(ref)) < 1e-12
    assert row["w_n_saturating"] == 2


def test_study_over_reference_layout(study, tmp_path):
    w = tmp_path / "weights"
    w.mkdir()
    _blobs(w, [0, 1], 256, 512)
    rows = study.run(w, x_kind="dataflow")
    assert [(r["layer"], r["proj"]) for r in rows] == [(0, "down_proj"), (0, "gate_proj"), (0, "up_proj"),
                                                     (1, "down_proj"), (1, "gate_proj"), (1, "up_proj")]
    for r in rows:
        for m in study.MODES:
            assert 0.99 < r[f"cos_{m}"] <= 1.0 and r[f"rel_l2_{m}"] < 0.15, (r["proj"], m)
        # N(0, 0.02) weights: about 56 % sit below E4M3's smallest normal without a scale
        # (subnormal codes: a fixed 2^-9 step), so the per-channel rules do better
        assert 0.5 < r["w_frac_below_min_normal"] < 0.62
        assert r["rel_l2_channel_fp32"] < r["rel_l2_none"]
        assert r["x_source"] == "dataflow"
    s = study.summary(rows)
    assert set(s) == set(study.MODES) and s["channel_fp32"]["all_pass"]
    # down's input is SiLU(gate) * up: heavier tails than the RMSNorm'd gate/up input
    kd = np.mean([r["x_kurtosis"] for r in rows if r["proj"] == "down_proj"])
    kg = np.mean([r["x_kurtosis"] for r in rows if r["proj"] == "gate_proj"])
    assert kd > kg


def test_captured_activations_and_cli(study, tmp_path):
    w = tmp_path / "weights"
    acts = tmp_path / "acts"
    w.mkdir()
    acts.mkdir()
    _blobs(w, [3], 128, 256, seed=1)
    rng = np.random.default_rng(2)
    for proj, K in (("gate_proj", 128), ("up_proj", 128), ("down_proj", 256)):
        rng.standard_normal(K).astype(np.float16).tofile(acts / f"L03.{proj}.K{K}.x.fp16.bin")
    out = tmp_path / "rows.json"
    assert study.main(["--weights", str(w), "--acts", str(acts), "--out", str(out)]) == 0
    doc = json.loads(out.read_text())
    assert len(doc["rows"]) == 3 and all(r["x_source"] == "captured" for r in doc["rows"])
    assert set(doc["summary"]) == set(study.MODES)
    (acts / "L03.down_proj.K256.x.fp16.bin").write_bytes(b"\0" * 100)
    with pytest.raises(ValueError, match="activation"):
        study.run(w, acts)
