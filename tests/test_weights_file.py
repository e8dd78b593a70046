"""Weight files on CPU: the binary format, the reference-blob importer and the
loader's orchestration (which records fill which layer, full-matrix
quantisation before sharding, packed reloads, layout checks).  The device
steps (quantise, prepack) are stood in for by the oracle's quantiser and by
ops whose prepack returns its input; the GPU test runs the real ones."""
from __future__ import annotations

import importlib
import json

import numpy as np
import pytest
import torch

from conftest import load_b2g, load_oracle


@pytest.fixture(scope="module")
def wfm():
    load_b2g()
    return importlib.import_module("b2g.weights_file")


def _fp16(rng, K, N):
    return (rng.standard_normal((K, N), dtype=np.float32) * 0.02).astype(np.float16)


# --------------------------------------------------------------------------
# Format
# --------------------------------------------------------------------------
def test_round_trip_all_kinds(wfm, tmp_path):
    rng = np.random.default_rng(1)
    w16 = _fp16(rng, 64, 48)
    codes = rng.integers(0, 256, (64, 48), dtype=np.uint8)
    s32 = rng.random(48, dtype=np.float32)
    packed = rng.integers(0, 256, 5000, dtype=np.uint8)
    s16 = rng.random(96).astype(np.float16)
    R = wfm.Record
    items = [(R(0, "gate_proj", wfm.KIND_FP16_KN, 0, 0, 64, 48), w16, None),
             (R(0, "up_proj", wfm.KIND_E4M3_KN, 1, 3, 64, 48), codes, s32),
             (R(0, "gate_up", wfm.KIND_PACKED, 1, 2, 64, 48, planes=2, ksplit=1, tp_rank=1, tp_size=2),
              torch.from_numpy(packed), torch.from_numpy(s16))]
    path = tmp_path / "w.b2gw"
    wfm.write(path, items)
    f = wfm.WeightFile(path)
    assert [r.name for r in f.records] == ["L00.gate_proj", "L00.up_proj", "L00.gate_up.tp1of2"]
    for r in f.records:
        assert r.data_offset % wfm.ALIGN == 0 and r.scales_offset % wfm.ALIGN == 0
    d, s = f.read(f.find(0, "gate_proj"))
    assert d.dtype == np.float16 and np.array_equal(d, w16) and s is None
    d, s = f.read(f.find(0, "up_proj", wfm.KIND_E4M3_KN))
    assert np.array_equal(d, codes) and s.dtype == np.float32 and np.array_equal(s, s32)
    r = f.find(0, "gate_up", wfm.KIND_PACKED, tp_rank=1, tp_size=2)
    assert (r.planes, r.ksplit, r.weight_dtype, r.scale_mode) == (2, 1, 1, 2)
    d, s = f.read(r)
    assert np.array_equal(d, packed) and s.dtype == np.float16 and np.array_equal(s, s16)
    with pytest.raises(KeyError):
        f.find(0, "gate_up", wfm.KIND_PACKED)  # tp 0/1 is not in the file
    assert f.layers() == [0]


def test_damage_is_detected(wfm, tmp_path):
    rng = np.random.default_rng(2)
    w16 = _fp16(rng, 32, 32)
    path = tmp_path / "w.b2gw"
    (rec,) = wfm.write(path, [(wfm.Record(3, "down_proj", wfm.KIND_FP16_KN, 0, 0, 32, 32), w16, None)])
    raw = bytearray(path.read_bytes())
    raw[rec.data_offset + 7] ^= 0x40  # one flipped bit in the weights
    bad = tmp_path / "bad.b2gw"
    bad.write_bytes(raw)
    f = wfm.WeightFile(bad)
    with pytest.raises(wfm.WeightFileError, match="CRC"):
        f.read(f.records[0])
    d, _ = f.read(f.records[0], verify=False)
    assert not np.array_equal(d, w16)

    (tmp_path / "magic.b2gw").write_bytes(b"NOTAWGHT" + bytes(raw[8:]))
    with pytest.raises(wfm.WeightFileError, match="not a weight file"):
        wfm.WeightFile(tmp_path / "magic.b2gw")
    (tmp_path / "short.b2gw").write_bytes(bytes(path.read_bytes()[:-100]))
    with pytest.raises(wfm.WeightFileError, match="truncated"):
        wfm.WeightFile(tmp_path / "short.b2gw")
    raw = bytearray(path.read_bytes())
    idx = raw.rfind(b"L03.down_proj")
    raw[idx + 2] = ord("4")  # the index name no longer matches its fields
    (tmp_path / "name.b2gw").write_bytes(raw)
    with pytest.raises(wfm.WeightFileError, match="does not match"):
        wfm.WeightFile(tmp_path / "name.b2gw")


# --------------------------------------------------------------------------
# The reference's blobs
# --------------------------------------------------------------------------
def _write_blobs(d, layers, hidden, inter, with_manifest, rng):
    shapes = {"gate_proj": (hidden, inter), "up_proj": (hidden, inter), "down_proj": (inter, hidden)}
    man, ws = [], {}
    for layer in layers:
        for proj, (K, N) in shapes.items():
            w = _fp16(rng, K, N)
            p = d / f"L{layer:02d}.{proj}.K{K}.N{N}.fp16.bin"
            w.tofile(p)
            ws[(layer, proj)] = w
            # as the reference's extractor writes it, with a path from the machine that ran it
            man.append({"layer": layer, "proj": proj, "init": f"onnx::MatMul_{layer}_{proj}", "K": K, "N": N,
                        "bytes": K * N * 2, "path": f"/workspace/.fp8_tools/weights/{p.name}"})
    if with_manifest:
        (d / "manifest.json").write_text(json.dumps(man, indent=2))
    return ws


def test_reference_blob_names(wfm):
    assert wfm.parse_reference_blob_name("L13.up_proj.K3072.N8192.fp16.bin") == (13, "up_proj", 3072, 8192)
    assert wfm.parse_reference_blob_name("/x/y/L00.down_proj.K8192.N3072.fp16.bin") == (0, "down_proj", 8192, 3072)
    for bad in ("L13.up_proj.K3072.fp16.bin", "L13.q_proj.K3072.N8192.fp16.bin", "L13.up_proj.K3072.N8192.bin",
                "L13.up_proj.K3072.synth.x.fp16.bin"):
        with pytest.raises(wfm.WeightFileError):
            wfm.parse_reference_blob_name(bad)


@pytest.mark.parametrize("with_manifest", [True, False])
def test_import_reference_blobs(wfm, tmp_path, with_manifest):
    src = tmp_path / "weights"
    src.mkdir()
    ws = _write_blobs(src, [0, 1, 13], 64, 128, with_manifest, np.random.default_rng(3))
    (src / "L13.up_proj.K64.synth.x.fp16.bin").write_bytes(b"\0" * 128)  # an activation file: skipped
    out = tmp_path / "model.b2gw"
    recs = wfm.import_reference_blobs(src, out, layers=[0, 13])
    assert [r.name for r in recs] == ["L00.gate_proj", "L00.up_proj", "L00.down_proj",
                                      "L13.gate_proj", "L13.up_proj", "L13.down_proj"]
    f = wfm.WeightFile(out)
    for (layer, proj), w in ws.items():
        if layer == 1:
            continue
        r = f.find(layer, proj, wfm.KIND_FP16_KN)
        assert (r.K, r.N) == w.shape
        d, _ = f.read(r)
        assert d.tobytes() == w.tobytes()  # the blob's bytes, unchanged


def test_import_rejects_bad_blobs(wfm, tmp_path):
    src = tmp_path / "w"
    src.mkdir()
    _write_blobs(src, [0], 32, 64, True, np.random.default_rng(4))
    p = src / "L00.down_proj.K64.N32.fp16.bin"
    p.write_bytes(p.read_bytes()[:-2])  # one element short
    with pytest.raises(wfm.WeightFileError, match="K\\*N\\*2"):
        wfm.import_reference_blobs(src, tmp_path / "o.b2gw")
    man = json.loads((src / "manifest.json").read_text())
    man[0]["K"] = 33
    (src / "manifest.json").write_text(json.dumps(man))
    with pytest.raises(wfm.WeightFileError, match="disagrees"):
        wfm.reference_blobs(src)
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(wfm.WeightFileError, match="no reference weight blobs"):
        wfm.import_reference_blobs(empty, tmp_path / "e.b2gw")


# --------------------------------------------------------------------------
# Loader orchestration (device steps stood in for on CPU)
# --------------------------------------------------------------------------
class FakeOp:
    """The attributes the loader reads from a GemvOp; prepack returns its
    inputs stacked (so what was packed can be checked)."""

    def __init__(self, K, N, planes, ksplit=1, weight_dtype=1, scale_mode=3, max_m=8):
        self.K, self.N, self.planes, self.weight_dtype, self.scale_mode, self.max_m = (
            K, N, planes, weight_dtype, scale_mode, max_m)
        self._ksplit = ksplit

    def plan(self, m):
        return {"ksplit": self._ksplit}

    def packed_bytes(self):
        return self.K * self.N * self.planes * (1 if self.weight_dtype == 1 else 2)

    def prepack(self, w0, w1=None):
        w = w0 if w1 is None else torch.stack([w0, w1])
        return w.contiguous().view(torch.uint8).flatten()


class FakeStack:
    def __init__(self, hidden, inter, n_layers, ksplit=1):
        self.n_layers = n_layers
        self.gate_up = FakeOp(hidden, inter, 2, ksplit)
        self.down = FakeOp(inter, hidden, 1, ksplit)
        self._keep = {}

    def set_layer(self, layer, pgu, sgu, pd, sd):
        self._keep[layer] = (pgu, sgu, pd, sd)


def _oracle_quantize(orc):
    def q(w, mode):
        c, s = orc.quantize_e4m3(w.numpy(), mode)
        return torch.from_numpy(c), torch.from_numpy(s)
    return q


def test_load_source_records_into_stack(wfm, tmp_path):
    orc = load_oracle()
    src = tmp_path / "w"
    src.mkdir()
    ws = _write_blobs(src, [0, 1], 64, 128, True, np.random.default_rng(5))
    wfm.import_reference_blobs(src, tmp_path / "m.b2gw")
    st = FakeStack(64, 128, 2)
    wfm.load_layers(wfm.WeightFile(tmp_path / "m.b2gw"), st, "cpu", quantize=_oracle_quantize(orc))
    for layer in (0, 1):
        pgu, sgu, pd, sd = st._keep[layer]
        (qg, sg), (qu, su), (qd, sd_want) = (orc.quantize_e4m3(ws[(layer, p)], orc.SCALE_CHANNEL_FP32)
                                              for p in ("gate_proj", "up_proj", "down_proj"))
        assert np.array_equal(pgu.numpy(), np.stack([qg, qu]).ravel())
        assert np.array_equal(sgu.numpy(), np.concatenate([sg, su]))
        assert np.array_equal(pd.numpy(), qd.ravel()) and np.array_equal(sd.numpy(), sd_want)


def test_load_tp_shards_quantise_whole_matrix_first(wfm, tmp_path):
    """Rank 1 of 2: gate/up columns and down rows of the codes quantised over
    the whole matrices -- down's per-channel scales stay the unsharded ones."""
    orc = load_oracle()
    tpm = importlib.import_module("b2g.tp")
    src = tmp_path / "w"
    src.mkdir()
    ws = _write_blobs(src, [0], 64, 128, False, np.random.default_rng(6))
    wfm.import_reference_blobs(src, tmp_path / "m.b2gw")
    st = tpm.TPStack(64, 128, 1, rank=1, world=2, build_ops=False)
    st.gate_up, st.down = FakeOp(64, 64, 2), FakeOp(64, 64, 1)
    wfm.load_layers(wfm.WeightFile(tmp_path / "m.b2gw"), st, "cpu", quantize=_oracle_quantize(orc))
    pgu, sgu, pd, sd = st.layers[0]
    (qg, sg), (qu, su), (qd, sdw) = (orc.quantize_e4m3(ws[(0, p)], orc.SCALE_CHANNEL_FP32)
                                      for p in ("gate_proj", "up_proj", "down_proj"))
    cs = slice(64, 128)
    assert np.array_equal(pgu.numpy(), np.stack([qg[:, cs], qu[:, cs]]).ravel())
    assert np.array_equal(sgu.numpy(), np.concatenate([sg[cs], su[cs]]))
    assert np.array_equal(pd.numpy(), qd[cs, :].ravel())
    assert np.array_equal(sd.numpy(), sdw)
    # quantising the shard alone would give other down scales
    _, s_shard = orc.quantize_e4m3(ws[(0, "down_proj")][cs, :], orc.SCALE_CHANNEL_FP32)
    assert not np.array_equal(s_shard, sdw)


def test_packed_export_reload_and_layout_check(wfm, tmp_path):
    orc = load_oracle()
    src = tmp_path / "w"
    src.mkdir()
    _write_blobs(src, [0, 1], 64, 128, True, np.random.default_rng(7))
    wfm.import_reference_blobs(src, tmp_path / "m.b2gw")
    st = FakeStack(64, 128, 2)
    wfm.load_layers(wfm.WeightFile(tmp_path / "m.b2gw"), st, "cpu", quantize=_oracle_quantize(orc))
    recs = wfm.export_packed(tmp_path / "p.b2gw", st)
    assert [(r.name, r.kind, r.planes, r.ksplit) for r in recs] == [
        ("L00.gate_up", wfm.KIND_PACKED, 2, 1), ("L00.down_proj", wfm.KIND_PACKED, 1, 1),
        ("L01.gate_up", wfm.KIND_PACKED, 2, 1), ("L01.down_proj", wfm.KIND_PACKED, 1, 1)]

    def no_quantize(w, mode):
        raise AssertionError("a packed reload must not quantise")
    st2 = FakeStack(64, 128, 2)
    wfm.load_layers(wfm.WeightFile(tmp_path / "p.b2gw"), st2, "cpu", quantize=no_quantize)
    for layer in (0, 1):
        for a, b in zip(st._keep[layer], st2._keep[layer]):
            assert torch.equal(a, b)
    # an op with another K split cannot take these streams, and the file has nothing else
    with pytest.raises(wfm.WeightFileError, match="another op plan"):
        wfm.load_layers(wfm.WeightFile(tmp_path / "p.b2gw"), FakeStack(64, 128, 2, ksplit=2), "cpu",
                        quantize=no_quantize)


def test_tp_rank_packed_export_reload(wfm, tmp_path):
    """A TPStack rank exports its own shard's streams (records named for the
    rank); the same rank reloads them without quantising, another rank finds
    none of its own and falls back to the source records."""
    orc = load_oracle()
    tpm = importlib.import_module("b2g.tp")
    src = tmp_path / "w"
    src.mkdir()
    _write_blobs(src, [0], 64, 128, True, np.random.default_rng(8))
    wfm.import_reference_blobs(src, tmp_path / "m.b2gw")

    def rank_stack(rank):
        st = tpm.TPStack(64, 128, 1, rank=rank, world=2, build_ops=False)
        st.gate_up, st.down = FakeOp(64, 64, 2), FakeOp(64, 64, 1)
        return st
    r1 = rank_stack(1)
    wfm.load_layers(wfm.WeightFile(tmp_path / "m.b2gw"), r1, "cpu", quantize=_oracle_quantize(orc))
    recs = wfm.export_packed(tmp_path / "r1.b2gw", r1)
    assert [r.name for r in recs] == ["L00.gate_up.tp1of2", "L00.down_proj.tp1of2"]

    def no_quantize(w, mode):
        raise AssertionError("a packed reload must not quantise")
    again = rank_stack(1)
    wfm.load_layers(wfm.WeightFile(tmp_path / "r1.b2gw"), again, "cpu", quantize=no_quantize)
    for a, b in zip(r1.layers[0], again.layers[0]):
        assert torch.equal(a, b)
    with pytest.raises(wfm.WeightFileError, match="rank 0 of 2"):  # no records of its own, no source weights
        wfm.load_layers(wfm.WeightFile(tmp_path / "r1.b2gw"), rank_stack(0), "cpu", quantize=no_quantize)


def _e4m3_items(wfm, rng, hidden, inter, mode, n_scales=None, shape=None):
    """One layer of E4M3_KN records with scale mode `mode` (codes random)."""
    R = wfm.Record
    items = []
    for proj, (K, N) in (("gate_proj", (hidden, inter)), ("up_proj", (hidden, inter)),
                         ("down_proj", (inter, hidden))):
        if shape is not None and proj == "down_proj":
            K, N = shape
        codes = rng.integers(0, 0x7F, (K, N), dtype=np.uint8)
        n = N if n_scales is None else n_scales
        s = None if mode == 0 else (rng.random(n).astype(np.float32 if mode == 3 else np.float16))
        items.append((R(0, proj, wfm.KIND_E4M3_KN, 1, mode, K, N), codes, s))
    return items


def test_e4m3_source_records_checked_against_op(wfm, tmp_path):
    """E4M3 codes are used without re-quantising, so a record whose scale
    rule, scale count or shape is not the op's is refused: the kernel would
    otherwise read N per-channel scales from a one-value buffer."""
    rng = np.random.default_rng(9)

    def no_quantize(w, mode):
        raise AssertionError("E4M3 records are not re-quantised")
    # matching records load (per-channel FP32, the op's rule)
    wfm.write(tmp_path / "ok.b2gw", _e4m3_items(wfm, rng, 64, 128, 3))
    st = FakeStack(64, 128, 1)
    wfm.load_layers(wfm.WeightFile(tmp_path / "ok.b2gw"), st, "cpu", quantize=no_quantize)
    assert st._keep[0][3].numel() == 64
    # per-tensor codes into a per-channel op
    wfm.write(tmp_path / "tensor.b2gw", _e4m3_items(wfm, rng, 64, 128, 1, n_scales=1))
    with pytest.raises(wfm.WeightFileError, match="scale mode 1"):
        wfm.load_layers(wfm.WeightFile(tmp_path / "tensor.b2gw"), FakeStack(64, 128, 1), "cpu",
                        quantize=no_quantize)
    # right rule, wrong number of scales
    wfm.write(tmp_path / "count.b2gw", _e4m3_items(wfm, rng, 64, 128, 3, n_scales=5))
    with pytest.raises(wfm.WeightFileError, match="5 scales"):
        wfm.load_layers(wfm.WeightFile(tmp_path / "count.b2gw"), FakeStack(64, 128, 1), "cpu",
                        quantize=no_quantize)
    # a down projection of another shape
    wfm.write(tmp_path / "shape.b2gw", _e4m3_items(wfm, rng, 64, 128, 3, shape=(96, 64)))
    with pytest.raises(wfm.WeightFileError, match="96x64"):
        wfm.load_layers(wfm.WeightFile(tmp_path / "shape.b2gw"), FakeStack(64, 128, 1), "cpu",
                        quantize=no_quantize)
