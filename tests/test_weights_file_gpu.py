"""Weight files on the GPU, full Llama-3.2-3B shapes: reference blobs ->
weight file -> Stack (quantised and packed on the device) gives bitwise the
rows of the same stack built directly from the weights; its packed export
reloads without quantising to bitwise the same rows again."""
from __future__ import annotations

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu

HIDDEN, INTER, LAYERS, M = 3072, 8192, 2, 8


def test_file_to_stack_bitwise(b2g, syn, cuda, tmp_path):
    wfm = importlib.import_module("b2g.weights_file")
    src = tmp_path / "weights"
    src.mkdir()
    ws = {}
    for layer in range(LAYERS):
        seeds = syn.layer_seeds(layer)
        for proj, (K, N), seed in (("gate_proj", (HIDDEN, INTER), seeds[0]), ("up_proj", (HIDDEN, INTER), seeds[1]),
                                   ("down_proj", (INTER, HIDDEN), seeds[2])):
            w = syn.weights(seed, K, N)
            w.tofile(src / f"L{layer:02d}.{proj}.K{K}.N{N}.fp16.bin")  # the reference's blob naming
            ws[(layer, proj)] = w
    wfm.import_reference_blobs(src, tmp_path / "model.b2gw")

    direct = b2g.Stack(HIDDEN, INTER, LAYERS, max_m=8)
    for layer in range(LAYERS):
        (qg, sg), (qu, su), (qd, sd) = (b2g.quantize_e4m3(torch.from_numpy(ws[(layer, p)]).to(cuda), "channel_fp32")
                                        for p in ("gate_proj", "up_proj", "down_proj"))
        direct.set_layer(layer, direct.gate_up.prepack(qg, qu), torch.cat([sg, su]), direct.down.prepack(qd), sd)

    loaded = b2g.Stack(HIDDEN, INTER, LAYERS, max_m=8)
    wfm.load_layers(wfm.WeightFile(tmp_path / "model.b2gw"), loaded, cuda)
    recs = wfm.export_packed(tmp_path / "packed.b2gw", loaded)
    assert all(r.kind == wfm.KIND_PACKED for r in recs) and len(recs) == 2 * LAYERS

    def no_quantize(w, mode):
        raise AssertionError("a packed reload must not quantise")
    reloaded = b2g.Stack(HIDDEN, INTER, LAYERS, max_m=8)
    wfm.load_layers(wfm.WeightFile(tmp_path / "packed.b2gw"), reloaded, cuda, quantize=no_quantize)

    h0 = torch.from_numpy(syn.hidden_state(M, HIDDEN)).to(cuda)
    outs = []
    for st in (direct, loaded, reloaded):
        h = h0.clone()
        act = torch.empty((M, INTER), dtype=torch.float16, device=cuda)
        st.enqueue(h, act, st.workspace(cuda))
        torch.cuda.synchronize()
        outs.append(h)
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(outs[0], outs[2])
    assert b2g.device_error() == 0
