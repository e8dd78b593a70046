"""Tensor-parallel stack host logic on CPU: gloo ranks (world size 2 and 4).

Each rank runs the package's TPStack orchestration -- shard ranges, which
weights and scales each rank slices, the residual on rank 0 only, the
all-reduce -- with the GEMVs replaced by the oracle on CPU (no GPU here).
Rank 0's result is checked against the oracle's single-process restatement
of the sharded layer (mlp_layer_tp) and against the unsharded stack.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_b2g, load_oracle, load_synthetic

HIDDEN, INTER, LAYERS, M = 64, 128, 3, 4


def _layers(orc, syn):
    out = []
    for l in range(LAYERS):
        wg, wu, wd = (syn.weights(2000 + 3 * l + j, K, N)
                      for j, (K, N) in enumerate(((HIDDEN, INTER), (HIDDEN, INTER), (INTER, HIDDEN))))
        (qg, sg), (qu, su), (qd, sd) = (orc.quantize_e4m3(w, orc.SCALE_CHANNEL_FP32) for w in (wg, wu, wd))
        out.append({"wg": qg, "wu": qu, "wd": qd, "sg": sg, "su": su, "sd": sd})
    return out


def _worker(rank, world, port, result_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    load_b2g()  # registers the package as module b2g in this process
    tp_mod = __import__("b2g.tp", fromlist=["TPStack"])
    orc, syn = load_oracle(), load_synthetic()
    layers = _layers(orc, syn)

    class OracleTPStack(tp_mod.TPStack):
        """The GEMV steps on the CPU oracle; everything else is TPStack's."""

        def gate_up_step(self, layer, h, act, workspace):
            wg, wu, _, sg, su, _ = self.layers[layer]
            a = orc.gate_up_silu(orc.rmsnorm(h.numpy()), wg, wu, orc.WTYPE_FP8, orc.SCALE_CHANNEL_FP32, sg, su)
            act.copy_(torch.from_numpy(np.asarray(a, np.float16)))

        def down_step(self, layer, act, h, workspace):
            _, _, wd, _, _, sd = self.layers[layer]
            y = orc.to_f16(orc.gemv(wd, orc.WTYPE_FP8, act.numpy(), orc.SCALE_CHANNEL_FP32, sd))
            if self.rank == 0:
                y = orc.residual_add(h.numpy(), y)
            h.copy_(torch.from_numpy(np.asarray(y, np.float16)))

    st = OracleTPStack(HIDDEN, INTER, LAYERS, rank=rank, world=world, build_ops=False)
    for l, L in enumerate(layers):
        # the oracle steps take this rank's numpy slices in place of packed buffers
        st.layers[l] = st.slice_layer(L["wg"], L["wu"], L["wd"], L["sg"], L["su"], L["sd"])
    h0 = syn.hidden_state(M, HIDDEN)
    h = torch.from_numpy(h0.copy())
    act = torch.zeros(M, st.shard, dtype=torch.float16)
    st.enqueue(h, act, None)  # the package's layer loop: gate_up_step, down_step, reduce_step (gloo)
    if rank == 0:
        np.save(result_path, np.stack([h.numpy(), h0]))
        with open(result_path + ".shards", "w") as f:
            f.write(f"{st.lo} {st.hi}\n")
    else:
        with open(result_path + f".shards{rank}", "w") as f:
            f.write(f"{st.lo} {st.hi}\n")
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range(b2g):
    tp = __import__("b2g.tp", fromlist=["shard_range"])
    assert [tp.shard_range(8192, r, 4) for r in range(4)] == [(0, 2048), (2048, 4096), (4096, 6144),
                                                              (6144, 8192)]
    with pytest.raises(ValueError):
        tp.shard_range(8192, 0, 3)
    with pytest.raises(ValueError):
        tp.shard_range(8192, 2, 2)


@pytest.mark.parametrize("world", [2, 4])
def test_tp_stack_gloo_ranks(b2g, orc, syn, tmp_path, world):
    out = str(tmp_path / "h.npy")
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    got, h0 = np.load(out)
    shards = [tuple(map(int, open(out + (".shards" if r == 0 else f".shards{r}")).read().split()))
              for r in range(world)]
    step = INTER // world
    assert shards == [(r * step, (r + 1) * step) for r in range(world)]
    layers = _layers(orc, syn)
    want_tp = h0
    for L in layers:
        want_tp = orc.mlp_layer_tp(want_tp, L, world)
    r = orc.compare(got, want_tp.astype(np.float64))
    assert r["rel_l2"] <= 2e-3, r
    r_full = orc.compare(got, orc.mlp_stack(h0, layers).astype(np.float64))
    assert r_full["rel_l2"] <= 5e-3, r_full


@pytest.mark.parametrize("exchange", ["reduce", "gather_kernel", "gather_launch"])
def test_fused_exchange_schedule(b2g, monkeypatch, exchange):
    """TPStack(fused=True)'s launch order on one rank, with recording stand-ins
    for the ops.  REDUCE (default): every layer is a plain gate||up and a down
    launch in REDUCE mode writing h, nothing after the last layer.  The PUSH
    exchanges: layer 0 stages h plainly; before every later gate||up the
    previous push is summed into h -- by the separate gather kernel followed
    by a plain gate||up, or by the gate||up launch itself in GATHER mode --
    and one final gather reads the last push's buffer.  Exchange number r
    (counted over all calls) goes to buffer r % 2, with the residual on rank 0
    only.  Each GEMV launch prefetches the next one's weights."""
    tp_mod = __import__("b2g.tp", fromlist=["TPStack"])
    calls = []

    class Rec:
        def __init__(self, name):
            self.name = name

        def enqueue(self, x, packed, scales=None, **kw):
            calls.append((self.name, "plain", None, packed, kw.get("prefetch")[1]))

        def enqueue_tp(self, comm, mode, buf, x, packed, scales=None, **kw):
            assert comm is st.comm
            if mode == tp_mod.TP_GATHER:
                assert kw["push_op"] is st.down and kw["h_out"] is h
            else:
                assert kw["residual"] is (h if st.rank == 0 else None) and kw["y"] is h
            pf = kw.get("prefetch")
            calls.append((self.name, mode, buf, packed, None if pf is None else pf[1]))

    def gather(comm, buf, op, hh):
        assert comm is st.comm and op is st.down and hh is h
        calls.append(("tp_gather", buf))
    monkeypatch.setattr(tp_mod, "tp_gather", gather)
    G, Pu, R = tp_mod.TP_GATHER, tp_mod.TP_PUSH, tp_mod.TP_REDUCE

    def gu(layer, buf):  # the gate||up of a layer > 0 and the gather before it
        if exchange == "gather_kernel":
            return [("tp_gather", buf), ("gu", "plain", None, f"pgu{layer}", f"pd{layer}")]
        return [("gu", G, buf, f"pgu{layer}", f"pd{layer}")]

    def want(first_buf):
        b = [first_buf, 1 - first_buf, first_buf]
        if exchange == "reduce":
            return [c for l in range(3) for c in (("gu", "plain", None, f"pgu{l}", f"pd{l}"),
                                                   ("dn", R, b[l], f"pd{l}", f"pgu{(l + 1) % 3}"))]
        return ([("gu", "plain", None, "pgu0", "pd0"), ("dn", Pu, b[0], "pd0", "pgu1")] + gu(1, b[0]) +
                [("dn", Pu, b[1], "pd1", "pgu2")] + gu(2, b[1]) +
                [("dn", Pu, b[2], "pd2", "pgu0"), ("tp_gather", b[2])])
    for rank in (0, 1):
        calls.clear()
        st = tp_mod.TPStack(64, 128, 3, rank=rank, world=2, build_ops=False, fused=True)
        if exchange != "reduce":
            st.exchange = exchange
        assert st.exchange == exchange
        st.gate_up, st.down = Rec("gu"), Rec("dn")
        st.layers = [(f"pgu{l}", f"sgu{l}", f"pd{l}", f"sd{l}") for l in range(3)]
        h, act = torch.zeros(4, 64, dtype=torch.float16), torch.zeros(4, 64, dtype=torch.float16)
        with pytest.raises(RuntimeError, match="setup_comm"):
            st.enqueue(h, act, None)
        st.comm = object()
        st.enqueue(h, act, None)
        assert calls == want(0), rank
        # A second call continues the alternation: with 3 layers the first
        # exchange of this call goes to buffer 1, not to buffer 0, which a
        # peer may still be reading from the previous call's last exchange.
        calls.clear()
        st.enqueue(h, act, None)
        assert calls == want(1), rank
    st.exchange = "bogus"
    with pytest.raises(ValueError, match="exchange"):
        st.enqueue(h, act, None)
