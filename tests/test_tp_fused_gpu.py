"""The all-reduce fused into the GEMVs through peer memory (b2g_enqueue_tp).

* world = 1 on one GPU: every fused exchange (REDUCE; PUSH with the gather
  kernel; PUSH with GATHER launches) must give bitwise the rows of the plain
  path;
* a wait that nothing satisfies expires (bounded) and reports through the
  device error word, leaving the rows untouched;
* two ranks on two GPUs, and every GPU of the machine (up to 8) when it
  has more: rank 0's result against the oracle's sharded restatement, every
  rank's rows bitwise equal.
"""
from __future__ import annotations

import os
import socket
import time

import numpy as np
import pytest
import torch

from conftest import load_b2g, load_oracle, load_synthetic

pytestmark = pytest.mark.gpu


def _tp(b2g):
    return __import__("b2g.tp", fromlist=["TPStack"])


def _weights(orc, syn, hidden, inter, n_layers, seed0):
    out = []
    for l in range(n_layers):
        ws = [syn.weights(seed0 + 3 * l + j, K, N)
              for j, (K, N) in enumerate(((hidden, inter), (hidden, inter), (inter, hidden)))]
        (qg, sg), (qu, su), (qd, sd) = (orc.quantize_e4m3(w, orc.SCALE_CHANNEL_FP32) for w in ws)
        out.append({"wg": qg, "wu": qu, "wd": qd, "sg": sg, "su": su, "sd": sd})
    return out


def _load_layers(st, layers, dev):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    for l, L in enumerate(layers):
        st.prepack_layer(l, t(L["wg"]), t(L["wu"]), t(L["wd"]), t(L["sg"]), t(L["su"]), t(L["sd"]))


@pytest.mark.parametrize("exchange", ["reduce", "gather_kernel", "gather_launch"])
@pytest.mark.parametrize("hidden,inter,n_layers", [(256, 512, 3), (3072, 8192, 2)])
def test_fused_world1_matches_plain(b2g, orc, syn, cuda, hidden, inter, n_layers, exchange):
    """The fused exchange (rows summed by each down CTA after its counterparts
    arrive, by the separate gather kernel, or by the gate||up launch in GATHER
    mode) gives bitwise the rows of the plain path."""
    tp = _tp(b2g)
    layers = _weights(orc, syn, hidden, inter, n_layers, 3000)
    plain = tp.TPStack(hidden, inter, n_layers, rank=0, world=1, max_m=8)
    fused = tp.TPStack(hidden, inter, n_layers, rank=0, world=1, max_m=8, fused=True)
    fused.exchange = exchange
    _load_layers(plain, layers, cuda)
    _load_layers(fused, layers, cuda)
    fused.setup_comm(cuda)
    ws_p, ws_f = plain.workspace(cuda), fused.workspace(cuda)
    for M in (1, 8):
        h0 = syn.hidden_state(M, hidden)
        hp = torch.from_numpy(h0).to(cuda)
        hf = hp.clone()
        act_p = torch.empty(M, inter, dtype=torch.float16, device=cuda)
        act_f = act_p.clone()
        for _ in range(2):  # a second step reuses the inbox buffers and counters
            plain.enqueue(hp, act_p, ws_p)
            fused.enqueue(hf, act_f, ws_f)
        torch.cuda.synchronize()
        assert torch.equal(hp, hf), M
        want = orc.mlp_stack(orc.mlp_stack(h0, layers), layers)
        r = orc.compare(hf.cpu().numpy(), want.astype(np.float64))
        assert r["rel_l2"] <= 5e-3, r
    assert b2g.device_error() == 0
    fused.close_comm()


def test_gather_wait_expires(b2g, orc, syn, cuda):
    """An arrival that never comes: the bounded wait gives up, records the
    peer-wait code and leaves h as it was."""
    tp = _tp(b2g)
    st = tp.TPStack(256, 512, 1, rank=0, world=1, max_m=8, fused=True)
    comm = st.setup_comm(cuda)
    _, _, epoch = b2g.tp_comm_layout(st._comm_buf.data_ptr(), 1, 8, 256)
    off = epoch - st._comm_buf.data_ptr()
    st._comm_buf[off:off + 4].view(torch.int32).fill_(1)  # one round expected, none pushed
    h = torch.full((2, 256), 3.0, dtype=torch.float16, device=cuda)
    b2g.tp_gather(comm, 0, st.down, h)
    torch.cuda.synchronize()
    assert b2g.device_error(clear=False) == 4  # peer wait expired
    assert bool((h == 3.0).all())
    # while the error word is set, a later wait gives up at once
    t0 = time.perf_counter()
    b2g.tp_gather(comm, 0, st.down, h)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.5
    assert b2g.device_error(clear=True) == 4
    assert bool((h == 3.0).all())
    st.close_comm()


def test_reduce_wait_expires_writes_nothing(b2g, orc, syn, cuda):
    """A down launch in REDUCE mode whose peer never writes: rank 0 of a
    two-rank exchange whose rank 1 is a second buffer on this GPU that no
    launch fills.  Every poll gives up after the bounded wait, records the
    peer-wait code, and y is left as it was; while the error word is set, a
    later launch gives up at once.  After the word is cleared and the buffers
    re-zeroed, the same op gives the plain result at world 1."""
    tp = _tp(b2g)
    H, I = 256, 512
    nbytes = b2g.tp_comm_bytes(2, 8, H)
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(2)]
    comm = b2g.TpComm()
    comm.world, comm.rank, comm.max_m, comm.width = 2, 0, 8, H
    for r, b in enumerate(bufs):
        inbox, counters, epoch = b2g.tp_comm_layout(b.data_ptr(), 2, 8, H)
        comm.inbox[r], comm.counters[r] = inbox, counters
        if r == 0:
            comm.epoch = epoch
    st = tp.TPStack(H, I, 1, rank=0, world=1, max_m=8, fused=True)
    wd, sd = b2g.quantize_e4m3(torch.from_numpy(syn.weights(83, I, H)).to(cuda), "channel_fp32")
    pd = st.down.prepack(wd)
    act = torch.from_numpy(syn.activations(84, 2, I)).to(cuda)
    h = torch.full((2, H), 3.0, dtype=torch.float16, device=cuda)
    ws = st.workspace(cuda)
    st.down.enqueue_tp(comm, b2g.TP_REDUCE, 0, act, pd, sd, y=h, residual=h, workspace=ws)
    torch.cuda.synchronize()
    assert b2g.device_error(clear=False) == 4  # peer wait expired
    assert bool((h == 3.0).all())
    t0 = time.perf_counter()
    st.down.enqueue_tp(comm, b2g.TP_REDUCE, 1, act, pd, sd, y=h, residual=h, workspace=ws)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.5
    assert b2g.device_error(clear=True) == 4
    assert bool((h == 3.0).all())
    # recovery: the word cleared, the exchange buffer re-zeroed
    one = st.setup_comm(cuda)
    st.down.enqueue_tp(one, b2g.TP_REDUCE, 0, act, pd, sd, y=h, residual=h, workspace=ws)
    torch.cuda.synchronize()
    want = 3.0 + orc.gemv(wd.cpu().numpy(), orc.WTYPE_FP8, act.cpu().numpy(), orc.SCALE_CHANNEL_FP32,
                          sd.cpu().numpy())
    assert orc.compare(h.cpu().numpy(), want)["rel_l2"] <= 5e-3
    assert b2g.device_error() == 0
    st.close_comm()


def test_reduce_refuses_unfit_plans(b2g, cuda):
    """REDUCE needs whole tiles and the register pipeline: a K-split down op
    and the TMA pipeline are refused before anything is launched."""
    tp = _tp(b2g)
    H, I = 256, 512
    st = tp.TPStack(H, I, 1, rank=0, world=1, max_m=8, fused=True)
    comm = st.setup_comm(cuda)
    act = torch.zeros(2, I, dtype=torch.float16, device=cuda)
    h = torch.zeros(2, H, dtype=torch.float16, device=cuda)
    ws = st.workspace(cuda)
    st.down.set_option(b2g.OPT_PIPE, b2g.PIPE_TMA)
    pd = st.down.prepack(torch.zeros(I, H, dtype=torch.uint8, device=cuda))
    sd = torch.ones(H, dtype=torch.float32, device=cuda)
    with pytest.raises(b2g.B2GError) as e:
        st.down.enqueue_tp(comm, b2g.TP_REDUCE, 0, act, pd, sd, y=h, residual=h, workspace=ws)
    assert e.value.status == b2g.ERR_UNSUPPORTED
    split = b2g.GemvOp(I, H, max_m=8, fuse=b2g.FUSE_RESIDUAL_ADD)
    split.set_option(b2g.OPT_KSPLIT, 2)
    assert split.plan(2)["ksplit"] == 2
    ps = split.prepack(torch.zeros(I, H, dtype=torch.uint8, device=cuda))
    with pytest.raises(b2g.B2GError) as e:
        split.enqueue_tp(comm, b2g.TP_REDUCE, 0, act, ps, sd, y=h, residual=h, workspace=split.workspace(cuda))
    assert e.value.status == b2g.ERR_INVALID
    torch.cuda.synchronize()
    assert bool((h == 0).all()) and b2g.device_error() == 0
    st.close_comm()


@pytest.mark.parametrize("pipe", ["registers", "tma"])
def test_gather_gemv_wait_expires_writes_nothing(b2g, orc, syn, cuda, pipe):
    """A gate||up launch in GATHER mode whose wait for the peers' arrivals
    expires records the peer-wait code and writes neither h (the all-reduced
    rows) nor its own output rows."""
    tp = _tp(b2g)
    H, I = 256, 512
    st = tp.TPStack(H, I, 1, rank=0, world=1, max_m=8, fused=True)
    code = {"registers": b2g.PIPE_REGISTERS, "tma": b2g.PIPE_TMA}[pipe]
    st.gate_up.set_option(b2g.OPT_PIPE, code)
    assert st.gate_up.plan(2)["pipe"] == code
    comm = st.setup_comm(cuda)
    wg, wu = (b2g.quantize_e4m3(torch.from_numpy(syn.weights(s, H, I)).to(cuda), "channel_fp32") for s in (81, 82))
    pgu = st.gate_up.prepack(wg[0], wu[0])
    sgu = torch.cat([wg[1], wu[1]])
    _, _, epoch = b2g.tp_comm_layout(st._comm_buf.data_ptr(), 1, 8, H)
    off = epoch - st._comm_buf.data_ptr()
    st._comm_buf[off:off + 4].view(torch.int32).fill_(1)  # one round expected, none pushed
    h = torch.full((2, H), 3.0, dtype=torch.float16, device=cuda)
    act = torch.full((2, I), 5.0, dtype=torch.float16, device=cuda)
    ws = st.workspace(cuda)
    st.gate_up.enqueue_tp(comm, b2g.TP_GATHER, 0, h, pgu, sgu, y=act, workspace=ws, push_op=st.down, h_out=h)
    torch.cuda.synchronize()
    assert b2g.device_error(clear=True) == 4  # peer wait expired
    assert bool((h == 3.0).all()) and bool((act == 5.0).all())
    # the workspace's tile counters are back at zero: the op runs normally afterwards
    st._comm_buf.zero_()
    y = st.gate_up.enqueue(h, pgu, sgu, workspace=ws)
    torch.cuda.synchronize()
    want = orc.gate_up_silu(orc.rmsnorm(h.cpu().numpy()), wg[0].cpu().numpy(), wu[0].cpu().numpy(),
                            orc.WTYPE_FP8, orc.SCALE_CHANNEL_FP32, wg[1].cpu().numpy(), wu[1].cpu().numpy())
    assert orc.compare(y.cpu().numpy(), want.astype(np.float64))["rel_l2"] <= 5e-3
    assert b2g.device_error() == 0
    st.close_comm()


# --------------------------------------------------------------------------
# Two ranks, one GPU each
# --------------------------------------------------------------------------
HID, INT, NL, MM = 3072, 8192, 2, 8


def _rank(rank, world, port, out, nl=NL, steps=1, exchange="reduce"):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)  # handle exchange only
    b2g, orc, syn = load_b2g(), load_oracle(), load_synthetic()
    tp = __import__("b2g.tp", fromlist=["TPStack"])
    layers = _weights(orc, syn, HID, INT, nl, 4000)
    st = tp.TPStack(HID, INT, nl, rank=rank, world=world, max_m=8, fused=True)
    st.exchange = exchange
    _load_layers(st, layers, dev)
    st.setup_comm(dev)
    h = torch.from_numpy(syn.hidden_state(MM, HID)).to(dev)
    act = torch.empty(MM, st.shard, dtype=torch.float16, device=dev)
    ws = st.workspace(dev)
    outs = []
    for _ in range(steps):  # consecutive steps: inbox buffers, counters and epochs carry over
        st.enqueue(h, act, ws)
        outs.append(h.cpu().numpy())
    torch.cuda.synchronize()
    err = b2g.device_error()
    dist.barrier()
    st.close_comm()
    np.save(out + f".{rank}.npy", np.stack(outs))
    with open(out + f".{rank}.err", "w") as f:
        f.write(str(err))
    dist.barrier()
    dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("which,nl,steps,exchange", [("two", NL, 1, "reduce"), ("two", 2, 2, "reduce"),
                                                     ("two", 3, 2, "reduce"), ("two", 3, 2, "gather_kernel"),
                                                     ("all", NL, 1, "reduce"), ("all", 2, 2, "gather_kernel")])
def test_fused_ranks(b2g, orc, syn, cuda, tmp_path, which, nl, steps, exchange):
    """Every rank's rows bitwise equal and, on rank 0, the oracle's sharded
    stack, after each of `steps` consecutive steps (an odd layer count makes
    the second step start on the other inbox buffer)."""
    n = min(torch.cuda.device_count(), 8)
    if n < 2 or (which == "all" and n == 2):
        pytest.skip("needs two GPUs" if n < 2 else "all = two here")
    world = 2 if which == "two" else n
    import torch.multiprocessing as mp
    out = str(tmp_path / "h")
    mp.spawn(_rank, args=(world, _port(), out, nl, steps, exchange), nprocs=world, join=True)
    got = [np.load(out + f".{r}.npy") for r in range(world)]
    assert [open(out + f".{r}.err").read() for r in range(world)] == ["0"] * world
    for r in range(1, world):
        assert np.array_equal(got[r], got[0]), r  # the same sum, in the same order, on every rank
    layers = _weights(orc, syn, HID, INT, nl, 4000)
    want = syn.hidden_state(MM, HID)
    for step in range(steps):
        for L in layers:
            want = orc.mlp_layer_tp(want, L, world)
        r = orc.compare(got[0][step], want.astype(np.float64))
        assert r["rel_l2"] <= 5e-3 * (step + 1), (step, r)
        want = got[0][step]  # the next step starts from the rows the GPU produced
