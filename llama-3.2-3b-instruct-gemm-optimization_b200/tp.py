"""Tensor-parallel decode-MLP stack: one process (one GPU) per rank.

The layer shards the way the MLP's algebra allows (no reference counterpart:
the reference runs on one GPU):

* gate and up are split by output columns: rank r owns intermediate channels
  [r*I/tp, (r+1)*I/tp) of both and computes its slice of act = SiLU(g)*u with
  no communication (SiLU*up is elementwise per channel);
* down is split by K over the same channel range, so each rank multiplies its
  own act slice and produces a full-width [M, hidden] fp16 partial;
* one all-reduce (sum) of the partials per layer; rank 0's down adds the
  residual in its epilogue and the others write a bare partial, so the sum is
  h + down(act) with the residual counted once.

RMSNorm runs replicated (each rank normalises the same h).  The GEMVs run in
the C-ABI library (``GemvOp``).  The all-reduce is either
torch.distributed's (NCCL on GPUs), or -- ``fused=True`` -- fused into the
down launch through peer memory (``exchange``):

* "reduce" (default, b2g_enqueue_tp REDUCE): the down GEMV's epilogue stores
  its rows into every rank's inbox over NVLink, each CTA waits for the CTAs
  with its index on the other ranks (they own the same output tiles) and sums
  its tiles' slots in rank order into h; the next gate||up is a plain launch;
* "gather_kernel" (PUSH, then b2g_tp_gather): the down launch only pushes;
  before the next gate||up a small kernel waits for every rank's arrivals
  and sums the slots into h;
* "gather_launch" (PUSH, then GATHER): the gate||up launch sums the slots
  itself while it stages its activations.
"""
from __future__ import annotations

from . import (FUSE_GATE_UP_SILU, FUSE_NONE, FUSE_RESIDUAL_ADD, FUSE_RMSNORM_INPUT, TP_GATHER, TP_PUSH,
               TP_REDUCE, GemvOp, TpComm, ipc_close, ipc_handle, ipc_open, tp_comm_bytes, tp_comm_layout,
               tp_gather)

EXCHANGES = ("reduce", "gather_kernel", "gather_launch")


def shard_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of rank's equal share of n channels (n must divide evenly)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if n % world:
        raise ValueError(f"{n} channels do not split evenly over {world} ranks")
    step = n // world
    return rank * step, (rank + 1) * step


class TPStack:
    """n_layers x [RMSNorm -> gate||up + SiLU*up -> down + residual], sharded
    over the ranks of ``group`` (default: the world group)."""

    def __init__(self, hidden: int = 3072, intermediate: int = 8192, n_layers: int = 28,
                 rank: int = 0, world: int = 1, weight_dtype="fp8_e4m3", scale_mode="channel_fp32",
                 max_m: int = 8, rms_eps: float = 1e-5, group=None, build_ops: bool = True,
                 fused: bool = False):
        self.hidden, self.intermediate, self.n_layers = hidden, intermediate, n_layers
        self.rank, self.world, self.group = rank, world, group
        self.lo, self.hi = shard_range(intermediate, rank, world)
        self.shard = self.hi - self.lo
        self.max_m, self.rms_eps = max_m, rms_eps
        self.layers = [None] * n_layers
        self.gate_up = self.down = None
        self.fused = fused
        # Fused exchange (one of EXCHANGES).  Measured on one B200 with
        # world = 1 (28 layers, M = 8): gather_kernel 27.8 us per layer,
        # gather_launch 30.5 (the gate||up launch loses its lean code and
        # every CTA sums the rows).
        self.exchange = "reduce"
        # Exchange rounds pushed so far (one per layer, carried across calls):
        # round r uses inbox buffer r % 2, so consecutive pushes always
        # alternate, also from the last layer of one call to the first of the next.
        self._round = 0
        self.comm = None
        self._comm_buf = None
        self._peer_bases = []
        if build_ops:
            kw = dict(weight_dtype=weight_dtype, scale_mode=scale_mode, max_m=max_m,
                      tp_rank=rank, tp_size=world)
            self.gate_up = GemvOp(hidden, self.shard, fuse=FUSE_GATE_UP_SILU | FUSE_RMSNORM_INPUT, **kw)
            self.down = GemvOp(self.shard, hidden,
                               fuse=FUSE_RESIDUAL_ADD if rank == 0 else FUSE_NONE, **kw)

    # -- weights -------------------------------------------------------------
    def slice_layer(self, wg, wu, wd, sg=None, su=None, sd=None):
        """This rank's shard of full [K, N] layer weights and per-channel scales:
        gate/up columns and their scales, down rows (K); down's scales are per
        output channel and stay whole."""
        cs = slice(self.lo, self.hi)

        def cols(s):
            return None if s is None else s[cs]
        return wg[:, cs], wu[:, cs], wd[cs, :], cols(sg), cols(su), sd

    def set_layer(self, layer: int, packed_gu, scales_gu, packed_d, scales_d):
        self.layers[layer] = (packed_gu, scales_gu, packed_d, scales_d)

    def prepack_layer(self, layer: int, wg, wu, wd, sg=None, su=None, sd=None):
        """Slice full device weights for this rank, prepack and register them."""
        import torch
        g, u, d, sg_, su_, sd_ = self.slice_layer(wg, wu, wd, sg, su, sd)
        pgu = self.gate_up.prepack(g.contiguous(), u.contiguous())
        pd = self.down.prepack(d.contiguous())
        sgu = None if sg_ is None else torch.cat([sg_, su_]).contiguous()
        self.set_layer(layer, pgu, sgu, pd, sd_)

    def workspace(self, device="cuda"):
        import torch
        n = max(self.gate_up.workspace_bytes(), self.down.workspace_bytes())
        return torch.zeros(n, dtype=torch.uint8, device=device)

    # -- one layer -----------------------------------------------------------
    def gate_up_step(self, layer: int, h, act, workspace):
        """act[:, shard] = SiLU(RMSNorm(h) . Wg_shard) * (RMSNorm(h) . Wu_shard);
        L2 meanwhile fetches the start of this layer's down shard."""
        pgu, sgu, pd, _ = self.layers[layer]
        self.gate_up.enqueue(h, pgu, sgu, y=act, workspace=workspace, rms_eps=self.rms_eps, pdl=True,
                             prefetch=(self.down, pd))

    def down_step(self, layer: int, act, h, workspace):
        """h <- h + act . Wd_shard on rank 0, h <- act . Wd_shard elsewhere;
        L2 meanwhile fetches the start of the next layer's gate||up shard."""
        _, _, pd, sd = self.layers[layer]
        nxt = self.layers[(layer + 1) % self.n_layers]
        self.down.enqueue(act, pd, sd, y=h, residual=h if self.rank == 0 else None,
                          workspace=workspace, pdl=True,
                          prefetch=None if nxt is None else (self.gate_up, nxt[0]))

    def reduce_step(self, h):
        """Sum the ranks' [M, hidden] partials in place (h on every rank)."""
        if self.world > 1:
            import torch.distributed as dist
            dist.all_reduce(h, group=self.group)

    def layer_step(self, layer: int, h, act, workspace):
        if self.layers[layer] is None:
            raise RuntimeError(f"layer {layer} has no weights")
        self.gate_up_step(layer, h, act, workspace)
        self.down_step(layer, act, h, workspace)
        self.reduce_step(h)

    def enqueue(self, h, act, workspace):
        """All layers on h [M, hidden] fp16 in place; act is [M, I/tp] scratch."""
        if self.fused:
            return self._enqueue_fused(h, act, workspace)
        for layer in range(self.n_layers):
            self.layer_step(layer, h, act, workspace)
        return h

    # -- the all-reduce fused into the GEMVs -------------------------------------
    def setup_comm(self, device="cuda"):
        """Allocate this rank's zero-filled exchange buffer, share it with the
        other ranks (CUDA IPC) and map theirs.  Collective: every rank calls it."""
        import torch
        import torch.distributed as dist
        nbytes = tp_comm_bytes(self.world, self.max_m, self.hidden)
        self._comm_buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        torch.cuda.synchronize()
        handles = [ipc_handle(self._comm_buf)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, ipc_handle(self._comm_buf), group=self.group)
        comm = TpComm()
        comm.world, comm.rank, comm.max_m, comm.width = self.world, self.rank, self.max_m, self.hidden
        for r in range(self.world):
            if r == self.rank:
                base = self._comm_buf.data_ptr()
            else:
                base = ipc_open(handles[r])
                self._peer_bases.append(base)
            inbox, counters, epoch = tp_comm_layout(base, self.world, self.max_m, self.hidden)
            comm.inbox[r], comm.counters[r] = inbox, counters
            if r == self.rank:
                comm.epoch = epoch
        self.comm = comm
        if self.world > 1:
            dist.barrier(group=self.group)  # every buffer is zeroed and mapped before any push
        return comm

    def close_comm(self):
        """Unmap the peers' buffers (before the process group goes away)."""
        for base in self._peer_bases:
            ipc_close(base)
        self._peer_bases = []
        self.comm = None

    def _enqueue_fused(self, h, act, workspace):
        if self.comm is None:
            raise RuntimeError("fused TPStack needs setup_comm() first")
        n = self.n_layers
        import torch
        if n % 2 and torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            # A graph fixes each launch's buffer; with an odd layer count the
            # replays would not alternate (the last push of one replay and the
            # first of the next would share a buffer a peer may still read).
            raise ValueError(f"a CUDA graph of the fused exchange needs an even layer count, not {n}")
        if self.exchange not in EXCHANGES:
            raise ValueError(f"exchange {self.exchange!r} is not one of {EXCHANGES}")
        if self.exchange == "reduce":
            for layer in range(n):
                pgu, sgu, pd, sd = self.layers[layer]
                nxt = self.layers[(layer + 1) % n]
                self.gate_up.enqueue(h, pgu, sgu, y=act, workspace=workspace, rms_eps=self.rms_eps, pdl=True,
                                     prefetch=(self.down, pd))
                self.down.enqueue_tp(self.comm, TP_REDUCE, self._round % 2, act, pd, sd, y=h, workspace=workspace,
                                     residual=h if self.rank == 0 else None, pdl=True,
                                     prefetch=None if nxt is None else (self.gate_up, nxt[0]))
                self._round += 1
            return h
        for layer in range(n):
            pgu, sgu, pd, sd = self.layers[layer]
            if layer == 0:
                self.gate_up.enqueue(h, pgu, sgu, y=act, workspace=workspace, rms_eps=self.rms_eps, pdl=True,
                                     prefetch=(self.down, pd))
            elif self.exchange == "gather_kernel":
                # h = sum of the ranks' previous down outputs, then a plain gate||up
                tp_gather(self.comm, (self._round - 1) % 2, self.down, h)
                self.gate_up.enqueue(h, pgu, sgu, y=act, workspace=workspace, rms_eps=self.rms_eps, pdl=True,
                                     prefetch=(self.down, pd))
            else:
                # h = sum of the ranks' previous down outputs, summed here
                self.gate_up.enqueue_tp(self.comm, TP_GATHER, (self._round - 1) % 2, h, pgu, sgu, y=act,
                                        workspace=workspace, rms_eps=self.rms_eps, pdl=True,
                                        prefetch=(self.down, pd), push_op=self.down, h_out=h)
            nxt = self.layers[(layer + 1) % n]
            self.down.enqueue_tp(self.comm, TP_PUSH, self._round % 2, act, pd, sd, y=h, workspace=workspace,
                                 residual=h if self.rank == 0 else None, pdl=True,
                                 prefetch=None if nxt is None else (self.gate_up, nxt[0]))
            self._round += 1
        tp_gather(self.comm, (self._round - 1) % 2, self.down, h)
        return h
