"""Python binding of the b200gemv C ABI (include/b200gemv.h).

The library is the C ABI; this module only marshals arguments.  Device memory
comes from torch tensors (plumbing: allocation, streams); every computation
runs in ``libb200gemv.so``.  There is no fallback: if the library is missing,
``lib()`` raises.

The class names mirror the reference's operator surface:
``GemvOp(in_features, out_features, weight_dtype, scale_mode)`` is the planned
IPluginV3 creator (tensorrt_custom_tactic_kernel_b07f17a4.plan.md:57-58) and
``GemvOp.enqueue(x, W, scales) -> y`` replaces ``run_gemv``
(kernels/gemv_fp8.cu:276-283).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libb200gemv.so"

OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_PEER_TIMEOUT, ERR_OOM, ERR_DEVICE, ERR_SCRATCH_LIMIT = range(8)
STATIC_SCRATCH_BYTES = 2 * 1024 * 1024  # B2G_STATIC_SCRATCH_BYTES
DTYPE = {"fp16": 0, "fp8_e4m3": 1}
SCALE = {"none": 0, "tensor_fp16": 1, "channel_fp16": 2, "channel_fp32": 3}
LAYOUT = {"KN": 0, "NK": 1}
FUSE_NONE, FUSE_GATE_UP_SILU, FUSE_RMSNORM_INPUT, FUSE_RESIDUAL_ADD = 0, 1, 2, 4
OPT_MATH, OPT_GRID, OPT_PARTITION, OPT_KSPLIT, OPT_PIPE = 1, 2, 3, 4, 5
PIPE_AUTO, PIPE_REGISTERS, PIPE_TMA = 0, 1, 2
PARTITION_AUTO, PARTITION_UNITS, PARTITION_TILES = 0, 1, 2
MATH_MMA, MATH_FFMA = 0, 1
STACK_OPT_MODE = 1
STACK_MODE_PERSISTENT, STACK_MODE_PER_LAYER, STACK_MODE_PERSISTENT_TMA = 0, 1, 2


class B2GError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {lib().b2g_status_string(status).decode()} (status {status})")


class Fields(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "in_features", "out_features", "weight_dtype", "scale_mode", "weight_layout", "max_m",
        "fuse", "tp_rank", "tp_size")]


class EnqueueArgs(ctypes.Structure):
    _fields_ = [("m", ctypes.c_int32), ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
                ("packed_w", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64), ("y", ctypes.c_void_p),
                ("ldy", ctypes.c_int64), ("workspace", ctypes.c_void_p), ("rms_eps", ctypes.c_float),
                ("pdl", ctypes.c_int32), ("prefetch_packed", ctypes.c_void_p),
                ("prefetch_op", ctypes.c_void_p)]


class PlanInfo(ctypes.Structure):
    _fields_ = [("grid", ctypes.c_int32), ("ksplit", ctypes.c_int32),
                ("kblocks_per_vtile", ctypes.c_int32), ("n_tiles", ctypes.c_int32),
                ("total_units", ctypes.c_int64), ("unit_bytes", ctypes.c_int32),
                ("inflight_bytes_per_cta", ctypes.c_int64), ("smem_bytes", ctypes.c_int64), ("max_contrib", ctypes.c_int32),
                ("partition", ctypes.c_int32),
                ("n_slots", ctypes.c_int32), ("x_kblocks", ctypes.c_int32), ("math", ctypes.c_int32),
                ("pipe", ctypes.c_int32), ("n_stages", ctypes.c_int32), ("stage_bytes", ctypes.c_int32)]

    def as_dict(self):
        return {n: getattr(self, n) for n, _ in self._fields_}


class StackFields(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("n_layers", ctypes.c_int32), ("weight_dtype", ctypes.c_int32),
                ("scale_mode", ctypes.c_int32), ("max_m", ctypes.c_int32),
                ("rms_eps", ctypes.c_float), ("tp_rank", ctypes.c_int32), ("tp_size", ctypes.c_int32)]


TP_NONE, TP_PUSH, TP_GATHER, TP_REDUCE = 0, 1, 2, 3
TP_MAX_RANKS = 8
TP_MAX_CTAS = 256


class TpComm(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("max_m", ctypes.c_int32),
                ("width", ctypes.c_int32), ("inbox", ctypes.c_void_p * TP_MAX_RANKS),
                ("counters", ctypes.c_void_p * TP_MAX_RANKS), ("epoch", ctypes.c_void_p)]


# Every exported entry point and its ctypes signature (kept in step with
# include/b200gemv.h; the tests check the two agree).
_P, _I32, _I64, _SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = {
    "b2g_status_string": ([ctypes.c_int], ctypes.c_char_p),
    "b2g_version": ([], ctypes.c_int32),
    "b2g_create": ([ctypes.POINTER(Fields), ctypes.POINTER(_P)], ctypes.c_int),
    "b2g_destroy": ([_P], ctypes.c_int),
    "b2g_op_set_option": ([_P, _I32, _I32], ctypes.c_int),
    "b2g_op_query": ([_P, _I32, ctypes.POINTER(PlanInfo)], ctypes.c_int),
    "b2g_plan_for_device": ([ctypes.POINTER(Fields), _I32, _I32, _I32, ctypes.POINTER(PlanInfo),
                             ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)], ctypes.c_int),
    "b2g_prepack_size": ([_P, ctypes.POINTER(_SZ)], ctypes.c_int),
    "b2g_prepack": ([_P, _P, _P, _I64, _P, _P], ctypes.c_int),
    "b2g_quantize_e4m3": ([_P, _I32, _I32, _I32, _I32, _P, _P, _P], ctypes.c_int),
    "b2g_workspace_size": ([_P, _I32, ctypes.POINTER(_SZ)], ctypes.c_int),
    "b2g_workspace_init": ([_P, _P, _P], ctypes.c_int),
    "b2g_enqueue": ([_P, _I32, _P, _P, _P, _P, _P, _P], ctypes.c_int),
    "b2g_enqueue_ex": ([_P, ctypes.POINTER(EnqueueArgs), _P], ctypes.c_int),
    "b2g_device_error": ([ctypes.POINTER(_I32), _I32], ctypes.c_int),
    "b2g_enqueue_static": ([_P, ctypes.POINTER(EnqueueArgs), _P], ctypes.c_int),
    "b2g_tp_comm_bytes": ([_I32, _I32, _I32], _SZ),
    "b2g_tp_comm_layout": ([_P, _I32, _I32, _I32, ctypes.POINTER(_P), ctypes.POINTER(_P), ctypes.POINTER(_P)],
                           ctypes.c_int),
    "b2g_ipc_handle": ([_P, _P], ctypes.c_int),
    "b2g_ipc_open": ([_P, ctypes.POINTER(_P)], ctypes.c_int),
    "b2g_ipc_close": ([_P], ctypes.c_int),
    "b2g_enqueue_tp": ([_P, ctypes.POINTER(EnqueueArgs), ctypes.POINTER(TpComm), _I32, _I32, _P, _P, _I64, _P],
                       ctypes.c_int),
    "b2g_tp_gather": ([ctypes.POINTER(TpComm), _I32, _P, _I32, _P, _I64, _P], ctypes.c_int),
    "b2g_stack_create": ([ctypes.POINTER(StackFields), ctypes.POINTER(_P)], ctypes.c_int),
    "b2g_stack_destroy": ([_P], ctypes.c_int),
    "b2g_stack_ops": ([_P, ctypes.POINTER(_P), ctypes.POINTER(_P)], ctypes.c_int),
    "b2g_stack_set_option": ([_P, _I32, _I32], ctypes.c_int),
    "b2g_stack_set_layer": ([_P, _I32, _P, _P, _P, _P], ctypes.c_int),
    "b2g_stack_workspace_size": ([_P, _I32, ctypes.POINTER(_SZ)], ctypes.c_int),
    "b2g_stack_workspace_init": ([_P, _P, _P], ctypes.c_int),
    "b2g_stack_enqueue": ([_P, _I32, _P, _P, _P, _P], ctypes.c_int),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The C-ABI library.  Raises if it has not been built -- no fallback."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with build.py (nvcc, sm_100a)")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: int, what: str):
    if status != OK:
        raise B2GError(status, what)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return ctypes.c_void_p(s.cuda_stream)


def _rows_stride(t):
    """Row stride in elements (a size-1 leading axis may carry any stride)."""
    return t.stride(0) if t.shape[0] > 1 else t.shape[1]


def _code(table, v):
    return table[v] if isinstance(v, str) else int(v)


class GemvOp:
    """One GEMV operator: y[m, N] = epilogue(x[m, K] . W[K, N] * s)."""

    def __init__(self, in_features: int, out_features: int, weight_dtype="fp8_e4m3",
                 scale_mode="channel_fp32", layout="KN", max_m: int = 8, fuse: int = FUSE_NONE,
                 tp_rank: int = 0, tp_size: int = 1, _handle=None):
        self.K, self.N = in_features, out_features
        self.weight_dtype = _code(DTYPE, weight_dtype)
        self.scale_mode = _code(SCALE, scale_mode)
        self.layout = _code(LAYOUT, layout)
        self.max_m, self.fuse = max_m, fuse
        self.planes = 2 if fuse & FUSE_GATE_UP_SILU else 1
        self._owned = _handle is None
        if _handle is None:
            f = Fields(in_features, out_features, self.weight_dtype, self.scale_mode, self.layout,
                       max_m, fuse, tp_rank, tp_size)
            h = ctypes.c_void_p()
            check(lib().b2g_create(ctypes.byref(f), ctypes.byref(h)), "b2g_create")
            self.h = h
        else:
            self.h = _handle

    def __del__(self):
        if getattr(self, "_owned", False) and getattr(self, "h", None) and _lib is not None:
            _lib.b2g_destroy(self.h)
            self.h = None

    # -- planning -------------------------------------------------------
    def set_option(self, key: int, value: int):
        check(lib().b2g_op_set_option(self.h, key, value), "b2g_op_set_option")

    def plan(self, m: int) -> dict:
        info = PlanInfo()
        check(lib().b2g_op_query(self.h, m, ctypes.byref(info)), "b2g_op_query")
        return info.as_dict()

    # -- weights -------------------------------------------------------
    def packed_bytes(self) -> int:
        n = ctypes.c_size_t()
        check(lib().b2g_prepack_size(self.h, ctypes.byref(n)), "b2g_prepack_size")
        return n.value

    def prepack(self, w0, w1=None, out=None, ld: int = 0, stream=None):
        """Repack device weights (op dtype/layout; E4M3 given as uint8) into the stream layout."""
        import torch
        if out is None:
            out = torch.empty(self.packed_bytes(), dtype=torch.uint8, device=w0.device)
        check(lib().b2g_prepack(self.h, _ptr(w0), _ptr(w1), ld, _ptr(out), _stream(stream)),
              "b2g_prepack")
        return out

    # -- workspace ------------------------------------------------------
    def workspace_bytes(self, m=None) -> int:
        n = ctypes.c_size_t()
        check(lib().b2g_workspace_size(self.h, m or self.max_m, ctypes.byref(n)), "b2g_workspace_size")
        return n.value

    def workspace(self, device="cuda", stream=None):
        import torch
        ws = torch.empty(self.workspace_bytes(), dtype=torch.uint8, device=device)
        check(lib().b2g_workspace_init(self.h, _ptr(ws), _stream(stream)), "b2g_workspace_init")
        return ws

    # -- enqueue --------------------------------------------------------
    def enqueue(self, x, packed, scales=None, y=None, workspace=None, residual=None,
                rms_eps: float = 1e-5, pdl: bool = False, stream=None, prefetch=None):
        """y = op(x, W, scales).  prefetch=(next_op, next_packed) warms L2 with the
        start of the weights the next launch in the stream will read."""
        import torch
        m = x.shape[0]
        if y is None:
            y = torch.empty((m, self.N), dtype=torch.float16, device=x.device)
        if workspace is None:
            workspace = self.workspace(x.device, stream)
        if x.stride(-1) != 1 or y.stride(-1) != 1 or (residual is not None and residual.stride(-1) != 1):
            raise ValueError("x, y and residual rows must be contiguous")
        a = EnqueueArgs(m, x.data_ptr(), _rows_stride(x), packed.data_ptr(),
                        0 if scales is None else scales.data_ptr(),
                        0 if residual is None else residual.data_ptr(),
                        0 if residual is None else _rows_stride(residual), y.data_ptr(),
                        _rows_stride(y), workspace.data_ptr(), rms_eps, 1 if pdl else 0,
                        None if prefetch is None else prefetch[1].data_ptr(),
                        None if prefetch is None else prefetch[0].h)
        check(lib().b2g_enqueue_ex(self.h, ctypes.byref(a), _stream(stream)), "b2g_enqueue_ex")
        return y

    def enqueue_tp(self, comm, mode, buf, x, packed, scales=None, y=None, workspace=None, residual=None,
                   rms_eps: float = 1e-5, pdl: bool = False, stream=None, prefetch=None, push_op=None,
                   h_out=None):
        """b2g_enqueue_tp: REDUCE (this op's rows to every rank's inbox, then
        y = the all-reduced rows on every rank), PUSH (the rows to every
        rank's inbox only) or GATHER (stage the all-reduced rows from the
        local inbox, writing them to h_out)."""
        m = x.shape[0]
        a = EnqueueArgs(m, x.data_ptr(), _rows_stride(x), packed.data_ptr(),
                        0 if scales is None else scales.data_ptr(),
                        0 if residual is None else residual.data_ptr(),
                        0 if residual is None else _rows_stride(residual),
                        (x if y is None else y).data_ptr(), self.N if y is None else _rows_stride(y),
                        workspace.data_ptr(), rms_eps, 1 if pdl else 0,
                        None if prefetch is None else prefetch[1].data_ptr(),
                        None if prefetch is None else prefetch[0].h)
        check(lib().b2g_enqueue_tp(self.h, ctypes.byref(a), ctypes.byref(comm), mode, buf,
                                   None if push_op is None else push_op.h,
                                   None if h_out is None else h_out.data_ptr(),
                                   0 if h_out is None else _rows_stride(h_out), _stream(stream)),
              "b2g_enqueue_tp")

    def enqueue_static(self, x, packed, y, scales=None, residual=None, rms_eps: float = 1e-5,
                       stream=None):
        """y = op(x, W, scales) on the library's static scratch (b2g_enqueue_static).

        The library call allocates nothing, so y must be given.  Calls that
        overlap on the device (other streams or threads) race on the scratch.
        """
        if x.stride(-1) != 1 or y.stride(-1) != 1 or (residual is not None and residual.stride(-1) != 1):
            raise ValueError("x, y and residual rows must be contiguous")
        a = EnqueueArgs(x.shape[0], x.data_ptr(), _rows_stride(x), packed.data_ptr(),
                        0 if scales is None else scales.data_ptr(),
                        0 if residual is None else residual.data_ptr(),
                        0 if residual is None else _rows_stride(residual), y.data_ptr(),
                        _rows_stride(y), None, rms_eps, 0, None, None)
        check(lib().b2g_enqueue_static(self.h, ctypes.byref(a), _stream(stream)), "b2g_enqueue_static")
        return y


B200_SMS, B200_SMEM_OPTIN = 148, 232448


def plan_for_device(in_features: int, out_features: int, weight_dtype="fp8_e4m3", scale_mode="channel_fp32",
                    layout="KN", max_m: int = 8, fuse: int = FUSE_NONE, m=None, num_sms: int = B200_SMS,
                    smem_optin: int = B200_SMEM_OPTIN) -> dict:
    """The plan GemvOp would make on a GPU with num_sms SMs (b2g_plan_for_device;
    no device needed), with its packed-weight and workspace bytes."""
    f = Fields(in_features, out_features, _code(DTYPE, weight_dtype), _code(SCALE, scale_mode),
               _code(LAYOUT, layout), max_m, fuse, 0, 1)
    info, pb, wb = PlanInfo(), ctypes.c_size_t(), ctypes.c_size_t()
    check(lib().b2g_plan_for_device(ctypes.byref(f), num_sms, smem_optin, m or max_m, ctypes.byref(info),
                                    ctypes.byref(pb), ctypes.byref(wb)), "b2g_plan_for_device")
    d = info.as_dict()
    d.update(packed_bytes=pb.value, workspace_bytes=wb.value)
    return d


def quantize_e4m3(w16, scale_mode="channel_fp32", layout="KN", stream=None):
    """Device E4M3 quantisation: returns (codes uint8 like w16, scales or None)."""
    import torch
    sm = _code(SCALE, scale_mode)
    lay = _code(LAYOUT, layout)
    K, N = (w16.shape if lay == 0 else w16.shape[::-1])
    q = torch.empty(w16.shape, dtype=torch.uint8, device=w16.device)
    if sm == 0:
        s = None
    elif sm == 1:
        s = torch.empty(1, dtype=torch.float16, device=w16.device)
    elif sm == 2:
        s = torch.empty(N, dtype=torch.float16, device=w16.device)
    else:
        s = torch.empty(N, dtype=torch.float32, device=w16.device)
    check(lib().b2g_quantize_e4m3(_ptr(w16), K, N, lay, sm, _ptr(q), _ptr(s), _stream(stream)),
          "b2g_quantize_e4m3")
    return q, s


def device_error(clear: bool = True) -> int:
    v = ctypes.c_int32()
    check(lib().b2g_device_error(ctypes.byref(v), 1 if clear else 0), "b2g_device_error")
    return v.value


class Stack:
    """The decode-MLP layer stack (RMSNorm -> gate||up+SiLU*up -> down + residual)."""

    def __init__(self, hidden=3072, intermediate=8192, n_layers=28, weight_dtype="fp8_e4m3",
                 scale_mode="channel_fp32", max_m=8, rms_eps=1e-5, tp_rank=0, tp_size=1):
        f = StackFields(hidden, intermediate, n_layers, _code(DTYPE, weight_dtype),
                        _code(SCALE, scale_mode), max_m, rms_eps, tp_rank, tp_size)
        h = ctypes.c_void_p()
        check(lib().b2g_stack_create(ctypes.byref(f), ctypes.byref(h)), "b2g_stack_create")
        self.h = h
        self.hidden, self.intermediate, self.n_layers, self.max_m = hidden, intermediate, n_layers, max_m
        g, d = ctypes.c_void_p(), ctypes.c_void_p()
        check(lib().b2g_stack_ops(self.h, ctypes.byref(g), ctypes.byref(d)), "b2g_stack_ops")
        kw = dict(weight_dtype=weight_dtype, scale_mode=scale_mode, max_m=max_m)
        self.gate_up = GemvOp(hidden, intermediate, fuse=FUSE_GATE_UP_SILU | FUSE_RMSNORM_INPUT,
                              _handle=g, **kw)
        self.down = GemvOp(intermediate, hidden, fuse=FUSE_RESIDUAL_ADD, _handle=d, **kw)
        self._keep = {}

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.b2g_stack_destroy(self.h)
            self.h = None

    def set_mode(self, mode):
        """"per_layer" (two chained launches per layer), "persistent" (one
        cooperative launch) or "persistent_tma" (one cooperative launch, weights
        through the TMA pipeline)."""
        check(lib().b2g_stack_set_option(self.h, STACK_OPT_MODE, _code(
            {"persistent": STACK_MODE_PERSISTENT, "per_layer": STACK_MODE_PER_LAYER,
             "persistent_tma": STACK_MODE_PERSISTENT_TMA}, mode)),
            "b2g_stack_set_option")

    def set_layer(self, layer, packed_gu, scales_gu, packed_d, scales_d):
        self._keep[layer] = (packed_gu, scales_gu, packed_d, scales_d)
        check(lib().b2g_stack_set_layer(self.h, layer, _ptr(packed_gu), _ptr(scales_gu),
                                        _ptr(packed_d), _ptr(scales_d)), "b2g_stack_set_layer")

    def workspace(self, device="cuda", stream=None):
        import torch
        n = ctypes.c_size_t()
        check(lib().b2g_stack_workspace_size(self.h, self.max_m, ctypes.byref(n)),
              "b2g_stack_workspace_size")
        ws = torch.empty(n.value, dtype=torch.uint8, device=device)
        check(lib().b2g_stack_workspace_init(self.h, _ptr(ws), _stream(stream)),
              "b2g_stack_workspace_init")
        return ws

    def enqueue(self, h, act, workspace, stream=None):
        check(lib().b2g_stack_enqueue(self.h, h.shape[0], _ptr(h), _ptr(act), _ptr(workspace),
                                      _stream(stream)), "b2g_stack_enqueue")
        return h


def tp_comm_bytes(world: int, max_m: int, width: int) -> int:
    return lib().b2g_tp_comm_bytes(world, max_m, width)


def tp_comm_layout(base: int, world: int, max_m: int, width: int):
    """(inbox, counters, epoch) device addresses inside a comm buffer at base."""
    i, c, e = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    check(lib().b2g_tp_comm_layout(ctypes.c_void_p(base), world, max_m, width, ctypes.byref(i),
                                   ctypes.byref(c), ctypes.byref(e)), "b2g_tp_comm_layout")
    return i.value, c.value, e.value


IPC_RECORD_BYTES = 72


def ipc_handle(t) -> bytes:
    buf = ctypes.create_string_buffer(IPC_RECORD_BYTES)
    check(lib().b2g_ipc_handle(ctypes.c_void_p(t.data_ptr()), buf), "b2g_ipc_handle")
    return buf.raw


def ipc_open(record: bytes) -> int:
    p = ctypes.c_void_p()
    check(lib().b2g_ipc_open(ctypes.create_string_buffer(record, IPC_RECORD_BYTES), ctypes.byref(p)),
          "b2g_ipc_open")
    return p.value


def ipc_close(addr: int):
    check(lib().b2g_ipc_close(ctypes.c_void_p(addr)), "b2g_ipc_close")


def tp_gather(comm, buf: int, push_op, h, stream=None):
    check(lib().b2g_tp_gather(ctypes.byref(comm), buf, push_op.h, h.shape[0], ctypes.c_void_p(h.data_ptr()),
                              _rows_stride(h), _stream(stream)), "b2g_tp_gather")
    return h
