"""Weight files for the decode-MLP stack: one file per model, read per rank.

The reference keeps each MLP projection as a raw blob
``L{ll}.{proj}.K{K}.N{N}.fp16.bin`` (fp16, [K, N] row-major, written by
kernels/opt_loop/fp8_accuracy/extract_real_weights.py:65-73, with a
manifest.json beside them; read back by kernels/gemv_fp8.cu:448-457, which
takes K and N from the name).  This module gathers such blobs into one
indexed file, and also stores what the GEMV kernels consume directly: the
prepacked weight stream of one rank for one op plan, so a later load is a
plain host-to-device copy.

Record kinds:

* ``KIND_FP16_KN``  fp16 weights [K, N] (the reference's blob, byte for byte);
* ``KIND_E4M3_KN``  E4M3 codes [K, N] + scales (quantised, not packed);
* ``KIND_PACKED``   the packed stream of one op (``GemvOp.prepack``) + the
  scales as the op takes them; valid only for the same packed layout
  (K, N, bytes per weight, planes, K split), which the record carries.

Binary layout (little-endian):

* bytes [0, 64): header -- magic ``b"B2GWEIGH"``, u32 version (1), u32
  record count, u64 index offset, u64 index bytes, u64 file bytes, 24 zero
  bytes;
* data and scale blobs, each starting at a multiple of 4096 bytes;
* the index: one 192-byte record per blob pair -- char name[48]; i32 layer,
  proj, kind, weight_dtype, scale_mode, K, N, planes, ksplit, tp_rank,
  tp_size, scales_dtype; u64 data_offset, data_bytes, scales_offset,
  scales_bytes; u32 data_crc32, scales_crc32; 56 zero bytes.

proj: 0 gate_proj, 1 up_proj, 2 down_proj, 3 gate_up (the fused pair, packed
records only).  scales_dtype: 0 none, 1 fp16, 2 fp32.  Loading never does
arithmetic on the host: quantisation and packing run on the GPU through the
library (``quantize_e4m3``, ``GemvOp.prepack``).
"""
from __future__ import annotations

import json
import re
import struct
import zlib
from dataclasses import dataclass
from pathlib import Path

import numpy as np

MAGIC = b"B2GWEIGH"
VERSION = 1
ALIGN = 4096
_HEADER = struct.Struct("<8sIIQQQ24x")
_RECORD = struct.Struct("<48s12i4Q2I56x")
assert _HEADER.size == 64 and _RECORD.size == 192

KIND_FP16_KN, KIND_E4M3_KN, KIND_PACKED = 0, 1, 2
PROJS = ("gate_proj", "up_proj", "down_proj", "gate_up")
SCALES_NONE, SCALES_FP16, SCALES_FP32 = 0, 1, 2
_SCALE_NP = {SCALES_FP16: np.float16, SCALES_FP32: np.float32}

# kernels/gemv_fp8.cu:448-457 takes K and N from ".K<k>" and ".N<n>" in this name.
REFERENCE_BLOB = re.compile(r"^L(\d+)\.(gate_proj|up_proj|down_proj)\.K(\d+)\.N(\d+)\.fp16\.bin$")


class WeightFileError(ValueError):
    """A file that is not a weight file, is damaged, or does not fit the op."""


@dataclass
class Record:
    layer: int
    proj: str
    kind: int
    weight_dtype: int  # 0 fp16, 1 E4M3 (the library's B2G_DTYPE_* codes)
    scale_mode: int    # the library's B2G_SCALE_* codes
    K: int
    N: int
    planes: int = 1
    ksplit: int = 0    # packed records: the op's K split; 0 otherwise
    tp_rank: int = 0
    tp_size: int = 1
    scales_dtype: int = SCALES_NONE
    data_offset: int = 0
    data_bytes: int = 0
    scales_offset: int = 0
    scales_bytes: int = 0
    data_crc32: int = 0
    scales_crc32: int = 0

    @property
    def name(self) -> str:
        s = f"L{self.layer:02d}.{self.proj}"
        return s if self.tp_size == 1 else f"{s}.tp{self.tp_rank}of{self.tp_size}"

    def pack(self) -> bytes:
        name = self.name.encode()
        if len(name) > 48:
            raise WeightFileError(f"record name {self.name!r} longer than 48 bytes")
        return _RECORD.pack(name, self.layer, PROJS.index(self.proj), self.kind, self.weight_dtype,
                            self.scale_mode, self.K, self.N, self.planes, self.ksplit, self.tp_rank,
                            self.tp_size, self.scales_dtype, self.data_offset, self.data_bytes,
                            self.scales_offset, self.scales_bytes, self.data_crc32, self.scales_crc32)

    @classmethod
    def unpack(cls, raw: bytes) -> "Record":
        (name, layer, proj, kind, wd, sm, K, N, planes, ksplit, tr, ts, sd, do, db, so, sb, dc,
         sc) = _RECORD.unpack(raw)
        name = name.rstrip(b"\0").decode(errors="replace")
        if not 0 <= proj < len(PROJS) or kind not in (KIND_FP16_KN, KIND_E4M3_KN, KIND_PACKED):
            raise WeightFileError(f"record {name!r}: unknown projection or kind")
        r = cls(layer, PROJS[proj], kind, wd, sm, K, N, planes, ksplit, tr, ts, sd, do, db, so, sb, dc, sc)
        if r.name != name:
            raise WeightFileError(f"record {name!r} does not match its fields ({r.name})")
        return r


def _bytes_view(a) -> memoryview:
    """A flat byte view of a host array or CPU tensor (no copy when contiguous)."""
    if hasattr(a, "numpy") and not isinstance(a, np.ndarray):  # torch tensor
        a = a.detach().cpu().contiguous().numpy()
    return memoryview(np.ascontiguousarray(a)).cast("B")


def write(path, items) -> list[Record]:
    """Write a weight file.  items: iterable of (Record, data, scales or None);
    data/scales are host arrays or CPU tensors.  Offsets, sizes and CRCs are
    filled in; returns the records as written."""
    path = Path(path)
    recs = []
    with open(path, "wb") as f:
        f.write(b"\0" * _HEADER.size)

        def put(buf: memoryview) -> tuple[int, int, int]:
            pos = f.tell()
            pad = (-pos) % ALIGN
            f.write(b"\0" * pad)
            off = pos + pad
            f.write(buf)
            return off, buf.nbytes, zlib.crc32(buf) & 0xFFFFFFFF

        for rec, data, scales in items:
            rec.data_offset, rec.data_bytes, rec.data_crc32 = put(_bytes_view(data))
            if scales is None:
                rec.scales_dtype, rec.scales_offset, rec.scales_bytes, rec.scales_crc32 = SCALES_NONE, 0, 0, 0
            else:
                s = scales.detach().cpu().numpy() if hasattr(scales, "detach") else np.asarray(scales)
                rec.scales_dtype = SCALES_FP32 if s.dtype == np.float32 else SCALES_FP16
                if s.dtype not in (np.float32, np.float16):
                    raise WeightFileError(f"{rec.name}: scales must be fp16 or fp32, not {s.dtype}")
                rec.scales_offset, rec.scales_bytes, rec.scales_crc32 = put(_bytes_view(s))
            recs.append(rec)
        index = b"".join(r.pack() for r in recs)
        index_off = f.tell() + (-f.tell()) % 8
        f.write(b"\0" * (index_off - f.tell()))
        f.write(index)
        total = f.tell()
        f.seek(0)
        f.write(_HEADER.pack(MAGIC, VERSION, len(recs), index_off, len(index), total))
    return recs


class WeightFile:
    """Index of a weight file; blobs are read on demand (by offset, so a rank
    reads only its own records)."""

    def __init__(self, path):
        self.path = Path(path)
        size = self.path.stat().st_size
        with open(self.path, "rb") as f:
            head = f.read(_HEADER.size)
            if len(head) < _HEADER.size:
                raise WeightFileError(f"{self.path}: shorter than a header")
            magic, version, n, index_off, index_bytes, total = _HEADER.unpack(head)
            if magic != MAGIC:
                raise WeightFileError(f"{self.path}: not a weight file (magic {magic!r})")
            if version != VERSION:
                raise WeightFileError(f"{self.path}: version {version}, this reader reads {VERSION}")
            if total != size or index_bytes != n * _RECORD.size or index_off + index_bytes > size:
                raise WeightFileError(f"{self.path}: truncated or inconsistent "
                                      f"(header says {total} B, index {index_off}+{index_bytes}; file {size} B)")
            f.seek(index_off)
            raw = f.read(index_bytes)
        self.records = [Record.unpack(raw[i:i + _RECORD.size]) for i in range(0, index_bytes, _RECORD.size)]
        for r in self.records:
            for off, nb in ((r.data_offset, r.data_bytes), (r.scales_offset, r.scales_bytes)):
                if nb and (off % ALIGN or off + nb > index_off):
                    raise WeightFileError(f"{self.path}: {r.name} blob [{off}, {off + nb}) outside the data area")

    def find(self, layer: int, proj: str, kind=None, tp_rank: int = 0, tp_size: int = 1) -> Record:
        for r in self.records:
            if (r.layer == layer and r.proj == proj and r.tp_rank == tp_rank and r.tp_size == tp_size
                    and (kind is None or r.kind == kind)):
                return r
        raise KeyError(f"no record L{layer:02d}.{proj} (kind {kind}, tp {tp_rank}/{tp_size}) in {self.path}")

    def layers(self) -> list[int]:
        return sorted({r.layer for r in self.records})

    def _blob(self, f, off: int, nbytes: int, crc: int, what: str, verify: bool) -> np.ndarray:
        f.seek(off)
        a = np.fromfile(f, dtype=np.uint8, count=nbytes)
        if a.size != nbytes:
            raise WeightFileError(f"{self.path}: short read of {what}")
        if verify and (zlib.crc32(memoryview(a)) & 0xFFFFFFFF) != crc:
            raise WeightFileError(f"{self.path}: {what} fails its CRC-32")
        return a

    def read(self, rec: Record, verify: bool = True):
        """(data, scales or None) as host arrays: fp16 [K, N] for FP16_KN,
        uint8 [K, N] for E4M3_KN, flat uint8 for PACKED."""
        with open(self.path, "rb") as f:
            d = self._blob(f, rec.data_offset, rec.data_bytes, rec.data_crc32, rec.name, verify)
            s = None
            if rec.scales_dtype != SCALES_NONE:
                s = self._blob(f, rec.scales_offset, rec.scales_bytes, rec.scales_crc32,
                               rec.name + " scales", verify).view(_SCALE_NP[rec.scales_dtype])
        if rec.kind == KIND_FP16_KN:
            if rec.data_bytes != rec.K * rec.N * 2:
                raise WeightFileError(f"{rec.name}: {rec.data_bytes} B is not K*N*2 for K={rec.K}, N={rec.N}")
            d = d.view(np.float16).reshape(rec.K, rec.N)
        elif rec.kind == KIND_E4M3_KN:
            if rec.data_bytes != rec.K * rec.N:
                raise WeightFileError(f"{rec.name}: {rec.data_bytes} B is not K*N for K={rec.K}, N={rec.N}")
            d = d.reshape(rec.K, rec.N)
        return d, s


# ---------------------------------------------------------------------------
# The reference's raw blobs
# ---------------------------------------------------------------------------
def parse_reference_blob_name(name: str):
    """(layer, proj, K, N) from a name like L00.up_proj.K3072.N8192.fp16.bin."""
    m = REFERENCE_BLOB.match(Path(name).name)
    if not m:
        raise WeightFileError(f"{name!r} is not a reference weight blob name (L<l>.<proj>.K<k>.N<n>.fp16.bin)")
    return int(m.group(1)), m.group(2), int(m.group(3)), int(m.group(4))


def reference_blobs(src) -> list[tuple[int, str, int, int, Path]]:
    """The blobs of a reference weight directory, sorted by (layer, proj):
    from its manifest.json when present (records layer, proj, K, N, bytes,
    path; a path that does not exist here is looked up by its file name in
    the directory), else every file whose name matches."""
    src = Path(src)
    out = []
    man = src / "manifest.json"
    if man.exists():
        for r in json.loads(man.read_text()):
            p = Path(r["path"])
            if not p.exists():
                p = src / p.name
            layer, proj, K, N = parse_reference_blob_name(p.name)
            if (layer, proj, K, N) != (r["layer"], r["proj"], r["K"], r["N"]):
                raise WeightFileError(f"manifest entry {r} disagrees with its file name {p.name}")
            if int(r["bytes"]) != K * N * 2:
                raise WeightFileError(f"manifest entry {p.name}: {r['bytes']} B is not K*N*2")
            out.append((layer, proj, K, N, p))
    else:
        for p in src.iterdir():
            if REFERENCE_BLOB.match(p.name):
                out.append((*parse_reference_blob_name(p.name), p))
    for layer, proj, K, N, p in out:
        if not p.exists():
            raise WeightFileError(f"{p} listed but missing")
        if p.stat().st_size != K * N * 2:
            raise WeightFileError(f"{p}: {p.stat().st_size} B, expected K*N*2 = {K * N * 2}")
    return sorted(out, key=lambda t: (t[0], PROJS.index(t[1])))


def import_reference_blobs(src, out_path, layers=None) -> list[Record]:
    """Gather a reference weight directory into one file of FP16_KN records
    (the blob bytes unchanged).  layers: the layers to take (default all)."""
    blobs = [b for b in reference_blobs(src) if layers is None or b[0] in set(layers)]
    if not blobs:
        raise WeightFileError(f"no reference weight blobs in {src}")

    def items():
        for layer, proj, K, N, p in blobs:
            data = np.fromfile(p, dtype=np.float16)
            yield Record(layer, proj, KIND_FP16_KN, 0, 0, K, N), data, None
    return write(out_path, items())


# ---------------------------------------------------------------------------
# Stacks: load and export
# ---------------------------------------------------------------------------
def _stack_shape(st):
    tp = hasattr(st, "prepack_layer")  # TPStack: rank's shard; Stack: whole layer
    return (st.rank, st.world) if tp else (0, 1)


def _layer_tensors(st, layer):
    held = st.layers[layer] if hasattr(st, "prepack_layer") else st._keep.get(layer)
    if held is None:
        raise KeyError(f"layer {layer} has no weights")
    return held


def load_layers(wf: WeightFile, st, device, layers=None, quantize=None, verify: bool = True):
    """Fill the layers of a Stack (one GPU) or of this rank's TPStack from wf.

    For each layer, PACKED records of this rank's shard are copied straight
    to the device when their packed layout is the op's; otherwise the
    layer's full-matrix records (FP16_KN, quantised on the device with the
    op's scale rule, or E4M3_KN) are uploaded and packed there -- a TPStack
    quantises the whole matrices first and slices them after, so its shards
    carry the unsharded per-channel scales.  quantize(w16_device, scale_mode)
    -> (codes, scales) defaults to the library's device quantiser."""
    import torch

    from . import quantize_e4m3
    quantize = quantize or quantize_e4m3
    rank, world = _stack_shape(st)
    gu_op, dn_op = st.gate_up, st.down
    e4m3 = gu_op.weight_dtype == 1
    for layer in (wf.layers() if layers is None else layers):
        try:
            pg = wf.find(layer, "gate_up", KIND_PACKED, rank, world)
            pd = wf.find(layer, "down_proj", KIND_PACKED, rank, world)
        except KeyError:
            pg = pd = None
        packed_ok = pg is not None and check_packed_layout(pg, gu_op) and check_packed_layout(pd, dn_op)
        if pg is not None and not packed_ok and not any(
                r.layer == layer and r.kind != KIND_PACKED for r in wf.records):
            raise WeightFileError(f"layer {layer}: the packed records are laid out for another op plan "
                                  f"({pg.K}x{pg.N}, K split {pg.ksplit}) and the file has no source weights")
        if packed_ok:
            tens = []
            for rec in (pg, pd):
                d, s = wf.read(rec, verify)
                tens += [torch.from_numpy(d).to(device), None if s is None else torch.from_numpy(s).to(device)]
            st.set_layer(layer, *tens)
            continue
        full = {}
        hidden, inter = gu_op.K, gu_op.N * world  # whole matrices (a TP op holds one shard of I)
        for proj in ("gate_proj", "up_proj", "down_proj"):
            src = [r for r in wf.records if r.layer == layer and r.proj == proj and r.tp_size == 1
                   and r.kind in (KIND_FP16_KN, KIND_E4M3_KN)]
            if not src:
                raise WeightFileError(f"layer {layer}: no packed records for rank {rank} of {world} that fit "
                                      f"this op, and no source weights for {proj}")
            rec = min(src, key=lambda r: r.kind)  # fp16 source first, else E4M3 codes
            want_kn = (inter, hidden) if proj == "down_proj" else (hidden, inter)
            if (rec.K, rec.N) != want_kn:
                raise WeightFileError(f"{rec.name}: {rec.K}x{rec.N} weights, the stack needs "
                                      f"{want_kn[0]}x{want_kn[1]}")
            d, s = wf.read(rec, verify)
            if rec.kind == KIND_E4M3_KN:
                _check_code_scales(rec, s, gu_op.scale_mode)
            w = torch.from_numpy(d).to(device)
            if rec.kind == KIND_FP16_KN and e4m3:
                full[proj] = quantize(w, gu_op.scale_mode)
            elif rec.kind == KIND_E4M3_KN and not e4m3:
                raise WeightFileError(f"{rec.name}: E4M3 codes cannot fill an FP16 stack")
            else:
                full[proj] = (w, None if s is None else torch.from_numpy(s).to(device))
        (qg, sg), (qu, su), (qd, sd) = full["gate_proj"], full["up_proj"], full["down_proj"]
        if hasattr(st, "prepack_layer"):
            st.prepack_layer(layer, qg, qu, qd, sg, su, sd)
        else:
            sgu = None if sg is None else torch.cat([sg, su]).contiguous()
            st.set_layer(layer, gu_op.prepack(qg, qu), sgu, dn_op.prepack(qd), sd)


def _check_code_scales(rec: Record, s, scale_mode: int) -> None:
    """E4M3 codes are used as they are, so their scale rule must be the op's
    and their scales exactly what the kernel reads for it: none, one fp16
    (tensor), N fp16 or N fp32 (per channel)."""
    if rec.scale_mode != scale_mode:
        raise WeightFileError(f"{rec.name}: codes quantised with scale mode {rec.scale_mode}, "
                              f"the op uses {scale_mode}")
    want = {0: (0, None), 1: (1, np.float16), 2: (rec.N, np.float16), 3: (rec.N, np.float32)}[scale_mode]
    have = (0, None) if s is None else (s.size, s.dtype.type)
    if have != want:
        raise WeightFileError(f"{rec.name}: {have[0]} scales of {have[1]}, scale mode {scale_mode} "
                              f"needs {want[0]} of {want[1]}")


def packed_layout(op) -> tuple:
    """(K, N, bytes per weight, planes, K split) of op's packed stream."""
    return (op.K, op.N, 1 if op.weight_dtype == 1 else 2, op.planes, op.plan(op.max_m)["ksplit"])


def check_packed_layout(rec: Record, op) -> bool:
    """Whether a PACKED record's stream is laid out for op (and of its size)."""
    want = packed_layout(op)
    have = (rec.K, rec.N, 1 if rec.weight_dtype == 1 else 2, rec.planes, rec.ksplit)
    return have == want and rec.data_bytes == op.packed_bytes() and rec.scale_mode == op.scale_mode


def export_packed(path, st, layers=None) -> list[Record]:
    """Write this rank's packed layers of a Stack or TPStack (their device
    streams, copied to the host) as PACKED records, for direct reloads."""
    rank, world = _stack_shape(st)
    todo = list(range(st.n_layers)) if layers is None else list(layers)

    def items():
        for layer in todo:
            pgu, sgu, pd, sd = _layer_tensors(st, layer)
            for proj, op, d, s in (("gate_up", st.gate_up, pgu, sgu), ("down_proj", st.down, pd, sd)):
                K, N, wb, planes, ks = packed_layout(op)
                rec = Record(layer, proj, KIND_PACKED, op.weight_dtype, op.scale_mode, K, N, planes, ks,
                             rank, world)
                yield rec, d.cpu(), None if s is None else s.cpu()
    return write(path, items())
