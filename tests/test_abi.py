"""The C-ABI library loads and exports what include/b200gemv.h declares (CPU).

No kernel is launched here: argument validation happens before any CUDA
call, so invalid requests are rejected identically with or without a GPU.
"""
from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "b200gemv.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(b2g_\w+)\s*\(", text)))


def test_header_declarations_have_bindings(b2g):
    decl = declared_functions()
    assert len(decl) >= 20
    assert sorted(b2g.SIGNATURES) == decl


def test_library_exports_every_declared_symbol(b2g):
    L = b2g.lib()
    for name in declared_functions():
        assert hasattr(L, name), name


def test_status_strings_and_version(b2g):
    L = b2g.lib()
    assert L.b2g_version() >= 100
    for s in range(8):
        assert L.b2g_status_string(s)
    assert L.b2g_status_string(0) == b"ok"


@pytest.mark.parametrize("bad", [
    dict(in_features=0), dict(out_features=-1), dict(weight_dtype=7), dict(scale_mode=9),
    dict(weight_layout=3), dict(fuse=64), dict(tp_size=2, tp_rank=2),
])
def test_create_rejects_bad_fields(b2g, bad):
    f = dict(in_features=3072, out_features=8192, weight_dtype=1, scale_mode=3, weight_layout=0,
             max_m=8, fuse=0, tp_rank=0, tp_size=1)
    f.update(bad)
    h = ctypes.c_void_p()
    st = b2g.lib().b2g_create(ctypes.byref(b2g.Fields(**f)), ctypes.byref(h))
    assert st == b2g.ERR_INVALID and not h.value


def test_create_rejects_unsupported(b2g):
    h = ctypes.c_void_p()
    f = b2g.Fields(3072, 8192, 1, 3, 0, 16, 0, 0, 1)  # max_m 16 > 8
    assert b2g.lib().b2g_create(ctypes.byref(f), ctypes.byref(h)) == b2g.ERR_UNSUPPORTED
    f = b2g.Fields(3072, 8192, 1, 3, 0, 8, b2g.FUSE_GATE_UP_SILU | b2g.FUSE_RESIDUAL_ADD, 0, 1)
    assert b2g.lib().b2g_create(ctypes.byref(f), ctypes.byref(h)) == b2g.ERR_UNSUPPORTED


def test_null_arguments_rejected(b2g):
    L = b2g.lib()
    assert L.b2g_create(None, None) == b2g.ERR_INVALID
    n = ctypes.c_size_t()
    assert L.b2g_prepack_size(None, ctypes.byref(n)) == b2g.ERR_INVALID
    assert L.b2g_enqueue_ex(None, None, None) == b2g.ERR_INVALID
    assert L.b2g_enqueue_static(None, None, None) == b2g.ERR_INVALID
    assert L.b2g_quantize_e4m3(None, 4, 4, 0, 0, None, None, None) == b2g.ERR_INVALID
    assert L.b2g_stack_create(None, None) == b2g.ERR_INVALID
    assert L.b2g_destroy(None) == b2g.OK


def test_product_raises_without_library(b2g, monkeypatch, tmp_path):
    """No silent fallback: a missing library is an error, not a CPU path."""
    monkeypatch.setattr(b2g, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(b2g, "_lib", None)
    with pytest.raises(RuntimeError, match="missing"):
        b2g.lib()


def test_package_does_not_reference_the_oracle():
    pkg = ROOT / "llama-3.2-3b-instruct-gemm-optimization_b200"
    for p in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.cpp")) + \
            list(pkg.rglob("*.cuh")) + list(pkg.rglob("*.h")):
        assert "oracle" not in p.read_text().lower(), p


def test_refused_option_keeps_plan(b2g):
    """Options are validated without a GPU only as far as the arguments go;
    an invalid key or value is refused before any CUDA call."""
    L = b2g.lib()
    assert L.b2g_op_set_option(None, b2g.OPT_GRID, 0) == b2g.ERR_INVALID


def test_header_is_plain_c_and_plans_without_a_device(b2g, tmp_path):
    """A C11 consumer (what a cgo / JNI / N-API binding compiles against):
    the header compiles with warnings as errors, every entry point links, and
    the device-free calls run -- the decode shapes' plans for a B200."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    refs = ",\n    ".join(f"(void (*)(void))&{f}" for f in declared_functions())
    src = tmp_path / "consumer.c"
    src.write_text(f"""#include <stdio.h>
#include "b200gemv.h"
static void (*const every_entry[])(void) = {{
    {refs}
}};
static int plan(int K, int N, int fuse) {{
  b2g_fields f = {{K, N, B2G_DTYPE_FP8_E4M3, B2G_SCALE_CHANNEL_FP32, B2G_LAYOUT_KN, 8, fuse, 0, 1}};
  b2g_plan_info info;
  size_t packed = 0, ws = 0;
  b2g_status st = b2g_plan_for_device(&f, 148, 232448, 8, &info, &packed, &ws);
  if (st != B2G_OK) {{ printf("error %s\\n", b2g_status_string(st)); return 1; }}
  printf("%d %d %d %d %zu\\n", K, N, info.grid, info.partition, packed);
  return 0;
}}
int main(void) {{
  printf("version %d entries %zu\\n", (int)b2g_version(), sizeof every_entry / sizeof every_entry[0]);
  return plan(3072, 8192, B2G_FUSE_GATE_UP_SILU | B2G_FUSE_RMSNORM_INPUT) | plan(8192, 3072, B2G_FUSE_RESIDUAL_ADD);
}}
""")
    libdir = b2g.LIB_PATH.parent
    exe = tmp_path / "consumer"
    subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-Wno-cast-function-type", "-I", str(ROOT / "include"),
                    str(src), "-L", str(libdir), "-lb200gemv", f"-Wl,-rpath,{libdir}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    assert out[0].startswith("version ") and out[0].endswith(f"entries {len(declared_functions())}")
    assert out[1] == f"3072 8192 128 2 {2 * 3072 * 8192}"
    assert out[2] == f"8192 3072 96 2 {8192 * 3072}"


@pytest.mark.parametrize("world,max_m,width", [(1, 8, 256), (2, 8, 3072), (8, 8, 3072), (4, 1, 3072)])
def test_tp_comm_layout_without_a_device(b2g, world, max_m, width):
    """The exchange buffer's layout is arithmetic on the base address: the
    inbox first (big enough for the REDUCE words, [2][world][max_m][width/2]
    x 8 B, which also covers the fp16 PUSH slots), then the 256-byte counter
    region, then the epoch region with the per-CTA round counts (word 64
    on, B2G_TP_MAX_CTAS of them); every region 256-byte aligned."""
    n = b2g.tp_comm_bytes(world, max_m, width)
    inbox_bytes = -(-2 * world * max_m * (width // 2) * 8 // 256) * 256
    epoch_bytes = -(-(64 + b2g.TP_MAX_CTAS) * 4 // 256) * 256
    assert n == inbox_bytes + 256 + epoch_bytes
    base = 1 << 40  # never dereferenced
    inbox, counters, epoch = b2g.tp_comm_layout(base, world, max_m, width)
    assert (inbox, counters, epoch) == (base, base + inbox_bytes, base + inbox_bytes + 256)
    assert epoch + (64 + b2g.TP_MAX_CTAS) * 4 <= base + n
    assert 2 * world * max_m * width * 2 <= inbox_bytes  # the fp16 slots fit as well


@pytest.mark.parametrize("world,max_m,width", [(0, 8, 256), (9, 8, 256), (2, 0, 256), (2, 8, 4)])
def test_tp_comm_rejects_bad_sizes(b2g, world, max_m, width):
    assert b2g.tp_comm_bytes(world, max_m, width) == 0
    with pytest.raises(b2g.B2GError):
        b2g.tp_comm_layout(1 << 40, world, max_m, width)
