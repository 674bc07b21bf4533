"""The C-ABI library loads and exports every function include/seoulkv_b200.h declares."""

import re
from pathlib import Path

import pytest
import torch

from seoulkv_b200 import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "seoulkv_b200.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(skv_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_core_entry_points():
    names = declared()
    for must in ("skv_create", "skv_destroy", "skv_upload_index", "skv_upload_kv", "skv_bind_query",
                 "skv_run", "skv_sync", "skv_status", "skv_output", "skv_debug_ids", "skv_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.skv_version().startswith(b"seoulkv_b200")
    assert lib.skv_kernels_per_step() > 0
    assert lib.skv_kernel_name(0) != b""


def test_flag_and_stage_constants_match_the_header():
    """The Python binding's flag bits and stage ids are the header's."""
    text = HEADER.read_text()
    defs = {m.group(1): int(m.group(2)) for m in re.finditer(r"#define\s+(SKV_\w+)\s+(\d+)", text)}
    assert defs["SKV_FLAG_STAGED"] == _native.SKV_FLAG_STAGED
    assert defs["SKV_FLAG_NO_LEAD"] == _native.SKV_FLAG_NO_LEAD
    assert defs["SKV_FLAG_TRACE"] == _native.SKV_FLAG_TRACE
    assert len({_native.SKV_FLAG_STAGED, _native.SKV_FLAG_NO_LEAD, _native.SKV_FLAG_TRACE}) == 3
    stage = {k[len("SKV_STAGE_"):].lower(): v for k, v in defs.items() if k.startswith("SKV_STAGE_")}
    for name, v in _native.STAGE.items():
        assert stage.get(name) == v, name


def test_create_rejects_bad_descriptors():
    lib = _native.load()
    import ctypes

    h = ctypes.c_void_p()
    for kw in (dict(n_slots=0), dict(nc=33), dict(context=0), dict(sink=9000), dict(stage15_capacity=100)):
        d = dict(n_slots=1, context=8192, sink=128, local=256, nc=1952, stage15_capacity=13056, device=0)
        d.update(kw)
        rc = lib.skv_create(ctypes.byref(_native.SkvDesc(**d)), ctypes.byref(h))
        assert rc == -1, kw
        assert lib.skv_last_error()


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU error path")
def test_no_gpu_fails_loudly():
    with pytest.raises(_native.NativeError) as exc:
        _native.Engine(n_slots=1, context=8192, sink=128, local=256, nc=1952, capacity=13056, device=0)
    assert exc.value.code == -2


C_CONSUMER = r"""
#include <stdio.h>
#include <string.h>
#include "seoulkv_b200.h"

int main(void) {
  SkvDesc d;
  void *h = NULL;
  memset(&d, 0, sizeof d);
  d.n_slots = 0;  /* invalid: rejected before any CUDA call */
  d.context = 8192; d.sink = 128; d.local = 256; d.nc = 1952; d.stage15_capacity = 13056;
  int rc = skv_create(&d, &h);
  const char *msg = skv_last_error();
  printf("%d %s|%s\n", rc, h == NULL ? "null" : "set", msg ? msg : "");
  return rc == SKV_E_INVALID && h == NULL && msg && msg[0] ? 0 : 1;
}
"""


def test_header_compiles_as_c_and_cxx(tmp_path):
    """The boundary header is plain C (what cgo, JNI or a C++ runtime includes)."""
    import shutil
    import subprocess

    for cc, std in (("gcc", "-std=c99"), ("g++", "-std=c++17")):
        if not shutil.which(cc):
            pytest.skip(f"{cc} not found")
        src = tmp_path / ("h.c" if cc == "gcc" else "h.cc")
        src.write_text('#include "seoulkv_b200.h"\nint main(void) { return sizeof(SkvDesc) == 0; }\n')
        r = subprocess.run([cc, std, "-Wall", "-Werror", "-pedantic", "-fsyntax-only", f"-I{HEADER.parent}",
                            str(src)], capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_c_program_links_and_gets_the_error_contract(tmp_path):
    """A plain C program linked against the library: a bad descriptor gives
    SKV_E_INVALID, no handle and a message from skv_last_error()."""
    import shutil
    import subprocess

    if not shutil.which("gcc"):
        pytest.skip("gcc not found")
    _native.load()  # (builds the library first when it is stale)
    lib = _native.library_path()
    src, exe = tmp_path / "consumer.c", tmp_path / "consumer"
    src.write_text(C_CONSUMER)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", f"-I{HEADER.parent}", str(src), str(lib),
                        f"-Wl,-rpath,{lib.parent}", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, (run.stdout, run.stderr)
    assert run.stdout.startswith(f"{-1} null|")
