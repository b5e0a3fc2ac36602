"""The C ABI library without a GPU: it loads, it exports exactly what
include/*.h declares, and its entry points fail cleanly when no device exists
(no compute calls here)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = ["gemv_dev.h", "gemv2_dev.h", "udmabuf.h", "b200_engine.h", "b200_comm.h", "b200_decoder.h", "b200_gguf.h"]


def declared_symbols() -> set[str]:
    names = set()
    for h in HEADERS:
        with open(os.path.join(ROOT, "include", h)) as fh:
            for m in re.finditer(r"^B200_API\s+[\w\s\*]+?\b(\w+)\s*\(", fh.read(), re.M):
                names.add(m.group(1))
    return names


def exported_symbols(path: str) -> set[str]:
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_headers_declare_the_reference_interfaces():
    names = declared_symbols()
    # board/kv260gemv/gemv_dev.h:15-35, gemv2_dev.h:63-80, udmabuf.h:23-36
    for ref in ["gemv_dev_open", "gemv_dev_open_named", "gemv_dev_close", "gemv_dev_run", "gemv_dev_start",
                "gemv_dev_wait", "gemv_dev_start4", "gemv2_dev_open", "gemv2_dev_close", "gemv2_fetch_start",
                "gemv2_fetch_wait", "gemv2_mac_start", "gemv2_mac_wait", "gemv2_mac_idle", "gemv2_drain",
                "udmabuf_open", "udmabuf_close", "udmabuf_alloc", "udmabuf_clean", "udmabuf_invalidate"]:
        assert ref in names, ref


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg.lib()
    exported = exported_symbols(pkg.capi.LIB_PATH)
    missing = declared_symbols() - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    extra = exported - declared_symbols()
    assert not extra, f"exported but not declared in include/*.h: {sorted(extra)}"
    for name in declared_symbols():
        assert hasattr(lib, name)


def test_ctypes_signatures_cover_the_headers(pkg):
    assert declared_symbols() == set(pkg.capi.SIGNATURES)


def test_inline_helpers_match_the_oracle(oracle):
    """gemv2_chunk_offset is a static inline in gemv2_dev.h; compile it and compare."""
    import subprocess
    import tempfile
    src = ('#include <stdio.h>\n#include "gemv2_dev.h"\nint main(void){int p;'
           'for(int r=0;r<64;++r)for(int c=0;c<4;++c){size_t o=gemv2_chunk_offset(r,c,64,1024,&p);'
           'printf("%zu %d\\n",o,p);}return 0;}\n')
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "t.c"), "w") as fh:
            fh.write(src)
        exe = os.path.join(d, "t")
        subprocess.run(["gcc", "-std=c11", "-I", os.path.join(ROOT, "include"), os.path.join(d, "t.c"), "-o", exe],
                       check=True)
        lines = subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split("\n")
    i = 0
    for r in range(64):
        for c in range(4):
            off, port = (int(v) for v in lines[i].split())
            assert (off, port) == oracle.gemv2_chunk_offset(r, c, 64, 1024)
            i += 1


def _no_gpu() -> bool:
    try:
        import torch
        return not torch.cuda.is_available()
    except Exception:
        return True


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-device error paths")
def test_entry_points_fail_cleanly_without_a_device(pkg):
    capi, lib = pkg.capi, pkg.lib()
    assert lib.b200_device_count() == 0
    h = ctypes.c_void_p()
    assert lib.b200_engine_open(ctypes.byref(h), 0) == -19        # -ENODEV
    assert b"no CUDA device" in lib.b200_last_error()
    d = capi.gemv_dev_t()
    assert lib.gemv_dev_open_named(ctypes.byref(d), b"gemv_q4_0", 1) == -1
    d2 = capi.gemv2_dev_t()
    assert lib.gemv2_dev_open(ctypes.byref(d2)) == -1
    assert lib.gemv_dev_start(ctypes.byref(d), 0, 0, 0, 256, 16) == -22   # engine not open
    b = capi.udmabuf_t()
    assert lib.udmabuf_clean(ctypes.c_void_p(12345), 16) == -22          # not inside a pool
    with pytest.raises(pkg.B200Error):
        pkg.Engine(0, stream=0)
