"""The C-ABI library loads on a CPU-only machine and exports exactly the
reference's 19 helper symbols (src/minicpmo/gpu_bridge.c:72-90) plus every
extension declared in include/minicpmo_gpu.h.  No compute calls."""
from __future__ import annotations

import ctypes
import re
import subprocess

from conftest import ROOT

HEADER = ROOT / "include" / "minicpmo_gpu.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(minicpmo_gpu_\w+)\s*\(", text)))


def test_library_loads_and_exports_header_symbols(pkg):
    lib = pkg.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_reference_symbol_set(pkg):
    from minicpmo_b200.gpu import REFERENCE_SYMBOLS

    assert len(REFERENCE_SYMBOLS) == 19
    declared = set(declared_functions())
    assert set(REFERENCE_SYMBOLS) <= declared


def test_dynamic_symbol_table_matches_header(pkg):
    out = subprocess.run(["nm", "-D", "--defined-only", str(pkg.lib_path())], capture_output=True, text=True).stdout
    exported = sorted({l.split()[-1] for l in out.splitlines() if " T " in l and "minicpmo" in l})
    assert exported == declared_functions()


def test_abi_version(pkg):
    assert pkg.lib().minicpmo_gpu_abi_version() == 1


def test_null_handles_are_rejected(pkg):
    lib = pkg.lib()
    err = ctypes.create_string_buffer(512)
    assert lib.minicpmo_gpu_context_smoke(None, err, 512) == 0
    assert err.value.startswith(b"error:")
    lib.minicpmo_gpu_context_destroy(None)  # NULL-safe (gpu_shim.c:2349-2352)
    assert lib.minicpmo_gpu_context_create(0, 0, None, err, 512) == 0


def test_no_alloc_attention_limits_are_checked_on_the_host(pkg):
    """Shapes beyond the fixed scratch are refused before any CUDA call."""
    import ctypes as C

    lib = pkg.lib()
    buf = (C.c_float * 4)()
    err = C.create_string_buffer(512)
    fn = lib.minicpmo_gpu_attention_no_alloc
    fn.argtypes = [C.c_void_p] * 3 + [C.c_int] + [C.c_size_t] * 5 + [C.c_void_p] * 2 + [C.c_char_p, C.c_size_t]
    p = C.cast(buf, C.c_void_p)
    # 32 heads, head_dim 128, a 4096-position cache -> 128 blocks x 132 floats x 32 heads = 2162688 B > 2 MiB
    assert fn(p, p, p, 0, 0, 32, 8, 128, 4096, p, None, err, 512) == 0
    assert b"scratch bytes" in err.value and b"2097152" in err.value
    assert fn(p, p, p, 0, 0, 2048, 2048, 64, 1, p, None, err, 512) == 0
    assert b"kv heads exceed" in err.value
    assert fn(p, p, p, 0, 0, 32, 2, 128, 1, p, None, err, 512) == 0  # group of 16
    assert b"group" in err.value
    assert fn(p, p, p, 0, 0, 4, 8, 128, 1, p, None, err, 512) == 0  # 4 heads over 8 kv heads
    assert b"fewer than 8 kv heads" in err.value
    assert fn(p, p, p, 0, 5, 8, 8, 128, 5, p, None, err, 512) == 0  # pos outside the context
    assert b"outside context" in err.value
    assert fn(None, p, p, 0, 0, 8, 8, 128, 1, p, None, err, 512) == 0
    assert b"null buffer" in err.value
