"""minicpmo_b200 -- B200-native Qwen3 quantised decode path of minicpm-o-uya.

The product is ``libminicpmo_gpu_helper.so`` (C ABI, ``include/minicpmo_gpu.h``):
a drop-in for the reference helper that ``src/minicpmo/gpu_bridge.c`` loads.
This package is the Python mirror of the reference host side above that ABI:

* :mod:`.gpu`   -- ctypes façade over the helper, mirroring ``src/minicpmo/gpu.uya``
* :mod:`.gguf`  -- GGUF v3 reader/writer and the Q4_K/Q6_K/Q8_0 block
  quantisers used to build seeded synthetic models
* :mod:`.qwen3` -- the Qwen3 runtime mirroring ``src/minicpmo/qwen3.uya``
  (open runtime, tokenwise prefill, greedy generate, bench)

There is no CPU fallback: if the helper library is missing or no B200 is
present, the entry points raise.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_NAME = "libminicpmo_gpu_helper.so"

# Uya TensorDType ordinals (src/minicpmo/tensor.uya:31-54)
F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 6, 10, 12, 20
DTYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K", BF16: "BF16"}

_lib = None


def lib_path() -> Path:
    return Path(os.environ.get("MINICPMO_GPU_HELPER", PKG_DIR / LIB_NAME))


def lib() -> ctypes.CDLL:
    """Load the helper library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        path = lib_path()
        if not path.exists():
            raise RuntimeError(f"{path} is missing: build it with __graft_entry__.build() (make -C minicpm-o-uya_b200/csrc)")
        _lib = ctypes.CDLL(str(path))
        from . import gpu

        gpu.declare(_lib)
    return _lib


def build(verbose: bool = False) -> Path:
    """Compile the helper for sm_100a (nvcc cross-compiles without a GPU)."""
    import subprocess

    cmd = ["make", "-C", str(PKG_DIR / "csrc"), "-j4"]
    res = subprocess.run(cmd, capture_output=not verbose, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"helper build failed:\n{res.stdout}\n{res.stderr}")
    return lib_path()
