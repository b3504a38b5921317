#!/usr/bin/env python3
"""Generates tests/golden/reference_vectors.npz from the reference's own code.

Run where the reference tree is available (``make -C oracle REF=<tree>`` builds
oracle/_ref/ from it first).  Every output array is computed by reference
code compiled from its sources, not by this repository:

* f16_bits       -- gpu_shim.c:2157-2192 (minicpmo_gpu_f32_to_f16) on f16_inputs
* q8_1_bytes     -- gpu_shim.c:380-401 (host Q8_1 quantiser) on q8_1_inputs
* kq_y_<dt>      -- the shim's CUDA Q4_K/Q6_K x Q8_1 matvec kernels
                    (gpu_shim.c:746-925) evaluated on the host
* cpu_y_<dt>     -- cpu_kernels.c:791-851 f32-activation matvec
* rope_out       -- gpu_shim.c:665-693 rope kernel body
* silu_out       -- gpu_shim.c:659-664
* rms_out        -- gpu_shim.c:694-718 RMSNorm kernel (one block of 256)
* hn_out         -- gpu_shim.c:719-745 head-norm kernel (a block per head)
* att_out        -- gpu_shim.c:926-979 decode-attention kernel (a block
                    per head), scale 1/minicpmo_gpu_sqrtf_positive(head_dim)

Inputs are seeded (numpy PCG64) and stored alongside.  Usage:
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402


def load_pkg():
    pkg_dir = ROOT / "minicpm-o-uya_b200"
    spec = importlib.util.spec_from_file_location("minicpmo_b200", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["minicpmo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    O.build()
    for n in ("cpu", "shim", "kernels"):
        if O.ref_lib(n) is None:
            raise SystemExit(f"oracle/_ref/libref_{n}.so missing: the reference tree is needed")
    import torch

    load_pkg()
    from minicpmo_b200 import gguf

    rng = np.random.Generator(np.random.PCG64(20261201))
    out = {}
    # f16 rounding: random magnitudes across the whole range + edge cases
    f = np.concatenate([
        (rng.standard_normal(4096) * np.exp2(rng.integers(-30, 20, 4096))).astype(np.float32),
        np.array([0.0, -0.0, 1.0, -2.0, 65504.0, 65520.0, 1e-8, 6.1e-5, 5.96e-8, 2.98e-8, np.inf, -np.inf, np.nan],
                 np.float32),
        # values exactly halfway between f16 neighbours
        (np.arange(1, 257, dtype=np.float32) * np.float32(2.0 ** -10) + np.float32(2.0 ** -11)).astype(np.float32) + 1.0,
    ]).astype(np.float32)
    out["f16_inputs"] = f
    out["f16_bits"] = np.array([O.ref_lib("shim").minicpmo_gpu_f32_to_f16(float(v)) for v in f], np.uint16)

    # Q8_1 quantisation
    xs = [rng.standard_normal(1024).astype(np.float32)]
    z = rng.standard_normal(512).astype(np.float32)
    z[32:64] = 0.0
    z[64:96] = -0.0
    z[96] = 1e-30
    xs.append(z)
    xs.append((rng.standard_normal(768) * 1e-4).astype(np.float32))
    ties = np.tile(np.arange(-16, 16, dtype=np.float32) * 0.5, 8)  # x/d lands on .5 boundaries
    ties[::32] = 127.0 * 0.5
    xs.append(ties.astype(np.float32))
    xs.append((rng.standard_normal(256) * 1e4).astype(np.float32))
    qin = np.concatenate(xs)
    out["q8_1_inputs"] = qin
    out["q8_1_bytes"] = O.ref_shim_q8_1(qin)

    # K-quant matvec through the reference kernels, and the CPU f32 path
    rows, cols = 24, 768
    w32 = torch.randn((rows, cols), generator=torch.Generator().manual_seed(5)) * 0.02
    x = rng.standard_normal(cols).astype(np.float32)
    xq = O.ref_shim_q8_1(x)
    out["mv_x"] = x
    for dt, name in ((gguf.Q4_K, "q4_k"), (gguf.Q6_K, "q6_k"), (gguf.Q8_0, "q8_0")):
        w = gguf.quantize(w32, dt).numpy()
        out[f"w_{name}"] = w
        if dt != gguf.Q8_0:
            out[f"kq_y_{name}"] = O.ref_kernel_matvec(dt, w, rows, cols, xq)
        out[f"cpu_y_{name}"] = O.ref_cpu_matvec(dt, w, rows, cols, x)

    # rope and silu kernel bodies
    heads, hd, ctx = 3, 128, 16
    cos_t, sin_t = O.rope_table(ctx, hd, 1e6, 1.0)
    vec = rng.standard_normal(heads * hd).astype(np.float32)
    r = vec.copy()
    O.ref_lib("kernels").refk_apply_rope(r.ctypes.data_as(O.fp), heads, hd, 11, cos_t.ctypes.data_as(O.fp),
                                          sin_t.ctypes.data_as(O.fp))
    out["rope_in"] = vec
    out["rope_cos"] = cos_t
    out["rope_sin"] = sin_t
    out["rope_out"] = r
    g = (rng.standard_normal(700) * 4).astype(np.float32)
    u = rng.standard_normal(700).astype(np.float32)
    s = np.empty_like(g)
    O.ref_lib("kernels").refk_silu_mul(s.ctypes.data_as(O.fp), g.ctypes.data_as(O.fp), u.ctypes.data_as(O.fp), g.size)
    out["silu_g"], out["silu_u"], out["silu_out"] = g, u, s

    # RMSNorm, head-norm and decode-attention kernel bodies (gpu_shim.c:694-745,
    # 926-979), one host thread per CUDA thread, phases split at __syncthreads
    K = O.ref_lib("kernels")
    n = 4096
    xr = (rng.standard_normal(n) * 3).astype(np.float32)
    wr = (1.0 + rng.standard_normal(n) * 0.02).astype(np.float32)
    ro = np.empty(n, np.float32)
    K.refk_rms_norm(ro.ctypes.data_as(O.fp), xr.ctypes.data_as(O.fp), wr.view(np.uint8).ctypes.data_as(O.u8p), 0, n,
                    1e-6)
    out["rms_x"], out["rms_w"], out["rms_out"] = xr, wr, ro
    heads, hd = 6, 128
    hv = (rng.standard_normal(heads * hd) * 2).astype(np.float32)
    hw = (1.0 + rng.standard_normal(hd) * 0.02).astype(np.float32)
    ho = hv.copy()
    K.refk_head_norm(ho.ctypes.data_as(O.fp), hw.view(np.uint8).ctypes.data_as(O.u8p), 0, heads, hd)
    out["hn_in"], out["hn_w"], out["hn_out"] = hv, hw, ho
    layers, ctx, ah, akv, ahd, apos = 2, 80, 8, 2, 128, 70
    aq = rng.standard_normal(ah * ahd).astype(np.float32)
    ak = rng.standard_normal((layers, ctx, akv * ahd)).astype(np.float32)
    av = rng.standard_normal((layers, ctx, akv * ahd)).astype(np.float32)
    scale = O.ref_lib("shim").minicpmo_gpu_sqrtf_positive(float(ahd))
    scale = np.float32(1.0) / np.float32(scale)
    ao = np.empty(ah * ahd, np.float32)
    K.refk_attention_decode(aq.ctypes.data_as(O.fp), ak.ctypes.data_as(O.fp), av.ctypes.data_as(O.fp),
                            ao.ctypes.data_as(O.fp), 1, apos, ah, akv, ahd, ctx, float(scale))
    out["att_q"], out["att_k"], out["att_v"], out["att_out"] = aq, ak, av, ao
    out["att_shape"] = np.array([layers, ctx, ah, akv, ahd, apos], np.int32)
    out["att_scale"] = np.array([scale], np.float32)

    path = Path(__file__).resolve().parent / "reference_vectors.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
