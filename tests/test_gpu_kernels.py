"""Parity of the sm_100a kernels with the CPU oracle, through the C ABI.

Everything is bit-exact against the oracle's device-order restatement:
integer and byte work by construction (Q8_1 blocks, per-block int32 dots,
embedding dequant), float work because the kernels use only correctly
rounded IEEE operations in the documented order (oracle/oracle.h, "device
evaluation order").  Against the reference's natural summation order the
float results are held to the stated tolerances.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_row_err

pytestmark = pytest.mark.gpu

Q4_K, Q6_K, Q8_0, F32, F16, BF16 = 10, 12, 6, 0, 1, 20
MATVEC_TOL = 1e-5  # vs the oracle on identical Q8_1 activations (summation order only)
NORTH_STAR_TOL = 1e-3  # per-row error / ||y||_2


def make_tensor(pkg, name, dt, rows, cols, seed, std=0.02, offset=0.0):
    from minicpmo_b200 import gguf
    from minicpmo_b200.gpu import Tensor

    x = torch.randn((rows, cols), generator=torch.Generator().manual_seed(seed)) * std + offset
    return Tensor(name, gguf.quantize(x, dt).numpy(), dt, rows, cols), x


def rvec(n, seed, scale=1.0):
    return (np.random.Generator(np.random.PCG64(seed)).standard_normal(n) * scale).astype(np.float32)


# ----------------------------------------------------------------- Q8_1
def test_q8_1_bit_exact_golden(gpu_ctx, O, golden):
    x = golden["q8_1_inputs"]
    assert np.array_equal(gpu_ctx.q8_1_quantize(x), golden["q8_1_bytes"])


@pytest.mark.parametrize("scale", [1e-7, 1e-3, 1.0, 1e3])
def test_q8_1_bit_exact_random(gpu_ctx, O, scale):
    x = rvec(4096 + 32 * 7, 11, scale)
    x[64:96] = 0.0
    assert np.array_equal(gpu_ctx.q8_1_quantize(x), O.q8_1_quantize(x))


def test_q8_1_bit_exact_near_half_integers(gpu_ctx, O):
    """Values whose quotient x/d sits on or a few ulp from a rounding boundary
    k + 0.5 (where the kernels switch from x*rcp(d) to the exact division)."""
    rng = np.random.Generator(np.random.PCG64(99))
    blocks = []
    for amax in [127.0, 100.0, 1.0, 3.3e-3, 7.77e4, 1e-30]:
        d = np.float32(np.float32(amax) / np.float32(127.0))
        for _ in range(24):
            k = rng.integers(-127, 127, 31)
            x = ((k + 0.5) * np.float64(d)).astype(np.float32)
            ulps = rng.integers(-3, 4, 31).astype(np.int32)
            x = (x.view(np.int32) + ulps).view(np.float32)
            x = np.clip(x, -np.float32(amax), np.float32(amax))
            blocks.append(np.concatenate([[np.float32(amax)], x]).astype(np.float32))
    x = np.concatenate(blocks)
    assert np.array_equal(gpu_ctx.q8_1_quantize(x), O.q8_1_quantize(x))


@pytest.mark.parametrize("wdt", [F32, F16, BF16])
@pytest.mark.parametrize("n", [1024, 4096, 5120, 12288])
def test_rms_norm_q8_1_bit_exact(pkg, gpu_ctx, O, wdt, n):
    from minicpmo_b200 import gguf
    from minicpmo_b200.gpu import Tensor

    w32 = torch.randn((1, n), generator=torch.Generator().manual_seed(n)) * 0.02 + 1.0
    w = Tensor(f"norm{n}_{wdt}", gguf.quantize(w32, wdt).numpy(), wdt, 1, n)
    gpu_ctx.upload_tensor(w)
    x = rvec(n, n + 1, 3.0)
    out, xq = gpu_ctx.rms_norm_q8_1(x, w)
    ref = O.rms_norm(x, w.data.view(np.float32 if wdt == F32 else np.uint16), wdt, 1e-6, order=1)
    assert np.array_equal(out, ref)
    assert np.array_equal(xq, O.q8_1_quantize(ref))


# ---------------------------------------------------------- quant GEMV
SHAPES = [(37, 256), (64, 512), (130, 3072), (24, 5120), (40, 12288), (300, 1024), (1, 8192)]


@pytest.mark.parametrize("dt", [Q4_K, Q6_K, Q8_0])
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_matvec_dots_bit_exact_and_rows_close(pkg, gpu_ctx, O, dt, rows, cols):
    t, _ = make_tensor(pkg, f"w{dt}_{rows}_{cols}", dt, rows, cols, seed=rows * 31 + cols)
    gpu_ctx.upload_tensor(t)
    xq = O.q8_1_quantize(rvec(cols, cols))
    y, dots = gpu_ctx.matvec_q8_1(t, xq, dots=True)
    assert np.array_equal(dots, O.block_dots(dt, t.data, rows, cols, xq))
    assert np.array_equal(y, O.matvec_q8_1_dev(dt, t.data, rows, cols, xq))
    assert rel_row_err(y, O.matvec_q8_1(dt, t.data, rows, cols, xq)) < MATVEC_TOL


@pytest.mark.parametrize("dt", [Q4_K, Q6_K, Q8_0])
@pytest.mark.parametrize("rows,cols", [(130, 3072), (64, 4096), (40, 12288), (37, 256)])
@pytest.mark.parametrize("wdt", [None, F32, F16, BF16])
def test_matvec_fused_input_matches_two_kernel_path(pkg, gpu_ctx, dt, rows, cols, wdt):
    """The GEMV prologue's own RMSNorm/quantisation gives the bits of
    rms_norm_q8_1 (or q8_1_quantize) followed by matvec_q8_1."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.gpu import Tensor

    t, _ = make_tensor(pkg, f"fin{dt}_{rows}_{cols}", dt, rows, cols, seed=rows + cols)
    gpu_ctx.upload_tensor(t)
    x = rvec(cols, cols + 3, 2.0)
    x[32:64] = 0.0  # an all-zero Q8_1 block
    if wdt is None:
        y = gpu_ctx.matvec_f32_input(t, x)
        xq = gpu_ctx.q8_1_quantize(x)
    else:
        w32 = torch.randn((1, cols), generator=torch.Generator().manual_seed(cols + wdt)) * 0.05 + 1.0
        w = Tensor(f"finw{cols}_{wdt}", gguf.quantize(w32, wdt).numpy(), wdt, 1, cols)
        gpu_ctx.upload_tensor(w)
        y = gpu_ctx.matvec_f32_input(t, x, w, 1e-6)
        _, xq = gpu_ctx.rms_norm_q8_1(x, w, 1e-6)
    assert np.array_equal(y, gpu_ctx.matvec_q8_1(t, xq))


def _near_half_integer_blocks(n, seed):
    """n values in 32-value blocks whose quotients x/d sit on or a few ulp from
    k + 0.5 (the rounding boundaries of the Q8_1 quantiser)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    amaxes = [127.0, 100.0, 1.0, 3.3e-3, 7.77e4]
    for i in range(n // 32):
        amax = amaxes[i % len(amaxes)]
        d = np.float32(np.float32(amax) / np.float32(127.0))
        k = rng.integers(-127, 127, 31)
        x = ((k + 0.5) * np.float64(d)).astype(np.float32)
        x = (x.view(np.int32) + rng.integers(-3, 4, 31).astype(np.int32)).view(np.float32)
        x = np.clip(x, -np.float32(amax), np.float32(amax))
        out.append(np.concatenate([[np.float32(amax)], x]).astype(np.float32))
    return np.concatenate(out)


@pytest.mark.parametrize("dt", [Q4_K, Q6_K])
@pytest.mark.parametrize("cols", [4096, 12288])
def test_matvec_fused_input_near_half_integers(pkg, gpu_ctx, dt, cols):
    """The f32-input prologue (one thread per block, approximate reciprocal
    with an exact fallback) on values placed at the rounding boundaries."""
    t, _ = make_tensor(pkg, f"fhb{dt}_{cols}", dt, 64, cols, seed=cols + dt)
    gpu_ctx.upload_tensor(t)
    x = _near_half_integer_blocks(cols, cols)
    assert np.array_equal(gpu_ctx.matvec_f32_input(t, x), gpu_ctx.matvec_q8_1(t, gpu_ctx.q8_1_quantize(x)))


@pytest.mark.parametrize("dt", [Q4_K, Q6_K])
def test_matvec_vs_reference_cuda_kernels(pkg, gpu_ctx, O, dt):
    if O.ref_lib("kernels") is None:
        pytest.skip("oracle/_ref not built")
    rows, cols = 96, 4096
    t, _ = make_tensor(pkg, f"refk{dt}", dt, rows, cols, seed=dt)
    gpu_ctx.upload_tensor(t)
    xq = O.q8_1_quantize(rvec(cols, 5))
    assert rel_row_err(gpu_ctx.matvec_q8_1(t, xq), O.ref_kernel_matvec(dt, t.data, rows, cols, xq)) < MATVEC_TOL


@pytest.mark.parametrize("dt", [Q4_K, Q6_K, Q8_0])
def test_reference_matvec_entry(pkg, gpu_ctx, O, dt):
    """minicpmo_gpu_context_matvec (host x in, host y out, gpu_shim.c:2529-2719)."""
    rows, cols = 512, 4096
    t, _ = make_tensor(pkg, f"hostmv{dt}", dt, rows, cols, seed=dt + 100)
    gpu_ctx.upload_tensor(t)
    x = rvec(cols, dt)
    y = gpu_ctx.matvec(t, x)
    assert rel_row_err(y, O.matvec_q8_1(dt, t.data, rows, cols, O.q8_1_quantize(x))) < MATVEC_TOL
    # against the reference CPU path (f32 activations): activation quantisation error only
    assert rel_row_err(y, O.matvec_f32(dt, t.data, rows, cols, x)) < NORTH_STAR_TOL * 10


@pytest.mark.parametrize("dt", [F32, F16, BF16])
def test_dense_matvec(pkg, gpu_ctx, O, dt):
    rows, cols = 70, 333
    t, _ = make_tensor(pkg, f"dense{dt}", dt, rows, cols, seed=dt + 7)
    gpu_ctx.upload_tensor(t)
    x = rvec(cols, 9)
    y = gpu_ctx.matvec(t, x)
    assert np.array_equal(y, O.matvec_dense_dev(dt, t.data, rows, cols, x))
    assert rel_row_err(y, O.matvec_f32(dt, t.data, rows, cols, x)) < 1e-5


def test_grouped_slot_matvec_mixed_dtypes(pkg, gpu_ctx, O):
    """q/k/v with Q4_K, Q4_K, Q6_K in one launch (the reference falls back to 3 calls, gpu_shim.c:3067-3074)."""
    h = 1024
    tq, _ = make_tensor(pkg, "g.q", Q4_K, 512, h, 1)
    tk, _ = make_tensor(pkg, "g.k", Q4_K, 128, h, 2)
    tv, _ = make_tensor(pkg, "g.v", Q6_K, 128, h, 3)
    for t in (tq, tk, tv):
        gpu_ctx.upload_tensor(t)
    x = rvec(h, 4)
    gpu_ctx.slot_upload(1, x)
    gpu_ctx.slot_matvec3(3, tq, 4, tk, 5, tv, 1)
    xq = O.q8_1_quantize(x)
    for slot, t in ((3, tq), (4, tk), (5, tv)):
        assert np.array_equal(gpu_ctx.slot_download(slot, t.rows), O.matvec_q8_1_dev(t.dtype, t.data, t.rows, h, xq))
    gpu_ctx.slot_matvec2(6, tk, 7, tv, 1)
    assert np.array_equal(gpu_ctx.slot_download(7, tv.rows), O.matvec_q8_1_dev(Q6_K, tv.data, tv.rows, h, xq))


# -------------------------------------------------------------- slot ops
def test_slot_norms_rope_bit_exact(pkg, gpu_ctx, O):
    from minicpmo_b200 import gguf
    from minicpmo_b200.gpu import Tensor

    heads, hd, ctx, pos = 6, 128, 32, 17
    w32 = torch.randn((1, hd), generator=torch.Generator().manual_seed(3)) * 0.02 + 1.0
    w = Tensor("hn", gguf.quantize(w32, F32).numpy(), F32, 1, hd)
    gpu_ctx.upload_tensor(w)
    wf = w.data.view(np.float32).reshape(-1)
    v = rvec(heads * hd, 21, 2.0)
    gpu_ctx.slot_upload(2, v)
    gpu_ctx.slot_head_norm(2, w, heads, hd)
    ref = O.head_norm(v, wf, heads, hd, 0, order=1)
    assert np.array_equal(gpu_ctx.slot_download(2, heads * hd), ref)
    cos_t, sin_t = O.rope_table(ctx, hd, 1e6, 1.0)
    gpu_ctx.slot_rope(2, heads, hd, pos, 1e6, 1.0, cos_t, sin_t, ctx)
    assert np.array_equal(gpu_ctx.slot_download(2, heads * hd), O.rope_apply(ref, heads, hd, pos, cos_t, sin_t))
    # big RMSNorm through the slot API
    hw32 = torch.randn((1, 2048), generator=torch.Generator().manual_seed(4)) * 0.02 + 1.0
    hwt = Tensor("rms2048", gguf.quantize(hw32, F32).numpy(), F32, 1, 2048)
    gpu_ctx.upload_tensor(hwt)
    x = rvec(2048, 5)
    gpu_ctx.slot_upload(8, x)
    gpu_ctx.slot_rms_norm(9, 8, hwt, 2048, 1e-6)
    assert np.array_equal(gpu_ctx.slot_download(9, 2048), O.rms_norm(x, hwt.data.view(np.float32).reshape(-1), 0, 1e-6, 1))


def test_slot_add_silu(gpu_ctx, O):
    g, u = rvec(3000, 1, 4.0), rvec(3000, 2)
    gpu_ctx.slot_upload(10, g)
    gpu_ctx.slot_upload(11, u)
    gpu_ctx.slot_silu_mul(12, 10, 11, 3000)
    out = gpu_ctx.slot_download(12, 3000)
    assert np.array_equal(out, O.silu_mul_dev(g, u))
    assert np.allclose(out, O.silu_mul(g, u), rtol=4e-7 * 4, atol=1e-30)  # within a few ulp of libm expf
    gpu_ctx.slot_add_inplace(10, 11, 3000)
    assert np.array_equal(gpu_ctx.slot_download(10, 3000), g + u)


@pytest.mark.parametrize("heads,kv,hd", [(16, 8, 128), (32, 8, 128), (2, 1, 4), (8, 2, 64), (4, 4, 256)])
def test_attention_slots_vs_oracle(gpu_ctx, O, heads, kv, hd):
    ctx, layers = 300, 2
    kvd = kv * hd
    gpu_ctx.prepare_attention(layers, ctx, kvd)
    kc = np.zeros((layers, ctx, kvd), np.float32)
    vc = np.zeros_like(kc)
    rng = np.random.Generator(np.random.PCG64(heads * hd))
    layer = 1
    for pos in range(0, 260):
        k = rng.standard_normal(kvd).astype(np.float32)
        v = rng.standard_normal(kvd).astype(np.float32)
        kc[layer, pos], vc[layer, pos] = k, v
        if pos in (0, 1, 31, 32, 33, 150, 259):
            q = rng.standard_normal(heads * hd).astype(np.float32)
            gpu_ctx.slot_upload(0, q)
            gpu_ctx.slot_upload(1, k)
            gpu_ctx.slot_upload(2, v)
            gpu_ctx.attention_slots(3, 0, 1, 2, layer, pos, heads, kv, hd, ctx)
            out = gpu_ctx.slot_download(3, heads * hd)
            dev = O.attention_dev(q, kc, vc, kc[layer, pos], vc[layer, pos], layer, pos, heads, kv, hd, ctx)
            assert np.array_equal(out, dev), (pos, np.abs(out - dev).max())
            ref = O.attention(q, kc, vc, layer, pos, heads, kv, hd, ctx)
            assert np.allclose(out, ref, rtol=1e-4, atol=1e-5), (pos, np.abs(out - ref).max())
        else:
            # host-buffer entry point appends too (gpu_shim.c:1456-1590)
            q = rng.standard_normal(heads * hd).astype(np.float32)
            out = gpu_ctx.attention(q, k, v, layer, pos, heads, kv, hd, ctx)
            if pos % 64 == 5:
                dev = O.attention_dev(q, kc, vc, kc[layer, pos], vc[layer, pos], layer, pos, heads, kv, hd, ctx)
                assert np.array_equal(out, dev)


@pytest.mark.parametrize("dt,rows,cols", [(Q6_K, 64, 1024), (Q4_K, 50, 512), (Q8_0, 33, 768), (F16, 20, 96), (F32, 9, 40)])
def test_embed_lookup_bit_exact(pkg, gpu_ctx, O, dt, rows, cols):
    t, _ = make_tensor(pkg, f"emb{dt}", dt, rows, cols, seed=dt * 3)
    gpu_ctx.upload_tensor(t)
    deq = O.dequant(dt, t.data, rows, cols)
    for tok in (0, 1, rows // 2, rows - 1):
        gpu_ctx.embed_lookup(13, t, tok)
        assert np.array_equal(gpu_ctx.slot_download(13, cols), deq[tok])


def test_argmax_penalized(gpu_ctx, O):
    n = 151936
    v = rvec(n, 77)
    v[1234] = v[99999] = 9.0  # tie: the first index wins (qwen3.uya:1748 strict >)
    gpu_ctx.slot_upload(14, v)
    tok, gap = gpu_ctx.argmax_penalized(14, n)
    rt, rg = O.argmax_penalized(v)
    assert (tok, gap) == (rt, rg) == (1234, 0.0)
    seen = [1234, 99999, 5, 17]
    for pen in (1.0, 1.3):
        tok, gap = gpu_ctx.argmax_penalized(14, n, seen, pen)
        rt, rg = O.argmax_penalized(v, seen, pen)
        assert tok == rt and gap == pytest.approx(rg, abs=0)


def test_error_paths(pkg, gpu_ctx):
    from minicpmo_b200.gpu import GpuError, Tensor

    with pytest.raises(GpuError, match="invalid gpu slot"):
        gpu_ctx.slot_download(16, 4)
    bad = Tensor("bad", np.zeros(10, np.uint8), Q4_K, 1, 100)
    with pytest.raises(GpuError, match="multiple of 256"):
        gpu_ctx.upload_tensor(bad)
    missing = Tensor("missing", np.zeros(144, np.uint8), Q4_K, 1, 256)
    with pytest.raises(GpuError, match="not uploaded"):
        gpu_ctx.matvec(missing, np.zeros(256, np.float32))
    with pytest.raises(GpuError, match="cache shape mismatch|not prepared|slots not ready"):
        gpu_ctx.attention_slots(0, 1, 2, 3, 99, 0, 2, 1, 4, 300)
    gpu_ctx.smoke()
