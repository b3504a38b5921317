"""Pins the CPU oracle to the reference before it is trusted as a checker.

1. Known-answer tests of the reference's own self-tests
   (src/minicpmo/kernels.uya:264-326 kernels_smoke, 749-852 quant_smoke).
2. Golden vectors produced by the reference's code (tests/golden/make_golden.py).
3. Live comparison with the reference builds in oracle/_ref/ when present.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import rel_row_err

Q4_K, Q6_K, Q8_0 = 10, 12, 6


# ---------------------------------------------------------------- 1. KATs
def test_f16_known_answers(O):
    # kernels.uya:278-279, 325
    assert O.f16_to_f32(0x3C00) == 1.0
    assert O.f16_to_f32(0xC000) == -2.0
    assert math.isnan(O.f16_to_f32(0x7E00))
    assert O.f16_to_f32(0x7C00) > 1e6
    assert O.f32_to_f16(1.0) == 0x3C00
    assert O.f32_to_f16(-2.0) == 0xC000


def test_rms_norm_known_answer(O):
    # kernels.uya:283-284: rms_norm([1,2,3,4], w=1, eps=0)[0] ~ 0.365148
    x = np.array([1, 2, 3, 4], np.float32)
    w = np.ones(4, np.float32)
    for order in (0, 1):
        y = O.rms_norm(x, w, 0, eps=0.0, order=order)
        assert abs(y[0] - 0.365148) < 1e-3


def test_rope_known_answer(O):
    # kernels.uya:289-290: rotating (1, 0) by pi/2 gives (0, 1)
    cos_t = np.array([math.cos(1.5707963)], np.float32)
    sin_t = np.array([math.sin(1.5707963)], np.float32)
    v = O.rope_apply(np.array([1.0, 0.0], np.float32), 1, 2, 0, cos_t, sin_t)
    assert abs(v[0]) < 1e-3 and abs(v[1] - 1.0) < 1e-3


def test_softmax_through_attention(O):
    # kernels.uya:291-294: softmax of [1, 2, 3] sums to 1 and is increasing.
    # One head, head_dim 1, k = scores*sqrt(1), v = one-hot positions.
    ctx = 3
    kc = np.array([1.0, 2.0, 3.0], np.float32)
    out = []
    for t in range(3):
        vc = np.zeros(3, np.float32)
        vc[t] = 1.0
        out.append(O.attention(np.array([1.0], np.float32), kc, vc, 0, 2, 1, 1, 1, ctx)[0])
    assert abs(sum(out) - 1.0) < 1e-6 and out[2] > out[1] > out[0]


def _pack_nibble(buf, i, v):
    b = i // 2
    buf[b] = (buf[b] & 0xF0) | (v & 15) if i % 2 == 0 else (buf[b] & 0x0F) | ((v & 15) << 4)


def quant_smoke_blocks(O):
    """The constructed blocks of quant_smoke_cli (kernels.uya:784-831)."""
    x = np.array([(i % 7) - 3 for i in range(256)], np.float32)
    q4 = np.zeros(144, np.uint8)
    q4[0:2] = np.frombuffer(np.uint16(O.f32_to_f16(0.0625)).tobytes(), np.uint8)
    q4[2:4] = np.frombuffer(np.uint16(O.f32_to_f16(0.03125)).tobytes(), np.uint8)
    sc = [3 + i for i in range(8)]
    mn = [1 + (i % 5) for i in range(8)]
    for i in range(4):  # q4_k_pack_scales_mins (kernels.uya:401-409)
        q4[4 + i] = (sc[i] & 63) | (((sc[i + 4] >> 4) & 3) << 6)
        q4[4 + i + 4] = (mn[i] & 63) | (((mn[i + 4] >> 4) & 3) << 6)
        q4[4 + i + 8] = (sc[i + 4] & 15) | ((mn[i + 4] & 15) << 4)
    qs = np.zeros(128, np.uint8)
    for i in range(256):
        _pack_nibble(qs, i, (i * 3 + 5) % 16)
    q4[16:] = qs
    q6 = np.zeros(210, np.uint8)
    q6[208:210] = np.frombuffer(np.uint16(O.f32_to_f16(0.125)).tobytes(), np.uint8)
    for i in range(128):
        q6[i] = ((i + 3) % 16) | (((i * 5) % 16) << 4)
    for i in range(64):
        q6[128 + i] = ((i + 1) % 4) | (((i + 2) % 4) << 2) | (((i + 3) % 4) << 4) | (((i + 0) % 4) << 6)
    for i in range(16):
        q6[192 + i] = np.uint8(np.int8((i % 11) - 5))
    return x, q4, q6


def test_quant_smoke_blocks(O):
    # kernels.uya:832-840: Q8_1 x K-quant dot within 0.05 of dequant . dequant(Q8_1)
    x, q4, q6 = quant_smoke_blocks(O)
    xq = O.q8_1_quantize(x)
    xd = np.array([O.f16_to_f32(int(xq[b * 36]) | (int(xq[b * 36 + 1]) << 8)) * np.int8(xq[b * 36 + 4 + i])
                   for b in range(8) for i in range(32)], np.float32)
    for dt, blk in ((Q4_K, q4), (Q6_K, q6)):
        y = O.matvec_q8_1(dt, blk, 1, 256, xq)[0]
        ref = float(np.dot(O.dequant(dt, blk, 1, 256)[0].astype(np.float64), xd))
        assert abs(y - ref) < 0.05, (dt, y, ref)


# ------------------------------------------------------- 2. golden vectors
def test_f16_rounding_golden(O, golden):
    f, bits = golden["f16_inputs"], golden["f16_bits"]
    mine = np.array([O.f32_to_f16(float(v)) for v in f], np.uint16)
    assert np.array_equal(mine, bits)


def test_q8_1_quantize_golden(O, golden):
    assert np.array_equal(O.q8_1_quantize(golden["q8_1_inputs"]), golden["q8_1_bytes"])


@pytest.mark.parametrize("name,dt", [("q4_k", Q4_K), ("q6_k", Q6_K)])
def test_kquant_matvec_golden(O, golden, name, dt):
    w, x = golden[f"w_{name}"], golden["mv_x"]
    xq = O.q8_1_quantize(x)
    y = O.matvec_q8_1(dt, w, w.shape[0], x.size, xq)
    # the reference kernel sums in its own thread/tree order: tolerance, not bits
    assert rel_row_err(y, golden[f"kq_y_{name}"]) < 1e-5
    # the integer part is exact: recompute each row from the oracle's block dots
    dots = O.block_dots(dt, w, w.shape[0], x.size, xq)
    assert dots.shape[0] == w.shape[0]


@pytest.mark.parametrize("name,dt", [("q4_k", Q4_K), ("q6_k", Q6_K), ("q8_0", Q8_0)])
def test_cpu_f32_matvec_golden(O, golden, name, dt):
    w, x = golden[f"w_{name}"], golden["mv_x"]
    y = O.matvec_f32(dt, w, w.shape[0], x.size, x)
    assert rel_row_err(y, golden[f"cpu_y_{name}"]) < 1e-5


def test_rope_golden(O, golden):
    v = O.rope_apply(golden["rope_in"], 3, 128, 11, golden["rope_cos"], golden["rope_sin"])
    assert np.array_equal(v, golden["rope_out"])  # same mul/sub sequence: bit-exact


def test_silu_golden(O, golden):
    assert np.array_equal(O.silu_mul(golden["silu_g"], golden["silu_u"]), golden["silu_out"])


# ------------------------------------------- 3. live reference (oracle/_ref)
def _need(O, name):
    if O.ref_lib(name) is None:
        pytest.skip(f"oracle/_ref/libref_{name}.so not built (reference tree absent)")


def test_q8_1_live_vs_reference_shim(O):
    _need(O, "shim")
    rng = np.random.Generator(np.random.PCG64(3))
    for scale in (1e-6, 1e-2, 1.0, 300.0):
        x = (rng.standard_normal(2048) * scale).astype(np.float32)
        assert np.array_equal(O.q8_1_quantize(x), O.ref_shim_q8_1(x))


@pytest.mark.parametrize("dt", [Q4_K, Q6_K])
def test_kquant_live_vs_reference_kernels(O, pkg, dt):
    _need(O, "kernels")
    import torch
    from minicpmo_b200 import gguf

    rows, cols = 40, 1536
    w = gguf.quantize(torch.randn((rows, cols), generator=torch.Generator().manual_seed(dt)) * 0.02, dt).numpy()
    x = np.random.Generator(np.random.PCG64(dt)).standard_normal(cols).astype(np.float32)
    xq = O.q8_1_quantize(x)
    assert rel_row_err(O.matvec_q8_1(dt, w, rows, cols, xq), O.ref_kernel_matvec(dt, w, rows, cols, xq)) < 1e-5


@pytest.mark.parametrize("dt", [Q4_K, Q6_K, Q8_0])
def test_cpu_matvec_live_vs_reference(O, pkg, dt):
    _need(O, "cpu")
    import torch
    from minicpmo_b200 import gguf

    rows, cols = 33, 1024
    w = gguf.quantize(torch.randn((rows, cols), generator=torch.Generator().manual_seed(7)) * 0.02, dt).numpy()
    x = np.random.Generator(np.random.PCG64(8)).standard_normal(cols).astype(np.float32)
    assert rel_row_err(O.matvec_f32(dt, w, rows, cols, x), O.ref_cpu_matvec(dt, w, rows, cols, x)) < 1e-5


# ------------------------------------------- 4. deterministic exp accuracy
def test_expf_det_accuracy(O):
    """orc_expf_det (shared by the kernels) stays within 2 ulp of libm expf."""
    xs = np.concatenate([np.linspace(-103.9, 88.7, 20001, dtype=np.float32),
                         np.random.Generator(np.random.PCG64(1)).uniform(-20, 20, 20000).astype(np.float32),
                         np.array([0.0, -0.0, 1e-30, -1e-30, 88.72, -87.3, -100.0], np.float32)])
    got = O.expf_det(xs)
    ref = np.exp(xs.astype(np.float64))
    ok = ref > np.finfo(np.float32).tiny
    ulp = np.spacing(ref[ok].astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(got[ok] - ref[ok]) / ulp) <= 2.0
    assert O.expf_det(np.array([-np.inf]))[0] == 0.0 and np.isinf(O.expf_det(np.array([np.inf]))[0])


def test_pooled_q8_1_oracle_matches_single_thread(O):
    """The row pool used for the full-shape parity tests gives the bits of the
    single-threaded oracle in both evaluation orders."""
    from conftest import load_pkg

    load_pkg()
    from minicpmo_b200 import gguf

    shape = gguf.Qwen3Shape(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=64, ffn=1536, vocab=2048, context=16)
    tensors = gguf.synth_model(shape, gguf.Q4_K_M)
    tmap = {n: (dt, r, c, d) for n, dt, r, c, d in tensors}
    for order in (True, False):
        one = O.OracleModel(shape, tmap, 16, q8_1=True, device_order=order)
        many = O.OracleModel(shape, tmap, 16, q8_1=True, device_order=order, pool_threads=3)
        for pos, tok in enumerate((3, 1000, 77)):
            a, _ = one.forward(tok, pos)
            b, _ = many.forward(tok, pos)
            assert np.array_equal(a, b), (order, pos)
        one.close()
        many.close()


# ------------------------------------- 2b. norm and attention kernel bodies
def test_rms_norm_pinned_to_reference_kernel(O, golden):
    """gpu_shim.c:694-718 run on the host (256 threads, phases at __syncthreads):
    the device-order RMSNorm restatement gives its bits (rsqrtf taken as 1/sqrtf)."""
    y = O.rms_norm(golden["rms_x"], golden["rms_w"], 0, 1e-6, order=1)
    assert np.array_equal(y, golden["rms_out"])
    # the reference CPU order (sequential sum) within a few ulp
    assert rel_row_err(O.rms_norm(golden["rms_x"], golden["rms_w"], 0, 1e-6, order=0), golden["rms_out"]) < 1e-6


def test_head_norm_pinned_to_reference_kernel(O, golden):
    """gpu_shim.c:719-745, one 256-thread block per head."""
    heads, hd = 6, 128
    y = O.head_norm(golden["hn_in"], golden["hn_w"], heads, hd, 0, order=1)
    assert np.array_equal(y, golden["hn_out"])
    assert rel_row_err(O.head_norm(golden["hn_in"], golden["hn_w"], heads, hd, 0, order=0), golden["hn_out"]) < 1e-6


def test_attention_pinned_to_reference_kernel(O, golden):
    """gpu_shim.c:926-979 (online softmax per position, 256-thread dot trees):
    the natural-order and device-order attention restatements within 1e-5."""
    layers, ctx, heads, kv, hd, pos = (int(v) for v in golden["att_shape"])
    assert golden["att_scale"][0] == np.float32(1.0) / np.float32(np.sqrt(np.float32(hd)))
    kc, vc = golden["att_k"], golden["att_v"]
    ref = golden["att_out"]
    nat = O.attention(golden["att_q"], kc, vc, 1, pos, heads, kv, hd, ctx)
    dev = O.attention_dev(golden["att_q"], kc, vc, kc[1, pos], vc[1, pos], 1, pos, heads, kv, hd, ctx)
    assert rel_row_err(nat, ref) < 1e-5
    assert rel_row_err(dev, ref) < 1e-5


def test_norm_and_attention_kernels_live(O):
    """The same pins on fresh inputs when oracle/_ref is built here."""
    K = O.ref_lib("kernels")
    if K is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.Generator(np.random.PCG64(4242))
    for n in (1024, 5120, 12288):
        x = (rng.standard_normal(n) * 2).astype(np.float32)
        w = (1 + rng.standard_normal(n) * 0.02).astype(np.float32)
        out = np.empty(n, np.float32)
        K.refk_rms_norm(out.ctypes.data_as(O.fp), x.ctypes.data_as(O.fp), w.view(np.uint8).ctypes.data_as(O.u8p), 0,
                        n, 1e-6)
        assert np.array_equal(O.rms_norm(x, w, 0, 1e-6, order=1), out), n
    layers, ctx, heads, kv, hd = 1, 40, 4, 1, 64
    q = rng.standard_normal(heads * hd).astype(np.float32)
    kc = rng.standard_normal((layers, ctx, kv * hd)).astype(np.float32)
    vc = rng.standard_normal((layers, ctx, kv * hd)).astype(np.float32)
    for pos in (0, 31, 39):
        out = np.empty(heads * hd, np.float32)
        scale = float(np.float32(1.0) / np.float32(np.sqrt(np.float32(hd))))
        K.refk_attention_decode(q.ctypes.data_as(O.fp), kc.ctypes.data_as(O.fp), vc.ctypes.data_as(O.fp),
                                out.ctypes.data_as(O.fp), 0, pos, heads, kv, hd, ctx, scale)
        assert rel_row_err(O.attention(q, kc, vc, 0, pos, heads, kv, hd, ctx), out) < 1e-5
