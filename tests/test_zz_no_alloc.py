"""minicpmo_gpu_attention_no_alloc: decode attention for callers that cannot
allocate device memory while they run (a serving loop that reserved all of
its memory up front, a host whose device memory belongs to its own pool).
Its split-K scratch is a static device array instead of allocated memory.

Checked through the C ABI, two calls in a row each (the counters in the
shared scratch must be clear again for the second call):

* f32 cache: bit-identical to the context entry point
  minicpmo_gpu_context_attention on the same cache and query (both launch
  the same kernel with the same split count and merge order);
* f32 and f16 caches: bit-identical to the oracle's device-order attention
  (an f16 cache is the f32 oracle cache rounded to f16 and widened back).

The file name sorts last so that, in a full run, the entry is also exercised
after every other GPU test has run in the same process; it passes alone too.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import rel_row_err

CASES = [(32, 8, 128, 300), (16, 16, 64, 40), (8, 2, 256, 700), (4, 1, 32, 5), (64, 8, 128, 1023)]
F16_CASES = [(32, 8, 128, 300), (8, 2, 64, 129), (4, 1, 32, 5), (6, 2, 16, 70)]


def _call(lib, q, kc, vc, kv_f16, pos, heads, kv, hd, ctx, out, stream):
    err = ctypes.create_string_buffer(512)
    ok = lib.minicpmo_gpu_attention_no_alloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kv_f16, pos, heads, kv, hd,
                                             ctx, out.data_ptr(), stream, err, 512)
    assert ok == 1, err.value.decode()


def _run_twice(lib, q, kc, vc, kv_f16, pos, heads, kv, hd, ctx):
    import torch

    dev = torch.device("cuda", 0)
    q_d = torch.from_numpy(q).to(dev)
    kc_d = torch.from_numpy(kc).to(dev)
    vc_d = torch.from_numpy(vc).to(dev)
    stream = torch.cuda.current_stream(dev)
    outs = []
    for _ in range(2):
        out_d = torch.full((heads * hd,), float("nan"), dtype=torch.float32, device=dev)
        _call(lib, q_d, kc_d, vc_d, kv_f16, pos, heads, kv, hd, ctx, out_d, ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()
        outs.append(out_d.cpu().numpy())
    return outs


@pytest.mark.gpu
@pytest.mark.parametrize("heads,kv,hd,pos", CASES)
def test_no_alloc_matches_context_entry(gpu_ctx, O, heads, kv, hd, pos):
    ctx, kvd = pos + 1, kv * hd
    gpu_ctx.prepare_attention(1, ctx, kvd)
    rng = np.random.Generator(np.random.PCG64(heads * 1000 + pos))
    kc = rng.standard_normal((ctx, kvd), dtype=np.float32)
    vc = rng.standard_normal((ctx, kvd), dtype=np.float32)
    q = rng.standard_normal(heads * hd, dtype=np.float32)
    # the context entry appends row t at position t; the last call attends
    for t in range(pos + 1):
        ref = gpu_ctx.attention(q, kc[t], vc[t], 0, t, heads, kv, hd, ctx)
    dev_ref = O.attention_dev(q, kc[None], vc[None], kc[pos], vc[pos], 0, pos, heads, kv, hd, ctx)
    for out in _run_twice(gpu_ctx.lib, q, kc, vc, 0, pos, heads, kv, hd, ctx):
        assert np.isfinite(out).all()
        assert np.array_equal(out, ref), rel_row_err(out, ref)
        assert np.array_equal(out, dev_ref), rel_row_err(out, dev_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("heads,kv,hd,pos", F16_CASES)
def test_no_alloc_f16_cache_matches_oracle(gpu_ctx, O, heads, kv, hd, pos):
    ctx, kvd = pos + 1, kv * hd
    rng = np.random.Generator(np.random.PCG64(heads * 77 + pos + hd))
    kc16 = rng.standard_normal((ctx, kvd), dtype=np.float32).astype(np.float16)
    vc16 = rng.standard_normal((ctx, kvd), dtype=np.float32).astype(np.float16)
    q = rng.standard_normal(heads * hd, dtype=np.float32)
    kc, vc = kc16.astype(np.float32), vc16.astype(np.float32)
    dev_ref = O.attention_dev(q, kc[None], vc[None], kc[pos], vc[pos], 0, pos, heads, kv, hd, ctx)
    nat = O.attention(q, kc[None], vc[None], 0, pos, heads, kv, hd, ctx)
    for out in _run_twice(gpu_ctx.lib, q, kc16, vc16, 1, pos, heads, kv, hd, ctx):
        assert np.isfinite(out).all()
        assert np.array_equal(out, dev_ref), rel_row_err(out, dev_ref)
        assert rel_row_err(out, nat) < 1e-5
