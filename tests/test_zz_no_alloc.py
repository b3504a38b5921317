"""minicpmo_gpu_attention_no_alloc (decode attention with a static device
scratch array, no allocation) against the context entry point
minicpmo_gpu_context_attention on the same cache and query.

The file name sorts last so that, in a full run, the entry is also exercised
after every other GPU test has run in the same process; it passes alone too.
Both entries launch the same kernel with the same split count, so the
tolerance below is expected to hold with zero difference."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import rel_row_err

TOL = 1e-6  # max |diff| / ||ref||_2 per call

CASES = [(32, 8, 128, 300), (16, 16, 64, 40), (8, 2, 256, 700), (4, 1, 32, 5), (64, 8, 128, 1023)]


def _call(lib, q, kc, vc, pos, heads, kv, hd, ctx, out, stream):
    err = ctypes.create_string_buffer(512)
    ok = lib.minicpmo_gpu_attention_no_alloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), 0, pos, heads, kv, hd, ctx,
                                             out.data_ptr(), stream, err, 512)
    assert ok == 1, err.value.decode()


@pytest.mark.gpu
@pytest.mark.parametrize("heads,kv,hd,pos", CASES)
def test_no_alloc_matches_context_entry(gpu_ctx, heads, kv, hd, pos):
    import torch

    ctx, kvd = pos + 1, kv * hd
    gpu_ctx.prepare_attention(1, ctx, kvd)
    rng = np.random.Generator(np.random.PCG64(heads * 1000 + pos))
    kc = rng.standard_normal((ctx, kvd), dtype=np.float32)
    vc = rng.standard_normal((ctx, kvd), dtype=np.float32)
    q = rng.standard_normal(heads * hd, dtype=np.float32)
    # the context entry appends row t at position t; the last call attends
    for t in range(pos + 1):
        ref = gpu_ctx.attention(q, kc[t], vc[t], 0, t, heads, kv, hd, ctx)

    dev = torch.device("cuda", 0)
    q_d = torch.from_numpy(q).to(dev)
    kc_d = torch.from_numpy(kc).to(dev)
    vc_d = torch.from_numpy(vc).to(dev)
    stream = torch.cuda.current_stream(dev)
    lib = gpu_ctx.lib
    for _ in range(2):  # two calls in a row: the counters must be clear again
        out_d = torch.full((heads * hd,), float("nan"), dtype=torch.float32, device=dev)
        _call(lib, q_d, kc_d, vc_d, pos, heads, kv, hd, ctx, out_d, ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()
        out = out_d.cpu().numpy()
        assert np.isfinite(out).all()
        assert rel_row_err(out, ref) <= TOL, rel_row_err(out, ref)
