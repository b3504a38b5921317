"""Batched decode of independent sequences (all linear weights Q8_0, the
projections on the tensor cores) against the reference's CPU path
(OracleModel q8_1=False: Q8_0 x f32, qwen3.uya:1200-1231), one oracle per
sequence, teacher-forced; sequences run at different positions.  With
batch_exact the batch runs its projections as the prompt prefill does and
equals the single-sequence decode bit for bit.

The default projections round weights and activations to f16 (relative
2^-11); the exact mode quantises activations to Q8_1 as the reference's GPU
arithmetic does.  Logits differ from the f32-activation reference by up to
~1e-3 of their norm; LOGIT_TOL bounds that.  Greedy tokens must match
wherever the reference's top-2 gap exceeds TOKEN_GAP and twice the step's
largest logit difference (a smaller gap can flip on that difference alone),
as for the single-sequence decode (test_gpu_baseline_shapes.py)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_row_err

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3
TOKEN_GAP = 1e-3  # the north star: identical greedy tokens wherever the top-2 gap exceeds 1e-3


def small_shape(**kw):
    from minicpmo_b200 import gguf

    d = dict(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1536, vocab=2048, context=64)
    d.update(kw)
    return gguf.Qwen3Shape(**d)


@pytest.mark.parametrize("kv_f16,B,exact", [(False, 4, False), (True, 3, False), (True, 17, False), (False, 4, True)])
def test_batched_decode_vs_reference_cpu(pkg, O, kv_f16, B, exact):
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape()
    tensors = gguf.synth_model(shape, gguf.ALL_Q8_0, seed_base=5)
    tmap = {n: (dt, r, c, d) for n, dt, r, c, d in tensors}
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16, max_batch=B, batch_exact=exact)
    assert rt.gpu.qwen3_batch_kernels(True) > 0
    check = list(range(min(B, 4)))  # sequences compared against an oracle (CPU time)
    oracles = {b: O.OracleModel(shape, tmap, shape.context, q8_1=False) for b in check}
    steps = 24
    ids = np.stack([gguf.prompt_ids(steps, shape.vocab, seed=11 + b) for b in range(B)]).astype(np.uint32)
    lag = np.arange(B) % 3  # sequence b starts lag[b] steps late: positions differ across the batch
    worst, compared, flips = 0.0, 0, 0
    for i in range(steps + 2):
        pos = i - lag
        live = (pos >= 0) & (pos < steps)
        tok = np.where(live, ids[np.arange(B), np.clip(pos, 0, steps - 1)], 0).astype(np.uint32)
        p = np.clip(pos, 0, steps - 1).astype(np.uint32)
        nxt, gaps, lg = rt.forward_batch(tok, p, logits=True, want_logits=True)
        assert np.isfinite(lg).all()
        for b in check:
            if not live[b]:
                continue
            ref, _ = oracles[b].forward(int(tok[b]), int(p[b]))
            worst = max(worst, rel_row_err(lg[b], ref))
            dmax = float(np.max(np.abs(lg[b].astype(np.float64) - ref)))
            t_ref, g_ref = O.argmax_penalized(ref)
            compared += 1
            if g_ref > max(TOKEN_GAP, 2 * dmax):
                assert nxt[b] == t_ref, (i, b, g_ref, dmax)
            elif nxt[b] != t_ref:
                flips += 1
    print(f"[batch] B={B} kv_f16={kv_f16}: {compared} steps compared, worst logit err {worst:.2e}, "
          f"near-tie flips {flips}")
    assert worst < LOGIT_TOL
    for o in oracles.values():
        o.close()
    rt.close()


@pytest.mark.parametrize("kv_f16,B", [(False, 3), (True, 5)])
def test_batched_decode_equals_single_sequence(pkg, kv_f16, B):
    """Each sequence of the batch gets the logits, tokens and gaps of its own
    single-sequence runtime bit for bit: the batch's projections run on the
    tensor-core prefill path, whose dots and float order are the decode
    GEMV's, and its attention merges blocks in the same order."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape()
    tensors = gguf.synth_model(shape, gguf.ALL_Q8_0, seed_base=9)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16, max_batch=B, batch_exact=True)
    # embed; per layer 4 activation operands, 7 projections and the attention; final norm, lm_head, sampler
    assert rt.gpu.qwen3_batch_kernels(True) == 1 + 12 * shape.layers + 3
    singles = [Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16) for _ in range(B)]
    steps = 20
    ids = np.stack([gguf.prompt_ids(steps, shape.vocab, seed=40 + b) for b in range(B)]).astype(np.uint32)
    lag = np.arange(B) % 3
    one = np.empty(shape.vocab, np.float32)
    for i in range(steps + 2):
        pos = i - lag
        live = (pos >= 0) & (pos < steps)
        tok = np.where(live, ids[np.arange(B), np.clip(pos, 0, steps - 1)], 0).astype(np.uint32)
        p = np.clip(pos, 0, steps - 1).astype(np.uint32)
        nxt, gaps, lg = rt.forward_batch(tok, p, logits=True, want_logits=True)
        for b in range(B):
            if not live[b]:
                continue
            t1, g1 = singles[b].forward(int(tok[b]), int(p[b]), want_logits=one)
            assert np.array_equal(lg[b], one), (i, b, rel_row_err(lg[b], one))
            assert (int(nxt[b]), float(gaps[b])) == (t1, g1), (i, b)
    for r in singles:
        r.close()
    rt.close()


def test_decode_batch_matches_host_loop(pkg):
    """The device loop (sampled tokens fed back on the GPU) gives the tokens of
    the host loop over forward_batch: same kernels, deterministic sums."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape(context=48)
    tensors = gguf.synth_model(shape, gguf.ALL_Q8_0, seed_base=6)
    B, P, n = 5, 8, 12
    prompts = np.stack([gguf.prompt_ids(P, shape.vocab, seed=30 + b) for b in range(B)])
    a = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=True, max_batch=B)
    a.append_prompt_batch(prompts)
    dev = a.generate_batch(n)
    a.close()
    b = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=True, max_batch=B)
    nxt, _ = b.append_prompt_batch(prompts)
    host = [nxt.copy()]
    for i in range(n - 1):
        nxt, _, _ = b.forward_batch(nxt, np.full(B, P + i, np.uint32))
        host.append(nxt.copy())
    b.close()
    assert np.array_equal(dev, np.stack(host, axis=1))


def test_batch_bind_rejects_k_quants(pkg):
    from minicpmo_b200 import gguf
    from minicpmo_b200.gpu import GpuError
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape(layers=1, context=16)
    tensors = gguf.synth_model(shape, gguf.Q4_K_M, seed_base=7)
    with pytest.raises(GpuError):
        Qwen3Runtime.open(tensors, shape=shape, context=shape.context, max_batch=4)
