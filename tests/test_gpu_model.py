"""End-to-end decode parity: the fused whole-token decode step (one CUDA
graph) against the oracle's restatement of the reference forward
(qwen3.uya:1920-1995 with the CUDA path's Q8_1 arithmetic), teacher-forced.

Against the oracle in device evaluation order the logits are bit-identical
at every step, so greedy tokens are identical (a stronger statement than the
BASELINE bar "identical wherever the top-2 gap exceeds 1e-3").  Against the
oracle in the reference's natural summation order the logits agree within
LOGIT_TOL of their L2 norm.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_row_err

pytestmark = pytest.mark.gpu

GAP = 1e-3
# max |dlogit| / ||logits||_2.  The GPU reassociates float sums (matvec,
# attention), which moves activations by ~1e-7 relative; an occasional value
# then lands on the other side of a Q8_1 rounding boundary in the next
# layer's quantisation (one step = amax/127), so logits drift by ~1e-4..1e-3
# of their norm.  Tokens are the contract; logits get this bound.
LOGIT_TOL = 5e-3


def build(pkg, shape, mix, seed=1):
    from minicpmo_b200 import gguf

    return gguf.synth_model(shape, mix, seed_base=seed)


def run_parity(pkg, O, shape, mix, steps, kv_f16=False, seed=1, tol=LOGIT_TOL, decode_mode=0):
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    tensors = build(pkg, shape, mix, seed)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16, decode_mode=decode_mode)
    tmap = {n: (dt, r, c, d) for n, dt, r, c, d in tensors}
    orc = O.OracleModel(shape, tmap, shape.context, q8_1=True, kv_f16=kv_f16)
    nat = O.OracleModel(shape, tmap, shape.context, q8_1=True, device_order=False) if not kv_f16 else None
    ids = gguf.prompt_ids(steps, shape.vocab, seed=7)
    lg = np.empty(shape.vocab, np.float32)
    worst = 0.0
    for pos in range(steps):
        tok_gpu, gap_gpu = rt.forward(int(ids[pos]), pos, logits=True, want_logits=lg)
        ref_logits, _ = orc.forward(int(ids[pos]), pos)
        tok_ref, gap_ref = O.argmax_penalized(ref_logits)
        assert np.array_equal(lg, ref_logits), (pos, rel_row_err(lg, ref_logits))
        assert tok_gpu == tok_ref and gap_gpu == gap_ref, pos
        if nat is not None:
            nat_logits, _ = nat.forward(int(ids[pos]), pos)
            worst = max(worst, rel_row_err(lg, nat_logits))
    rt.close()
    orc.close()
    if nat is not None:
        nat.close()
        print(f"[parity] {shape} steps={steps}: bit-exact; vs natural order worst logit err={worst:.3e}")
        assert worst < tol
    return worst


def small_shape(**kw):
    from minicpmo_b200 import gguf

    d = dict(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1536, vocab=2048, context=96)
    d.update(kw)
    return gguf.Qwen3Shape(**d)


def test_forward_q4_k_m_gqa4(pkg, O):
    from minicpmo_b200 import gguf

    run_parity(pkg, O, small_shape(), gguf.Q4_K_M, steps=40)


def test_forward_tied_06b_layout(pkg, O):
    """0.6B-like head layout (16 q / 8 kv heads, tied Q6_K lm_head)."""
    from minicpmo_b200 import gguf

    run_parity(pkg, O, small_shape(hidden=1024, heads=16, kv_heads=8, ffn=3072, tied=True), gguf.Q4_K_M, steps=24)


def test_forward_q8_0(pkg, O):
    from minicpmo_b200 import gguf

    run_parity(pkg, O, small_shape(layers=3), gguf.ALL_Q8_0, steps=24)


def test_forward_head_dim_64_and_long_positions(pkg, O):
    from minicpmo_b200 import gguf

    # crosses several 32-position attention chunks
    run_parity(pkg, O, small_shape(head_dim=64, heads=8, kv_heads=4, context=160), gguf.Q4_K_M, steps=150)


def test_forward_f16_kv_cache(pkg, O):
    from minicpmo_b200 import gguf

    # f16 KV is a new capability (the reference keeps f32 KV): looser logits bound
    run_parity(pkg, O, small_shape(), gguf.Q4_K_M, steps=32, kv_f16=True, tol=5e-3)


def test_device_decode_matches_host_loop(pkg, O):
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape()
    tensors = build(pkg, shape, gguf.Q4_K_M)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    prompt = gguf.prompt_ids(12, shape.vocab, seed=3)
    rt.append_prompt_ids(prompt)
    host = rt.generate(20)
    rt.reset()
    rt.append_prompt_ids(prompt)
    dev = rt.generate_device(20)
    assert host == dev
    rt.close()


def test_runtime_bench_and_output_lines(pkg, O):
    """Qwen3Runtime.bench (the reference's `bench` loop, qwen3.uya:2774-2973: prompt, then n_gen
    decode steps feeding the seed ids cyclically) and its output lines with the context's stats."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime, format_bench_lines

    shape = small_shape()
    tensors = build(pkg, shape, gguf.Q4_K_M)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    prompt = gguf.prompt_ids(9, shape.vocab, seed=5)
    r = rt.bench(prompt, n_gen=6, repetitions=2)
    assert r["prompt_tokens"] == 18 and r["decode_tokens"] == 12
    assert r["prompt_us"] > 0 and r["decode_us"] > 0 and 0 < r["first_token_us"] <= r["decode_us"]
    assert rt.total_tokens == 9 + 6  # each repetition starts from an empty context
    stats = rt.gpu.snapshot()
    lines = format_bench_lines(r, 2, stats)
    assert lines[0].startswith("bench text_prompt: ") and " units=18 " in lines[0]
    assert lines[1].startswith("bench text_decode: ") and " units=12 " in lines[1]
    assert f"weights_uploaded={stats['uploaded_weight_count']}" in lines[3]
    assert stats["uploaded_weight_count"] >= len(tensors) and lines[-1] == "bench: PASS"
    # the same prompt after bench gives the tokens of a fresh context
    rt.reset()
    a = rt.append_prompt_ids(prompt)
    rt2 = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    assert rt2.append_prompt_ids(prompt) == a
    rt.close()
    rt2.close()


def test_slot_api_forward_matches_fused(pkg, O):
    """Drive the reference's per-op orchestration (qwen3_forward_embedding_runtime_cuda,
    qwen3.uya:1865-1918) through the 19-symbol ABI and compare with the fused step."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.gpu import Tensor
    from minicpmo_b200.qwen3 import Qwen3Runtime, rope_table

    shape = small_shape()
    tensors = build(pkg, shape, gguf.Q4_K_M)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    g = rt.gpu
    T = rt.tensors
    h, qd, kvd, f = shape.hidden, shape.q_dim, shape.kv_dim, shape.ffn
    HID, NRM, Q, K, V, CTX, AO, GATE, UP, FUS, DOWN, LOG = range(12)
    g.prepare_attention(shape.layers, shape.context, kvd)
    cos_t, sin_t = rope_table(shape.context, shape.head_dim, shape.rope_base)
    ids = gguf.prompt_ids(10, shape.vocab, seed=9)
    lg = np.empty(shape.vocab, np.float32)
    emb = T["token_embd.weight"]
    for pos, tok in enumerate(ids):
        g.embed_lookup(HID, emb, int(tok))
        for l in range(shape.layers):
            p = f"blk.{l}."
            g.slot_rms_norm(NRM, HID, T[p + "attn_norm.weight"], h)
            g.slot_matvec3(Q, T[p + "attn_q.weight"], K, T[p + "attn_k.weight"], V, T[p + "attn_v.weight"], NRM)
            g.slot_head_norm(Q, T[p + "attn_q_norm.weight"], shape.heads, shape.head_dim)
            g.slot_head_norm(K, T[p + "attn_k_norm.weight"], shape.kv_heads, shape.head_dim)
            g.slot_rope(Q, shape.heads, shape.head_dim, pos, shape.rope_base, 1.0, cos_t, sin_t, shape.context)
            g.slot_rope(K, shape.kv_heads, shape.head_dim, pos, shape.rope_base, 1.0, cos_t, sin_t, shape.context)
            g.attention_slots(CTX, Q, K, V, l, pos, shape.heads, shape.kv_heads, shape.head_dim, shape.context)
            g.slot_matvec(AO, T[p + "attn_output.weight"], CTX)
            g.slot_add_inplace(HID, AO, h)
            g.slot_rms_norm(NRM, HID, T[p + "ffn_norm.weight"], h)
            g.slot_matvec2(GATE, T[p + "ffn_gate.weight"], UP, T[p + "ffn_up.weight"], NRM)
            g.slot_silu_mul(FUS, GATE, UP, f)
            g.slot_matvec(DOWN, T[p + "ffn_down.weight"], FUS)
            g.slot_add_inplace(HID, DOWN, h)
        g.slot_rms_norm(NRM, HID, T["output_norm.weight"], h)
        g.slot_matvec(LOG, T["output.weight"], NRM)
        slot_logits = g.slot_download(LOG, shape.vocab)
        tok_slot, _ = g.argmax_penalized(LOG, shape.vocab)
        tok_fused, _ = rt.forward(int(tok), pos, logits=True, want_logits=lg)
        # the slot path rounds through the same kernels in the same order
        assert np.array_equal(slot_logits, lg)
        assert tok_slot == tok_fused == int(np.argmax(slot_logits))
    st = g.snapshot()
    assert st["native_quant_matvec_count"] > 0 and st["attention_kernel_calls"] > 0
    rt.close()


@pytest.mark.parametrize("kv_f16", [False, True])
def test_persistent_step_matches_per_kernel_graph(pkg, O, kv_f16):
    """decode_mode 2 (the whole step in one persistent kernel) and decode_mode
    1 (one kernel per operation) give identical logits, tokens and gaps, on
    the 8B attention layout (32 q / 8 kv heads, head_dim 128) far enough into
    the context that attention merges many splits."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape(hidden=512, heads=32, kv_heads=8, head_dim=128, ffn=1024, vocab=1024, context=400)
    tensors = build(pkg, shape, gguf.Q4_K_M, seed=3)
    rt0 = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16, decode_mode=2)
    rt1 = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16, decode_mode=1)
    assert rt0.gpu.qwen3_step_kernels(True) == 4  # embed, seen-set, the step, sampler
    assert rt1.gpu.qwen3_step_kernels(True) > 4 * shape.layers
    ids = gguf.prompt_ids(330, shape.vocab, seed=9)
    l0 = np.empty(shape.vocab, np.float32)
    l1 = np.empty(shape.vocab, np.float32)
    for pos in range(330):
        t0, g0 = rt0.forward(int(ids[pos]), pos, logits=pos % 3 == 0 or pos > 300, want_logits=l0)
        t1, g1 = rt1.forward(int(ids[pos]), pos, logits=pos % 3 == 0 or pos > 300, want_logits=l1)
        if pos % 3 == 0 or pos > 300:
            assert np.array_equal(l0, l1), (pos, rel_row_err(l0, l1))
            assert (t0, g0) == (t1, g1), pos
    # device-side greedy loop from the same state
    a = rt0.gpu.qwen3_decode(int(ids[0]), 330, 40)
    b = rt1.gpu.qwen3_decode(int(ids[0]), 330, 40)
    assert np.array_equal(a, b)
    rt0.close()
    rt1.close()



@pytest.mark.parametrize("mix,kv_f16", [("Q4_K_M", False), ("Q4_K_M", True), ("ALL_Q8_0", False)])
def test_gemv_chain_matches_per_kernel_graph(pkg, O, mix, kv_f16):
    """decode_mode 3 (per layer the attention plus one launch chaining the o,
    gate/up, down and next q/k/v GEMVs through grid barriers) and decode_mode
    1 give identical logits, tokens and gaps, with and without the logits
    (the last layer's chain then ends after its down GEMV), and the same
    device-side greedy loop."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape(layers=3, hidden=512, heads=32, kv_heads=8, head_dim=128, ffn=1024, vocab=1024, context=200)
    tensors = build(pkg, shape, getattr(gguf, mix), seed=4)
    rt3 = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16, decode_mode=3)
    rt1 = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16, decode_mode=1)
    # embed, seen-set, the first q/k/v, per layer attention + chain, sampler
    assert rt3.gpu.qwen3_step_kernels(True) == 3 + 2 * shape.layers + 1
    ids = gguf.prompt_ids(150, shape.vocab, seed=9)
    l3 = np.empty(shape.vocab, np.float32)
    l1 = np.empty(shape.vocab, np.float32)
    for pos in range(150):
        want = pos % 4 == 0 or pos > 140
        t3, g3 = rt3.forward(int(ids[pos]), pos, logits=want, want_logits=l3)
        t1, g1 = rt1.forward(int(ids[pos]), pos, logits=want, want_logits=l1)
        if want:
            assert np.array_equal(l3, l1), (pos, rel_row_err(l3, l1))
            assert (t3, g3) == (t1, g1), pos
    a = rt3.gpu.qwen3_decode(int(ids[0]), 150, 30)
    b = rt1.gpu.qwen3_decode(int(ids[0]), 150, 30)
    assert np.array_equal(a, b)
    rt3.close()
    rt1.close()


def test_gemv_chain_vs_oracle(pkg, O):
    """The chained step against the oracle in device order: bit-identical logits."""
    from minicpmo_b200 import gguf

    run_parity(pkg, O, small_shape(layers=3), gguf.Q4_K_M, steps=24, decode_mode=3)


@pytest.mark.parametrize("mix", ["Q4_K_M", "ALL_Q8_0"])
def test_persistent_step_vs_oracle(pkg, O, mix):
    """The persistent step kernel (both of its weight classes) against the
    oracle in device order: bit-identical logits."""
    from minicpmo_b200 import gguf

    run_parity(pkg, O, small_shape(layers=3), getattr(gguf, mix), steps=24, decode_mode=2)


@pytest.mark.parametrize("decode_mode", [1, 2])
def test_prompt_embeddings_match_oracle(pkg, O, decode_mode):
    """qwen3_append_prompt_embeddings (qwen3.uya:2534-2557): caller-given f32
    rows forwarded in place of token embeddings, interleaved with tokens, give
    logits bit-identical to the oracle's device-order forward on the same
    rows, in the per-operation graph and in the persistent step kernel."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape()
    tensors = build(pkg, shape, gguf.Q4_K_M)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, decode_mode=decode_mode)
    tmap = {n: (dt, r, c, d) for n, dt, r, c, d in tensors}
    orc = O.OracleModel(shape, tmap, shape.context, q8_1=True)
    rng = np.random.default_rng(5)
    ids = gguf.prompt_ids(10, shape.vocab, seed=9)
    lg = np.empty(shape.vocab, np.float32)
    for pos in range(10):
        if pos in (1, 2, 5, 9):
            emb = (rng.standard_normal(shape.hidden) * 0.5).astype(np.float32)
            tok, gap = rt.gpu.qwen3_forward_embedding(emb, 3, pos, want_logits=lg)
            ref, _ = orc.forward_embedding(emb, pos)
        else:
            tok, gap = rt.forward(int(ids[pos]), pos, want_logits=lg)
            ref, _ = orc.forward(int(ids[pos]), pos)
        assert np.array_equal(lg, ref), (pos, rel_row_err(lg, ref))
        tok_ref, gap_ref = O.argmax_penalized(ref)
        assert tok == tok_ref and gap == gap_ref, pos
    rt.close()
    orc.close()


def test_runtime_append_prompt_embeddings(pkg, O):
    """The runtime loop: a span of embedding rows after a token prompt takes
    one position per row, and its last row's logits and greedy token equal
    the oracle's; a wrong row length is refused."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape()
    tensors = build(pkg, shape, gguf.Q4_K_M, seed=2)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    tmap = {n: (dt, r, c, d) for n, dt, r, c, d in tensors}
    orc = O.OracleModel(shape, tmap, shape.context, q8_1=True)
    ids = [int(t) for t in gguf.prompt_ids(4, shape.vocab, seed=3)]
    rt.append_prompt_ids(ids)
    for pos, t in enumerate(ids):
        orc.forward(t, pos, logits=False)
    span = (np.random.default_rng(8).standard_normal((3, shape.hidden)) * 0.3).astype(np.float32)
    lg = np.empty(shape.vocab, np.float32)
    nxt, _ = rt.append_prompt_embeddings(7, span, want_logits=lg)
    assert rt.total_tokens == len(ids) + 3
    for i in range(3):
        ref, _ = orc.forward_embedding(span[i], len(ids) + i, logits=i == 2)
    assert np.array_equal(lg, ref)
    assert nxt == O.argmax_penalized(ref)[0]
    with pytest.raises(RuntimeError):
        rt.gpu.qwen3_forward_embedding(np.zeros(shape.hidden - 1, np.float32), 7, rt.total_tokens)
    rt.close()
    orc.close()


def _sampler_model(pkg, vocab):
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape(vocab=vocab)
    tensors = build(pkg, shape, gguf.Q4_K_M, seed=4)
    return shape, Qwen3Runtime.open(tensors, shape=shape, context=shape.context)


@pytest.mark.parametrize("vocab", [256, 200])
def test_device_sampler_matches_reference_restatement(pkg, O, vocab):
    """qwen3_sample (qwen3.uya:2073-2138) on the device against the oracle's
    restatement, for vocabularies where the reference samples: penalty per
    history entry, temperature, softmax, top-k / top-p / min-p and the
    xorshift32 draw.  Tokens and seed states must agree; the only allowed
    difference is a draw within 1e-5 of a cumulative boundary (CUDA's expf
    and libm's may differ in the last bit)."""
    shape, rt = _sampler_model(pkg, vocab)
    lg = np.empty(shape.vocab, np.float32)
    history = [int(t) for t in np.random.default_rng(3).integers(0, shape.vocab, 12)]
    history += history[:4]  # repeats: the penalty applies once per entry
    settings = [(0.7, 40, 0.9, 0.05, 1.3), (1.0, 0, 1.0, 0.0, 1.0), (1.5, 8, 0.5, 0.0, 1.1), (0.3, 256, 0.95, 0.2, 1.5),
                (0.0, 40, 0.9, 0.0, 1.3), (0.8, 1, 0.9, 0.0, 1.2)]
    seed_gpu = seed_ref = 2463534242
    near = 0
    for pos in range(8):
        rt.forward(int(history[pos]), pos, logits=True, want_logits=lg)
        for temp, k, p, mp, pen in settings:
            tok, seed_gpu = rt.gpu.qwen3_sample(history, temp, k, p, mp, pen, seed_gpu)
            ref, seed_ref, margin = O.sample(lg, history, temp, k, p, mp, pen, seed_ref)
            assert seed_gpu == seed_ref, (pos, temp, k)
            if tok != ref:
                assert margin < 1e-5, (pos, temp, k, tok, ref, margin)
                near += 1
    assert near <= 2
    rt.close()


def test_device_sampler_large_vocab_is_greedy(pkg, O):
    """Above 256 tokens the reference samples greedily whatever the settings:
    the penalised argmax of the last logits, the seed untouched."""
    shape, rt = _sampler_model(pkg, 2048)
    lg = np.empty(shape.vocab, np.float32)
    history = [5, 9, 9, 700]
    for pos, t in enumerate(history):
        rt.forward(t, pos, logits=True, want_logits=lg)
    tok, seed = rt.gpu.qwen3_sample(history, 0.8, 40, 0.9, 0.05, 1.3, 777)
    assert seed == 777
    assert tok == O.argmax_penalized(lg, history, 1.3)[0]
    rt.close()


@pytest.mark.parametrize("decode_mode", [1, 2])
def test_layered_q4_k_m_file_matches_oracle(pkg, O, tmp_path, decode_mode):
    """A model with the per-layer dtype pattern of real llama.cpp Q4_K_M files
    (attn_v / ffn_down Q6_K in some layers, Q4_K in the rest; Q4_K token
    embeddings), written to a GGUF file and loaded from it, decodes with
    logits bit-identical to the oracle in both decode modes."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape(layers=8)
    tensors = gguf.synth_model(shape, gguf.Q4_K_M_LAYERED, seed_base=11)
    path = tmp_path / "layered.gguf"
    gguf.write_gguf(path, gguf.qwen3_metadata(shape), tensors)
    rt = Qwen3Runtime.open(str(path), context=shape.context, decode_mode=decode_mode)
    tmap = {n: (dt, r, c, d) for n, dt, r, c, d in tensors}
    orc = O.OracleModel(shape, tmap, shape.context, q8_1=True)
    ids = gguf.prompt_ids(10, shape.vocab, seed=4)
    lg = np.empty(shape.vocab, np.float32)
    for pos in range(10):
        tok, gap = rt.forward(int(ids[pos]), pos, want_logits=lg)
        ref, _ = orc.forward(int(ids[pos]), pos)
        assert np.array_equal(lg, ref), (pos, rel_row_err(lg, ref))
        assert (tok, gap) == O.argmax_penalized(ref), pos
    rt.close()
    orc.close()


@pytest.mark.parametrize(
    "mix,kv_f16,shape_kw,n_prompt",
    [("Q4_K_M", False, {}, 10), ("Q4_K_M", True, {}, 7), ("ALL_Q8_0", False, {}, 4), ("Q4_K_M", False, {"head_dim": 64}, 9),
     ("Q4_K_M_LAYERED", False, {"layers": 4}, 13), ("Q4_K_M", False, {}, 1),
     # 16 tokens or more: the projections on the tensor cores (pgemm.cu)
     ("Q4_K_M", False, {}, 40), ("Q4_K_M", True, {}, 70), ("ALL_Q8_0", False, {}, 33), ("Q4_K_M", False, {"head_dim": 64}, 16),
     ("Q4_K_M_LAYERED", False, {"layers": 4}, 57), ("Q4_K_M", False, {"hidden": 1024, "ffn": 3072}, 48)],
)
def test_prefill_matches_token_by_token(pkg, O, mix, kv_f16, shape_kw, n_prompt):
    """qwen3_prefill against the reference's token-by-token prefill
    (qwen3.uya:2485-2506, which the forward reproduces bit-exactly): prompts
    under 16 tokens go through the multi-vector GEMVs (up to 4 tokens per
    pass over the weights), longer ones through the tensor-core projections
    (tcgen05 kind::i8, 32-token tiles).  Either way the last token's logits
    and greedy token are bit-identical, and so is every decode step after it
    (the KV caches agree)."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape(**shape_kw)
    tensors = build(pkg, shape, getattr(gguf, mix), seed=6)
    a = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16)
    b = Qwen3Runtime.open(tensors, shape=shape, context=shape.context, kv_f16=kv_f16)
    ids = [int(t) for t in gguf.prompt_ids(n_prompt, shape.vocab, seed=12)]
    la, lb = np.empty(shape.vocab, np.float32), np.empty(shape.vocab, np.float32)
    for pos, t in enumerate(ids):
        ta, ga = a.forward(t, pos, logits=pos == len(ids) - 1, penalty=1.2, want_logits=la if pos == len(ids) - 1 else None)
    tb, gb = b.gpu.qwen3_prefill(ids, 0, penalty=1.2, want_logits=lb)
    tc, gv = b.gpu.qwen3_prefill_passes()
    assert (tc, gv) == ((1, 0) if n_prompt >= 16 else (0, (n_prompt + 3) // 4))  # the path the test names
    assert np.array_equal(la, lb), rel_row_err(la, lb)
    assert (ta, ga) == (tb, gb)
    for step in range(5):
        pos = len(ids) + step
        ta, ga = a.forward(ta, pos, penalty=1.2, want_logits=la)
        tb, gb = b.forward(tb, pos, penalty=1.2, want_logits=lb)
        assert np.array_equal(la, lb), (step, rel_row_err(la, lb))
        assert (ta, ga) == (tb, gb), step
    a.close()
    b.close()


@pytest.mark.parametrize("mix", ["Q4_K_M", "ALL_Q8_0"])
def test_prefill_tensor_core_passes(pkg, O, mix):
    """A prompt longer than one tensor-core pass (256 tokens) after a
    token-by-token start: positions continue across passes, the cache rows
    of every pass are what the token-by-token forwards write, and the last
    token's logits and the decode after it are bit-identical."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape(context=400, ffn=1024)
    tensors = build(pkg, shape, getattr(gguf, mix), seed=13)
    a = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    b = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    ids = [int(t) for t in gguf.prompt_ids(300, shape.vocab, seed=21)]
    la, lb = np.empty(shape.vocab, np.float32), np.empty(shape.vocab, np.float32)
    for pos, t in enumerate(ids):
        ta, ga = a.forward(t, pos, logits=pos == len(ids) - 1, want_logits=la if pos == len(ids) - 1 else None)
    for pos in range(3):  # the first tokens one by one, the rest in one call
        b.forward(ids[pos], pos, logits=False)
    tb, gb = b.gpu.qwen3_prefill(ids[3:], 3, want_logits=lb)
    assert b.gpu.qwen3_prefill_passes() == (2, 0)  # 256 + 41 tokens on the tensor cores
    assert np.array_equal(la, lb), rel_row_err(la, lb)
    assert (ta, ga) == (tb, gb)
    for step in range(4):
        pos = len(ids) + step
        ta, ga = a.forward(ta, pos, want_logits=la)
        tb, gb = b.forward(tb, pos, want_logits=lb)
        assert np.array_equal(la, lb), (step, rel_row_err(la, lb))
        assert (ta, ga) == (tb, gb), step
    a.close()
    b.close()


def test_runtime_prefill_prompt_ids(pkg, O):
    """The runtime wrapper: positions advance by the prompt length and the
    next token equals the token-by-token loop's."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape()
    tensors = build(pkg, shape, gguf.Q4_K_M, seed=8)
    a = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    b = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    ids = [int(t) for t in gguf.prompt_ids(11, shape.vocab, seed=2)]
    na, _ = a.append_prompt_ids(ids)
    nb, _ = b.prefill_prompt_ids(ids)
    assert (na, a.total_tokens) == (nb, b.total_tokens)
    assert a.generate(6) == b.generate(6)
    a.close()
    b.close()


def test_time_ffn_leaves_decode_unchanged(pkg, O):
    """qwen3_time_ffn reports a positive launch time and the launch's bytes,
    and touches only scratch activations: decoding afterwards gives the same
    tokens as a runtime that never timed."""
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = small_shape()
    tensors = build(pkg, shape, gguf.Q4_K_M, seed=9)
    a = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    b = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    ids = [int(t) for t in gguf.prompt_ids(7, shape.vocab, seed=3)]
    a.append_prompt_ids(ids)
    b.append_prompt_ids(ids)
    us, nbytes = b.gpu.qwen3_time_ffn(iters=2 * shape.layers)
    assert us > 0.0
    gate, up = b.tensors["blk.0.ffn_gate.weight"], b.tensors["blk.0.ffn_up.weight"]
    assert nbytes >= gate.nbytes + up.nbytes
    assert a.generate(5) == b.generate(5)
    a.close()
    b.close()
