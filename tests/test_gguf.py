"""GGUF writer/reader round trip and the synthetic-model quantisers (CPU)."""
from __future__ import annotations

import numpy as np
import pytest
import torch


@pytest.mark.parametrize("dt,tol", [(6, 0.01), (10, 0.08), (12, 0.04)])
def test_quantisers_produce_valid_blocks(pkg, O, dt, tol):
    from minicpmo_b200 import gguf

    x = torch.randn((8, 512), generator=torch.Generator().manual_seed(1)) * 0.02
    w = gguf.quantize(x, dt).numpy()
    assert w.shape == (8, gguf.row_bytes(dt, 512))
    deq = O.dequant(dt, w, 8, 512)
    err = np.abs(deq - x.numpy()).max() / np.abs(x.numpy()).max()
    assert err < tol


def test_gguf_round_trip(pkg, tmp_path):
    from minicpmo_b200 import gguf

    shape = gguf.Qwen3Shape(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=300, context=128)
    tensors = gguf.synth_model(shape, gguf.Q4_K_M)
    path = tmp_path / "m.gguf"
    gguf.write_gguf(path, gguf.qwen3_metadata(shape), tensors)
    f = gguf.GgufFile(path)
    s2 = f.shape()
    assert (s2.layers, s2.hidden, s2.heads, s2.kv_heads, s2.head_dim, s2.ffn, s2.vocab) == (2, 256, 4, 2, 64, 512, 300)
    assert len(f.metadata["tokenizer.ggml.tokens"]) == 300
    for name, dt, rows, cols, data in tensors:
        t = f.tensors[name]
        assert (t.dtype, t.rows, t.cols) == (dt, rows, cols)
        assert np.array_equal(np.asarray(t.data), data.reshape(-1))


def test_synthetic_seeds_are_stable(pkg):
    from minicpmo_b200 import gguf

    a = gguf.synth_tensor("blk.0.attn_q.weight", gguf.Q4_K, 4, 256, "w")
    b = gguf.synth_tensor("blk.0.attn_q.weight", gguf.Q4_K, 4, 256, "w")
    c = gguf.synth_tensor("blk.1.attn_q.weight", gguf.Q4_K, 4, 256, "w")
    assert np.array_equal(a, b) and not np.array_equal(a, c)


def test_layered_q4_k_m_pattern(pkg):
    """Q4_K_M_LAYERED: attn_v / ffn_down are Q6_K in the first and last
    eighth of the layers and every third layer between, Q4_K elsewhere."""
    from minicpmo_b200 import gguf

    shape = gguf.Qwen3Shape(layers=16, hidden=256, heads=4, kv_heads=2, head_dim=64, ffn=512, vocab=300, context=64)
    specs = {n: dt for n, dt, _, _, _ in gguf.tensor_specs(shape, gguf.Q4_K_M_LAYERED)}
    hi = [l for l in range(16) if specs[f"blk.{l}.attn_v.weight"] == gguf.Q6_K]
    assert hi == [0, 1, 4, 7, 10, 13, 14, 15]
    assert all(specs[f"blk.{l}.ffn_down.weight"] == (gguf.Q6_K if l in hi else gguf.Q4_K) for l in range(16))
    assert specs["token_embd.weight"] == gguf.Q4_K and specs["output.weight"] == gguf.Q6_K
    assert all(specs[f"blk.{l}.attn_q.weight"] == gguf.Q4_K for l in range(16))
