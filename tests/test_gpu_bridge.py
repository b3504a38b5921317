"""The drop-in through the reference's own loader: oracle/_ref/bridge_host is
the reference's src/minicpmo/gpu_bridge.c, unmodified, linked with a small C
host (tests/bridge_host.c).  The bridge dlmopen()s the helper next to its
executable into a private link-map namespace (LM_ID_NEWLM,
gpu_bridge.c:107-176) -- the statically linked CUDA runtime has to work
there -- and every call goes through its 19 forwarders.  The host runs the
reference's per-operation decode of a 2-layer model; its logits must equal,
bit for bit, the same model's fused decode step run in this process."""
from __future__ import annotations

import json
import shutil
import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

BRIDGE = ROOT / "oracle" / "_ref" / "bridge_host"


def test_reference_bridge_drives_the_helper(pkg, tmp_path):
    if not BRIDGE.exists():
        pytest.skip("oracle/_ref/bridge_host not built (needs the reference tree at build time)")
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime, rope_table

    shape = gguf.Qwen3Shape(layers=2, hidden=512, heads=8, kv_heads=2, head_dim=128, ffn=1536, vocab=2048, context=32)
    tensors = gguf.synth_model(shape, gguf.Q4_K_M, seed_base=11)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    ids = gguf.prompt_ids(8, shape.vocab, seed=5)
    emb = rt.tensors["token_embd.weight"]
    rows = []
    for tok in ids:  # the reference host dequantises the embedding row itself (qwen3.uya:1164-1174)
        rt.gpu.embed_lookup(0, emb, int(tok))
        rows.append(rt.gpu.slot_download(0, shape.hidden))
    cos_t, sin_t = rope_table(shape.context, shape.head_dim, shape.rope_base)
    blob = struct.pack("<10I", shape.layers, shape.hidden, shape.heads, shape.kv_heads, shape.head_dim, shape.ffn,
                       shape.vocab, shape.context, len(ids), len(tensors))
    for name, dt, r, c, data in tensors:
        nb = name.encode()
        blob += struct.pack("<I", len(nb)) + nb + struct.pack("<iQQQ", dt, r, c, data.nbytes) + data.tobytes()
    blob += cos_t.astype(np.float32).tobytes() + sin_t.astype(np.float32).tobytes()
    blob += np.stack(rows).astype(np.float32).tobytes()
    (tmp_path / "in.bin").write_bytes(blob)
    exe = tmp_path / "bridge_host"
    shutil.copy(BRIDGE, exe)
    shutil.copy(pkg.lib_path(), tmp_path / "libminicpmo_gpu_helper.so")
    out = subprocess.run([str(exe), str(tmp_path / "in.bin"), str(tmp_path / "out.bin")], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    stats = json.loads(out.stdout.strip().splitlines()[-1])
    assert stats["native_quant_matvec_count"] > 0 and stats["attention_kernel_calls"] == len(ids) * shape.layers
    got = np.fromfile(tmp_path / "out.bin", np.float32).reshape(len(ids), shape.vocab)
    lg = np.empty(shape.vocab, np.float32)
    for pos, tok in enumerate(ids):
        rt.forward(int(tok), pos, logits=True, want_logits=lg)
        assert np.array_equal(got[pos], lg), pos
    rt.close()
