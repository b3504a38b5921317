"""The reference's own GPU helper on the same B200, through the same host.

oracle/_ref/refhelper/libminicpmo_gpu_helper.so is the reference's
src/minicpmo/gpu_shim.c built as its Makefile builds it (NVRTC-compiled
kernels and cuBLAS at run time).  The C host oracle/_ref/bridge_host (the
reference's gpu_bridge.c plus the per-operation decode of
qwen3.uya:1865-1918) runs the same four layers of the Qwen3-8B shape
(vocab 151936, untied Q6_K lm_head) once next to the reference helper and
once next to this repository's helper.  Both perform the reference's CUDA
arithmetic (Q8_1 activations, int32 block dots), in different summation
orders, so the logits agree within LOGIT_TOL of their norm; the greedy
tokens agree wherever the top-2 gap exceeds twice the largest logit
difference.  The decode rates of the two helpers under the same host loop
(every call a bridge forwarder, logits downloaded each token) are
printed."""
from __future__ import annotations

import json
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

from conftest import ROOT, rel_row_err

pytestmark = pytest.mark.gpu

BRIDGE = ROOT / "oracle" / "_ref" / "bridge_host"
REF_HELPER = ROOT / "oracle" / "_ref" / "refhelper" / "libminicpmo_gpu_helper.so"
LOGIT_TOL = 5e-3
NTOK = 12


def _write_input(path, shape, tensors, rows, cos_t, sin_t):
    with open(path, "wb") as fh:
        fh.write(struct.pack("<10I", shape.layers, shape.hidden, shape.heads, shape.kv_heads, shape.head_dim,
                             shape.ffn, shape.vocab, shape.context, len(rows), len(tensors)))
        for name, dt, r, c, data in tensors:
            nb = name.encode()
            fh.write(struct.pack("<I", len(nb)) + nb + struct.pack("<iQQQ", dt, r, c, data.nbytes))
            fh.write(np.ascontiguousarray(data).tobytes())
        fh.write(cos_t.astype(np.float32).tobytes() + sin_t.astype(np.float32).tobytes())
        fh.write(np.stack(rows).astype(np.float32).tobytes())


def _run(tmp_path, helper, label, inp):
    d = tmp_path / label
    d.mkdir()
    shutil.copy(BRIDGE, d / "bridge_host")
    shutil.copy(helper, d / "libminicpmo_gpu_helper.so")
    env = dict(os.environ)
    env["LD_LIBRARY_PATH"] = "/usr/local/cuda/lib64:" + env.get("LD_LIBRARY_PATH", "")
    out = subprocess.run([str(d / "bridge_host"), str(inp), str(d / "out.bin")], capture_output=True, text=True,
                         timeout=600, env=env)
    assert out.returncode == 0, (label, out.stderr[-2000:])
    stats = json.loads(out.stdout.strip().splitlines()[-1])
    return np.fromfile(d / "out.bin", np.float32), stats


def test_reference_gpu_helper_same_host(pkg, O, tmp_path):
    if not BRIDGE.exists() or not REF_HELPER.exists():
        pytest.skip("oracle/_ref not built (needs the reference tree at build time)")
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime, rope_table

    shape = gguf.Qwen3Shape(**{**gguf.SHAPES["qwen3-8b"].__dict__, "layers": 4, "context": 64})
    tensors = gguf.synth_model(shape, gguf.Q4_K_M, device="cuda", seed_base=13)
    rt = Qwen3Runtime.open(tensors, shape=shape, context=shape.context)
    ids = gguf.prompt_ids(NTOK, shape.vocab, seed=21)
    emb = rt.tensors["token_embd.weight"]
    rows = []
    for tok in ids:
        rt.gpu.embed_lookup(0, emb, int(tok))
        rows.append(rt.gpu.slot_download(0, shape.hidden))
    rt.close()
    cos_t, sin_t = rope_table(shape.context, shape.head_dim, shape.rope_base)
    inp = tmp_path / "in.bin"
    _write_input(inp, shape, tensors, rows, cos_t, sin_t)
    ref, ref_stats = _run(tmp_path, REF_HELPER, "reference", inp)
    ours, our_stats = _run(tmp_path, pkg.lib_path(), "b200", inp)
    ref = ref.reshape(NTOK, shape.vocab)
    ours = ours.reshape(NTOK, shape.vocab)
    worst, flips = 0.0, 0
    for t in range(NTOK):
        err = rel_row_err(ours[t], ref[t])
        worst = max(worst, err)
        assert err < LOGIT_TOL, (t, err)
        tr, gr = O.argmax_penalized(ref[t])
        to, _ = O.argmax_penalized(ours[t])
        if tr != to:
            flips += 1
            assert gr <= 2 * float(np.max(np.abs(ours[t].astype(np.float64) - ref[t]))), t
    print(f"[ref-shim] qwen3-8b shape, 4 layers, same bridge host: reference helper {ref_stats['tok_per_s']:.1f} tok/s, "
          f"this helper {our_stats['tok_per_s']:.1f} tok/s (per-operation calls); worst logit err {worst:.2e}, "
          f"{flips} greedy flips")
