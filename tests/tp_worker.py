"""Tensor-parallel decode worker, launched by tests/test_gpu_tp.py under
torch.distributed.run (one process per GPU).  Every rank binds its shards of
the same seeded model and decodes the same teacher-forced tokens; rank 0 also
runs the single-GPU runtime and prints one JSON line comparing the two."""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parent))
from conftest import load_pkg, rel_row_err  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    import datetime

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    load_pkg()
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime, TensorParallel

    steps = int(os.environ.get("TP_STEPS", "48"))
    if os.environ.get("TP_SHAPE", "small") == "qwen3-8b-4l":
        shape = gguf.Qwen3Shape(**{**gguf.SHAPES["qwen3-8b"].__dict__, "layers": 4, "context": 64})
        tensors = gguf.synth_model(shape, gguf.Q4_K_M, device=f"cuda:{local}", seed_base=5)
    else:
        kv = max(2, world)  # every rank keeps >= 1 kv head and 512 q columns
        shape = gguf.Qwen3Shape(layers=2, hidden=512, heads=4 * kv, kv_heads=kv, head_dim=128, ffn=2048, vocab=2048,
                                context=96)
        tensors = gguf.synth_model(shape, gguf.Q4_K_M, seed_base=5)
    rt = Qwen3Runtime.open(tensors, shape=shape, device_index=local, context=shape.context,
                           tp=TensorParallel(rank, world))
    ids = gguf.prompt_ids(steps, shape.vocab, seed=3)
    lg = np.zeros(shape.vocab, np.float32)
    toks, gaps, slices = [], [], []
    for pos in range(steps):
        t, g = rt.forward(int(ids[pos]), pos, logits=True, want_logits=lg)
        toks.append(int(t))
        gaps.append(float(g))
        slices.append(lg.copy())
    dec = rt.gpu.qwen3_decode(int(ids[0]), steps, 16).tolist()
    # prompt tokens without logits (the graph that ends with the finalising exchange), then one more step
    for pos in range(steps + 16, steps + 20):
        rt.forward(int(ids[pos % steps]), pos, logits=False)
    t_last, _ = rt.forward(int(ids[0]), steps + 20, logits=True, want_logits=lg)
    everyone = [None] * world
    spans = []
    for sl in slices:  # this rank's vocab slice of every step's logits (zeros elsewhere)
        nz = np.nonzero(sl)[0]
        lo, hi = (int(nz.min()), int(nz.max()) + 1) if nz.size else (0, 0)
        spans.append((lo, hi, sl[lo:hi].copy()))
    dist.all_gather_object(everyone, {"toks": toks, "dec": dec, "last": int(t_last), "spans": spans})
    if rank == 0:
        ref = Qwen3Runtime.open(tensors, shape=shape, device_index=local, context=shape.context)
        rl = np.zeros(shape.vocab, np.float32)
        mism, flips, worst = 0, 0, 0.0
        lo, hi = None, None
        for pos in range(steps):
            t, g = ref.forward(int(ids[pos]), pos, logits=True, want_logits=rl)
            full = np.zeros(shape.vocab, np.float32)  # every rank's slice of this step's logits
            for e in everyone:
                lo, hi, vals = e["spans"][pos]
                full[lo:hi] = vals
            worst = max(worst, rel_row_err(full, rl))
            dmax = float(np.max(np.abs(full.astype(np.float64) - rl)))
            if t != toks[pos]:
                flips += 1
                # a flip is allowed only where the gap is within twice the step's largest logit difference
                if g > 1e-3 and g > 2 * dmax:
                    mism += 1
        ref_dec = ref.gpu.qwen3_decode(int(ids[0]), steps, 16).tolist()
        for pos in range(steps + 16, steps + 20):
            ref.forward(int(ids[pos % steps]), pos, logits=False)
        ref_last, ref_gap = ref.forward(int(ids[0]), steps + 20, logits=True, want_logits=rl)
        if ref_last != t_last:
            flips += 1
        agree = all(e["toks"] == toks and e["dec"] == dec and e["last"] == int(t_last) for e in everyone)
        print(json.dumps({"world": world, "ranks_agree": agree, "token_mismatch_large_gap": mism, "flips": flips,
                          "worst_logit_err": worst, "decode_equal": dec == ref_dec, "min_gap": min(gaps)}))
        ref.close()
    dist.barrier()  # no rank unmaps its exchange buffer while a peer may still read it
    rt.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
