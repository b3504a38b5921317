"""Per-stage timing of the persistent decode-step kernel (decode_mode 2).

    python minicpm-o-uya_b200/step_trace.py [--shape qwen3-8b] [--prompt 560] [--layers N]

Binds a synthetic model of the shape, prefills `--prompt` tokens, decodes a
few tokens with MCPO_STEP_TRACE=1 and prints, per stage kind, the mean time
from the stage's start to its activations being ready (the prologue), the
mean and max of the weight-loop time over CTAs, the stage's span, and the
gap from the previous stage's last CTA to this stage's first start (the grid
barrier).  Times are globaltimer nanoseconds written by the kernel.
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _pkg():
    if "minicpmo_b200" in sys.modules:
        return sys.modules["minicpmo_b200"]
    spec = importlib.util.spec_from_file_location("minicpmo_b200", HERE / "__init__.py",
                                                  submodule_search_locations=[str(HERE)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["minicpmo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shape", default="qwen3-8b")
    ap.add_argument("--prompt", type=int, default=560)
    ap.add_argument("--layers", type=int, default=0)
    args = ap.parse_args()
    os.environ["MCPO_STEP_TRACE"] = "1"
    _pkg()
    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    shape = gguf.SHAPES[args.shape]
    if args.layers > 0:
        shape = gguf.Qwen3Shape(**{**shape.__dict__, "layers": args.layers})
    tensors = gguf.synth_model(shape, gguf.Q4_K_M, device="cuda")
    rt = Qwen3Runtime.open(tensors, shape=shape, context=args.prompt + 64, decode_mode=2)
    if rt.gpu.qwen3_step_kernels(True) > 4:
        print("the model does not fit the persistent step kernel")
        return 1
    nxt, _ = rt.append_prompt_ids(list(gguf.prompt_ids(args.prompt, shape.vocab)))
    for _ in range(3):
        nxt, _ = rt.forward(nxt, rt.total_tokens)
        rt.total_tokens += 1
    tr = rt.gpu.qwen3_step_trace()
    if tr is None:
        print("tracing unavailable")
        return 1
    tr = tr.astype(np.int64)
    ns = tr.shape[0]
    names = (["qkv", "attn", "o", "gateup", "down"] * shape.layers + ["lm_head"])[:ns]
    t0 = tr[0, :, 0].min()
    agg = {}
    prev_end = None
    for s in range(ns):
        st, rd, en = tr[s, :, 0] - t0, tr[s, :, 1] - t0, tr[s, :, 2] - t0
        gemv = names[s] != "attn"
        pro = (rd - st) if gemv else np.zeros_like(st)
        work = (en - rd) if gemv else (en - st)
        gap = (st.min() - prev_end) if prev_end is not None else 0
        a = agg.setdefault(names[s], np.zeros(6))
        a += [1, pro.mean(), work.mean(), work.max(), (en - st).max(), gap]
        prev_end = en.max()
    span = tr[:, :, 2].max() - t0
    print(f"step kernel span {span / 1e3:.1f} us over {ns} stages at position {rt.total_tokens - 1}")
    print(f"{'stage':8s} {'n':>3s} {'prologue':>9s} {'work_mean':>10s} {'work_max':>9s} {'stage_max':>10s} {'gap':>7s}"
          "  (us per stage, mean over layers)")
    for k, a in agg.items():
        n = a[0]
        print(f"{k:8s} {int(n):3d} {a[1] / n / 1e3:9.2f} {a[2] / n / 1e3:10.2f} {a[3] / n / 1e3:9.2f} "
              f"{a[4] / n / 1e3:10.2f} {a[5] / n / 1e3:7.2f}")
    ms = rt.gpu.qwen3_time_decode(nxt, rt.total_tokens, 20)
    print(f"decode ms/step {ms / 20:.4f}")
    rt.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
