#!/usr/bin/env python3
"""Benchmark: Qwen3-8B-shape Q4_K_M greedy decode on B200.

One step = one decode token: embedding lookup, 36 layers of fused
RMSNorm->Q8_1->GEMV / QK-norm+RoPE+KV-append+split-K attention / SwiGLU /
residual, final norm, lm_head GEMV and the greedy sampler, all on the device
as one CUDA-graph replay.

* value  -- decode tokens/s with everything resident in HBM: K graph replays,
            each feeding its own sampled token back on the device, timed with
            CUDA events on the helper's stream (weights 4.9 GB >> 126 MB L2,
            so every step streams them from HBM).
* e2e    -- the same decode through the public C ABI call a host makes per
            token (minicpmo_gpu_context_qwen3_forward): each step copies the
            token/position state host->device, replays, and reads the sampled
            token back (pinned buffers), timed on the host clock.
* roofline -- the dominant kernel (the quantised GEMV) timed alone on the
            model's largest per-layer shape, against MEASURED_PEAKS.json.
* cpu_baseline -- the reference's own CPU matvec (src/minicpmo/cpu_kernels.c,
            compiled from the reference tree into oracle/_ref/) plus the
            oracle's restatement of the decode glue, all host threads, on a
            bounded sample of the same workload.

--impl reference runs only that CPU reference arm.  Under torchrun with N > 1
the N GPUs decode one sequence with tensor parallelism (q/k/v and gate/up
column-parallel, o and down row-parallel with the hidden-vector exchange
fused into those GEMVs over NVLink, the lm_head vocab-parallel; strong
scaling); --replicas runs N independent sequences instead (weak scaling).
Weights are seeded synthetic N(0, 0.02)
quantised Q4_K_M-style (no real checkpoint exists here).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT = 512  # 512 random prompt ids, then greedy decode
STATE_BYTES = 36  # StepState copied each way per e2e step


def load_pkg():
    if "minicpmo_b200" in sys.modules:
        return sys.modules["minicpmo_b200"]
    pkg_dir = ROOT / "minicpm-o-uya_b200"
    spec = importlib.util.spec_from_file_location("minicpmo_b200", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["minicpmo_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def metric_name(shape_key: str) -> str:
    label = {"qwen3-0.6b": "Qwen3-0.6B", "qwen3-8b": "Qwen3-8B", "qwen3-32b": "Qwen3-32B"}.get(shape_key, shape_key)
    return f"{label} Q4_K_M decode tok/s"


def model_bytes(tensors, shape, pos_mean):
    """Bytes one decode step must read: every weight once, except the token
    embedding (one row per step), plus the f32 KV rows attended."""
    w = 0
    for name, _, rows, _, d in tensors:
        w += int(d.nbytes) // rows if name == "token_embd.weight" else int(d.nbytes)
    kv = 2 * shape.layers * shape.kv_dim * 4 * (pos_mean + 1)
    return w, kv


def clock_csv(rank: int) -> Path:
    """A private temporary file for one rank's nvidia-smi samples."""
    import tempfile

    fd, name = tempfile.mkstemp(prefix=f"mcpo_clocks_rank{rank}_", suffix=".csv")
    os.close(fd)
    return Path(name)


class ClockSampler:
    """nvidia-smi clocks during the timed region (the recipe's clocks line)."""

    def __init__(self, device: int, path: Path):
        self.path = path
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(device),
                 "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        try:
            self.path.unlink()
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def build_weights(shape, mix, device):
    from minicpmo_b200 import gguf

    return gguf.synth_model(shape, mix, device=device)


def cpu_reference(shape, tensors, n_tokens, start_pos, threads):
    """The reference CPU path: cpu_kernels.c matvec (oracle/_ref) in a row-partitioned
    pthread pool (qwen3.uya:1247-1499) + the oracle's restatement of the glue.
    The KV cache holds seeded values for the start_pos earlier positions, so each
    timed token attends over start_pos+1.. positions as in the GPU run."""
    from oracle import oracle as O

    ctx = start_pos + 3 * n_tokens + 1
    tmap = {n: (dt, r, c, d) for n, dt, r, c, d in tensors}
    m = O.OracleModel(shape, tmap, ctx, q8_1=False, pool_threads=threads, use_reference_matvec=True)
    rng = np.random.Generator(np.random.PCG64(5))
    m.kc[:] = rng.standard_normal(m.kc.size, dtype=np.float32)
    m.vc[:] = rng.standard_normal(m.vc.size, dtype=np.float32)
    kind = "reference" if m.uses_reference_matvec else "port"
    ids = np.random.Generator(np.random.PCG64(11)).integers(0, shape.vocab, 3 * n_tokens + 1)
    m.forward(int(ids[0]), start_pos)  # untimed warm-up token (page in the weights)
    rates = []
    pos = start_pos + 1
    for rep in range(3):  # median of 3 timed windows of n_tokens each
        t0 = time.perf_counter()
        for i in range(n_tokens):
            m.forward(int(ids[1 + rep * n_tokens + i]), pos)
            pos += 1
        rates.append(n_tokens / (time.perf_counter() - t0))
    m.close()
    return statistics.median(rates), kind


def run_reference(args, shape, mix):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import torch

    dev = "cuda" if torch.cuda.is_available() else "cpu"
    tensors = build_weights(shape, mix, dev)
    threads = os.cpu_count() or 1
    # each step is one decode token of the reference CPU path at position >= args.prompt
    n = args.steps
    from oracle import oracle as O

    ctx = args.prompt + args.warmup + n + 1
    tmap = {nm: (dt, r, c, d) for nm, dt, r, c, d in tensors}
    m = O.OracleModel(shape, tmap, ctx, q8_1=False, pool_threads=threads, use_reference_matvec=True)
    rng = np.random.Generator(np.random.PCG64(5))
    m.kc[:] = rng.standard_normal(m.kc.size, dtype=np.float32)
    m.vc[:] = rng.standard_normal(m.vc.size, dtype=np.float32)
    kind = "reference" if m.uses_reference_matvec else "port"
    ids = np.random.Generator(np.random.PCG64(11)).integers(0, shape.vocab, args.warmup + n)
    pos = args.prompt
    for i in range(args.warmup):
        m.forward(int(ids[i]), pos)
        pos += 1
    t0 = time.perf_counter()
    for i in range(n):
        m.forward(int(ids[args.warmup + i]), pos)
        pos += 1
    dt = time.perf_counter() - t0
    m.close()
    tps = n / dt
    line = {
        "impl": "reference",
        "metric": metric_name(args.shape),
        "value": tps,
        "unit": "tok/s",
        "n_gpus": 0,
        "steps": n,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 / tps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) weights quantised Q4_K_M-style; seeded KV for the 512-token prompt)",
        "config": {"workload": f"{args.shape}-shape Q4_K_M greedy decode, prompt 512", "layers": shape.layers,
                   "hidden": shape.hidden, "vocab": shape.vocab, "parallelism": "cpu threads"},
        "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": kind,
                         "sample": f"{n} decode tokens at positions {args.prompt + args.warmup}..{pos - 1} "
                                   "(f32 activations, reference cpu_kernels.c AVX2 matvec, pthread row pool)"},
        "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_kernel_sweep(args) -> int:
    """Config 1: y = W.x at the north-star shapes for Q4_K, Q6_K and Q8_0 weights (N(0, 0.02)), x N(0, 1)
    stand-in (a fixed pattern: the GEMV's time does not depend on the values).  Each GEMV is timed alone
    with CUDA events over weight copies rotated through more than 2x the L2; the hidden-input shapes are
    also timed with the fused RMSNorm -> Q8_1 prologue, the down shape with the f32 -> Q8_1 prologue (the
    SwiGLU output it consumes in the step)."""
    import torch
    from minicpmo_b200 import gguf
    from minicpmo_b200.gpu import GpuContext, Tensor

    local = int(os.environ.get("LOCAL_RANK", "0"))
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    torch.cuda.set_device(local)
    g = GpuContext(local)
    hbm, peak_kind = peaks()
    names = {10: "Q4_K", 12: "Q6_K", 6: "Q8_0"}
    if args.sweep_launches > 0:
        # for a profiler's launch list: each case's Q8_1-input GEMV launched a few times on its own, one
        # tensor resident at a time (no timing, no rotated copies)
        for rows, cols in [(4096, 4096), (12288, 4096), (4096, 12288), (151936, 4096)]:
            for dt in (10, 12, 6):
                name = f"sweep.{names[dt]}.{rows}x{cols}"
                t = Tensor(name, gguf.synth_tensor(name, dt, rows, cols, "weight", device="cuda"), dt, rows, cols)
                g.upload_tensor(t)
                xq = g.q8_1_quantize(np.ones(cols, np.float32))
                for _ in range(args.sweep_launches):
                    g.matvec_q8_1(t, xq)
                print(json.dumps({"kernel_sweep_launches": {"dtype": names[dt], "rows": rows, "cols": cols,
                                                            "launches": args.sweep_launches}}), flush=True)
                g.close()
                g = GpuContext(local)
        g.close()
        return 0
    norms = {}
    for rows, cols in [(4096, 4096), (12288, 4096), (4096, 12288), (151936, 4096)]:
        for dt in (10, 12, 6):
            name = f"sweep.{names[dt]}.{rows}x{cols}"
            t = Tensor(name, gguf.synth_tensor(name, dt, rows, cols, "weight", device="cuda"), dt, rows, cols)
            g.upload_tensor(t)
            w_bytes = t.nbytes
            modes = [("q8_1", 0, cols // 32 * 36)]
            if cols == 4096:
                if cols not in norms:
                    nt = Tensor(f"sweep.norm{cols}", gguf.synth_tensor(f"sweep.norm{cols}", 0, 1, cols, "norm",
                                                                        device="cuda"), 0, 1, cols)
                    g.upload_tensor(nt)
                    norms[cols] = nt
                modes.append(("rmsnorm_f32", 2, cols * 8))
            else:
                modes.append(("f32", 1, cols * 4))
            for label, mode, x_bytes in modes:
                us = g.time_matvec_input(t, mode, norms.get(cols) if mode == 2 else None, iters=20)
                alg = w_bytes + x_bytes + rows * 4
                print(json.dumps({"kernel_sweep": {"dtype": names[dt], "rows": rows, "cols": cols, "input": label,
                                                   "us": us, "bytes": alg, "gbs": alg / us / 1e3,
                                                   "frac": alg / us / 1e3 / hbm, "peak_gbs": hbm,
                                                   "peak_kind": peak_kind}}), flush=True)
    g.close()
    return 0


def _ncu_traffic(key):
    """Per-launch DRAM bytes of the roofline kernel from the committed ncu summary (or None)."""
    tf = ROOT / "profiles" / "ncu_traffic.json"
    if not tf.exists():
        return None
    try:
        return json.loads(tf.read_text()).get(key)
    except (ValueError, KeyError):
        return None


def run_prefill_bench(args, shape, mix) -> int:
    """Prompt prefill on 1 GPU: --prompt seeded ids through qwen3_prefill
    (16 ids or more: tensor-core passes of up to 256; fewer: GEMV passes of
    up to 4) and, over the same positions of a reset cache, through one
    qwen3_forward per id (the reference's qwen3_append_prompt_ids loop).
    Host wall time around each call, which synchronises; max(1, --steps //
    64) repetitions after one untimed (which also builds the tensor-core
    operand copy of the weights)."""
    import torch

    from minicpmo_b200.qwen3 import Qwen3Runtime
    from minicpmo_b200 import gguf

    torch.cuda.set_device(0)
    tensors = build_weights(shape, mix, "cuda:0")
    torch.cuda.empty_cache()
    rt = Qwen3Runtime.open(tensors, shape=shape, device_index=0, context=args.prompt + 8)
    prompt = gguf.prompt_ids(args.prompt, shape.vocab, seed=7)
    reps = max(1, args.steps // 64)

    def timed(fn):
        rt.reset()
        torch.cuda.synchronize()
        t = time.perf_counter()
        out = fn(prompt)
        torch.cuda.synchronize()
        return time.perf_counter() - t, out

    timed(rt.prefill_prompt_ids)
    pf = [timed(rt.prefill_prompt_ids) for _ in range(reps)]
    tw = [timed(rt.append_prompt_ids) for _ in range(reps)]
    assert all(p[1][0] == tw[0][1][0] for p in pf + tw), "prefill and token-by-token next tokens differ"
    t_pf = min(p[0] for p in pf)
    t_tw = min(p[0] for p in tw)
    print(json.dumps({
        "metric": f"{metric_name(args.shape).replace('decode', 'prefill')}",
        "value": args.prompt / t_pf, "unit": "tok/s", "n_gpus": 1, "steps": reps, "warmup": 1,
        "higher_is_better": True,
        "dtype": ("q4_k/q6_k x q8_1 (int8 block dots on tcgen05 kind::i8, f32 combine)" if args.prompt >= 16
                  else "q4_k/q6_k x q8_1 (int8 dp4a, f32 accumulate)"),
        "data": f"synthetic: seeded N(0,0.02) weights quantised Q4_K_M-style, {args.prompt} uniform random prompt ids",
        "config": {"workload": f"{args.shape}-shape Q4_K_M prompt prefill, {args.prompt} ids from position 0",
                   "layers": shape.layers,
                   "passes": (args.prompt + 255) // 256 if args.prompt >= 16 else (args.prompt + 3) // 4},
        "prefill_s": t_pf, "tokenwise_s": t_tw, "tokenwise_tok_s": args.prompt / t_tw,
        "speedup_vs_tokenwise": t_tw / t_pf, "next_token": int(pf[0][1][0]),
    }), flush=True)
    rt.close()
    return 0


def run_batch_bench(args, shape, world, rank, local, dist, barrier) -> int:
    """Qwen3-8B shape, every linear weight Q8_0, f16 KV cache at a 4096-token
    context, B independent sequences each after a prompt of --prompt ids (default 1024), greedy
    decode; the projections run on the tcgen05 tensor cores.  Under torchrun every rank decodes
    its own B sequences (replicas, weak scaling)."""
    import torch

    from minicpmo_b200 import gguf
    from minicpmo_b200.qwen3 import Qwen3Runtime

    B = args.batch
    prompt_len = args.prompt if args.prompt != PROMPT else 1024
    mix = gguf.ALL_Q8_0
    t_gen = time.perf_counter()
    tensors = build_weights(shape, mix, f"cuda:{local}")
    torch.cuda.empty_cache()
    t_gen = time.perf_counter() - t_gen
    t_load = time.perf_counter()
    ctx = max(4096, prompt_len + args.warmup + 2 * args.steps + 8)
    rt = Qwen3Runtime.open(tensors, shape=shape, device_index=local, context=ctx, kv_f16=True, max_batch=B,
                           batch_exact=args.batch_exact)
    t_load = time.perf_counter() - t_load
    g = rt.gpu
    prompts = np.stack([gguf.prompt_ids(prompt_len, shape.vocab, seed=7 + 1000 * rank + b) for b in range(B)])
    t_pf = time.perf_counter()
    nxt, _ = rt.append_prompt_batch(prompts)
    t_pf = time.perf_counter() - t_pf
    rt.generate_batch(args.warmup)  # untimed warm-up steps
    cur = np.asarray(rt.batch_last, np.uint32)
    pos0 = rt.batch_tokens

    clocks = ClockSampler(local, clock_csv(rank))
    barrier()
    wall0 = time.perf_counter()
    ms = g.qwen3_time_decode_batch(cur, np.full(B, pos0, np.uint32), args.steps)
    barrier()
    wall = time.perf_counter() - wall0
    clk = clocks.stop()
    start_pos = pos0
    pos1 = pos0 + args.steps
    # e2e: the public per-step batch call with host buffers (states in, tokens out)
    barrier()
    e0 = time.perf_counter()
    tok = cur
    for i in range(args.steps):
        tok, _, _ = g.qwen3_forward_batch(tok, np.full(B, pos1 + i, np.uint32))
    barrier()
    e2e_s = time.perf_counter() - e0

    ms_t = torch.tensor([ms / 1000.0, e2e_s], dtype=torch.float64, device=f"cuda:{local}")
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    step_s, e2e_s = float(ms_t[0]), float(ms_t[1])
    tokens_total = args.steps * B * world
    value = tokens_total / step_s
    e2e_v = tokens_total / e2e_s

    # roofline: the dominant kernel is the tensor-core projection; the gate
    # shape (12288 x 4096 Q8_0, one of the two matrices of the gate|up launch)
    # timed alone with the L2 flushed before each launch
    hbm, peak_kind = peaks()
    T = rt.tensors
    gate = T["blk.0.ffn_gate.weight"]
    us = g.time_matmul_q8_0_batch(gate, B, iters=10)
    alg = gate.nbytes + B * gate.cols * 2 + B * gate.rows * 4
    gemm_gbs = alg / us / 1e3
    flops = 2.0 * gate.rows * gate.cols * B
    w_bytes = 0
    for name, _, rows, _, d in tensors:
        w_bytes += int(d.nbytes) // rows if name == "token_embd.weight" else int(d.nbytes)
    kv_bytes = 2 * shape.layers * shape.kv_dim * 2 * (start_pos + args.steps // 2 + 1) * B
    step_bytes = w_bytes + kv_bytes
    kernels = g.qwen3_batch_kernels(True)
    line = {
        "metric": f"Qwen3-8B Q8_0 batched decode (B={B}) tok/s",
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * step_s / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": ("q8_0 x q8_1 int8 block dots on tcgen05 kind::i8 (single-sequence bits); f16 KV" if args.batch_exact
                  else "q8_0 weights and activations as f16 on tcgen05 (f32 accumulate); f16 KV"),
        "data": f"synthetic: seeded N(0,0.02) weights quantised Q8_0, {B} x {prompt_len} uniform random prompt ids",
        "config": {
            "workload": f"qwen3-8b-shape all-Q8_0 batched greedy decode, B={B}, prompt {prompt_len}, f16 KV at "
                        f"{ctx}-token context (BASELINE config 3)",
            "batch": B, "layers": shape.layers, "hidden": shape.hidden, "ffn": shape.ffn, "vocab": shape.vocab,
            "prompt": prompt_len, "context": ctx, "decode_positions": [start_pos, start_pos + args.steps],
            "kv_cache": "f16",
            "parallelism": f"replicas x{world} ({B} sequences per GPU)" if world > 1 else "single gpu",
            "l2": "weights 8.0 GB per step >> 126 MB L2 (no flush needed)",
            "weights_bytes": w_bytes, "step_bytes_mean": step_bytes,
            "step_hbm_frac": step_bytes / step_s * args.steps / 1e9 / hbm,
            "prefill_s": t_pf, "load_s": t_load, "synth_s": t_gen, "wall_timed_s": wall,
        },
        "e2e": {"value": e2e_v, "unit": "tok/s", "h2d_bytes_per_step": STATE_BYTES * B,
                "d2h_bytes_per_step": STATE_BYTES * B},
        "gpu_launches": kernels * args.steps,
        "roofline": {"bound": "hbm", "achieved": gemm_gbs, "peak": hbm, "unit": "GB/s", "frac": gemm_gbs / hbm,
                     "traffic": _ncu_traffic("gemm_q80_12288x4096_x32_bytes") if B == 32 else None,
                     "peak_kind": peak_kind,
                     "kernel": f"k_gemm_q80<{16 if B <= 16 else 32}> (tcgen05, Q8_0 12288x4096 x {B} sequences), "
                               "timed alone with the L2 flushed before each launch",
                     "algorithmic_bytes_per_launch": alg, "us_per_launch": us,
                     "tensor_tflops": flops / us / 1e6},
        "clocks": clk,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    rt.close()
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--shape", default="qwen3-8b")
    ap.add_argument("--cpu-sample", type=int, default=4, help="decode tokens for the CPU baseline sample (0: skip)")
    ap.add_argument("--replicas", action="store_true",
                    help="under torchrun: N independent replicas (one sequence each, weak scaling) instead of the "
                         "default tensor parallelism over the N GPUs (one sequence, strong scaling)")
    ap.add_argument("--tp", action="store_true", help="(the default under torchrun; kept for old command lines)")
    ap.add_argument("--sweep-launches", type=int, default=0,
                    help="with --kernel-sweep: launch each case's Q8_1-input GEMV this many times without timing "
                         "(a launch list for a profiler), one weight tensor resident at a time")
    ap.add_argument("--kernel-sweep", action="store_true",
                    help="BASELINE config 1: time the GEMV on each shape x dtype (and its fused prologues); "
                         "one JSON line per case")
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (smaller cases of the same shape, for profiler captures)")
    ap.add_argument("--decode-mode", type=int, default=0,
                    help="0: the library default; 1: one kernel per operation; 2: one persistent kernel per step; "
                         "3: per layer the attention and one chained GEMV launch")
    ap.add_argument("--batch", type=int, default=0,
                    help="BASELINE config 3: batched decode of this many sequences (2..32), all-Q8_0 weights on the "
                         "tensor cores, f16 KV, prompt 1024 unless --prompt is given")
    ap.add_argument("--batch-exact", action="store_true",
                    help="with --batch: the projections as the prompt prefill runs them (int8 block dots; every "
                         "sequence bit-identical to its single-sequence decode)")
    ap.add_argument("--prefill", action="store_true",
                    help="time the multi-token prompt prefill (qwen3_prefill) of --prompt ids on 1 GPU against "
                         "the token-by-token forwards over the same positions; one JSON line")
    ap.add_argument("--prompt", type=int, default=PROMPT,
                    help="prompt length before decode (default: the 512 of the headline config; shorter only for "
                         "profiler launch lists)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    load_pkg()
    from minicpmo_b200 import gguf

    shape = gguf.SHAPES[args.shape]
    if args.layers > 0:
        shape = gguf.Qwen3Shape(**{**shape.__dict__, "layers": args.layers})
    mix = gguf.Q4_K_M
    if args.impl == "reference":
        return run_reference(args, shape, mix)
    if args.kernel_sweep:
        return run_kernel_sweep(args)
    if args.prefill:
        return run_prefill_bench(args, shape, mix)

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))

    from minicpmo_b200.gpu import Tensor
    from minicpmo_b200.qwen3 import Qwen3Runtime

    if args.batch > 1:
        def barrier_b():
            if dist is not None:
                dist.barrier()
            torch.cuda.synchronize()

        rc = run_batch_bench(args, shape, world, rank, local, dist, barrier_b)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return rc

    t_gen = time.perf_counter()
    tensors = build_weights(shape, mix, f"cuda:{local}")
    torch.cuda.empty_cache()
    t_gen = time.perf_counter() - t_gen
    t_load = time.perf_counter()
    tp = None
    if world > 1 and not args.replicas:
        from minicpmo_b200.qwen3 import TensorParallel

        tp = TensorParallel(rank, world)
    rt = Qwen3Runtime.open(tensors, shape=shape, device_index=local, context=args.prompt + args.warmup + 2 * args.steps + 8,
                           decode_mode=args.decode_mode, tp=tp)
    t_load = time.perf_counter() - t_load
    g = rt.gpu
    prompt = gguf.prompt_ids(args.prompt, shape.vocab, seed=7 + (0 if tp is not None else rank))
    # prompt: the multi-token prefill (the same cache bits as token-by-token
    # forwards), then the token-by-token loop over the same positions for the
    # record (it rewrites identical values)
    t_pf = time.perf_counter()
    if tp is None:
        nxt, _ = rt.prefill_prompt_ids(prompt)
        torch.cuda.synchronize()
    else:
        nxt, _ = rt.append_prompt_ids(prompt)
    t_pf = time.perf_counter() - t_pf
    t_pf_tok = None
    if tp is None:
        t_pf_tok = time.perf_counter()
        for i, t in enumerate(prompt):
            g.qwen3_forward(int(t), i, logits=i + 1 == len(prompt))
        t_pf_tok = time.perf_counter() - t_pf_tok
    # warm-up decode steps (untimed)
    toks = g.qwen3_decode(nxt, rt.total_tokens, args.warmup)
    rt.total_tokens += args.warmup
    cur = int(toks[-1])

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- value: device-timed K decode steps (graph replays, token fed back on device)
    clocks = ClockSampler(local, clock_csv(rank))
    barrier()
    wall0 = time.perf_counter()
    ms = g.qwen3_time_decode(cur, rt.total_tokens, args.steps)
    barrier()
    wall = time.perf_counter() - wall0
    clk = clocks.stop()
    start_pos = rt.total_tokens
    rt.total_tokens += args.steps
    # ---- e2e: the public per-token ABI call with host buffers
    barrier()
    e0 = time.perf_counter()
    tok = cur
    for i in range(args.steps):
        tok, _ = g.qwen3_forward(tok, rt.total_tokens + i, logits=True)
    barrier()
    e2e_s = time.perf_counter() - e0
    rt.total_tokens += args.steps

    ms_t = torch.tensor([ms / 1000.0, e2e_s], dtype=torch.float64, device=f"cuda:{local}")
    if dist is not None:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    step_s, e2e_s = float(ms_t[0]), float(ms_t[1])
    tokens_total = args.steps * (1 if tp is not None else world)
    value = tokens_total / step_s
    e2e_v = tokens_total / e2e_s

    # ---- roofline.  Persistent mode: the dominant (only large) kernel is the
    # step kernel itself, one launch per token, so its achieved bandwidth is
    # the step's algorithmic bytes over the device-timed step.  Per-kernel
    # mode: the quantised GEMV on the gate/up shape, timed alone.
    hbm, peak_kind = peaks()
    T = rt.tensors
    persistent = g.qwen3_step_kernels(True) <= 4
    shapes = {}
    lm_name = "output.weight" if "output.weight" in T else "token_embd.weight"  # tied lm_head (0.6B)
    for name in (("blk.0.ffn_gate.weight", "blk.0.ffn_down.weight", "blk.0.attn_q.weight", lm_name)
                 if tp is None else ()):  # (under TP only the shards are resident)
        t = T[name]
        us = g.time_matvec(t, iters=20)
        alg = t.nbytes + t.cols // 32 * 36 + t.rows * 4
        shapes[name] = {"dtype": {10: "Q4_K", 12: "Q6_K", 6: "Q8_0"}[t.dtype], "rows": t.rows,
                        "cols": t.cols, "us": us, "gbs": alg / us / 1e3, "frac": alg / us / 1e3 / hbm}
    w_bytes, kv_bytes = model_bytes(tensors, shape, start_pos + args.steps // 2)
    step_bytes = w_bytes + kv_bytes
    traffic_key = "decode_step_qwen3_8b_bytes" if persistent else "gemv_q4_k_gateup_2x12288x4096_bytes"
    traffic = _ncu_traffic(traffic_key)
    if persistent:
        gbs = step_bytes / (step_s / args.steps) / 1e9
        dom = {"gbs": gbs, "frac": gbs / hbm}
        dom_desc = ("k_decode_step (the whole layer chain + lm_head in one persistent launch per token; "
                    "timed with CUDA events over the K graph replays, which add 3 small kernels)")
    else:
        # the fused gate/up launch (two Q4_K 12288x4096 matrices, RMSNorm
        # prologue, SwiGLU + Q8_1 epilogue), launched as the decode step
        # launches it, back to back over the layers (each launch streams its
        # own layer's weights from HBM)
        ffn_us, ffn_bytes = g.qwen3_time_ffn(iters=2 * shape.layers)
        dom = {"us": ffn_us, "gbs": ffn_bytes / ffn_us / 1e3, "frac": ffn_bytes / ffn_us / 1e3 / hbm,
               "bytes": ffn_bytes}
        dom_desc = (f"k_gemv<Q4_K> fused ffn gate/up (2 x {shape.ffn}x{shape.hidden} Q4_K + RMSNorm, SwiGLU, Q8_1 "
                    f"out) as the decode step launches it, CUDA events over {2 * shape.layers} back-to-back launches "
                    f"rotating the {shape.layers} layers")
    kernels = g.qwen3_step_kernels(True)

    line = {
        "metric": metric_name(args.shape),
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": 1000.0 * step_s / args.steps,
        "higher_is_better": True,
        "scaling": "strong" if tp is not None else "weak",
        "vs_baseline": None,
        "dtype": "q4_k/q6_k x q8_1 (int8 dp4a, f32 accumulate)",
        "data": "synthetic: seeded N(0,0.02) weights quantised Q4_K_M-style, 512 uniform random prompt ids",
        "config": {
            "workload": f"{args.shape}-shape Q4_K_M greedy decode after a {args.prompt}-token prompt "
                        f"(BASELINE config {4 if args.shape == 'qwen3-32b' else 0 if args.shape == 'qwen3-0.6b' else 2})",
            "layers": shape.layers, "hidden": shape.hidden, "heads": shape.heads, "kv_heads": shape.kv_heads,
            "ffn": shape.ffn, "vocab": shape.vocab, "prompt": args.prompt, "decode_positions": [start_pos, start_pos + args.steps],
            "kv_cache": "f32",
            "parallelism": (f"tp{world} (heads/FFN/vocab shards, P2P all-reduce over NVLink)" if tp is not None
                            else f"replicas x{world}" if world > 1 else "single gpu"),
            "l2": "weights 4.9 GB per step >> 126 MB L2 (no flush needed)",
            "weights_bytes": w_bytes,
            "step_bytes_mean": step_bytes,
            "step_hbm_frac": step_bytes / (1000.0 * step_s / args.steps) / 1e6 / hbm,
            "prefill_s": t_pf, "prefill_tokenwise_s": t_pf_tok, "load_s": t_load, "synth_s": t_gen,
            "wall_timed_s": wall,
        },
        "e2e": {"value": e2e_v, "unit": "tok/s", "h2d_bytes_per_step": STATE_BYTES, "d2h_bytes_per_step": STATE_BYTES},
        "gpu_launches": kernels * args.steps,
        "roofline": {"bound": "hbm", "achieved": dom["gbs"], "peak": hbm, "unit": "GB/s", "frac": dom["frac"],
                     "traffic": traffic, "peak_kind": peak_kind, "kernel": dom_desc,
                     "algorithmic_bytes_per_launch": step_bytes if persistent else dom["bytes"],
                     "gemv_sweep": shapes},
        "decode_mode": "persistent" if persistent else ("chained" if kernels == 4 + 2 * shape.layers else "per-kernel"),
        "clocks": clk,
    }
    if rank == 0 and world == 1 and args.cpu_sample > 0:
        try:
            cps, kind = cpu_reference(shape, tensors, args.cpu_sample, args.prompt, os.cpu_count() or 1)
            line["cpu_baseline"] = {"value": cps, "unit": "tok/s", "cores": os.cpu_count() or 1, "kind": kind,
                                    "sample": f"median of 3 windows of {args.cpu_sample} decode tokens (after one warm-up token) "
                                              f"following {args.prompt} seeded KV positions, reference cpu_kernels.c "
                                              "AVX2 matvec in a pthread row pool, f32 activations"}
        except Exception as exc:  # the GPU line must still print
            line["cpu_baseline"] = {"value": None, "error": str(exc)[:200]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    rt.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
