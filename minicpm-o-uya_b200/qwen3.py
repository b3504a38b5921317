"""Qwen3 text runtime over the B200 helper (mirror of src/minicpmo/qwen3.uya).

* :meth:`Qwen3Runtime.open`      -- qwen3_open_runtime (qwen3.uya:2728-2763): bind
  weights (GGUF file or in-memory synthetic tensors), upload them once,
  runtime context = min(context_length, 4096) (qwen3.uya:2238-2242)
* :meth:`append_prompt_ids`      -- tokenwise prefill, logits only for the last id
  (qwen3.uya:2485-2506)
* :meth:`generate`               -- greedy decode (qwen3_generate_capture_timed,
  qwen3.uya:2559-2639; argmax_penalized for vocab > 256, qwen3.uya:2078)
* :meth:`bench`                  -- the ``bench`` command's prompt/decode timing and
  its output lines (qwen3.uya:2774-2973), timed with a wall clock instead of
  the reference's process-CPU ``clock()`` (qwen3.uya:2365-2367)

Each forwarded token is one call of the helper's fused decode-step extension
(one CUDA graph launch) instead of ~20 ABI calls per layer.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from .gguf import GgufFile, Qwen3Shape
from .gpu import GpuContext, Qwen3Config, Tensor

RUNTIME_CONTEXT_CAP = 4096  # qwen3.uya:104 (QWEN3_FORWARD_MAX_CONTEXT)


def rope_table(context: int, head_dim: int, base: float, scale: float = 1.0) -> Tuple[np.ndarray, np.ndarray]:
    """qwen3_precompute_rope (qwen3.uya:1633-1662) in f32, as the host does."""
    half = head_dim // 2
    pos = np.arange(context, dtype=np.float32)[:, None]
    d = np.arange(half, dtype=np.float32)[None, :]
    theta = (pos * np.float32(scale)) / np.power(np.float32(base), (2 * d) / np.float32(head_dim)).astype(np.float32)
    return np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)


@dataclass
class Qwen3Runtime:
    shape: Qwen3Shape
    gpu: GpuContext
    tensors: Dict[str, Tensor]
    context: int
    total_tokens: int = 0
    last_token: int = 0
    seen: List[int] = field(default_factory=list)

    @classmethod
    def open(cls, weights, shape: Optional[Qwen3Shape] = None, device_index: int = 0, kv_f16: bool = False,
             context: Optional[int] = None, debug: bool = False, decode_mode: int = 0,
             tp: Optional["TensorParallel"] = None, max_batch: int = 0,
             batch_exact: bool = False) -> "Qwen3Runtime":
        """weights: a GGUF path/GgufFile, or a list of (name, dtype, rows, cols, uint8 bytes).
        decode_mode 0: the default (one kernel per operation); 1: one kernel per operation; 2: one
        persistent kernel per decode step where the model fits it; 3: per layer the attention and one
        launch chaining the o, gate/up, down and next q/k/v GEMVs (same results in every mode).
        tp: tensor parallelism over the ranks of one node (`TensorParallel`, one process per GPU);
        every rank opens with the same weights and drives the same tokens.
        max_batch 2..32: also bind the batched decode of that many independent sequences
        (every linear weight Q8_0; forward_batch / append_prompt_batch / generate_batch)."""
        if isinstance(weights, (str,)) or hasattr(weights, "__fspath__"):
            weights = GgufFile(weights)
        if isinstance(weights, GgufFile):
            shape = shape or weights.shape()
            items = [(t.name, t.dtype, t.rows, t.cols, t.data) for t in weights.tensors.values()]
        else:
            items = list(weights)
            if shape is None:
                raise ValueError("shape is required for in-memory weights")
        gpu = GpuContext(device_index, debug=debug)
        gpu.smoke()
        tensors = {}
        for name, dt, rows, cols, data in items:
            t = Tensor(name, np.ascontiguousarray(data), dt, rows, cols)
            gpu.upload_tensor(t)
            tensors[name] = t
        ctx = min(shape.context, RUNTIME_CONTEXT_CAP) if context is None else context
        cfg = Qwen3Config()
        cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads = shape.layers, shape.hidden, shape.heads, shape.kv_heads
        cfg.head_dim, cfg.ffn, cfg.vocab, cfg.context = shape.head_dim, shape.ffn, shape.vocab, ctx
        cfg.rms_eps = 1e-6  # the reference forward's fixed eps (qwen3.uya:108)
        cfg.rope_freq_base = shape.rope_base
        cfg.rope_freq_scale = 1.0
        cfg.kv_f16 = int(kv_f16)
        cfg.decode_mode = int(decode_mode)
        cfg.max_batch = int(max_batch)
        cfg.batch_exact = int(bool(batch_exact))
        if tp is not None and tp.world > 1:
            handles = tp.all_gather(gpu.tp_buffer(shape.hidden))
            gpu.qwen3_bind_tp(cfg, tp.rank, tp.world, handles)
            tp.all_gather(b"")  # every rank bound (exchange flags zeroed) before any decodes
        else:
            gpu.qwen3_bind(cfg)
        return cls(shape=shape, gpu=gpu, tensors=tensors, context=ctx)

    def close(self) -> None:
        self.gpu.close()

    # -- decode ------------------------------------------------------------
    def forward(self, token: int, pos: int, logits: bool = True, penalty: float = 1.0,
                want_logits: Optional[np.ndarray] = None) -> Tuple[int, float]:
        return self.gpu.qwen3_forward(int(token), int(pos), logits=logits, penalty=penalty, want_logits=want_logits)

    def append_prompt_ids(self, ids: Sequence[int], penalty: float = 1.0) -> Tuple[int, float]:
        if len(ids) == 0:
            raise ValueError("error: empty prompt")
        if self.total_tokens + len(ids) > self.context:
            raise ValueError(f"error: context overflow total_tokens={self.total_tokens} add_tokens={len(ids)} "
                             f"runtime_context={self.context}")
        nxt, gap = 0, 0.0
        for i, tok in enumerate(ids):
            last = i + 1 == len(ids)
            nxt, gap = self.forward(tok, self.total_tokens, logits=last, penalty=penalty)
            self.seen.append(int(tok))
            self.total_tokens += 1
        self.last_token = nxt
        return nxt, gap

    def prefill_prompt_ids(self, ids: Sequence[int], penalty: float = 1.0,
                           want_logits: Optional[np.ndarray] = None) -> Tuple[int, float]:
        """append_prompt_ids through the multi-token prefill (weights streamed once per 4 tokens);
        the same cache, logits and next token as the token-by-token loop."""
        if len(ids) == 0:
            raise ValueError("error: empty prompt")
        if self.total_tokens + len(ids) > self.context:
            raise ValueError(f"error: context overflow total_tokens={self.total_tokens} add_tokens={len(ids)} "
                             f"runtime_context={self.context}")
        nxt, gap = self.gpu.qwen3_prefill([int(t) for t in ids], self.total_tokens, logits=True, penalty=penalty,
                                          want_logits=want_logits)
        self.seen.extend(int(t) for t in ids)
        self.total_tokens += len(ids)
        self.last_token = nxt
        return nxt, gap

    def append_prompt_embeddings(self, placeholder_id: int, embeddings, penalty: float = 1.0,
                                 want_logits: Optional[np.ndarray] = None) -> Tuple[int, float]:
        """qwen3_append_prompt_embeddings (qwen3.uya:2534-2557): each row of
        embeddings [n][hidden] (f32) is forwarded in place of a token's
        embedding at the next position, recorded as placeholder_id; logits
        (and the greedy next token) only for the last row."""
        e = np.ascontiguousarray(embeddings, np.float32).reshape(-1, self.shape.hidden)
        n = e.shape[0]
        if n == 0:
            return self.last_token, 0.0
        if self.total_tokens + n > self.context:
            raise ValueError(f"error: context overflow total_tokens={self.total_tokens} add_embeddings={n} "
                             f"runtime_context={self.context}")
        nxt, gap = 0, 0.0
        for i in range(n):
            last = i + 1 == n
            nxt, gap = self.gpu.qwen3_forward_embedding(e[i], placeholder_id, self.total_tokens, logits=last,
                                                        penalty=penalty, want_logits=want_logits if last else None)
            self.seen.append(int(placeholder_id))
            self.total_tokens += 1
        self.last_token = nxt
        return nxt, gap

    def generate(self, n_new: int, penalty: float = 1.0, stop_token: Optional[int] = None) -> List[int]:
        """Greedy decode after append_prompt_ids; host loop, one forward per token."""
        out = []
        tok = self.last_token
        for _ in range(n_new):
            if self.total_tokens >= self.context:
                break
            out.append(tok)
            if stop_token is not None and tok == stop_token:
                break
            nxt, _ = self.forward(tok, self.total_tokens, logits=True, penalty=penalty)
            self.seen.append(tok)
            self.total_tokens += 1
            tok = nxt
        self.last_token = tok
        return out

    # -- batched decode (max_batch independent sequences) --------------------
    def forward_batch(self, tokens, positions, logits: bool = True, want_logits: bool = False):
        """One step of every sequence: (next tokens, top-2 gaps, logits [n, vocab] or None)."""
        return self.gpu.qwen3_forward_batch(tokens, positions, logits=logits, want_logits=want_logits)

    def append_prompt_batch(self, prompts) -> Tuple[np.ndarray, np.ndarray]:
        """Forward equal-length prompts [n_seq][P] position by position (logits only at the last);
        returns each sequence's next token and top-2 gap."""
        ids = np.asarray(prompts, dtype=np.uint32)
        if ids.ndim != 2 or ids.shape[1] == 0:
            raise ValueError("error: prompts must be [n_seq][P] with P > 0")
        n, P = ids.shape
        start = getattr(self, "batch_tokens", 0)
        if start + P > self.context:
            raise ValueError(f"error: context overflow total_tokens={start} add_tokens={P} runtime_context={self.context}")
        nxt, gap = None, None
        for i in range(P):
            pos = np.full(n, start + i, np.uint32)
            nxt, gap, _ = self.gpu.qwen3_forward_batch(ids[:, i], pos, logits=(i + 1 == P))
        self.batch_tokens = start + P
        self.batch_last = nxt
        return nxt, gap

    def generate_batch(self, n_new: int) -> np.ndarray:
        """Greedy decode of every sequence after append_prompt_batch, the sampled tokens fed back on
        the device; returns [n_seq][n] (the first column is the token sampled from the prompt)."""
        start = self.batch_tokens
        n = min(n_new, self.context - start)
        if n <= 0:
            return np.zeros((len(self.batch_last), 0), np.uint32)
        first = np.asarray(self.batch_last, np.uint32)
        toks = self.gpu.qwen3_decode_batch(first, np.full(first.size, start, np.uint32), n)
        out = np.concatenate([first[:, None], toks[:, :-1]], axis=1)
        self.batch_tokens = start + n
        self.batch_last = toks[:, -1].copy()
        return out

    def generate_device(self, n_new: int, penalty: float = 1.0) -> List[int]:
        """Greedy decode with the sampled token fed back on the device (no host round trip per token)."""
        n = min(n_new, self.context - self.total_tokens)
        if n <= 0:
            return []
        toks = self.gpu.qwen3_decode(self.last_token, self.total_tokens, n, penalty)
        out = [self.last_token] + [int(t) for t in toks[:-1]]
        self.total_tokens += n
        self.last_token = int(toks[-1])
        return out

    def reset(self) -> None:
        self.total_tokens = 0
        self.seen.clear()
        self.gpu.qwen3_reset()

    # -- bench (qwen3.uya:2774-2973) --------------------------------------
    def bench(self, prompt_ids: Sequence[int], n_gen: int, repetitions: int = 1) -> Dict[str, float]:
        prompt_us = decode_us = first_us = 0.0
        for _ in range(repetitions):
            self.reset()
            t0 = time.perf_counter()
            self.append_prompt_ids(prompt_ids)
            t1 = time.perf_counter()
            prompt_us += (t1 - t0) * 1e6
            # bench feeds the seed ids cyclically with logits every step (qwen3.uya:2412-2432)
            t2 = time.perf_counter()
            for i in range(n_gen):
                ts = time.perf_counter()
                self.forward(int(prompt_ids[i % len(prompt_ids)]), self.total_tokens, logits=True)
                self.total_tokens += 1
                if i == 0:
                    first_us += (time.perf_counter() - ts) * 1e6
            decode_us += (time.perf_counter() - t2) * 1e6
        return {
            "prompt_tokens": len(prompt_ids) * repetitions,
            "prompt_us": prompt_us,
            "decode_tokens": n_gen * repetitions,
            "decode_us": decode_us,
            "first_token_us": first_us,
        }


def format_bench_lines(r: Dict[str, float], repetitions: int, stats: dict) -> List[str]:
    """The reference's bench rate lines (qwen3.uya:2374-2399, 2950-2971), in its integer arithmetic:
    times are whole microseconds, the rate is units * 10^9 // micros (tokens/s x 1000)."""
    def rate(label, units, us):
        micros = int(us)
        scaled = units * 1_000_000_000 // micros if micros else 0
        return (f"bench {label}: {scaled // 1000}.{scaled % 1000:03d} tokens/s units={units} "
                f"ms={micros // 1000}.{micros % 1000:03d} repetitions={repetitions}")

    return [
        rate("text_prompt", int(r["prompt_tokens"]), r["prompt_us"]),
        rate("text_decode", int(r["decode_tokens"]), r["decode_us"]),
        f"bench first_token: us={int(r['first_token_us'])} avg_us={int(r['first_token_us']) // max(repetitions, 1)} "
        f"repetitions={repetitions}",
        "bench backend: hot_matvec=b200_sm100a_q8_1_dp4a_gemv attention=cuda kv_cache=device prefill=tokenwise "
        f"device_index=0 quant_path=native_q8_1_vecdot device_cache=resident weights_uploaded={stats['uploaded_weight_count']}",
        f"bench transfer: backend_init_ms={stats['backend_init_us'] // 1000}.{stats['backend_init_us'] % 1000:03d} "
        f"host_to_device_bytes={stats['host_to_device_bytes']} device_to_host_bytes={stats['device_to_host_bytes']} "
        f"weights_device_bytes={stats['weight_upload_bytes']} kv_device_bytes={stats['kv_device_bytes']}",
        "bench: PASS",
    ]


class TensorParallel:
    """Rank, world size and an all-gather of small byte strings between the ranks of one node.

    The default all-gather uses the initialised ``torch.distributed`` process group (any backend);
    a host embedding the library can pass its own (``gather(bytes) -> list of bytes in rank order``).
    """

    def __init__(self, rank: int, world: int, gather=None):
        self.rank, self.world = int(rank), int(world)
        self._gather = gather

    def all_gather(self, blob: bytes) -> List[bytes]:
        if self._gather is not None:
            return list(self._gather(blob))
        import torch.distributed as dist

        out: List[object] = [None] * self.world
        dist.all_gather_object(out, bytes(blob))
        return [bytes(b) for b in out]

    @classmethod
    def from_env(cls) -> "TensorParallel":
        import os

        return cls(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
