"""ctypes façade over libminicpmo_gpu_helper.so.

Mirrors the reference's Uya façade ``src/minicpmo/gpu.uya`` (``gpu_context_open``,
``gpu_context_upload_tensor``, ``gpu_context_slot_*``, ...): every call checks
the C return code and raises :class:`GpuError` carrying the helper's
``error: ...`` message, the way ``gpu.uya`` surfaces ``gpu_context_last_error``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence, Tuple

import numpy as np

ERR_CAP = 512  # gpu.uya:9

u32, i32, sz, f32, vp, cp = C.c_uint32, C.c_int, C.c_size_t, C.c_float, C.c_void_p, C.c_char_p
fptr = C.POINTER(C.c_float)
u32ptr = C.POINTER(C.c_uint32)
i32ptr = C.POINTER(C.c_int32)


class GpuStats(C.Structure):
    """gpu_bridge.c:11-25 (13 x u64)."""

    _fields_ = [
        (n, C.c_uint64)
        for n in (
            "backend_init_us",
            "host_to_device_bytes",
            "device_to_host_bytes",
            "weight_upload_bytes",
            "scratch_x_bytes",
            "scratch_y_bytes",
            "uploaded_weight_count",
            "native_quant_matvec_count",
            "staged_quant_matvec_count",
            "q8_1_x_bytes",
            "attention_kernel_calls",
            "kv_device_bytes",
            "kv_host_to_device_bytes",
        )
    ]

    def as_dict(self) -> dict:
        return {n: int(getattr(self, n)) for n, _ in self._fields_}


class Qwen3Config(C.Structure):
    """minicpmo_qwen3_config of include/minicpmo_gpu.h."""

    _fields_ = [
        ("layers", u32),
        ("hidden", u32),
        ("heads", u32),
        ("kv_heads", u32),
        ("head_dim", u32),
        ("ffn", u32),
        ("vocab", u32),
        ("context", u32),
        ("rms_eps", f32),
        ("rope_freq_base", f32),
        ("rope_freq_scale", f32),
        ("rope_cos", fptr),
        ("rope_sin", fptr),
        ("kv_f16", i32),
        ("max_batch", i32),
        ("decode_mode", i32),
        ("batch_exact", i32),
        ("reserved", i32 * 4),
    ]


REFERENCE_SYMBOLS = (
    "minicpmo_gpu_context_create",
    "minicpmo_gpu_context_destroy",
    "minicpmo_gpu_context_smoke",
    "minicpmo_gpu_context_upload_tensor",
    "minicpmo_gpu_context_matvec",
    "minicpmo_gpu_context_prepare_attention",
    "minicpmo_gpu_context_attention",
    "minicpmo_gpu_context_slot_upload_f32",
    "minicpmo_gpu_context_slot_download_f32",
    "minicpmo_gpu_context_slot_matvec",
    "minicpmo_gpu_context_slot_matvec2",
    "minicpmo_gpu_context_slot_matvec3",
    "minicpmo_gpu_context_slot_rms_norm",
    "minicpmo_gpu_context_slot_head_norm",
    "minicpmo_gpu_context_slot_rope",
    "minicpmo_gpu_context_slot_add_inplace",
    "minicpmo_gpu_context_slot_silu_mul",
    "minicpmo_gpu_context_attention_slots",
    "minicpmo_gpu_context_snapshot",
)

E = [cp, sz]  # (char *error, size_t error_cap)
SIGNATURES = {
    "minicpmo_gpu_context_create": (i32, [C.c_uint, i32, C.POINTER(vp)] + E),
    "minicpmo_gpu_context_destroy": (None, [vp]),
    "minicpmo_gpu_context_smoke": (i32, [vp] + E),
    "minicpmo_gpu_context_upload_tensor": (i32, [vp, cp, vp, sz, i32, sz, sz] + E),
    "minicpmo_gpu_context_matvec": (i32, [vp, cp, vp, i32, fptr, sz, sz, fptr] + E),
    "minicpmo_gpu_context_prepare_attention": (i32, [vp, sz, sz, sz] + E),
    "minicpmo_gpu_context_attention": (i32, [vp, fptr, fptr, fptr, sz, sz, sz, sz, sz, sz, fptr] + E),
    "minicpmo_gpu_context_slot_upload_f32": (i32, [vp, C.c_uint, fptr, sz] + E),
    "minicpmo_gpu_context_slot_download_f32": (i32, [vp, C.c_uint, fptr, sz] + E),
    "minicpmo_gpu_context_slot_matvec": (i32, [vp, C.c_uint, cp, vp, i32, C.c_uint, sz, sz] + E),
    "minicpmo_gpu_context_slot_matvec2": (i32, [vp, C.c_uint, cp, vp, i32, sz, C.c_uint, cp, vp, i32, sz, C.c_uint, sz] + E),
    "minicpmo_gpu_context_slot_matvec3": (
        i32,
        [vp, C.c_uint, cp, vp, i32, sz, C.c_uint, cp, vp, i32, sz, C.c_uint, cp, vp, i32, sz, C.c_uint, sz] + E,
    ),
    "minicpmo_gpu_context_slot_rms_norm": (i32, [vp, C.c_uint, C.c_uint, vp, sz, f32] + E),
    "minicpmo_gpu_context_slot_head_norm": (i32, [vp, C.c_uint, vp, sz, sz] + E),
    "minicpmo_gpu_context_slot_rope": (i32, [vp, C.c_uint, sz, sz, sz, f32, f32, fptr, fptr, sz] + E),
    "minicpmo_gpu_context_slot_add_inplace": (i32, [vp, C.c_uint, C.c_uint, sz] + E),
    "minicpmo_gpu_context_slot_silu_mul": (i32, [vp, C.c_uint, C.c_uint, C.c_uint, sz] + E),
    "minicpmo_gpu_context_attention_slots": (i32, [vp, C.c_uint, C.c_uint, C.c_uint, C.c_uint, sz, sz, sz, sz, sz, sz] + E),
    "minicpmo_gpu_context_snapshot": (None, [vp, C.POINTER(GpuStats)]),
    # extensions
    "minicpmo_gpu_abi_version": (i32, []),
    "minicpmo_gpu_context_stream": (vp, [vp]),
    "minicpmo_gpu_context_set_stream": (i32, [vp, vp] + E),
    "minicpmo_gpu_context_embed_lookup": (i32, [vp, C.c_uint, vp, i32, u32, sz] + E),
    "minicpmo_gpu_context_argmax_penalized": (i32, [vp, C.c_uint, sz, u32ptr, sz, f32, u32ptr, fptr] + E),
    "minicpmo_gpu_context_qwen3_bind": (i32, [vp, C.POINTER(Qwen3Config)] + E),
    "minicpmo_gpu_context_tp_buffer": (i32, [vp, sz, vp] + E),
    "minicpmo_gpu_context_qwen3_bind_tp": (i32, [vp, C.POINTER(Qwen3Config), i32, i32, vp] + E),
    "minicpmo_gpu_context_qwen3_forward": (i32, [vp, u32, sz, i32, f32, u32ptr, fptr, fptr, fptr] + E),
    "minicpmo_gpu_context_qwen3_forward_embedding": (i32, [vp, fptr, sz, u32, sz, i32, f32, u32ptr, fptr, fptr, fptr] + E),
    "minicpmo_gpu_context_qwen3_sample": (i32, [vp, u32ptr, sz, f32, u32, f32, f32, f32, u32ptr, u32ptr] + E),
    "minicpmo_gpu_context_qwen3_prefill": (i32, [vp, u32ptr, sz, sz, i32, f32, u32ptr, fptr, fptr] + E),
    "minicpmo_gpu_context_qwen3_reset": (i32, [vp] + E),
    "minicpmo_gpu_context_qwen3_kv_write": (i32, [vp, sz, sz, sz, vp, vp] + E),
    "minicpmo_gpu_context_qwen3_kv_read": (i32, [vp, sz, sz, sz, vp, vp] + E),
    "minicpmo_gpu_context_qwen3_decode": (i32, [vp, u32, sz, sz, f32, u32ptr] + E),
    "minicpmo_gpu_context_q8_1_quantize": (i32, [vp, fptr, sz, vp] + E),
    "minicpmo_gpu_context_rms_norm_q8_1": (i32, [vp, fptr, vp, sz, f32, fptr, vp] + E),
    "minicpmo_gpu_context_matvec_q8_1": (i32, [vp, vp, vp, sz, sz, fptr, i32ptr] + E),
    "minicpmo_gpu_context_matvec_f32_input": (i32, [vp, vp, fptr, vp, f32, sz, sz, fptr] + E),
    "minicpmo_gpu_context_time_matvec_input": (i32, [vp, vp, sz, sz, i32, i32, vp, fptr] + E),
    "minicpmo_gpu_context_matmul_q8_0_batch": (i32, [vp, vp, fptr, sz, sz, sz, fptr] + E),
    "minicpmo_gpu_context_time_matmul_q8_0_batch": (i32, [vp, vp, sz, i32, fptr] + E),
    "minicpmo_gpu_context_qwen3_forward_batch": (i32, [vp, sz, u32ptr, u32ptr, i32, u32ptr, fptr, fptr] + E),
    "minicpmo_gpu_context_qwen3_decode_batch": (i32, [vp, sz, u32ptr, u32ptr, sz, u32ptr] + E),
    "minicpmo_gpu_context_qwen3_time_decode_batch": (i32, [vp, sz, u32ptr, u32ptr, sz, fptr] + E),
    "minicpmo_gpu_context_qwen3_batch_kernels": (i32, [vp, i32]),
    "minicpmo_gpu_context_time_matvec": (i32, [vp, vp, sz, sz, i32, fptr] + E),
    "minicpmo_gpu_context_qwen3_time_ffn": (i32, [vp, i32, fptr, C.POINTER(C.c_double)] + E),
    "minicpmo_gpu_context_qwen3_time_decode": (i32, [vp, u32, sz, sz, fptr] + E),
    "minicpmo_gpu_context_tensor_device_bytes": (sz, [vp, vp]),
    "minicpmo_gpu_context_qwen3_step_kernels": (i32, [vp, i32]),
    "minicpmo_gpu_context_qwen3_prefill_passes": (C.c_longlong, [vp, C.POINTER(C.c_longlong)]),
    "minicpmo_gpu_context_qwen3_step_trace": (i32, [vp, vp, sz, u32ptr, u32ptr]),
    "minicpmo_gpu_context_qwen3_graph_trace": (i32, [vp, vp, sz, u32ptr, u32ptr]),
    "minicpmo_gpu_attention_no_alloc": (i32, [vp, vp, vp, i32, sz, sz, sz, sz, sz, vp, vp] + E),
}


def declare(lib: C.CDLL) -> None:
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


class GpuError(RuntimeError):
    pass


def _f(a: np.ndarray):
    return a.ctypes.data_as(fptr)


def _as_f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


@dataclass
class Tensor:
    """A host weight tensor kept alive while uploaded (the registry key is its pointer)."""

    name: str
    data: np.ndarray  # raw GGUF bytes (uint8) or f32/u16 values
    dtype: int
    rows: int
    cols: int

    @property
    def ptr(self) -> int:
        return self.data.ctypes.data

    @property
    def nbytes(self) -> int:
        return self.data.nbytes


class GpuContext:
    """gpu_context_open/close and the slot API (src/minicpmo/gpu.uya:96-315)."""

    def __init__(self, device_index: int = 0, debug: bool = False):
        from . import lib

        self.lib = lib()
        self._err = C.create_string_buffer(ERR_CAP)
        h = vp()
        if not self.lib.minicpmo_gpu_context_create(device_index, int(debug), C.byref(h), self._err, ERR_CAP):
            raise GpuError(self._err.value.decode())
        self.handle = h
        self._keep: dict = {}

    # -- plumbing --
    def _call(self, name: str, *args):
        ok = getattr(self.lib, name)(self.handle, *args, self._err, ERR_CAP)
        if not ok:
            raise GpuError(self._err.value.decode())
        return ok

    def close(self) -> None:
        if self.handle:
            self.lib.minicpmo_gpu_context_destroy(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- reference ABI --
    def smoke(self) -> None:
        self._call("minicpmo_gpu_context_smoke")

    def upload_tensor(self, t: Tensor) -> None:
        self._keep[t.ptr] = t
        self._call("minicpmo_gpu_context_upload_tensor", t.name.encode(), t.ptr, t.nbytes, t.dtype, t.rows, t.cols)

    def matvec(self, t: Tensor, x) -> np.ndarray:
        x = _as_f32(x)
        y = np.empty(t.rows, np.float32)
        self._call("minicpmo_gpu_context_matvec", t.name.encode(), t.ptr, t.dtype, _f(x), t.cols, t.rows, _f(y))
        return y

    def prepare_attention(self, layers: int, context: int, kv_dim: int) -> None:
        self._call("minicpmo_gpu_context_prepare_attention", layers, context, kv_dim)

    def attention(self, q, k, v, layer, pos, heads, kv_heads, head_dim, context) -> np.ndarray:
        q, k, v = _as_f32(q), _as_f32(k), _as_f32(v)
        out = np.empty(heads * head_dim, np.float32)
        self._call("minicpmo_gpu_context_attention", _f(q), _f(k), _f(v), layer, pos, heads, kv_heads, head_dim, context, _f(out))
        return out

    def slot_upload(self, slot: int, x) -> None:
        x = _as_f32(x)
        self._call("minicpmo_gpu_context_slot_upload_f32", slot, _f(x), x.size)

    def slot_download(self, slot: int, n: int) -> np.ndarray:
        y = np.empty(n, np.float32)
        self._call("minicpmo_gpu_context_slot_download_f32", slot, _f(y), n)
        return y

    def slot_matvec(self, dst: int, t: Tensor, src: int) -> None:
        self._call("minicpmo_gpu_context_slot_matvec", dst, t.name.encode(), t.ptr, t.dtype, src, t.cols, t.rows)

    def slot_matvec2(self, dst0: int, t0: Tensor, dst1: int, t1: Tensor, src: int) -> None:
        self._call(
            "minicpmo_gpu_context_slot_matvec2", dst0, t0.name.encode(), t0.ptr, t0.dtype, t0.rows,
            dst1, t1.name.encode(), t1.ptr, t1.dtype, t1.rows, src, t0.cols,
        )

    def slot_matvec3(self, dst0, t0: Tensor, dst1, t1: Tensor, dst2, t2: Tensor, src: int) -> None:
        self._call(
            "minicpmo_gpu_context_slot_matvec3", dst0, t0.name.encode(), t0.ptr, t0.dtype, t0.rows,
            dst1, t1.name.encode(), t1.ptr, t1.dtype, t1.rows, dst2, t2.name.encode(), t2.ptr, t2.dtype, t2.rows,
            src, t0.cols,
        )

    def slot_rms_norm(self, dst: int, src: int, w: Tensor, n: int, eps: float = 1e-6) -> None:
        self._call("minicpmo_gpu_context_slot_rms_norm", dst, src, w.ptr, n, eps)

    def slot_head_norm(self, slot: int, w: Tensor, heads: int, head_dim: int) -> None:
        self._call("minicpmo_gpu_context_slot_head_norm", slot, w.ptr, heads, head_dim)

    def slot_rope(self, slot, heads, head_dim, pos, base, scale, cos_t=None, sin_t=None, rope_ctx=0) -> None:
        if cos_t is not None:
            cos_t, sin_t = _as_f32(cos_t), _as_f32(sin_t)
            self._keep[("rope", cos_t.ctypes.data)] = (cos_t, sin_t)
            self._call("minicpmo_gpu_context_slot_rope", slot, heads, head_dim, pos, base, scale, _f(cos_t), _f(sin_t), rope_ctx)
        else:
            self._call("minicpmo_gpu_context_slot_rope", slot, heads, head_dim, pos, base, scale, None, None, 0)

    def slot_add_inplace(self, dst: int, src: int, n: int) -> None:
        self._call("minicpmo_gpu_context_slot_add_inplace", dst, src, n)

    def slot_silu_mul(self, dst: int, gate: int, up: int, n: int) -> None:
        self._call("minicpmo_gpu_context_slot_silu_mul", dst, gate, up, n)

    def attention_slots(self, dst, q, k, v, layer, pos, heads, kv_heads, head_dim, context) -> None:
        self._call("minicpmo_gpu_context_attention_slots", dst, q, k, v, layer, pos, heads, kv_heads, head_dim, context)

    def snapshot(self) -> dict:
        s = GpuStats()
        self.lib.minicpmo_gpu_context_snapshot(self.handle, C.byref(s))
        return s.as_dict()

    # -- extensions --
    @property
    def stream(self) -> int:
        return int(self.lib.minicpmo_gpu_context_stream(self.handle) or 0)

    def embed_lookup(self, dst: int, t: Tensor, token: int) -> None:
        self._call("minicpmo_gpu_context_embed_lookup", dst, t.ptr, t.dtype, token, t.cols)

    def argmax_penalized(self, slot: int, n: int, seen: Sequence[int] = (), penalty: float = 1.0):
        seen_a = np.ascontiguousarray(np.asarray(seen, dtype=np.uint32))
        out = u32()
        gap = f32()
        self._call(
            "minicpmo_gpu_context_argmax_penalized", slot, n, seen_a.ctypes.data_as(u32ptr), seen_a.size, penalty,
            C.byref(out), C.byref(gap),
        )
        return int(out.value), float(gap.value)

    def qwen3_bind(self, cfg: Qwen3Config) -> None:
        self._keep["qwen3_cfg"] = cfg
        self._vocab = int(cfg.vocab)
        self._call("minicpmo_gpu_context_qwen3_bind", C.byref(cfg))

    def tp_buffer(self, hidden: int) -> bytes:
        """Allocate this rank's tensor-parallel exchange buffer; returns its 64-byte CUDA IPC handle."""
        h = C.create_string_buffer(64)
        self._call("minicpmo_gpu_context_tp_buffer", hidden, C.cast(h, C.c_void_p))
        return h.raw

    def qwen3_bind_tp(self, cfg: Qwen3Config, rank: int, world: int, handles: Sequence[bytes]) -> None:
        blob = b"".join(handles)
        if len(blob) != 64 * world:
            raise GpuError("error: qwen3_bind_tp needs one 64-byte handle per rank")
        buf = C.create_string_buffer(blob, len(blob))
        self._keep["qwen3_cfg"] = cfg
        self._keep["tp_handles"] = buf
        self._call("minicpmo_gpu_context_qwen3_bind_tp", C.byref(cfg), rank, world, C.cast(buf, C.c_void_p))

    def qwen3_forward(self, token: int, pos: int, logits: bool = True, penalty: float = 1.0,
                      want_logits: Optional[np.ndarray] = None, want_hidden: Optional[np.ndarray] = None):
        out = u32()
        gap = f32()
        self._call(
            "minicpmo_gpu_context_qwen3_forward", token, pos, 0 if logits else 1, penalty, C.byref(out), C.byref(gap),
            _f(want_logits) if want_logits is not None else None,
            _f(want_hidden) if want_hidden is not None else None,
        )
        return int(out.value), float(gap.value)

    def qwen3_forward_embedding(self, embedding, placeholder_id: int, pos: int, logits: bool = True,
                                penalty: float = 1.0, want_logits: Optional[np.ndarray] = None,
                                want_hidden: Optional[np.ndarray] = None):
        """One step on a given f32 input row instead of a token's embedding
        (qwen3_append_prompt_embeddings, qwen3.uya:2534-2557); the
        placeholder id joins the repeat penalty's seen set."""
        e = _as_f32(embedding)
        out = u32()
        gap = f32()
        self._call(
            "minicpmo_gpu_context_qwen3_forward_embedding", _f(e), e.size, placeholder_id, pos, 0 if logits else 1,
            penalty, C.byref(out), C.byref(gap),
            _f(want_logits) if want_logits is not None else None,
            _f(want_hidden) if want_hidden is not None else None,
        )
        return int(out.value), float(gap.value)

    def qwen3_sample(self, seen, temperature: float, top_k: int, top_p: float, min_p: float, penalty: float,
                     seed: int) -> Tuple[int, int]:
        """qwen3_sample (qwen3.uya:2073-2138) on the last forward's logits -> (token, next seed state)."""
        s = np.ascontiguousarray(np.asarray(seen, dtype=np.uint32))
        st = u32(seed)
        out = u32()
        self._call("minicpmo_gpu_context_qwen3_sample", s.ctypes.data_as(u32ptr), s.size, temperature, top_k, top_p,
                   min_p, penalty, C.byref(st), C.byref(out))
        return int(out.value), int(st.value)

    def qwen3_prefill(self, tokens, first_pos: int, logits: bool = True, penalty: float = 1.0,
                      want_logits: Optional[np.ndarray] = None):
        """Prompt tokens in passes over the weights (qwen3_prefill: 16 tokens or more on the tensor cores, 256 per
        pass, else up to 4 per pass through the GEMVs); the same bits as token-by-token forwards."""
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        out = u32()
        gap = f32()
        self._call("minicpmo_gpu_context_qwen3_prefill", t.ctypes.data_as(u32ptr), t.size, first_pos,
                   0 if logits else 1, penalty, C.byref(out), C.byref(gap),
                   _f(want_logits) if want_logits is not None else None)
        return int(out.value), float(gap.value)

    def qwen3_reset(self) -> None:
        self._call("minicpmo_gpu_context_qwen3_reset")

    def qwen3_kv_write(self, layer: int, first_pos: int, k_rows: np.ndarray, v_rows: np.ndarray) -> None:
        """Rows [first_pos, first_pos + len) of one layer's K/V cache from host arrays (f32, or f16 for an
        f16 cache), each row kv_heads * head_dim values."""
        k = np.ascontiguousarray(k_rows)
        v = np.ascontiguousarray(v_rows)
        if k.shape != v.shape or k.ndim != 2:
            raise ValueError("k_rows and v_rows must be [n_pos][kv_dim] arrays of one shape")
        self._call("minicpmo_gpu_context_qwen3_kv_write", layer, first_pos, k.shape[0], k.ctypes.data, v.ctypes.data)

    def qwen3_kv_read(self, layer: int, first_pos: int, n_pos: int, kv_dim: int, dtype=np.float32):
        k = np.empty((n_pos, kv_dim), dtype)
        v = np.empty((n_pos, kv_dim), dtype)
        self._call("minicpmo_gpu_context_qwen3_kv_read", layer, first_pos, n_pos, k.ctypes.data, v.ctypes.data)
        return k, v

    def qwen3_decode(self, first_token: int, first_pos: int, steps: int, penalty: float = 1.0) -> np.ndarray:
        toks = np.empty(steps, np.uint32)
        self._call("minicpmo_gpu_context_qwen3_decode", first_token, first_pos, steps, penalty, toks.ctypes.data_as(u32ptr))
        return toks

    def qwen3_time_decode(self, first_token: int, first_pos: int, steps: int) -> float:
        ms = f32()
        self._call("minicpmo_gpu_context_qwen3_time_decode", first_token, first_pos, steps, C.byref(ms))
        return float(ms.value)

    def q8_1_quantize(self, x) -> np.ndarray:
        x = _as_f32(x)
        out = np.empty(x.size // 32 * 36, np.uint8)
        self._call("minicpmo_gpu_context_q8_1_quantize", _f(x), x.size, out.ctypes.data)
        return out

    def rms_norm_q8_1(self, x, w: Tensor, eps: float = 1e-6):
        x = _as_f32(x)
        out = np.empty(x.size, np.float32)
        xq = np.empty(x.size // 32 * 36, np.uint8) if x.size % 32 == 0 else None
        self._call("minicpmo_gpu_context_rms_norm_q8_1", _f(x), w.ptr, x.size, eps, _f(out),
                   xq.ctypes.data if xq is not None else None)
        return out, xq

    def matvec_q8_1(self, t: Tensor, xq: np.ndarray, dots: bool = False):
        xq = np.ascontiguousarray(xq, dtype=np.uint8)
        y = np.empty(t.rows, np.float32)
        per_row = t.cols // 16 if t.dtype == 12 else t.cols // 32
        d = np.empty((t.rows, per_row), np.int32) if dots else None
        self._call("minicpmo_gpu_context_matvec_q8_1", t.ptr, xq.ctypes.data, t.cols, t.rows, _f(y),
                   d.ctypes.data_as(i32ptr) if d is not None else None)
        return (y, d) if dots else y

    def matvec_f32_input(self, t: Tensor, x, norm: Tensor | None = None, eps: float = 1e-6) -> np.ndarray:
        """GEMV whose kernel quantises x (after RMSNorm with `norm`, if given)."""
        x = _as_f32(x)
        y = np.empty(t.rows, np.float32)
        self._call("minicpmo_gpu_context_matvec_f32_input", t.ptr, _f(x), norm.ptr if norm is not None else None, eps,
                   t.cols, t.rows, _f(y))
        return y

    def matmul_q8_0_batch(self, t: Tensor, x) -> np.ndarray:
        """Tensor-core batched projection: rows of x [n, cols] -> [n, rows] (f16 operands, f32 sums)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim != 2 or x.shape[1] != t.cols:
            raise ValueError("x must be [n_seq, cols]")
        y = np.empty((x.shape[0], t.rows), np.float32)
        self._call("minicpmo_gpu_context_matmul_q8_0_batch", t.ptr, _f(x), x.shape[0], t.cols, t.rows, _f(y))
        return y

    def time_matvec_input(self, t: Tensor, input_mode: int, norm: Optional[Tensor] = None, iters: int = 20) -> float:
        """Mean device time (us) of the GEMV with input mode 0 (Q8_1), 1 (f32) or 2 (RMSNorm + f32)."""
        us = f32()
        self._call("minicpmo_gpu_context_time_matvec_input", t.ptr, t.cols, t.rows, iters, input_mode,
                   norm.ptr if norm is not None else None, C.byref(us))
        return float(us.value)

    def qwen3_time_ffn(self, iters: int = 72) -> Tuple[float, float]:
        """Mean device time (us) of the bound model's fused gate/up GEMV as the
        decode step launches it, over the layers in turn, and its algorithmic
        bytes per launch."""
        us, nbytes = f32(), C.c_double()
        self._call("minicpmo_gpu_context_qwen3_time_ffn", iters, C.byref(us), C.byref(nbytes))
        return float(us.value), float(nbytes.value)

    def time_matvec(self, t: Tensor, iters: int = 20) -> float:
        us = f32()
        self._call("minicpmo_gpu_context_time_matvec", t.ptr, t.cols, t.rows, iters, C.byref(us))
        return float(us.value)

    def time_matmul_q8_0_batch(self, t: Tensor, n_seq: int, iters: int = 10) -> float:
        """Mean device time (us) of the tensor-core projection, L2 flushed before each launch."""
        us = f32()
        self._call("minicpmo_gpu_context_time_matmul_q8_0_batch", t.ptr, n_seq, iters, C.byref(us))
        return float(us.value)

    def qwen3_forward_batch(self, tokens, positions, logits: bool = True, want_logits: bool = False):
        """One batched step: (next tokens, top-2 gaps, logits [n, vocab] or None)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uint32)
        n = t.size
        out_t = np.zeros(n, np.uint32)
        gaps = np.zeros(n, np.float32)
        lg = np.empty((n, self._vocab), np.float32) if (want_logits and logits) else None
        self._call("minicpmo_gpu_context_qwen3_forward_batch", n, t.ctypes.data_as(u32ptr), p.ctypes.data_as(u32ptr),
                   0 if logits else 1, out_t.ctypes.data_as(u32ptr), _f(gaps), _f(lg) if lg is not None else None)
        return out_t, gaps, lg

    def qwen3_decode_batch(self, first_tokens, first_positions, n_steps: int) -> np.ndarray:
        """Greedy decode on the device: tokens [n_seq, n_steps]."""
        t = np.ascontiguousarray(first_tokens, dtype=np.uint32)
        p = np.ascontiguousarray(first_positions, dtype=np.uint32)
        out = np.zeros((t.size, n_steps), np.uint32)
        self._call("minicpmo_gpu_context_qwen3_decode_batch", t.size, t.ctypes.data_as(u32ptr), p.ctypes.data_as(u32ptr),
                   n_steps, out.ctypes.data_as(u32ptr))
        return out

    def qwen3_time_decode_batch(self, first_tokens, first_positions, n_steps: int) -> float:
        t = np.ascontiguousarray(first_tokens, dtype=np.uint32)
        p = np.ascontiguousarray(first_positions, dtype=np.uint32)
        ms = f32()
        self._call("minicpmo_gpu_context_qwen3_time_decode_batch", t.size, t.ctypes.data_as(u32ptr),
                   p.ctypes.data_as(u32ptr), n_steps, C.byref(ms))
        return float(ms.value)

    def qwen3_batch_kernels(self, with_logits: bool = True) -> int:
        return int(self.lib.minicpmo_gpu_context_qwen3_batch_kernels(self.handle, int(with_logits)))

    def qwen3_step_kernels(self, with_logits: bool = True) -> int:
        return int(self.lib.minicpmo_gpu_context_qwen3_step_kernels(self.handle, int(with_logits)))

    def qwen3_prefill_passes(self):
        """(tensor-core passes, multi-vector GEMV passes) of qwen3_prefill so far."""
        g = C.c_longlong()
        tc = self.lib.minicpmo_gpu_context_qwen3_prefill_passes(self.handle, C.byref(g))
        return int(tc), int(g.value)

    def qwen3_step_trace(self):
        """[stage][cta][start, ready, end] ns of the last persistent step (MCPO_STEP_TRACE=1 at bind), or None."""
        ns, nc = u32(), u32()
        self.lib.minicpmo_gpu_context_qwen3_step_trace(self.handle, None, 0, C.byref(ns), C.byref(nc))
        if ns.value == 0:
            return None
        out = np.empty((ns.value, nc.value, 3), np.uint64)
        if not self.lib.minicpmo_gpu_context_qwen3_step_trace(self.handle, out.ctypes.data, out.size, None, None):
            return None
        return out

    def qwen3_graph_trace(self):
        """[launch][cta][8] ns of the last per-operation step (MCPO_GRAPH_TRACE=1 at bind): start, past wait,
        ready, done (attention also blocks done, past the cluster barrier), or None."""
        nl, nc = u32(), u32()
        self.lib.minicpmo_gpu_context_qwen3_graph_trace(self.handle, None, 0, C.byref(nl), C.byref(nc))
        if nl.value == 0:
            return None
        out = np.empty((nl.value, nc.value, 8), np.uint64)
        if not self.lib.minicpmo_gpu_context_qwen3_graph_trace(self.handle, out.ctypes.data, out.size, None, None):
            return None
        return out

    def tensor_device_bytes(self, t: Tensor) -> int:
        return int(self.lib.minicpmo_gpu_context_tensor_device_bytes(self.handle, t.ptr))
