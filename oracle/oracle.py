"""ctypes bindings of the CPU oracle (liboracle.so) and of the reference
builds in oracle/_ref/.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the product package.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path
from typing import Dict, Optional, Sequence

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
REF_DIR = ORACLE_DIR / "_ref"

u8p = C.POINTER(C.c_uint8)
fp = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int32)
u32p = C.POINTER(C.c_uint32)
sz = C.c_size_t


def build(quiet: bool = True) -> None:
    res = subprocess.run(["make", "-C", str(ORACLE_DIR)], capture_output=quiet, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")


_orc = None


def orc() -> C.CDLL:
    global _orc
    if _orc is None:
        path = ORACLE_DIR / "liboracle.so"
        if not path.exists():
            build()
        lib = C.CDLL(str(path))
        sig = {
            "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
            "orc_row_bytes": (sz, [C.c_int, sz]),
            "orc_dequant_row": (C.c_int, [C.c_int, u8p, sz, fp]),
            "orc_q8_1_quantize": (C.c_int, [fp, sz, u8p]),
            "orc_q8_1_block_sums": (C.c_int, [u8p, sz, i32p]),
            "orc_q4_k_block_dots": (C.c_int, [u8p, u8p, sz, i32p, i32p]),
            "orc_q6_k_block_dots": (C.c_int, [u8p, u8p, sz, i32p]),
            "orc_q8_0_block_dots": (C.c_int, [u8p, u8p, sz, i32p]),
            "orc_matvec_q8_1": (C.c_int, [C.c_int, u8p, sz, sz, u8p, fp]),
            "orc_matvec_f32": (C.c_int, [C.c_int, u8p, sz, sz, fp, fp]),
            "orc_rms_norm": (C.c_int, [fp, C.c_void_p, C.c_int, sz, C.c_float, C.c_int, fp]),
            "orc_head_norm": (C.c_int, [fp, C.c_void_p, C.c_int, sz, sz, C.c_int]),
            "orc_rope_table": (C.c_int, [sz, sz, C.c_float, C.c_float, fp, fp]),
            "orc_rope_apply": (C.c_int, [fp, sz, sz, sz, fp, fp]),
            "orc_attention": (C.c_int, [fp, fp, fp, fp, sz, sz, sz, sz, sz, sz]),
            "orc_silu_mul": (None, [fp, fp, fp, sz]),
            "orc_argmax_penalized": (C.c_uint32, [fp, sz, u32p, sz, C.c_float, fp]),
            "orc_sample": (C.c_uint32, [fp, sz, u32p, sz, C.c_float, C.c_uint32, C.c_float, C.c_float, C.c_float,
                                        u32p, fp]),
            "orc_state_kv_floats": (sz, [C.c_void_p]),
            "orc_forward_token": (C.c_int, [C.c_void_p, C.c_void_p, C.c_uint32, sz, fp, fp]),
            "orc_forward_embedding": (C.c_int, [C.c_void_p, C.c_void_p, fp, sz, fp, fp]),
            "orc_pool_create": (C.c_void_p, [C.c_int, C.c_char_p]),
            "orc_pool_destroy": (None, [C.c_void_p]),
            "orc_pool_is_reference": (C.c_int, [C.c_void_p]),
            "orc_state_attach_pool": (None, [C.c_void_p, C.c_void_p]),
            "orc_expf_det": (C.c_float, [C.c_float]),
            "orc_attn_n_split": (C.c_int, [C.c_int]),
            "orc_f32_to_f16_rne": (C.c_uint16, [C.c_float]),
            "orc_matvec_q8_1_dev": (C.c_int, [C.c_int, u8p, sz, sz, u8p, fp]),
            "orc_matvec_dense_dev": (C.c_int, [C.c_int, u8p, sz, sz, fp, fp]),
            "orc_silu_mul_dev": (None, [fp, fp, fp, sz]),
            "orc_attention_dev": (C.c_int, [fp, fp, fp, fp, fp, fp, sz, sz, sz, sz, sz, sz]),
        }
        for n, (r, a) in sig.items():
            fn = getattr(lib, n)
            fn.restype = r
            fn.argtypes = a
        _orc = lib
    return _orc


def _u8(a: np.ndarray):
    return np.ascontiguousarray(a, dtype=np.uint8).ctypes.data_as(u8p)


def _f(a: np.ndarray):
    return a.ctypes.data_as(fp)


def f32_to_f16(v: float) -> int:
    return int(orc().orc_f32_to_f16(C.c_float(v)))


def f16_to_f32(b: int) -> float:
    return float(orc().orc_f16_to_f32(b))


def row_bytes(dtype: int, cols: int) -> int:
    return int(orc().orc_row_bytes(dtype, cols))


def dequant(dtype: int, w: np.ndarray, rows: int, cols: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(rows, -1)
    out = np.empty((rows, cols), np.float32)
    for r in range(rows):
        assert orc().orc_dequant_row(dtype, w[r].ctypes.data_as(u8p), cols, out[r].ctypes.data_as(fp))
    return out


def q8_1_quantize(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size // 32 * 36, np.uint8)
    assert orc().orc_q8_1_quantize(_f(x), x.size, out.ctypes.data_as(u8p))
    return out


def block_dots(dtype: int, w: np.ndarray, rows: int, cols: int, xq: np.ndarray) -> np.ndarray:
    """Per-block int32 dots, [rows][cols/32] (Q4_K, Q8_0) or [rows][cols/16] (Q6_K)."""
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(rows, -1)
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    per = cols // 16 if dtype == 12 else cols // 32
    out = np.empty((rows, per), np.int32)
    tmp = np.empty(per, np.int32)
    for r in range(rows):
        if dtype == 10:
            assert orc().orc_q4_k_block_dots(w[r].ctypes.data_as(u8p), xq.ctypes.data_as(u8p), cols,
                                             out[r].ctypes.data_as(i32p), tmp.ctypes.data_as(i32p))
        elif dtype == 12:
            assert orc().orc_q6_k_block_dots(w[r].ctypes.data_as(u8p), xq.ctypes.data_as(u8p), cols, out[r].ctypes.data_as(i32p))
        else:
            assert orc().orc_q8_0_block_dots(w[r].ctypes.data_as(u8p), xq.ctypes.data_as(u8p), cols, out[r].ctypes.data_as(i32p))
    return out


def matvec_q8_1(dtype: int, w: np.ndarray, rows: int, cols: int, xq: np.ndarray) -> np.ndarray:
    y = np.empty(rows, np.float32)
    assert orc().orc_matvec_q8_1(dtype, _u8(w), rows, cols, _u8(xq), _f(y))
    return y


def matvec_f32(dtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, np.float32)
    assert orc().orc_matvec_f32(dtype, _u8(w), rows, cols, _f(x), _f(y))
    return y


def rms_norm(x: np.ndarray, w: np.ndarray, w_dtype: int = 0, eps: float = 1e-6, order: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w)
    out = np.empty_like(x)
    assert orc().orc_rms_norm(_f(x), w.ctypes.data, w_dtype, x.size, eps, order, _f(out))
    return out


def head_norm(vec: np.ndarray, w: np.ndarray, heads: int, head_dim: int, w_dtype: int = 0, order: int = 1) -> np.ndarray:
    v = np.array(vec, dtype=np.float32, copy=True)
    w = np.ascontiguousarray(w)
    assert orc().orc_head_norm(_f(v), w.ctypes.data, w_dtype, heads, head_dim, order)
    return v


def rope_table(context: int, head_dim: int, base: float = 1e6, scale: float = 1.0):
    c = np.empty(context * (head_dim // 2), np.float32)
    s = np.empty_like(c)
    assert orc().orc_rope_table(context, head_dim, base, scale, _f(c), _f(s))
    return c, s


def rope_apply(vec: np.ndarray, heads: int, head_dim: int, pos: int, cos_t: np.ndarray, sin_t: np.ndarray) -> np.ndarray:
    v = np.array(vec, dtype=np.float32, copy=True)
    assert orc().orc_rope_apply(_f(v), heads, head_dim, pos, _f(cos_t), _f(sin_t))
    return v


def attention(q, k_cache, v_cache, layer, pos, heads, kv_heads, head_dim, context) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    kc = np.ascontiguousarray(k_cache, dtype=np.float32)
    vc = np.ascontiguousarray(v_cache, dtype=np.float32)
    out = np.empty(heads * head_dim, np.float32)
    assert orc().orc_attention(_f(out), _f(q), _f(kc), _f(vc), layer, pos, heads, kv_heads, head_dim, context)
    return out


def expf_det(x: np.ndarray) -> np.ndarray:
    return np.array([orc().orc_expf_det(float(v)) for v in np.asarray(x, np.float32).ravel()], np.float32)


def matvec_q8_1_dev(dtype: int, w: np.ndarray, rows: int, cols: int, xq: np.ndarray) -> np.ndarray:
    """Device evaluation order (bit-exact contract with the GEMV kernel)."""
    y = np.empty(rows, np.float32)
    assert orc().orc_matvec_q8_1_dev(dtype, _u8(w), rows, cols, _u8(xq), _f(y))
    return y


def matvec_dense_dev(dtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, np.float32)
    assert orc().orc_matvec_dense_dev(dtype, _u8(w), rows, cols, _f(x), _f(y))
    return y


def silu_mul_dev(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    orc().orc_silu_mul_dev(_f(out), _f(g), _f(u), g.size)
    return out


def attention_dev(q, k_cache, v_cache, cur_k, cur_v, layer, pos, heads, kv_heads, head_dim, context) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    kc = np.ascontiguousarray(k_cache, dtype=np.float32)
    vc = np.ascontiguousarray(v_cache, dtype=np.float32)
    ck = np.ascontiguousarray(cur_k, dtype=np.float32)
    cv = np.ascontiguousarray(cur_v, dtype=np.float32)
    out = np.empty(heads * head_dim, np.float32)
    assert orc().orc_attention_dev(_f(out), _f(q), _f(kc), _f(vc), _f(ck), _f(cv), layer, pos, heads, kv_heads,
                                   head_dim, context)
    return out


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    g = np.ascontiguousarray(g, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(g)
    orc().orc_silu_mul(_f(out), _f(g), _f(u), g.size)
    return out


def argmax_penalized(values: np.ndarray, seen: Sequence[int] = (), penalty: float = 1.0):
    v = np.ascontiguousarray(values, dtype=np.float32)
    s = np.ascontiguousarray(np.asarray(seen, dtype=np.uint32))
    gap = C.c_float()
    tok = orc().orc_argmax_penalized(_f(v), v.size, s.ctypes.data_as(u32p), s.size, penalty, C.byref(gap))
    return int(tok), float(gap.value)


def sample(values: np.ndarray, seen: Sequence[int], temp: float, top_k: int, top_p: float, min_p: float,
           penalty: float, seed: int):
    """qwen3_sample (qwen3.uya:2073-2138) -> (token, next seed state, margin of the draw)."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    s = np.ascontiguousarray(np.asarray(seen, dtype=np.uint32))
    st = C.c_uint32(seed)
    mg = C.c_float()
    tok = orc().orc_sample(_f(v), v.size, s.ctypes.data_as(u32p), s.size, temp, top_k, top_p, min_p, penalty,
                           C.byref(st), C.byref(mg))
    return int(tok), int(st.value), float(mg.value)


# ---------------------------------------------------------------------------
# whole-step oracle
# ---------------------------------------------------------------------------
class OrcLayer(C.Structure):
    _fields_ = [
        ("attn_norm", C.c_void_p), ("attn_norm_dtype", C.c_int),
        ("q", C.c_void_p), ("q_dtype", C.c_int),
        ("k", C.c_void_p), ("k_dtype", C.c_int),
        ("v", C.c_void_p), ("v_dtype", C.c_int),
        ("q_norm", C.c_void_p), ("q_norm_dtype", C.c_int),
        ("k_norm", C.c_void_p), ("k_norm_dtype", C.c_int),
        ("o", C.c_void_p), ("o_dtype", C.c_int),
        ("ffn_norm", C.c_void_p), ("ffn_norm_dtype", C.c_int),
        ("gate", C.c_void_p), ("gate_dtype", C.c_int),
        ("up", C.c_void_p), ("up_dtype", C.c_int),
        ("down", C.c_void_p), ("down_dtype", C.c_int),
    ]


class OrcModel(C.Structure):
    _fields_ = [
        ("layers", C.c_uint32), ("hidden", C.c_uint32), ("heads", C.c_uint32), ("kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32), ("ffn", C.c_uint32), ("vocab", C.c_uint32), ("context", C.c_uint32),
        ("eps", C.c_float),
        ("token_embd", C.c_void_p), ("token_embd_dtype", C.c_int),
        ("output_norm", C.c_void_p), ("output_norm_dtype", C.c_int),
        ("output", C.c_void_p), ("output_dtype", C.c_int),
        ("layer", C.POINTER(OrcLayer)),
        ("rope_cos", fp), ("rope_sin", fp),
    ]


class OrcState(C.Structure):
    _fields_ = [
        ("k_cache", fp), ("v_cache", fp), ("q8_1_activations", C.c_int), ("norm_order", C.c_int),
        ("kv_f16", C.c_int), ("matvec", C.c_void_p), ("matvec_user", C.c_void_p),
    ]


class OracleModel:
    """CPU decode of a model given as {name: (dtype, rows, cols, bytes)}.

    q8_1=True: the reference CUDA path's arithmetic (Q8_1 activations) in the
    device evaluation order (device_order=True, the bit-exact contract) or
    in natural order with libm expf (device_order=False); q8_1=False: the
    reference CPU path (f32 activations, sequential norms), optionally through
    a threaded pool calling the reference's own native matvec.
    """

    def __init__(self, shape, tensors: Dict[str, tuple], context: int, q8_1: bool = True, pool_threads: int = 0,
                 use_reference_matvec: bool = False, device_order: bool = True, kv_f16: bool = False):
        self.shape = shape
        self.context = context
        self._keep = {k: np.ascontiguousarray(v[3]) for k, v in tensors.items()}
        self.t = tensors
        L = shape.layers
        self.layers = (OrcLayer * L)()

        def ptr(name):
            return self._keep[name].ctypes.data if name in self._keep else None

        def dt(name):
            return tensors[name][0] if name in tensors else 0

        for l in range(L):
            p = f"blk.{l}."
            lw = self.layers[l]
            for field, suffix in (("attn_norm", "attn_norm"), ("q", "attn_q"), ("k", "attn_k"), ("v", "attn_v"),
                                  ("q_norm", "attn_q_norm"), ("k_norm", "attn_k_norm"), ("o", "attn_output"),
                                  ("ffn_norm", "ffn_norm"), ("gate", "ffn_gate"), ("up", "ffn_up"), ("down", "ffn_down")):
                setattr(lw, field, ptr(p + suffix + ".weight"))
                setattr(lw, field + "_dtype", dt(p + suffix + ".weight"))
        self.cos, self.sin = rope_table(context, shape.head_dim, shape.rope_base, 1.0)
        m = OrcModel()
        m.layers, m.hidden, m.heads, m.kv_heads = L, shape.hidden, shape.heads, shape.kv_heads
        m.head_dim, m.ffn, m.vocab, m.context = shape.head_dim, shape.ffn, shape.vocab, context
        m.eps = 1e-6
        m.token_embd, m.token_embd_dtype = ptr("token_embd.weight"), dt("token_embd.weight")
        m.output_norm, m.output_norm_dtype = ptr("output_norm.weight"), dt("output_norm.weight")
        out_name = "output.weight" if "output.weight" in tensors else "token_embd.weight"
        m.output, m.output_dtype = ptr(out_name), dt(out_name)
        m.layer = self.layers
        m.rope_cos, m.rope_sin = _f(self.cos), _f(self.sin)
        self.model = m
        kvf = L * context * shape.kv_heads * shape.head_dim
        self.kc = np.zeros(kvf, np.float32)
        self.vc = np.zeros(kvf, np.float32)
        st = OrcState()
        st.k_cache, st.v_cache = _f(self.kc), _f(self.vc)
        st.q8_1_activations = int(q8_1)
        st.norm_order = 1 if (q8_1 and device_order) else 0
        st.kv_f16 = int(kv_f16)
        self.state = st
        self.pool = None
        if pool_threads:
            ref = (str(REF_DIR / "libref_cpu.so")
                   if use_reference_matvec and not q8_1 and (REF_DIR / "libref_cpu.so").exists() else None)
            self.pool = orc().orc_pool_create(pool_threads, ref.encode() if ref else None)
            orc().orc_state_attach_pool(C.byref(self.state), self.pool)

    @property
    def uses_reference_matvec(self) -> bool:
        return bool(self.pool) and bool(orc().orc_pool_is_reference(self.pool))

    def forward(self, token: int, pos: int, logits: bool = True):
        lg = np.empty(self.shape.vocab, np.float32) if logits else None
        hid = np.empty(self.shape.hidden, np.float32)
        ok = orc().orc_forward_token(C.byref(self.model), C.byref(self.state), token, pos,
                                     _f(lg) if lg is not None else None, _f(hid))
        if not ok:
            raise RuntimeError("oracle forward failed")
        return lg, hid

    def forward_embedding(self, emb, pos: int, logits: bool = True):
        """The layer stack on a given f32 input row (qwen3_append_prompt_embeddings, qwen3.uya:2534-2557)."""
        e = np.ascontiguousarray(emb, np.float32)
        if e.size != self.shape.hidden:
            raise ValueError("embedding size != hidden")
        lg = np.empty(self.shape.vocab, np.float32) if logits else None
        hid = np.empty(self.shape.hidden, np.float32)
        ok = orc().orc_forward_embedding(C.byref(self.model), C.byref(self.state), _f(e), pos,
                                         _f(lg) if lg is not None else None, _f(hid))
        if not ok:
            raise RuntimeError("oracle forward_embedding failed")
        return lg, hid

    def close(self):
        if self.pool:
            orc().orc_pool_destroy(self.pool)
            self.pool = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# reference builds (oracle/_ref): present only where the reference tree was
# available at build time
# ---------------------------------------------------------------------------
_ref: Dict[str, Optional[C.CDLL]] = {}


def ref_lib(name: str) -> Optional[C.CDLL]:
    """'cpu' -> libref_cpu.so, 'shim' -> libref_shim.so, 'kernels' -> libref_kernels.so (None if absent)."""
    if name not in _ref:
        path = REF_DIR / f"libref_{name}.so"
        lib = C.CDLL(str(path)) if path.exists() else None
        if lib is not None and name == "cpu":
            lib.minicpmo_cpu_matvec_range.restype = C.c_int
            lib.minicpmo_cpu_matvec_range.argtypes = [fp, u8p, C.c_int, fp, sz, sz, sz]
            lib.minicpmo_cpu_quantize_q8_1.restype = C.c_int
            lib.minicpmo_cpu_quantize_q8_1.argtypes = [C.c_void_p, fp, sz]
            lib.minicpmo_cpu_matvec_q8_1_range.restype = C.c_int
            lib.minicpmo_cpu_matvec_q8_1_range.argtypes = [fp, u8p, C.c_int, C.c_void_p, sz, sz, sz]
        if lib is not None and name == "shim":
            lib.minicpmo_gpu_q8_1_quantize_row.restype = C.c_int
            lib.minicpmo_gpu_q8_1_quantize_row.argtypes = [u8p, fp, sz]
            lib.minicpmo_gpu_f32_to_f16.restype = C.c_uint16
            lib.minicpmo_gpu_f32_to_f16.argtypes = [C.c_float]
            lib.minicpmo_gpu_sqrtf_positive.restype = C.c_float
            lib.minicpmo_gpu_sqrtf_positive.argtypes = [C.c_float]
        if lib is not None and name == "kernels":
            for fn in ("refk_q4_k_matvec", "refk_q6_k_matvec"):
                getattr(lib, fn).restype = None
                getattr(lib, fn).argtypes = [u8p, u8p, fp, C.c_int, C.c_int]
            lib.refk_float_to_half.restype = C.c_uint16
            lib.refk_float_to_half.argtypes = [C.c_float]
            lib.refk_apply_rope.restype = None
            lib.refk_apply_rope.argtypes = [fp, C.c_int, C.c_int, C.c_int, fp, fp]
            lib.refk_silu_mul.restype = None
            lib.refk_silu_mul.argtypes = [fp, fp, fp, C.c_int]
            lib.refk_rms_norm.restype = None
            lib.refk_rms_norm.argtypes = [fp, fp, u8p, C.c_int, C.c_int, C.c_float]
            lib.refk_head_norm.restype = None
            lib.refk_head_norm.argtypes = [fp, u8p, C.c_int, C.c_int, C.c_int]
            lib.refk_attention_decode.restype = None
            lib.refk_attention_decode.argtypes = [fp, fp, fp, fp] + [C.c_int] * 6 + [C.c_float]
        _ref[name] = lib
    return _ref[name]


def ref_cpu_matvec(dtype: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    lib = ref_lib("cpu")
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(rows, np.float32)
    assert lib.minicpmo_cpu_matvec_range(_f(y), _u8(w), dtype, _f(x), cols, 0, rows)
    return y


def ref_shim_q8_1(x: np.ndarray) -> np.ndarray:
    """The reference GPU shim's own host quantiser (gpu_shim.c:380-401); n % 256 == 0."""
    lib = ref_lib("shim")
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.zeros(x.size // 32 * 36, np.uint8)
    assert lib.minicpmo_gpu_q8_1_quantize_row(out.ctypes.data_as(u8p), _f(x), x.size)
    return out


def ref_kernel_matvec(dtype: int, w: np.ndarray, rows: int, cols: int, xq: np.ndarray) -> np.ndarray:
    """The reference CUDA matvec kernels (gpu_shim.c:746-925) evaluated on the host."""
    lib = ref_lib("kernels")
    y = np.empty(rows, np.float32)
    fn = lib.refk_q4_k_matvec if dtype == 10 else lib.refk_q6_k_matvec
    fn(_u8(w), _u8(xq), _f(y), rows, cols)
    return y
