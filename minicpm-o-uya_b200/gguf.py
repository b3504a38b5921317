"""GGUF v3 files and GGML block quantisers for seeded synthetic Qwen3 models.

Formats (the reference's own readers: src/minicpmo/tensor.uya, gguf.uya;
block layouts qwen3.uya:847-1000):

* Q8_0  32 values / 34 B : f16 d, i8 q[32];            x = d*q
* Q4_K 256 values / 144 B: f16 d, f16 dmin, u8 scales[12], u8 qs[128];
                             x = d*sc_j*q - dmin*m_j (6-bit sc/m per 32 values)
* Q6_K 256 values / 210 B: u8 ql[128], u8 qh[64], i8 sc[16], f16 d;
                             x = d*sc_g*(q-32) (per 16 values)

The quantisers here only have to produce *valid* blocks of a given f32
matrix (the decode path never quantises weights); they use simple
min/max scale choices, vectorised in torch so that multi-GB synthetic models
can be built on a GPU in seconds.  Scale/min packing follows
``q4_k_pack_scales_mins`` (src/minicpmo/kernels.uya:401-409) and the element
order of ``qwen3_q6_k_copy_row`` (qwen3.uya:1069-1103).
"""
from __future__ import annotations

import struct
import zlib
from dataclasses import dataclass
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np

# Uya TensorDType ordinal <-> ggml type id (tensor.uya:166-189)
F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 6, 10, 12, 20
UYA_TO_GGML = {F32: 0, F16: 1, Q8_0: 8, Q4_K: 12, Q6_K: 14, BF16: 30}
GGML_TO_UYA = {v: k for k, v in UYA_TO_GGML.items()}
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

SEED_BASE = 20261201


def row_bytes(dtype: int, cols: int) -> int:
    if dtype == F32:
        return cols * 4
    if dtype in (F16, BF16):
        return cols * 2
    qk, nb = BLOCK[dtype]
    if cols % qk:
        raise ValueError(f"cols={cols} not a multiple of {qk} for dtype {dtype}")
    return cols // qk * nb


# ---------------------------------------------------------------------------
# quantisers (torch; any device)
# ---------------------------------------------------------------------------

def _torch():
    import torch

    return torch


def _f16_bytes(t):
    torch = _torch()
    return t.to(torch.float16).contiguous().view(torch.uint8).reshape(*t.shape, 2)


def quantize_q8_0(x):
    """x: float tensor [rows, cols] -> uint8 [rows, cols/32*34]."""
    torch = _torch()
    rows, cols = x.shape
    xb = x.float().reshape(rows, cols // 32, 32)
    d = (xb.abs().amax(-1) / 127.0).to(torch.float16)
    df = d.float()
    inv = torch.where(df > 0, 1.0 / df, torch.zeros_like(df))
    q = torch.round(xb * inv.unsqueeze(-1)).clamp(-127, 127).to(torch.int8)
    out = torch.cat([_f16_bytes(d), q.view(torch.uint8)], dim=-1)
    return out.reshape(rows, -1)


def quantize_q4_k(x):
    """x: float tensor [rows, cols] -> uint8 [rows, cols/256*144]."""
    torch = _torch()
    rows, cols = x.shape
    xb = x.float().reshape(rows, cols // 256, 8, 32)
    mn = xb.amin(-1).clamp(max=0.0)
    mx = xb.amax(-1)
    scale = (mx - mn) / 15.0
    mins = -mn
    d = (scale.amax(-1) / 63.0).to(torch.float16)
    dmin = (mins.amax(-1) / 63.0).to(torch.float16)
    df, dmf = d.float().unsqueeze(-1), dmin.float().unsqueeze(-1)
    sc = torch.where(df > 0, torch.round(scale / df.clamp(min=1e-30)), torch.zeros_like(scale)).clamp(0, 63)
    m = torch.where(dmf > 0, torch.round(mins / dmf.clamp(min=1e-30)), torch.zeros_like(mins)).clamp(0, 63)
    eff = (df * sc).unsqueeze(-1)
    effm = (dmf * m).unsqueeze(-1)
    q = torch.where(eff > 0, torch.round((xb + effm) / eff.clamp(min=1e-30)), torch.zeros_like(xb)).clamp(0, 15)
    q = q.to(torch.uint8)
    sc = sc.to(torch.uint8)
    m = m.to(torch.uint8)
    # scales[12] (kernels.uya:401-409)
    s_lo = (sc[..., :4] & 63) | ((sc[..., 4:] >> 4) << 6)
    m_lo = (m[..., :4] & 63) | ((m[..., 4:] >> 4) << 6)
    s_hi = (sc[..., 4:] & 15) | ((m[..., 4:] & 15) << 4)
    scales = torch.cat([s_lo, m_lo, s_hi], dim=-1)
    # qs: group g -> bytes 32g..32g+31 = sub-block 2g (low) | 2g+1 (high)
    qs = (q[:, :, 0::2, :] | (q[:, :, 1::2, :] << 4)).reshape(rows, cols // 256, 128)
    out = torch.cat([_f16_bytes(d), _f16_bytes(dmin), scales, qs], dim=-1)
    return out.reshape(rows, -1)


def quantize_q6_k(x):
    """x: float tensor [rows, cols] -> uint8 [rows, cols/256*210]."""
    torch = _torch()
    rows, cols = x.shape
    xg = x.float().reshape(rows, cols // 256, 16, 16)
    amax = xg.abs().amax(-1)
    gscale = amax / 31.0
    d = (gscale.amax(-1) / 127.0).to(torch.float16)
    df = d.float().unsqueeze(-1)
    sc = torch.where(df > 0, torch.round(gscale / df.clamp(min=1e-30)), torch.zeros_like(gscale)).clamp(-127, 127)
    eff = (df * sc).unsqueeze(-1)
    q = torch.where(eff != 0, torch.round(xg / torch.where(eff != 0, eff, torch.ones_like(eff))), torch.zeros_like(xg))
    q = (q.clamp(-32, 31) + 32).to(torch.uint8).reshape(rows, cols // 256, 2, 4, 32)  # [n, quarter, l]
    ql0 = (q[:, :, :, 0] & 15) | ((q[:, :, :, 2] & 15) << 4)  # ql[n*64 + l]
    ql1 = (q[:, :, :, 1] & 15) | ((q[:, :, :, 3] & 15) << 4)  # ql[n*64 + 32 + l]
    ql = torch.stack([ql0, ql1], dim=3).reshape(rows, cols // 256, 128)
    qh = ((q[:, :, :, 0] >> 4) | ((q[:, :, :, 1] >> 4) << 2) | ((q[:, :, :, 2] >> 4) << 4) | ((q[:, :, :, 3] >> 4) << 6))
    qh = qh.reshape(rows, cols // 256, 64)
    sc8 = sc.to(torch.int8).view(torch.uint8)
    out = torch.cat([ql, qh, sc8, _f16_bytes(d)], dim=-1)
    return out.reshape(rows, -1)


def quantize(x, dtype: int):
    """f32 [rows, cols] (torch) -> raw GGUF bytes (torch uint8 or f32/f16 values)."""
    torch = _torch()
    if dtype == Q8_0:
        return quantize_q8_0(x)
    if dtype == Q4_K:
        return quantize_q4_k(x)
    if dtype == Q6_K:
        return quantize_q6_k(x)
    if dtype == F32:
        return x.float().contiguous().view(torch.uint8).reshape(x.shape[0], -1)
    if dtype == F16:
        return x.to(torch.float16).contiguous().view(torch.uint8).reshape(x.shape[0], -1)
    if dtype == BF16:
        return x.to(torch.bfloat16).contiguous().view(torch.uint8).reshape(x.shape[0], -1)
    raise ValueError(dtype)


# ---------------------------------------------------------------------------
# synthetic Qwen3 models (seeded configs of the benchmark shapes)
# ---------------------------------------------------------------------------

@dataclass
class Qwen3Shape:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    context: int = 4096
    tied: bool = False
    rms_eps: float = 1e-6
    rope_base: float = 1e6

    @property
    def q_dim(self) -> int:
        return self.heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


SHAPES = {
    "qwen3-0.6b": Qwen3Shape(28, 1024, 16, 8, 128, 3072, 151936, tied=True),
    "qwen3-8b": Qwen3Shape(36, 4096, 32, 8, 128, 12288, 151936),
    "qwen3-32b": Qwen3Shape(64, 5120, 64, 8, 128, 25600, 151936),
}

# Q4_K_M-style mix (BASELINE configs 0/2/4): Q4_K for q/k/o/gate/up, Q6_K for
# v, down, token_embd and the untied output.
Q4_K_M = {"attn_q": Q4_K, "attn_k": Q4_K, "attn_v": Q6_K, "attn_output": Q4_K, "ffn_gate": Q4_K, "ffn_up": Q4_K,
          "ffn_down": Q6_K, "token_embd": Q6_K, "output": Q6_K}
ALL_Q8_0 = {k: Q8_0 for k in Q4_K_M}

# The per-layer pattern of real llama.cpp Q4_K_M files: attn_v and ffn_down
# take the higher-precision Q6_K only in the "more bits" layers -- the first
# and last eighth of the stack and every third layer in between -- and Q4_K
# elsewhere; token_embd keeps the base Q4_K, the output Q6_K.  (The mixed
# classes this gives per layer -- q/k/v all Q4_K, or Q4_K with a Q6_K v --
# are what a loaded real file hands the decode step.)
Q4_K_M_LAYERED = {**Q4_K_M, "token_embd": Q4_K, "_more_bits": True}


def _more_bits(layer: int, n_layers: int) -> bool:
    return layer < n_layers // 8 or layer >= 7 * n_layers // 8 or (layer - n_layers // 8) % 3 == 2


def layer_mix(mix: Dict[str, int], layer: int, n_layers: int) -> Dict[str, int]:
    """The dtypes of one layer under `mix` (per-layer only for Q4_K_M_LAYERED-style mixes)."""
    if not mix.get("_more_bits"):
        return mix
    hi = _more_bits(layer, n_layers)
    return {**mix, "attn_v": Q6_K if hi else Q4_K, "ffn_down": Q6_K if hi else Q4_K}


def tensor_specs(shape: Qwen3Shape, mix: Dict[str, int]) -> List[Tuple[str, int, int, int, str]]:
    """(name, dtype, rows, cols, kind) in GGUF order; kind 'w' (N(0,0.02)) or 'norm' (1+N(0,0.02))."""
    h, q, kv, f, V = shape.hidden, shape.q_dim, shape.kv_dim, shape.ffn, shape.vocab
    out = [("token_embd.weight", mix["token_embd"], V, h, "w")]
    for l in range(shape.layers):
        p = f"blk.{l}."
        lm = layer_mix(mix, l, shape.layers)
        out += [
            (p + "attn_norm.weight", F32, 1, h, "norm"),
            (p + "attn_q.weight", lm["attn_q"], q, h, "w"),
            (p + "attn_k.weight", lm["attn_k"], kv, h, "w"),
            (p + "attn_v.weight", lm["attn_v"], kv, h, "w"),
            (p + "attn_q_norm.weight", F32, 1, shape.head_dim, "norm"),
            (p + "attn_k_norm.weight", F32, 1, shape.head_dim, "norm"),
            (p + "attn_output.weight", lm["attn_output"], h, q, "w"),
            (p + "ffn_norm.weight", F32, 1, h, "norm"),
            (p + "ffn_gate.weight", lm["ffn_gate"], f, h, "w"),
            (p + "ffn_up.weight", lm["ffn_up"], f, h, "w"),
            (p + "ffn_down.weight", lm["ffn_down"], h, f, "w"),
        ]
    out.append(("output_norm.weight", F32, 1, h, "norm"))
    if not shape.tied:
        out.append(("output.weight", mix["output"], V, h, "w"))
    return out


def synth_tensor(name: str, dtype: int, rows: int, cols: int, kind: str, device: str = "cpu", std: float = 0.02,
                 seed_base: int = SEED_BASE) -> np.ndarray:
    """Seeded tensor (seed = seed_base + crc32(name)) as GGUF bytes in a numpy uint8 array."""
    torch = _torch()
    g = torch.Generator(device=device)
    g.manual_seed(seed_base + zlib.crc32(name.encode()))
    out = np.empty((rows, row_bytes(dtype, cols)), np.uint8)
    step = max(1, (1 << 26) // max(cols, 1))  # ~64M values per chunk
    for r0 in range(0, rows, step):
        r1 = min(rows, r0 + step)
        x = torch.randn((r1 - r0, cols), generator=g, device=device, dtype=torch.float32) * std
        if kind == "norm":
            x = x + 1.0
        out[r0:r1] = quantize(x, dtype).cpu().numpy()
    return out


def synth_model(shape: Qwen3Shape, mix: Dict[str, int], device: str = "cpu", seed_base: int = SEED_BASE):
    """-> list of (name, dtype, rows, cols, uint8 bytes)."""
    return [(n, dt, r, c, synth_tensor(n, dt, r, c, k, device=device, seed_base=seed_base))
            for n, dt, r, c, k in tensor_specs(shape, mix)]


def prompt_ids(n: int, vocab: int, seed: int = 7) -> np.ndarray:
    """Prompt of n ids uniform over [0, vocab) (numpy PCG64(seed))."""
    return np.random.Generator(np.random.PCG64(seed)).integers(0, vocab, size=n, dtype=np.int64).astype(np.uint32)


# ---------------------------------------------------------------------------
# GGUF v3 (writer modelled on tests/make_tiny_gguf.py:138-201 of the reference)
# ---------------------------------------------------------------------------
T_U32, T_I32, T_F32, T_STR, T_ARR = 4, 5, 6, 8, 9


def _s(v: str) -> bytes:
    b = v.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, value) -> bytes:
    if isinstance(value, str):
        return _s(key) + struct.pack("<I", T_STR) + _s(value)
    if isinstance(value, float):
        return _s(key) + struct.pack("<If", T_F32, value)
    if isinstance(value, int):
        return _s(key) + struct.pack("<II", T_U32, value)
    if isinstance(value, list) and all(isinstance(v, str) for v in value):
        return _s(key) + struct.pack("<IIQ", T_ARR, T_STR, len(value)) + b"".join(_s(v) for v in value)
    raise TypeError(f"{key}: {type(value)}")


def qwen3_metadata(shape: Qwen3Shape, name: str = "synthetic qwen3") -> Dict[str, object]:
    return {
        "general.architecture": "qwen3",
        "general.name": name,
        "general.alignment": 32,
        "qwen3.context_length": shape.context,
        "qwen3.embedding_length": shape.hidden,
        "qwen3.block_count": shape.layers,
        "qwen3.feed_forward_length": shape.ffn,
        "qwen3.attention.head_count": shape.heads,
        "qwen3.attention.head_count_kv": shape.kv_heads,
        "qwen3.attention.key_length": shape.head_dim,
        "qwen3.attention.value_length": shape.head_dim,
        "qwen3.attention.layer_norm_rms_epsilon": float(shape.rms_eps),
        "qwen3.rope.freq_base": float(shape.rope_base),
        "qwen3.vocab_size": shape.vocab,
        "tokenizer.ggml.model": "gpt2",
        "tokenizer.ggml.tokens": [f"<t{i}>" for i in range(shape.vocab)],
    }


def write_gguf(path, metadata: Dict[str, object], tensors: Iterable[Tuple[str, int, int, int, np.ndarray]],
               alignment: int = 32) -> None:
    tensors = list(tensors)
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(metadata))
    head += b"".join(_kv(k, v) for k, v in metadata.items())
    offset = 0
    infos = b""
    for name, dt, rows, cols, data in tensors:
        dims = [cols] if rows == 1 else [cols, rows]
        infos += _s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        infos += struct.pack("<IQ", UYA_TO_GGML[dt], offset)
        offset += (data.nbytes + alignment - 1) // alignment * alignment
    with open(path, "wb") as fh:
        fh.write(head + infos)
        pad = (-fh.tell()) % alignment
        fh.write(b"\0" * pad)
        for _, _, _, _, data in tensors:
            fh.write(np.ascontiguousarray(data).tobytes())
            fh.write(b"\0" * ((-data.nbytes) % alignment))


@dataclass
class GgufTensor:
    name: str
    dtype: int
    rows: int
    cols: int
    data: np.ndarray  # uint8 view into the mmap


class GgufFile:
    """Minimal GGUF v3 reader (tensor.uya:414-509): metadata + mmap'd tensor views."""

    def __init__(self, path):
        self.path = Path(path)
        self.mm = np.memmap(self.path, dtype=np.uint8, mode="r")
        buf = self.mm
        pos = 0

        def rd(fmt):
            nonlocal pos
            n = struct.calcsize(fmt)
            v = struct.unpack_from(fmt, buf, pos)
            pos += n
            return v

        def rs():
            (n,) = rd("<Q")
            nonlocal pos
            v = bytes(buf[pos:pos + n]).decode("utf-8", "replace")
            pos += n
            return v

        def rval(t):
            if t == T_STR:
                return rs()
            if t == T_ARR:
                (et, n) = rd("<IQ")
                return [rval(et) for _ in range(n)]
            fmt = {0: "<B", 1: "<b", 2: "<H", 3: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f", 7: "<?", 10: "<Q",
                   11: "<q", 12: "<d"}[t]
            return rd(fmt)[0]

        magic = bytes(buf[:4])
        if magic != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        pos = 4
        ver, n_t, n_kv = rd("<IQQ")
        if ver != 3:
            raise ValueError(f"{path}: GGUF version {ver} unsupported")
        self.metadata = {}
        for _ in range(n_kv):
            k = rs()
            (t,) = rd("<I")
            self.metadata[k] = rval(t)
        infos = []
        for _ in range(n_t):
            name = rs()
            (nd,) = rd("<I")
            dims = [rd("<Q")[0] for _ in range(nd)]
            (gt, off) = rd("<IQ")
            infos.append((name, dims, gt, off))
        align = int(self.metadata.get("general.alignment", 32))
        base = (pos + align - 1) // align * align
        self.tensors: Dict[str, GgufTensor] = {}
        for name, dims, gt, off in infos:
            if gt not in GGML_TO_UYA:
                raise ValueError(f"{name}: ggml type {gt} unsupported by this path")
            dt = GGML_TO_UYA[gt]
            cols = dims[0]
            rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
            nbytes = rows * row_bytes(dt, cols)
            self.tensors[name] = GgufTensor(name, dt, rows, cols, self.mm[base + off: base + off + nbytes])

    def shape(self) -> Qwen3Shape:
        m = self.metadata
        arch = m.get("general.architecture", "qwen3")
        g = lambda k, d=None: m.get(f"{arch}.{k}", d)
        hidden = int(g("embedding_length"))
        heads = int(g("attention.head_count"))
        head_dim = int(g("attention.key_length", hidden // heads))
        emb = self.tensors["token_embd.weight"]
        return Qwen3Shape(
            layers=int(g("block_count")), hidden=hidden, heads=heads, kv_heads=int(g("attention.head_count_kv", heads)),
            head_dim=head_dim, ffn=int(g("feed_forward_length")), vocab=int(g("vocab_size", emb.rows)),
            context=int(g("context_length", 4096)), tied="output.weight" not in self.tensors,
            rms_eps=float(g("attention.layer_norm_rms_epsilon", 1e-6)), rope_base=float(g("rope.freq_base", 1e6)),
        )
