"""Synthetic GGUF models and GEMV operands for the benchmark workloads.

No real model files exist on the machines this runs on, so every workload is a
seeded synthetic GGUF (v3) whose quantized blocks are drawn field by field:

* ``llama_1b``  -- LLaMA architecture shaped like a 1.1B chat model (22 layers,
  dim 2048, 32/4 heads, ffn 5632, vocab 32000) in a Q4_K_M-style type mix.
* ``gpt2_124m`` -- GPT-2 (12 layers, dim 768, 12 heads, ffn 3072, vocab 50257,
  ctx 1024) with Q8_0 matrices and F16 embeddings.
* ``qwen2_05b`` -- Qwen2 (24 layers, dim 896, 14/2 heads, ffn 4864, vocab 151936).
  896 is not a multiple of 256, and the K-quant decoders reject rows that do
  not fill whole 256-element super-blocks (llamini.cpp gguf.c:505 and
  gguf.c:562), so tensors with 896-wide rows use Q5_0 where Q4_K was
  asked and Q8_0 where Q6_K was asked; ffn_down (rows of 4864 = 19*256) keeps
  Q4_K/Q6_K.
* ``llama_7b``  -- LLaMA at 7B shape (32 layers, dim 4096, 32/32 heads, ffn 11008).

Block fields (all from ``numpy.random.default_rng(seed)``):
  f16 scales d (and dmin, Q4_1's m) ~ U[1e-3, 4e-3] (Q4_1 m ~ U[-3e-2, 0]);
  packed integer fields (nibbles, 6-bit K-quant scale/min pairs, Q5/Q6 high
  bits) are uniform random bytes, which makes every packed field uniform over
  its own bit range; Q6_K sub-block scales are int8 ~ U{-63..63}; Q8_0 values
  int8 ~ U{-127..127}; F32 norm weights 1 + N(0, 0.05); biases N(0, 0.02);
  F16 embeddings (GPT-2) N(0, 0.02).

The file layout follows the GGUF v3 format read by gguf.c:117-231: header,
metadata key/values, tensor infos, padding to 32 bytes, tensor data (each
tensor 32-byte aligned).
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field

import numpy as np

# ggml type ids and block geometry (gguf.h:29-37, gguf.c:427-590)
F32, F16, Q4_0, Q4_1, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 2, 3, 6, 8, 12, 13, 14
BLOCK = {F32: (1, 4), F16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22),
         Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}
TYPE_NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0",
              Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K"}
QUANT_TYPES = [Q4_0, Q4_1, Q5_0, Q8_0, Q4_K, Q5_K, Q6_K]

# GGUF metadata value tags (gguf.h:10-24)
_U32, _I32, _F32, _STR, _ARR = 4, 5, 6, 8, 9


def type_bytes(t: int, n: int) -> int:
    be, bb = BLOCK[t]
    assert n % be == 0, (t, n)
    return n // be * bb


def _f16_bytes(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16).view(np.uint8).reshape(-1, 2)


def random_blocks(rng: np.random.Generator, t: int, n: int) -> np.ndarray:
    """Raw bytes of ``n`` elements of type ``t`` drawn with the field
    distributions above; returns a flat uint8 array."""
    if t == F32:
        return (1.0 + rng.normal(0, 0.05, n)).astype(np.float32).view(np.uint8)
    if t == F16:
        return rng.normal(0, 0.02, n).astype(np.float16).view(np.uint8)
    be, bb = BLOCK[t]
    nb = n // be
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    d = _f16_bytes(rng.uniform(1e-3, 4e-3, nb))
    if t in (Q4_0, Q5_0, Q8_0):
        raw[:, 0:2] = d
        if t == Q8_0:
            raw[:, 2:34] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
    elif t == Q4_1:
        raw[:, 0:2] = d
        raw[:, 2:4] = _f16_bytes(rng.uniform(-3e-2, 0.0, nb))
    elif t in (Q4_K, Q5_K):
        raw[:, 0:2] = d
        raw[:, 2:4] = _f16_bytes(rng.uniform(1e-3, 4e-3, nb))
    elif t == Q6_K:
        raw[:, 192:208] = rng.integers(-63, 64, size=(nb, 16), dtype=np.int8).view(np.uint8)
        raw[:, 208:210] = d
    return raw.reshape(-1)


# ----------------------------------------------------------------------------- writer

@dataclass
class TensorSpec:
    name: str
    ne: tuple          # ggml dims, fastest first: (in, out) for a weight matrix
    type: int
    kind: str = "q"    # "q" random blocks, "norm" 1+N(0,.05), "bias" N(0,.02), "emb16" N(0,.02)


@dataclass
class GGUFSpec:
    meta: list = field(default_factory=list)     # (key, tag, value)
    tensors: list = field(default_factory=list)  # TensorSpec


def _pack_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _pack_meta(key: str, tag: int, val) -> bytes:
    out = _pack_str(key) + struct.pack("<I", tag)
    if tag == _U32:
        out += struct.pack("<I", val)
    elif tag == _I32:
        out += struct.pack("<i", val)
    elif tag == _F32:
        out += struct.pack("<f", val)
    elif tag == _STR:
        out += _pack_str(val)
    elif tag == _ARR:
        etag, items = val
        out += struct.pack("<IQ", etag, len(items))
        if etag == _STR:
            out += b"".join(_pack_str(s) for s in items)
        elif etag == _F32:
            out += np.asarray(items, dtype="<f4").tobytes()
        elif etag == _I32:
            out += np.asarray(items, dtype="<i4").tobytes()
        else:
            raise ValueError(etag)
    else:
        raise ValueError(tag)
    return out


def _tensor_payload(rng, ts: TensorSpec) -> np.ndarray:
    n = int(np.prod(ts.ne))
    if ts.kind == "norm":
        return (1.0 + rng.normal(0, 0.05, n)).astype(np.float32).view(np.uint8)
    if ts.kind == "bias":
        return rng.normal(0, 0.02, n).astype(np.float32).view(np.uint8)
    if ts.kind == "emb16":
        return rng.normal(0, 0.02, n).astype(np.float16).view(np.uint8)
    return random_blocks(rng, ts.type, n)


def write_gguf(path: str, spec: GGUFSpec, seed: int, align: int = 32, payloads: dict | None = None) -> None:
    """Write ``spec`` to ``path``; tensor payloads are drawn in spec order from
    ``default_rng(seed)`` so a (spec, seed) pair always gives the same bytes.
    ``payloads`` may give the raw bytes of some tensors explicitly."""
    rng = np.random.default_rng(seed)
    sizes = [type_bytes(t.type, int(np.prod(t.ne))) for t in spec.tensors]
    offs, cur = [], 0
    for s in sizes:
        cur = (cur + align - 1) // align * align
        offs.append(cur)
        cur += s
    head = struct.pack("<IIQQ", 0x46554747, 3, len(spec.tensors), len(spec.meta))
    head += b"".join(_pack_meta(k, t, v) for k, t, v in spec.meta)
    for ts, off in zip(spec.tensors, offs):
        head += _pack_str(ts.name) + struct.pack("<I", len(ts.ne))
        head += b"".join(struct.pack("<Q", d) for d in ts.ne)
        head += struct.pack("<IQ", ts.type, off)
    pad = (-len(head)) % align
    tmp = path + ".tmp%d" % os.getpid()
    with open(tmp, "wb") as f:
        f.write(head + b"\0" * pad)
        pos = 0
        for ts, off, sz in zip(spec.tensors, offs, sizes):
            if off > pos:
                f.write(b"\0" * (off - pos))
            data = _tensor_payload(rng, ts)
            if payloads and ts.name in payloads:
                data = np.asarray(payloads[ts.name], dtype=np.uint8).reshape(-1)
            assert data.size == sz, (ts.name, data.size, sz)
            f.write(data.tobytes())
            pos = off + sz
    os.replace(tmp, path)


# ----------------------------------------------------------------------------- models

def _vocab_meta(n: int, model: str):
    toks = ["<t%d>" % i for i in range(n)]
    return [
        ("tokenizer.ggml.model", _STR, model),
        ("tokenizer.ggml.tokens", _ARR, (_STR, toks)),
        ("tokenizer.ggml.scores", _ARR, (_F32, [0.0] * n)),
        ("tokenizer.ggml.token_type", _ARR, (_I32, [1] * n)),
        ("tokenizer.ggml.bos_token_id", _U32, 1),
        ("tokenizer.ggml.eos_token_id", _U32, 2),
    ]


@dataclass
class LlamaShape:
    arch: str
    dim: int
    n_layers: int
    n_heads: int
    n_kv: int
    ffn: int
    vocab: int
    ctx: int
    rope_base: float
    eps: float
    qkv_bias: bool
    types: dict          # role -> callable(layer) -> ggml type, or a type for non-layer tensors
    head_dim: int = 0

    def hd(self) -> int:
        return self.head_dim or self.dim // self.n_heads


def llama_spec(s: LlamaShape) -> GGUFSpec:
    a = s.arch
    hd = s.hd()
    qd, kvd = s.n_heads * hd, s.n_kv * hd
    meta = [
        ("general.architecture", _STR, a),
        ("general.alignment", _U32, 32),
        (a + ".embedding_length", _U32, s.dim),
        (a + ".block_count", _U32, s.n_layers),
        (a + ".attention.head_count", _U32, s.n_heads),
        (a + ".attention.head_count_kv", _U32, s.n_kv),
        (a + ".feed_forward_length", _U32, s.ffn),
        (a + ".attention.layer_norm_rms_epsilon", _F32, s.eps),
        (a + ".rope.freq_base", _F32, s.rope_base),
        (a + ".context_length", _U32, s.ctx),
    ]
    if s.head_dim:
        meta.append((a + ".attention.key_length", _U32, s.head_dim))
    meta += _vocab_meta(s.vocab, "gpt2" if a == "qwen2" else "llama")
    T = s.types
    ts = [TensorSpec("token_embd.weight", (s.dim, s.vocab), T["embd"]),
          TensorSpec("output_norm.weight", (s.dim,), F32, "norm"),
          TensorSpec("output.weight", (s.dim, s.vocab), T["output"])]
    for l in range(s.n_layers):
        p = "blk.%d." % l
        ts += [TensorSpec(p + "attn_norm.weight", (s.dim,), F32, "norm"),
               TensorSpec(p + "attn_q.weight", (s.dim, qd), T["q"](l)),
               TensorSpec(p + "attn_k.weight", (s.dim, kvd), T["k"](l)),
               TensorSpec(p + "attn_v.weight", (s.dim, kvd), T["v"](l))]
        if s.qkv_bias:
            ts += [TensorSpec(p + "attn_q.bias", (qd,), F32, "bias"),
                   TensorSpec(p + "attn_k.bias", (kvd,), F32, "bias"),
                   TensorSpec(p + "attn_v.bias", (kvd,), F32, "bias")]
        ts += [TensorSpec(p + "attn_output.weight", (qd, s.dim), T["o"](l)),
               TensorSpec(p + "ffn_norm.weight", (s.dim,), F32, "norm"),
               TensorSpec(p + "ffn_gate.weight", (s.dim, s.ffn), T["gate"](l)),
               TensorSpec(p + "ffn_up.weight", (s.dim, s.ffn), T["up"](l)),
               TensorSpec(p + "ffn_down.weight", (s.ffn, s.dim), T["down"](l))]
    return GGUFSpec(meta, ts)


def _q4km_types(fallback_896: bool = False) -> dict:
    """The Q4_K_M mix: Q4_K everywhere, Q6_K for attn_v/ffn_down on layers with
    l % 3 == 0 and for output.weight."""
    def vq(l): return Q6_K if l % 3 == 0 else Q4_K
    t = {"embd": Q4_K, "output": Q6_K, "q": lambda l: Q4_K, "k": lambda l: Q4_K,
         "v": vq, "o": lambda l: Q4_K, "gate": lambda l: Q4_K, "up": lambda l: Q4_K,
         "down": vq}
    if fallback_896:
        sub = {Q4_K: Q5_0, Q6_K: Q8_0}
        def v896(l):
            return Q5_0 if l % 2 == 1 else sub[vq(l)]
        t = {"embd": Q5_0, "output": Q8_0, "q": lambda l: Q5_0, "k": lambda l: Q5_0,
             "v": v896, "o": lambda l: Q5_0, "gate": lambda l: Q5_0, "up": lambda l: Q5_0,
             "down": vq}
    return t


def shape_llama_1b(**kw) -> LlamaShape:
    d = dict(arch="llama", dim=2048, n_layers=22, n_heads=32, n_kv=4, ffn=5632, vocab=32000,
             ctx=2048, rope_base=10000.0, eps=1e-5, qkv_bias=False, types=_q4km_types())
    d.update(kw)
    return LlamaShape(**d)


def shape_llama_7b(**kw) -> LlamaShape:
    d = dict(arch="llama", dim=4096, n_layers=32, n_heads=32, n_kv=32, ffn=11008, vocab=32000,
             ctx=4096, rope_base=10000.0, eps=1e-5, qkv_bias=False, types=_q4km_types())
    d.update(kw)
    return LlamaShape(**d)


def shape_qwen2_05b(**kw) -> LlamaShape:
    d = dict(arch="qwen2", dim=896, n_layers=24, n_heads=14, n_kv=2, ffn=4864, vocab=151936,
             ctx=32768, rope_base=1e6, eps=1e-6, qkv_bias=True, types=_q4km_types(True))
    d.update(kw)
    return LlamaShape(**d)


@dataclass
class Gpt2Shape:
    dim: int = 768
    n_layers: int = 12
    n_heads: int = 12
    ffn: int = 3072
    vocab: int = 50257
    ctx: int = 1024
    wtype: int = Q8_0


def gpt2_spec(s: Gpt2Shape) -> GGUFSpec:
    meta = [
        ("general.architecture", _STR, "gpt2"),
        ("general.alignment", _U32, 32),
        ("gpt2.embedding_length", _U32, s.dim),
        ("gpt2.block_count", _U32, s.n_layers),
        ("gpt2.attention.head_count", _U32, s.n_heads),
        ("gpt2.feed_forward_length", _U32, s.ffn),
        ("gpt2.context_length", _U32, s.ctx),
    ] + _vocab_meta(s.vocab, "gpt2")
    d, f, w = s.dim, s.ffn, s.wtype
    ts = [TensorSpec("token_embd.weight", (d, s.vocab), F16, "emb16"),
          TensorSpec("position_embd.weight", (d, s.ctx), F16, "emb16"),
          TensorSpec("output_norm.weight", (d,), F32, "norm"),
          TensorSpec("output_norm.bias", (d,), F32, "bias"),
          TensorSpec("output.weight", (d, s.vocab), w)]
    for l in range(s.n_layers):
        p = "blk.%d." % l
        ts += [TensorSpec(p + "attn_norm.weight", (d,), F32, "norm"),
               TensorSpec(p + "attn_norm.bias", (d,), F32, "bias"),
               TensorSpec(p + "attn_qkv.weight", (d, 3 * d), w),
               TensorSpec(p + "attn_qkv.bias", (3 * d,), F32, "bias"),
               TensorSpec(p + "attn_output.weight", (d, d), w),
               TensorSpec(p + "attn_output.bias", (d,), F32, "bias"),
               TensorSpec(p + "ffn_norm.weight", (d,), F32, "norm"),
               TensorSpec(p + "ffn_norm.bias", (d,), F32, "bias"),
               TensorSpec(p + "ffn_up.weight", (d, f), w),
               TensorSpec(p + "ffn_up.bias", (f,), F32, "bias"),
               TensorSpec(p + "ffn_down.weight", (f, d), w),
               TensorSpec(p + "ffn_down.bias", (d,), F32, "bias")]
    return GGUFSpec(meta, ts)


# Named workloads: (spec builder, seed). Seeds follow the workload table:
# llama_1b 0, gemv sweep 1, gpt2_124m 2, qwen2_05b 3, llama_7b 4.
WORKLOADS = {
    "llama_1b": (lambda: llama_spec(shape_llama_1b()), 0),
    "gpt2_124m": (lambda: gpt2_spec(Gpt2Shape()), 2),
    "qwen2_05b": (lambda: llama_spec(shape_qwen2_05b()), 3),
    "llama_7b": (lambda: llama_spec(shape_llama_7b()), 4),
}


def workload_prompt(name: str, n: int) -> np.ndarray:
    """Prompt token ids of a workload: llama_1b ~U[3,32000) from seed 0 (drawn
    after the model), gpt2 ~U[0,50257) seed 2, qwen2 seed 3, llama_7b seed 4.
    A separate stream (seed + 1000) keeps the prompt independent of the file."""
    seed = WORKLOADS[name][1]
    rng = np.random.default_rng(seed + 1000)
    lo, hi = {"llama_1b": (3, 32000), "gpt2_124m": (0, 50257),
              "qwen2_05b": (3, 151936), "llama_7b": (3, 32000)}[name]
    return rng.integers(lo, hi, size=n, dtype=np.int64).astype(np.uint32)


def ensure_workload(name: str, directory: str | None = None) -> str:
    """Path of the workload's GGUF, writing it first if absent."""
    directory = directory or os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200")
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, name + ".gguf")
    if not os.path.exists(path):
        build, seed = WORKLOADS[name]
        write_gguf(path, build(), seed)
    return path


def ensure_spec(spec: GGUFSpec, seed: int, path: str) -> str:
    if not os.path.exists(path):
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        write_gguf(path, spec, seed)
    return path


# ----------------------------------------------------------------------------- reader

_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B",
           10: "<Q", 11: "<q", 12: "<d"}


class GGUFReader:
    """Minimal reader for files written above (and any GGUF v2/v3): metadata
    and tensor views straight from a read-only memory map."""

    def __init__(self, path: str):
        self.path = path
        self.buf = np.memmap(path, dtype=np.uint8, mode="r")
        b = self.buf
        self.pos = 0
        magic, ver = struct.unpack_from("<II", b, 0)
        assert magic == 0x46554747 and ver in (2, 3)
        n_t, n_kv = struct.unpack_from("<QQ", b, 8)
        self.pos = 24
        self.meta = {}
        for _ in range(n_kv):
            k = self._str()
            tag = self._u32()
            self.meta[k] = self._val(tag)
        self.tensors = {}
        for _ in range(n_t):
            name = self._str()
            nd = self._u32()
            ne = tuple(struct.unpack_from("<Q", b, self.pos + 8 * i)[0] for i in range(nd))
            self.pos += 8 * nd
            t = self._u32()
            off = struct.unpack_from("<Q", b, self.pos)[0]
            self.pos += 8
            self.tensors[name] = (t, ne, off)
        align = self.meta.get("general.alignment", 32)
        self.data_off = (self.pos + align - 1) // align * align

    def _u32(self):
        v = struct.unpack_from("<I", self.buf, self.pos)[0]
        self.pos += 4
        return v

    def _str(self):
        n = struct.unpack_from("<Q", self.buf, self.pos)[0]
        s = bytes(self.buf[self.pos + 8:self.pos + 8 + n]).decode()
        self.pos += 8 + n
        return s

    def _val(self, tag):
        if tag == _STR:
            return self._str()
        if tag == _ARR:
            et = self._u32()
            n = struct.unpack_from("<Q", self.buf, self.pos)[0]
            self.pos += 8
            if et == _STR:
                return [self._str() for _ in range(n)]
            fmt = _SCALAR[et]
            sz = struct.calcsize(fmt)
            arr = np.frombuffer(self.buf, dtype=np.dtype(fmt), count=n, offset=self.pos)
            self.pos += sz * n
            return arr
        fmt = _SCALAR[tag]
        v = struct.unpack_from(fmt, self.buf, self.pos)[0]
        self.pos += struct.calcsize(fmt)
        return v

    def raw(self, name: str) -> tuple:
        """(ggml type, ne, uint8 view of the tensor's bytes)."""
        t, ne, off = self.tensors[name]
        n = type_bytes(t, int(np.prod(ne)))
        start = self.data_off + off
        return t, ne, self.buf[start:start + n]
