"""ctypes binding of the CPU oracle (liboracle.so) and of the reference build
(_ref/libllamini_ref.so). TEST INFRASTRUCTURE: only tests/, the smoke check and
the benchmark's CPU-baseline leg use this module; the product never does.
"""
from __future__ import annotations

import ctypes as C
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libllamini_ref.so")
DROPIN_SO = os.path.join(HERE, "_ref", "libdriver_b200.so")

u32, u64, f32 = C.c_uint32, C.c_uint64, C.c_float
P = C.c_void_p
FP = C.POINTER(C.c_float)


def _synthetic():
    name = "llamini_b200_synthetic"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "llamini.cpp_b200", "synthetic.py"))
    m = importlib.util.module_from_spec(spec)
    sys.modules[name] = m
    spec.loader.exec_module(m)
    return m


class OrcMat(C.Structure):
    _fields_ = [("type", u32), ("rows", u32), ("cols", u32), ("data", P)]


class OrcLlamaLayer(C.Structure):
    _fields_ = [(n, OrcMat) for n in ("q", "k", "v", "o", "gate", "up", "down")] + \
               [(n, FP) for n in ("attn_norm", "ffn_norm", "bq", "bk", "bv")]


class OrcLlama(C.Structure):
    _fields_ = [(n, u32) for n in ("dim", "n_layers", "n_heads", "n_heads_kv", "head_dim", "ffn_dim",
                                   "vocab", "max_seq")] + \
               [("rms_eps", f32), ("rope_base", f32), ("emb_scale", f32), ("rope_neox", C.c_int),
                ("act_gelu", C.c_int), ("tok_embd", OrcMat), ("lm_head", OrcMat), ("final_norm", FP),
                ("layers", C.POINTER(OrcLlamaLayer))]


class OrcGpt2Layer(C.Structure):
    _fields_ = [("attn_norm_w", FP), ("attn_norm_b", FP), ("qkv", OrcMat), ("qkv_b", FP),
                ("out", OrcMat), ("out_b", FP), ("ffn_norm_w", FP), ("ffn_norm_b", FP),
                ("up", OrcMat), ("up_b", FP), ("down", OrcMat), ("down_b", FP)]


class OrcGpt2(C.Structure):
    _fields_ = [(n, u32) for n in ("dim", "n_layers", "n_heads", "ffn_dim", "vocab", "n_ctx", "max_seq")] + \
               [("ln_eps", f32), ("tok_embd", OrcMat), ("pos_embd", OrcMat), ("out_norm_w", FP),
                ("out_norm_b", FP), ("lm_head", OrcMat), ("layers", C.POINTER(OrcGpt2Layer))]


_orc = None


def oracle() -> C.CDLL:
    global _orc
    if _orc is None:
        if not os.path.exists(ORACLE_SO):
            raise FileNotFoundError("oracle not built: make -C oracle")
        L = C.CDLL(ORACLE_SO)
        L.orc_dequant.argtypes = [u32, P, u64, P]
        L.orc_dequant.restype = C.c_int
        L.orc_linear.argtypes = [C.POINTER(OrcMat), P, P]
        L.orc_rms_norm.argtypes = [P, P, P, u32, f32]
        L.orc_layer_norm.argtypes = [P, P, P, P, u32, f32]
        L.orc_ffn_glu.argtypes = [P, P, P, u32, C.c_int]
        L.orc_rope.argtypes = [P, u32, u32, u32, f32, C.c_int]
        L.orc_causal_mha.argtypes = [P, P, P, P, P, P, u32, u32, u32, u32]
        L.orc_greedy.argtypes = [P, u32]
        L.orc_greedy.restype = u32
        L.orc_f16_to_f32.argtypes = [C.c_uint16]
        L.orc_f16_to_f32.restype = f32
        L.orc_llama_state_new.argtypes = [C.POINTER(OrcLlama)]
        L.orc_llama_state_new.restype = P
        L.orc_gpt2_state_new.argtypes = [C.POINTER(OrcGpt2)]
        L.orc_gpt2_state_new.restype = P
        L.orc_state_free.argtypes = [P]
        L.orc_llama_forward.argtypes = [C.POINTER(OrcLlama), P, u32, u32, P, P]
        L.orc_gpt2_forward.argtypes = [C.POINTER(OrcGpt2), P, u32, u32, P, P]
        L.orc_llama_generate.argtypes = [C.POINTER(OrcLlama), P, P, u32, P, u32, u32]
        L.orc_llama_generate.restype = u32
        L.orc_gpt2_generate.argtypes = [C.POINTER(OrcGpt2), P, P, u32, P, u32, u32]
        L.orc_gpt2_generate.restype = u32
        _orc = L
    return _orc


def _bind_driver(L: C.CDLL) -> C.CDLL:
    L.drv_open.argtypes = [C.c_char_p, u32]
    L.drv_open.restype = C.c_int
    L.drv_open_file.argtypes = [C.c_char_p]
    L.drv_open_file.restype = C.c_int
    L.drv_vocab.restype = u32
    L.drv_forward.argtypes = [u32, u32, P]
    L.drv_generate.argtypes = [P, u32, P, u32, u32]
    L.drv_generate.restype = u32
    L.drv_generate_sampled.argtypes = [P, u32, P, u32, u32, f32, f32, u32]
    L.drv_generate_sampled.restype = u32
    L.sample_token.argtypes = [P, u32, f32, f32]
    L.sample_token.restype = u32
    L.drv_perplexity.argtypes = [P, u32]
    L.drv_perplexity.restype = f32
    L.drv_time_decode.argtypes = [u32, u32, u32, P]
    L.drv_time_decode.restype = C.c_double
    L.drv_dequant_rows.argtypes = [C.c_char_p, u32, u32, u32, P]
    L.drv_dequant_rows.restype = C.c_int
    L.drv_fake_generate.argtypes = [P]
    L.drv_fake_generate.restype = u32
    L.drv_rms_norm.argtypes = [P, P, P, u32, f32]
    L.drv_rope.argtypes = [P, u32, u32, u32, f32, C.c_int]
    L.drv_ffn_glu.argtypes = [P, P, P, u32, C.c_int]
    L.drv_causal_mha.argtypes = [P, P, P, P, P, u32, P, u32, u32, u32, u32]
    L.drv_linear_f32.argtypes = [P, P, P, u32, u32]
    L.drv_greedy.argtypes = [P, u32]
    L.drv_greedy.restype = u32
    return L


def reference() -> C.CDLL | None:
    """The reference's own C compiled from its sources, or None if not built."""
    if not os.path.exists(REF_SO):
        return None
    return _bind_driver(C.CDLL(REF_SO))


def dropin() -> C.CDLL | None:
    """The same driver compiled against include/ and linked to libllamini_cuda.so."""
    if not os.path.exists(DROPIN_SO):
        return None
    return _bind_driver(C.CDLL(DROPIN_SO))


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


# ----------------------------------------------------------------- models from GGUF

class _Keep:
    """Holds numpy views so the pointers in the ctypes structs stay valid."""

    def __init__(self):
        self.items = []

    def f32(self, reader, name):
        t, ne, raw = reader.raw(name)
        assert t == 0, (name, t)
        a = np.ascontiguousarray(raw).view(np.float32)
        self.items.append(a)
        return a.ctypes.data_as(FP)

    def mat(self, reader, name, rows, cols):
        t, ne, raw = reader.raw(name)
        assert int(np.prod(ne)) == rows * cols, (name, ne, rows, cols)
        self.items.append(raw)
        return OrcMat(t, rows, cols, raw.ctypes.data)


class OracleLlama:
    """Restated LLaMA-family forward pass over a GGUF file's raw bytes."""

    def __init__(self, path: str, max_seq: int = 0):
        S = _synthetic()
        r = S.GGUFReader(path)
        self.reader = r
        a = r.meta.get("general.architecture", "llama")
        g = lambda k, d=None: r.meta.get(a + "." + k, d)
        dim, nh = g("embedding_length"), g("attention.head_count")
        nkv = g("attention.head_count_kv", nh)
        hd = g("key_length", None) or g("attention.key_length", None) or dim // nh
        ffn = g("feed_forward_length")
        vocab = len(r.meta["tokenizer.ggml.tokens"])
        ctx = min(g("context_length", 2048), 2048)
        self.keep = k = _Keep()
        m = OrcLlama()
        m.dim, m.n_layers, m.n_heads, m.n_heads_kv, m.head_dim = dim, g("block_count"), nh, nkv, hd
        m.ffn_dim, m.vocab, m.max_seq = ffn, vocab, max_seq or ctx
        m.rms_eps = g("attention.layer_norm_rms_epsilon", 1e-5)
        m.rope_base = g("rope.freq_base", 10000.0)
        m.emb_scale = float(np.sqrt(np.float32(dim))) if a == "gemma" else 1.0
        m.rope_neox = 1 if a in ("qwen2", "gemma") else 0
        m.act_gelu = 1 if a == "gemma" else 0
        m.tok_embd = k.mat(r, "token_embd.weight", vocab, dim)
        m.lm_head = k.mat(r, "output.weight" if "output.weight" in r.tensors else "token_embd.weight", vocab, dim)
        m.final_norm = k.f32(r, "output_norm.weight")
        self.layers = (OrcLlamaLayer * m.n_layers)()
        qd, kvd = nh * hd, nkv * hd
        for l in range(m.n_layers):
            p = "blk.%d." % l
            L = self.layers[l]
            L.q = k.mat(r, p + "attn_q.weight", qd, dim)
            L.k = k.mat(r, p + "attn_k.weight", kvd, dim)
            L.v = k.mat(r, p + "attn_v.weight", kvd, dim)
            L.o = k.mat(r, p + "attn_output.weight", dim, qd)
            L.gate = k.mat(r, p + "ffn_gate.weight", ffn, dim)
            L.up = k.mat(r, p + "ffn_up.weight", ffn, dim)
            L.down = k.mat(r, p + "ffn_down.weight", dim, ffn)
            L.attn_norm = k.f32(r, p + "attn_norm.weight")
            L.ffn_norm = k.f32(r, p + "ffn_norm.weight")
            if a == "qwen2":
                L.bq, L.bk, L.bv = (k.f32(r, p + s) for s in ("attn_q.bias", "attn_k.bias", "attn_v.bias"))
        m.layers = self.layers
        self.m = m
        self.state = oracle().orc_llama_state_new(C.byref(m))

    def forward(self, pos, token, trace=False):
        logits = np.zeros(self.m.vocab, np.float32)
        tr = np.zeros((self.m.n_layers, self.m.dim), np.float32) if trace else None
        oracle().orc_llama_forward(C.byref(self.m), self.state, pos, token, ptr(logits),
                                   ptr(tr) if trace else None)
        return (logits, tr) if trace else logits

    def generate(self, prompt, max_gen, eos=0xFFFFFFFF):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(len(p) + max_gen + 1, np.uint32)
        self.reset()
        n = oracle().orc_llama_generate(C.byref(self.m), self.state, ptr(p), len(p), ptr(out), max_gen, eos)
        return out[:n]

    def reset(self):
        oracle().orc_state_free(self.state)
        self.state = oracle().orc_llama_state_new(C.byref(self.m))

    def __del__(self):
        try:
            oracle().orc_state_free(self.state)
        except Exception:
            pass


class OracleGpt2:
    """Restated GPT-2 forward pass over a GGUF file's raw bytes."""

    def __init__(self, path: str, max_seq: int = 0):
        S = _synthetic()
        r = S.GGUFReader(path)
        self.reader = r
        g = lambda k, d=None: r.meta.get("gpt2." + k, d)
        dim, nh, ffn = g("embedding_length"), g("attention.head_count"), g("feed_forward_length")
        vocab = len(r.meta["tokenizer.ggml.tokens"])
        ctx = min(g("context_length", 1024), 2048)
        self.keep = k = _Keep()
        m = OrcGpt2()
        m.dim, m.n_layers, m.n_heads, m.ffn_dim, m.vocab, m.n_ctx = dim, g("block_count"), nh, ffn, vocab, ctx
        m.max_seq = max_seq or ctx
        m.ln_eps = 1e-5
        m.tok_embd = k.mat(r, "token_embd.weight", vocab, dim)
        m.pos_embd = k.mat(r, "position_embd.weight", ctx, dim)
        m.out_norm_w = k.f32(r, "output_norm.weight")
        m.out_norm_b = k.f32(r, "output_norm.bias")
        m.lm_head = k.mat(r, "output.weight", vocab, dim)
        self.layers = (OrcGpt2Layer * m.n_layers)()
        for l in range(m.n_layers):
            p = "blk.%d." % l
            L = self.layers[l]
            L.attn_norm_w, L.attn_norm_b = k.f32(r, p + "attn_norm.weight"), k.f32(r, p + "attn_norm.bias")
            L.qkv, L.qkv_b = k.mat(r, p + "attn_qkv.weight", 3 * dim, dim), k.f32(r, p + "attn_qkv.bias")
            L.out, L.out_b = k.mat(r, p + "attn_output.weight", dim, dim), k.f32(r, p + "attn_output.bias")
            L.ffn_norm_w, L.ffn_norm_b = k.f32(r, p + "ffn_norm.weight"), k.f32(r, p + "ffn_norm.bias")
            L.up, L.up_b = k.mat(r, p + "ffn_up.weight", ffn, dim), k.f32(r, p + "ffn_up.bias")
            L.down, L.down_b = k.mat(r, p + "ffn_down.weight", dim, ffn), k.f32(r, p + "ffn_down.bias")
        m.layers = self.layers
        self.m = m
        self.state = oracle().orc_gpt2_state_new(C.byref(m))

    def forward(self, pos, token, trace=False):
        logits = np.zeros(self.m.vocab, np.float32)
        tr = np.zeros((self.m.n_layers, self.m.dim), np.float32) if trace else None
        oracle().orc_gpt2_forward(C.byref(self.m), self.state, pos, token, ptr(logits),
                                  ptr(tr) if trace else None)
        return (logits, tr) if trace else logits

    def generate(self, prompt, max_gen, eos=0xFFFFFFFF):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(len(p) + max_gen + 1, np.uint32)
        self.reset()
        n = oracle().orc_gpt2_generate(C.byref(self.m), self.state, ptr(p), len(p), ptr(out), max_gen, eos)
        return out[:n]

    def reset(self):
        oracle().orc_state_free(self.state)
        self.state = oracle().orc_gpt2_state_new(C.byref(self.m))


def oracle_model(path: str, max_seq: int = 0):
    r = _synthetic().GGUFReader(path)
    if r.meta.get("general.architecture") == "gpt2":
        return OracleGpt2(path, max_seq)
    return OracleLlama(path, max_seq)


def dequant(t: int, raw: np.ndarray, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    rc = oracle().orc_dequant(t, ptr(np.ascontiguousarray(raw)), n, ptr(out))
    assert rc == 0
    return out
