"""Python binding of libllamini_cuda.so (ctypes, plain pointers).

The library's API is the reference's C99 API (gguf.h, model.h, generate.h,
kv_cache.h, tensor.h, gpt2.h) plus the additive llamini_b200.h. This module
declares the caller-visible structs with the reference layouts and wraps the
calls that tests and the benchmark make. There is no fallback: if the shared
library is missing, importing this module raises.

Because the directory name contains a dot it is loaded by path, e.g.
``importlib`` with ``spec_from_file_location("llamini_b200", ".../__init__.py")``.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libllamini_cuda.so")

u32, u64, f32, i32 = C.c_uint32, C.c_uint64, C.c_float, C.c_int32
P = C.c_void_p


class GGUFHeader(C.Structure):           # gguf.h:62-67
    _fields_ = [("magic", u32), ("version", u32), ("n_tensors", u64), ("n_metadata", u64)]


class GGUFFile(C.Structure):             # gguf.h:70-82
    _fields_ = [("fd", C.c_int), ("data", P), ("size", C.c_size_t), ("hdr", GGUFHeader),
                ("tensor_offset", u64), ("kv", P), ("n_kv", u64), ("tensors", P), ("n_tensors", u64)]


class Tensor(C.Structure):               # tensor.h:16-23
    _fields_ = [("dims", u32 * 4), ("ndim", u32), ("size", u32), ("data", C.POINTER(f32)),
                ("src_gf", P), ("src_info", P)]


class LLaMAConfig(C.Structure):          # model.h:24-40
    _fields_ = [("dim", u32), ("n_layers", u32), ("n_heads", u32), ("n_heads_kv", u32),
                ("head_dim", u32), ("ffn_dim", u32), ("vocab_size", u32), ("seq_len", u32),
                ("rms_eps", f32), ("rope_freq_base", f32), ("rope_type", C.c_int),
                ("ffn_act", C.c_int), ("qkv_bias", C.c_int), ("embedding_scale", f32)]


class DecoderLayer(C.Structure):         # model.h:46-59
    _fields_ = [(n, C.POINTER(Tensor)) for n in
                ("attn_norm", "q_proj", "k_proj", "v_proj", "q_bias", "k_bias", "v_bias",
                 "o_proj", "ffn_norm", "gate_proj", "up_proj", "down_proj")]


class LLaMAModel(C.Structure):           # model.h:62-68
    _fields_ = [("cfg", LLaMAConfig), ("embeddings", C.POINTER(Tensor)),
                ("layers", C.POINTER(DecoderLayer)), ("final_norm", C.POINTER(Tensor)),
                ("lm_head", C.POINTER(Tensor))]


class KVCache(C.Structure):              # kv_cache.h:7-13
    _fields_ = [("key", C.POINTER(f32)), ("val", C.POINTER(f32)), ("dim", u32),
                ("max_seq", u32), ("cur_seq", u32)]


class GPT2Config(C.Structure):           # gpt2.h:18-21
    _fields_ = [("dim", u32), ("n_layers", u32), ("n_heads", u32), ("ffn_dim", u32),
                ("vocab_size", u32), ("n_ctx", u32), ("ln_eps", f32)]


class GPT2Layer(C.Structure):            # gpt2.h:23-30
    _fields_ = [(n, C.POINTER(Tensor)) for n in
                ("attn_norm_w", "attn_norm_b", "attn_qkv_w", "attn_qkv_b", "attn_out_w",
                 "attn_out_b", "ffn_norm_w", "ffn_norm_b", "ffn_up_w", "ffn_up_b",
                 "ffn_down_w", "ffn_down_b")]


class GPT2Model(C.Structure):            # gpt2.h:32-40
    _fields_ = [("cfg", GPT2Config), ("token_embd", C.POINTER(Tensor)),
                ("pos_embd", C.POINTER(Tensor)), ("output_norm_w", C.POINTER(Tensor)),
                ("output_norm_b", C.POINTER(Tensor)), ("lm_head", C.POINTER(Tensor)),
                ("layers", C.POINTER(GPT2Layer))]


# Every function of include/*.h, with its ctypes signature. The CPU test suite
# checks that the library exports each of these.
SIGNATURES = {
    # gguf.h
    "gguf_open": (C.c_int, [C.c_char_p, C.POINTER(GGUFFile)]),
    "gguf_close": (None, [C.POINTER(GGUFFile)]),
    "gguf_read_f32": (C.c_int, [C.POINTER(GGUFFile), u64, P, u64]),
    "gguf_get_u32": (u32, [C.POINTER(GGUFFile), C.c_char_p, u32]),
    "gguf_get_f32": (f32, [C.POINTER(GGUFFile), C.c_char_p, f32]),
    "gguf_get_str": (P, [C.POINTER(GGUFFile), C.c_char_p]),
    "gguf_meta_array_len": (u64, [C.POINTER(GGUFFile), C.c_char_p, P]),
    "gguf_get_string_array": (P, [C.POINTER(GGUFFile), C.c_char_p, P]),
    "gguf_get_f32_array": (P, [C.POINTER(GGUFFile), C.c_char_p, P]),
    "gguf_get_i32_array": (P, [C.POINTER(GGUFFile), C.c_char_p, P]),
    "gguf_find_tensor": (P, [C.POINTER(GGUFFile), C.c_char_p]),
    "gguf_tensor_count": (u64, [P]),
    "gguf_dequantize_tensor": (C.c_int, [C.POINTER(GGUFFile), P, P, u64]),
    "gguf_dequantize_rows": (C.c_int, [C.POINTER(GGUFFile), P, u32, u32, u32, P]),
    # tensor.h
    "tensor_create": (C.POINTER(Tensor), [u32, P]),
    "tensor_free": (None, [C.POINTER(Tensor)]),
    "matmul": (None, [C.POINTER(Tensor), C.POINTER(Tensor), C.POINTER(Tensor)]),
    "vec_add": (None, [P, P, P, u32]),
    "vec_scale": (None, [P, P, f32, u32]),
    "tensor_get_row": (None, [C.POINTER(Tensor), u32, u32, P]),
    # kv_cache.h
    "kv_cache_init": (None, [C.POINTER(KVCache), u32, u32]),
    "kv_cache_reset": (None, [C.POINTER(KVCache)]),
    # model.h
    "rms_norm": (None, [P, P, P, u32, f32]),
    "ffn_glu": (None, [P, P, P, u32, C.c_int]),
    "rope": (None, [P, u32, u32, u32, f32, C.c_int]),
    "linear": (None, [P, P, C.POINTER(Tensor), u32, u32]),
    "add_bias": (None, [P, P, u32]),
    "causal_mha": (None, [P, P, P, C.POINTER(KVCache), P, u32, u32, u32, u32]),
    "llama_model_init": (C.c_int, [C.POINTER(LLaMAModel), C.POINTER(LLaMAConfig)]),
    "llama_model_free": (None, [C.POINTER(LLaMAModel)]),
    "llama_config_from_gguf": (LLaMAConfig, [C.POINTER(GGUFFile), LLaMAConfig, P]),
    "llama_load_weights": (C.c_int, [C.POINTER(LLaMAModel), C.POINTER(GGUFFile)]),
    # generate.h
    "greedy_sample": (u32, [P, u32]),
    "sample_token": (u32, [P, u32, f32, f32]),
    "forward_step": (None, [C.POINTER(LLaMAModel), C.POINTER(KVCache), u32, u32, P]),
    "generate_autoregressive": (u32, [C.POINTER(LLaMAModel), C.POINTER(KVCache), P, u32, P, u32, u32, f32, f32]),
    "compute_perplexity": (f32, [C.POINTER(LLaMAModel), C.POINTER(KVCache), P, u32]),
    # gpt2.h
    "gpt2_config_from_gguf": (GPT2Config, [C.POINTER(GGUFFile)]),
    "gpt2_model_init": (C.c_int, [C.POINTER(GPT2Model), C.POINTER(GPT2Config)]),
    "gpt2_model_free": (None, [C.POINTER(GPT2Model)]),
    "gpt2_load_weights": (C.c_int, [C.POINTER(GPT2Model), C.POINTER(GGUFFile)]),
    "gpt2_forward_step": (None, [C.POINTER(GPT2Model), C.POINTER(KVCache), u32, u32, P]),
    "gpt2_generate": (u32, [C.POINTER(GPT2Model), C.POINTER(KVCache), P, u32, P, u32, u32, f32, f32]),
    "gpt2_compute_perplexity": (f32, [C.POINTER(GPT2Model), C.POINTER(KVCache), P, u32]),
    # llamini_b200.h
    "llamini_last_error": (C.c_char_p, []),
    "llamini_clear_error": (None, []),
    "llamini_device_count": (C.c_int, []),
    "llamini_set_device": (C.c_int, [C.c_int]),
    "llamini_stream": (P, []),
    "llamini_release": (None, []),
    "llamini_type_bytes": (u64, [u32, u64]),
    "llamini_dequant_host": (C.c_int, [u32, P, u64, P]),
    "llamini_sample_host": (u32, [P, u32, f32, f32, f32]),
    "llamini_dequant_device": (C.c_int, [u32, P, u64, P]),
    "llamini_gemv_host": (C.c_int, [u32, P, u32, u32, P, u32, P]),
    "llamini_gemv_device": (C.c_int, [u32, P, u32, u32, P, u32, P]),
    "llamini_llama_session": (P, [C.POINTER(LLaMAModel), C.POINTER(KVCache)]),
    "llamini_gpt2_session": (P, [C.POINTER(GPT2Model), C.POINTER(KVCache)]),
    "llamini_session_begin": (C.c_int, [P, P, u32]),
    "llamini_session_step": (C.c_int, [P, u32]),
    "llamini_session_tokens": (C.c_int, [P, P, u32]),
    "llamini_session_logits": (C.c_int, [P, P]),
    "llamini_session_pos": (u32, [P]),
    "llamini_llama_batch": (P, [P, u32, u32]),
    "llamini_gpt2_batch": (P, [P, u32, u32]),
    "llamini_batch_begin": (C.c_int, [P, u32, P, P]),
    "llamini_batch_step": (C.c_int, [P, u32]),
    "llamini_batch_tokens": (C.c_int, [P, u32, P, u32]),
    "llamini_batch_logits": (C.c_int, [P, u32, P]),
    "llamini_batch_pos": (u32, [P]),
    "llamini_batch_weight_bytes": (u64, [P]),
    "llamini_batch_gemm_kind": (C.c_int, [P]),
    "llamini_set_batch_gemm": (C.c_int, [C.c_int]),
    "llamini_set_prefill": (C.c_int, [C.c_int]),
    "llamini_session_prefill": (C.c_int, [P]),
    "llamini_tp_handle": (C.c_int, [P]),
    "llamini_tp_join": (C.c_int, [C.c_uint32, C.c_uint32, P]),
    "llamini_tp_leave": (C.c_int, []),
    "llamini_tp_plan": (C.c_int, [u32, u32, u32, u32, u32, u32, P]),
    "llamini_tp_rank": (C.c_int, []),
    "llamini_tp_world": (C.c_int, []),
    "llamini_batch_free": (None, [P]),
    "llamini_session_kernel": (C.c_int, [P]),
    "llamini_session_weight_bytes": (u64, [P]),
    "llamini_session_kv_bytes_per_pos": (u64, [P]),
    "llamini_set_kv_f16": (C.c_int, [C.c_int]),
    "llamini_causal_mha_noalloc": (C.c_int, [P, P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, P]),
    "llamini_session_trace": (C.c_int, [P, C.c_int]),
    "llamini_session_trace_read": (C.c_int, [P, P]),
}


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load the library and attach signatures. Raises if it is missing."""
    if not os.path.exists(path):
        raise FileNotFoundError("libllamini_cuda.so not built (%s); run llamini.cpp_b200/build.py" % path)
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = load()
    return _lib


_libc = C.CDLL(None)
_libc.free.argtypes = [P]
_libc.free.restype = None


def last_error() -> str:
    return (lib().llamini_last_error() or b"").decode()


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Model:
    """A GGUF model opened and loaded through the reference API
    (main.c:400-481's sequence), with one KV cache per layer."""

    def __init__(self, path: str, max_seq: int = 0):
        L = lib()
        self.gf = GGUFFile()
        if L.gguf_open(path.encode(), C.byref(self.gf)) != 0:
            raise RuntimeError("gguf_open failed: " + path)
        arch = L.gguf_get_str(C.byref(self.gf), b"general.architecture")
        self.arch = C.string_at(arch).decode() if arch else "llama"
        if arch:
            _libc.free(arch)
        self.is_gpt2 = self.arch == "gpt2"
        if self.is_gpt2:
            cfg = L.gpt2_config_from_gguf(C.byref(self.gf))
            self.model = GPT2Model()
            if L.gpt2_model_init(C.byref(self.model), C.byref(cfg)) != 0 or \
                    L.gpt2_load_weights(C.byref(self.model), C.byref(self.gf)) != 0:
                raise RuntimeError("gpt2 load failed: " + last_error())
            self.cfg = self.model.cfg
            self.vocab, self.n_layers, self.dim = cfg.vocab_size, cfg.n_layers, cfg.dim
            kv_dim, ms = cfg.dim, (max_seq or cfg.n_ctx)
        else:
            d = LLaMAConfig(dim=2048, n_layers=22, n_heads=32, n_heads_kv=4, ffn_dim=5632,
                            vocab_size=32000, seq_len=2048, rms_eps=1e-5, rope_freq_base=10000.0)
            cfg = L.llama_config_from_gguf(C.byref(self.gf), d, None)
            self.model = LLaMAModel()
            if L.llama_model_init(C.byref(self.model), C.byref(cfg)) != 0 or \
                    L.llama_load_weights(C.byref(self.model), C.byref(self.gf)) != 0:
                raise RuntimeError("llama load failed: " + last_error())
            self.cfg = self.model.cfg
            self.vocab, self.n_layers, self.dim = cfg.vocab_size, cfg.n_layers, cfg.dim
            kv_dim, ms = cfg.n_heads_kv * cfg.head_dim, (max_seq or cfg.seq_len)
        self.max_seq = ms
        self.caches = (KVCache * self.n_layers)()
        for i in range(self.n_layers):
            L.kv_cache_init(C.byref(self.caches[i]), kv_dim, ms)
        self._closed = False

    # reference-API calls -------------------------------------------------
    def generate(self, prompt, max_gen: int, eos: int = 0xFFFFFFFF, temp: float = 0.0,
                 top_p: float = 0.0) -> np.ndarray:
        """generate_autoregressive (generate.c:122-167); temp > 0 samples with
        the process's rand() stream, as the reference does."""
        L = lib()
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(len(p) + max_gen + 1, dtype=np.uint32)
        for i in range(self.n_layers):
            L.kv_cache_reset(C.byref(self.caches[i]))
        fn = L.gpt2_generate if self.is_gpt2 else L.generate_autoregressive
        n = fn(C.byref(self.model), self.caches, ptr(p), len(p), ptr(out), max_gen, eos, temp, top_p)
        return out[:n]

    def forward(self, pos: int, token: int) -> np.ndarray:
        logits = np.zeros(self.vocab, dtype=np.float32)
        fn = lib().gpt2_forward_step if self.is_gpt2 else lib().forward_step
        fn(C.byref(self.model), self.caches, pos, token, ptr(logits))
        return logits

    def perplexity(self, tokens) -> float:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        fn = lib().gpt2_compute_perplexity if self.is_gpt2 else lib().compute_perplexity
        return float(fn(C.byref(self.model), self.caches, ptr(t), len(t)))

    # device-resident session --------------------------------------------
    def session(self):
        L = lib()
        s = (L.llamini_gpt2_session if self.is_gpt2 else L.llamini_llama_session)(
            C.byref(self.model), self.caches)
        if not s:
            raise RuntimeError("session failed: " + last_error())
        return s

    def close(self):
        if self._closed:
            return
        L = lib()
        # same order as main.c:444-447: caches (plain free), model, file
        for i in range(self.n_layers):
            _libc.free(C.cast(self.caches[i].key, P))
            _libc.free(C.cast(self.caches[i].val, P))
        (L.gpt2_model_free if self.is_gpt2 else L.llama_model_free)(C.byref(self.model))
        L.gguf_close(C.byref(self.gf))
        self._closed = True
