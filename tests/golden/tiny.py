"""Small synthetic GGUF models used by the parity tests.

They exercise every code path of the token loop at sizes the CPU oracle and
the reference finish in seconds: K-quant and 32-block formats in every matrix
role, GQA, NORM and NEOX RoPE, q/k/v biases, tied embeddings, GPT-2's fused
QKV / LayerNorm / GELU / learned positions, and F16/F32 tables.
"""
from __future__ import annotations

import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def synthetic():
    name = "llamini_b200_synthetic"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "llamini.cpp_b200", "synthetic.py"))
    m = importlib.util.module_from_spec(spec)
    sys.modules[name] = m
    spec.loader.exec_module(m)
    return m


def _types(S, q, k, v, o, gate, up, down, embd, output):
    c = lambda t: (lambda l: t) if isinstance(t, int) else t
    return {"q": c(q), "k": c(k), "v": c(v), "o": c(o), "gate": c(gate), "up": c(up), "down": c(down),
            "embd": embd, "output": output}


def specs():
    """name -> (GGUFSpec, seed)"""
    S = synthetic()
    out = {}
    # LLaMA-family: the Q4_K_M mix at a small shape (Q6_K on layer 0's v/down).
    out["tiny_llama"] = (S.llama_spec(S.shape_llama_1b(
        dim=256, n_layers=3, n_heads=8, n_kv=2, ffn=512, vocab=1000, ctx=128)), 10)
    # Every other format in some matrix role, NORM RoPE, 4 heads of 64.
    out["tiny_mixed"] = (S.llama_spec(S.shape_llama_1b(
        dim=256, n_layers=2, n_heads=4, n_kv=4, ffn=768, vocab=512, ctx=96,
        types=_types(S, S.Q4_0, S.Q4_1, S.Q5_0, S.Q8_0, S.Q5_K, S.Q4_K, S.Q6_K, S.Q8_0, S.Q5_K))), 11)
    # Qwen2: NEOX RoPE, q/k/v biases, 192-wide rows (32-block formats only), theta 1e6.
    out["tiny_qwen2"] = (S.llama_spec(S.shape_qwen2_05b(
        dim=192, n_layers=2, n_heads=6, n_kv=2, ffn=512, vocab=800, ctx=128)), 12)
    # Tied lm_head: no output.weight, the embedding table is the head (model.c:447-452).
    tied = S.llama_spec(S.shape_llama_1b(dim=256, n_layers=2, n_heads=4, n_kv=1, ffn=512, vocab=600, ctx=64))
    tied.tensors = [t for t in tied.tensors if t.name != "output.weight"]
    out["tiny_tied"] = (tied, 14)
    # Tensor-parallel shape: 8 heads of 64 and 4 kv heads, FFN of 6 super-blocks,
    # so two ranks split o-proj and down on 256-column boundaries.
    out["tiny_tp"] = (S.llama_spec(S.shape_llama_1b(
        dim=512, n_layers=2, n_heads=8, n_kv=4, ffn=1536, vocab=1000, ctx=128)), 15)
    # Gemma: NEOX RoPE, GeGLU, embeddings scaled by sqrt(dim), lm_head tied to the
    # embeddings (model.c:296-299, 319, 447-452).
    g = S.shape_llama_1b(dim=256, n_layers=2, n_heads=4, n_kv=1, ffn=512, vocab=600, ctx=64)
    g.arch = "gemma"
    gemma = S.llama_spec(g)
    gemma.tensors = [t for t in gemma.tensors if t.name != "output.weight"]
    out["tiny_gemma"] = (gemma, 16)
    # GPT-2: Q8_0 matrices, F16 embeddings, LayerNorm + biases, GELU MLP.
    out["tiny_gpt2"] = (S.gpt2_spec(S.Gpt2Shape(dim=128, n_layers=2, n_heads=4, ffn=512, vocab=700, ctx=64)), 13)
    return out


def path_of(name: str, directory: str | None = None) -> str:
    directory = directory or os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200")
    return os.path.join(directory, name + ".gguf")


def ensure(name: str, directory: str | None = None) -> str:
    spec, seed = specs()[name]
    return synthetic().ensure_spec(spec, seed, path_of(name, directory))
