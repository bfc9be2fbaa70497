"""Gemma on the LLaMA path (model.c:296-299, 319, 447-452): NEOX RoPE, GeGLU,
embeddings scaled by sqrt(dim), lm_head tied to the embedding table.

The single-sequence path and the batched (tensor-core GEMM) path must both
reproduce the oracle's greedy stream, with logits within the 1e-3 bar.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _oracle_stream(orc, path, prompt, n_gen, keep):
    o = orc.oracle_model(path)
    toks, lg_keep = list(prompt), []
    for pos in range(len(prompt) + n_gen - 1):
        lg = o.forward(pos, toks[pos])
        if pos < keep:
            lg_keep.append(lg)
        if pos + 1 >= len(prompt):
            toks.append(int(np.argmax(lg)))
    return toks, lg_keep


def test_gemma_single_and_batch_match_oracle(gpu, orc, tiny):
    path = tiny.ensure("tiny_gemma")
    rng = np.random.default_rng(23)
    prompt = rng.integers(3, 600, 6).tolist()
    n_gen = 20
    want, want_lg = _oracle_stream(orc, path, prompt, n_gen, 5)
    m = gpu.Model(path)
    L = gpu.lib()
    try:
        got = m.generate(np.array(prompt, np.uint32), n_gen).tolist()
        assert got == want, (got, want)
        for pos in range(5):
            lg = m.forward(pos, want[pos])
            assert rel_l2(lg, want_lg[pos]) < TOL, (pos, rel_l2(lg, want_lg[pos]))
        b = L.llamini_llama_batch(C.byref(m.model), 3, m.max_seq)
        assert b, gpu.last_error()
        try:
            others = [rng.integers(3, 600, 9).tolist(), rng.integers(3, 600, 2).tolist()]
            prompts = [prompt] + others
            flat = np.concatenate([np.asarray(p, np.uint32) for p in prompts])
            lens = np.array([len(p) for p in prompts], np.uint32)
            assert L.llamini_batch_begin(b, 3, gpu.ptr(flat), gpu.ptr(lens)) == 0, gpu.last_error()
            steps = len(want) - 1
            assert L.llamini_batch_step(b, steps) == 0, gpu.last_error()
            out = np.zeros(steps + 1, np.uint32)
            assert L.llamini_batch_tokens(b, 0, gpu.ptr(out), steps + 1) >= 0, gpu.last_error()
            assert out.tolist() == want
            for s, p in enumerate(others, start=1):
                o2 = np.zeros(steps + 1, np.uint32)
                assert L.llamini_batch_tokens(b, s, gpu.ptr(o2), steps + 1) >= 0
                alone = m.generate(np.array(p, np.uint32), steps + 1 - len(p)).tolist()
                assert o2.tolist() == alone[:steps + 1], s
        finally:
            L.llamini_batch_free(b)
    finally:
        m.close()
