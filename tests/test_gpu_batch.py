"""Batched decode (llamini_*_batch) on the GPU.

Every sequence of a batch must decode exactly as it would alone: its greedy
token stream equals the single-sequence path's (and, for the golden prompts, the
reference's own stream), and its logits stay within the 1e-3 bar of the CPU
oracle. Prompts are ragged, so sequences switch from prompt to generated tokens
at different steps of the lockstep batch.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _batch(gpu, m, max_batch, max_seq):
    L = gpu.lib()
    fn = L.llamini_gpt2_batch if m.is_gpt2 else L.llamini_llama_batch
    b = fn(C.byref(m.model), max_batch, max_seq)
    assert b, gpu.last_error()
    return b


def _begin(gpu, b, prompts):
    flat = np.concatenate([np.asarray(p, np.uint32) for p in prompts])
    lens = np.array([len(p) for p in prompts], np.uint32)
    assert gpu.lib().llamini_batch_begin(b, len(prompts), gpu.ptr(flat), gpu.ptr(lens)) == 0, gpu.last_error()


def _tokens(gpu, b, seq, n):
    out = np.zeros(n, np.uint32)
    k = gpu.lib().llamini_batch_tokens(b, seq, gpu.ptr(out), n)
    assert k >= 0, gpu.last_error()
    return out[:min(k, n)].tolist()


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_tied", "tiny_gpt2", "tiny_mixed", "tiny_qwen2"])
def test_batch_streams_equal_single_sequence(gpu, orc, tiny, golden, name):
    path = tiny.ensure(name)
    m = gpu.Model(path)
    L = gpu.lib()
    g = golden["tokens"][name]
    rng = np.random.default_rng(7)
    vocab = m.vocab
    prompts = [g["prompt"], rng.integers(3, vocab, 3).tolist(), rng.integers(3, vocab, 9).tolist(),
               [1], rng.integers(3, vocab, 16).tolist()]
    steps = min(m.max_seq, 48) - 1
    b = _batch(gpu, m, 8, m.max_seq)
    try:
        _begin(gpu, b, prompts)
        assert L.llamini_batch_step(b, steps) == 0, gpu.last_error()
        assert L.llamini_batch_pos(b) == steps
        for s, p in enumerate(prompts):
            got = _tokens(gpu, b, s, steps + 1)
            assert len(got) == steps + 1
            alone = m.generate(np.array(p, np.uint32), steps + 1 - len(p)).tolist()
            assert got == alone[:steps + 1], (s, got, alone)
        ref = g["tokens"]
        n = min(len(ref), steps + 1)
        assert _tokens(gpu, b, 0, n) == ref[:n]
        # logits of the last step against the oracle, teacher-forced on the stream
        o = orc.oracle_model(path)
        for s in (0, 3):
            toks = _tokens(gpu, b, s, steps + 1)
            want = None
            for pos in range(steps):
                want = o.forward(pos, toks[pos])
            lg = np.zeros(vocab, np.float32)
            assert L.llamini_batch_logits(b, s, gpu.ptr(lg)) == 0
            assert rel_l2(lg, want) < TOL, (s, rel_l2(lg, want))
    finally:
        L.llamini_batch_free(b)
        m.close()


def test_batch_gemm_kinds(gpu, tiny):
    """Every block format takes the tensor-core GEMM; the mma.sync GEMM (kept
    behind llamini_set_batch_gemm(0)) refuses Q4_1, Q5_0 and Q5_K with a message."""
    L = gpu.lib()
    m = gpu.Model(tiny.ensure("tiny_mixed"))       # Q4_0 Q4_1 Q5_0 Q8_0 Q5_K Q4_K Q6_K matrices
    try:
        b = L.llamini_llama_batch(C.byref(m.model), 4, 32)
        assert b, gpu.last_error()
        assert L.llamini_batch_gemm_kind(b) == 1
        L.llamini_batch_free(b)
        assert L.llamini_set_batch_gemm(0) == 0
        try:
            assert not L.llamini_llama_batch(C.byref(m.model), 4, 32)
            assert "batched" in gpu.last_error()
            L.llamini_clear_error()
        finally:
            L.llamini_set_batch_gemm(-1)
    finally:
        m.close()


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_gpt2"])
def test_batch_mma_gemm_streams(gpu, tiny, golden, name):
    """The mma.sync GEMM (llamini_set_batch_gemm(0)) still decodes the golden
    prompt's stream."""
    L = gpu.lib()
    g = golden["tokens"][name]
    m = gpu.Model(tiny.ensure(name))
    assert L.llamini_set_batch_gemm(0) == 0
    try:
        b = _batch(gpu, m, 2, m.max_seq)
    finally:
        L.llamini_set_batch_gemm(-1)
    try:
        assert L.llamini_batch_gemm_kind(b) == 0
        _begin(gpu, b, [g["prompt"], g["prompt"][:3]])
        steps = min(m.max_seq, 40) - 1
        assert L.llamini_batch_step(b, steps) == 0, gpu.last_error()
        n = min(len(g["tokens"]), steps + 1)
        assert _tokens(gpu, b, 0, n) == g["tokens"][:n]
    finally:
        L.llamini_batch_free(b)
        m.close()


@pytest.mark.parametrize("name", ["llama_1b", "gpt2_124m"])
def test_batch_workload_golden_stream(gpu, synth, golden, name):
    """Full-size workloads, 4 sequences: the golden prompt's stream equals the
    reference's for 24 generated tokens; the others equal the single path."""
    g = golden["tokens"][name]
    m = gpu.Model(synth.ensure_workload(name), max_seq=512)
    L = gpu.lib()
    rng = np.random.default_rng(3)
    prompts = [g["prompt"], rng.integers(3, m.vocab, 40).tolist(), rng.integers(3, m.vocab, len(g["prompt"])).tolist(),
               rng.integers(3, m.vocab, 5).tolist()]
    steps = len(g["prompt"]) - 1 + 24
    b = _batch(gpu, m, 4, 512)
    try:
        _begin(gpu, b, prompts)
        assert L.llamini_batch_step(b, steps) == 0, gpu.last_error()
        assert _tokens(gpu, b, 0, steps + 1) == g["tokens"][:steps + 1]
        for s in (1, 3):
            got = _tokens(gpu, b, s, steps + 1)
            alone = m.generate(np.array(prompts[s], np.uint32), steps + 1 - len(prompts[s])).tolist()
            assert got == alone[:steps + 1], s
    finally:
        L.llamini_batch_free(b)
        m.close()


def _run_batch(gpu, m, prompts, calls, max_batch):
    """Tokens of every sequence after llamini_batch_step(b, n) for each n of `calls`."""
    L = gpu.lib()
    b = _batch(gpu, m, max_batch, m.max_seq)
    try:
        _begin(gpu, b, prompts)
        for n in calls:
            assert L.llamini_batch_step(b, n) == 0, gpu.last_error()
        steps = sum(calls)
        assert L.llamini_batch_pos(b) == steps
        toks = [_tokens(gpu, b, s, steps + 1) for s in range(len(prompts))]
        lg = np.zeros(m.vocab, np.float32)
        assert L.llamini_batch_logits(b, 0, gpu.ptr(lg)) == 0, gpu.last_error()
        return toks, lg
    finally:
        L.llamini_batch_free(b)


@pytest.mark.parametrize("name,n_seq", [("tiny_llama", 3), ("tiny_gpt2", 3), ("tiny_qwen2", 8), ("tiny_llama", 32),
                                        ("tiny_llama", 64)])
def test_batch_prompt_prefill(gpu, orc, tiny, golden, name, n_seq):
    """Lockstep positions inside every sequence's prompt run as prefill chunks of
    64 / B positions x B sequences (B = 3: 21 x 3, B = 8: 8 x 8, B = 32: 2 x
    32) into the batch's caches; B = 64 keeps the lockstep steps. The streams
    equal the one-position-at-a-time batch (prefill off), the single-sequence
    path and, for the golden prompt, the reference's; the last step's logits
    stay within 1e-3 of the oracle. Steps come in calls that stop inside the
    prompt, at its end and past it."""
    path = tiny.ensure(name)
    m = gpu.Model(path)
    L = gpu.lib()
    g = golden["tokens"][name]
    rng = np.random.default_rng(11)
    base = list(g["prompt"]) + rng.integers(3, m.vocab, 20).tolist()       # 36 tokens
    prompts = [base] + [rng.integers(3, m.vocab, int(rng.integers(24, 40))).tolist() for _ in range(n_seq - 1)]
    common = min(len(p) for p in prompts)
    steps = min(m.max_seq, 64) - 1
    calls = [5, common - 1 - 5 - 3, 3 + 4, steps - (common - 1) - 4]
    assert all(c > 0 for c in calls)
    try:
        got, lg = _run_batch(gpu, m, prompts, calls, n_seq)
        assert L.llamini_set_prefill(0) == 0
        try:
            want, lg_off = _run_batch(gpu, m, prompts, calls, n_seq)
        finally:
            L.llamini_set_prefill(-1)
        assert got == want
        for s in range(min(n_seq, 4)):
            alone = m.generate(np.array(prompts[s], np.uint32), steps + 1 - len(prompts[s])).tolist()
            assert got[s] == alone[:steps + 1], s
        # the golden prompt's first 16 tokens, then the sequence's own prompt
        o = orc.oracle_model(path)
        want_lg = None
        for pos in range(steps):
            want_lg = o.forward(pos, got[0][pos])
        assert rel_l2(lg, want_lg) < TOL, rel_l2(lg, want_lg)
        assert rel_l2(lg_off, want_lg) < TOL
    finally:
        m.close()


def test_batch_prefill_workload_golden(gpu, synth, golden):
    """llama_1b, 4 sequences sharing the golden 128-token prompt's length: 126
    positions of prefill (16 x 4 columns per chunk), then the reference's
    stream for 24 generated tokens on the golden sequence."""
    g = golden["tokens"]["llama_1b"]
    m = gpu.Model(synth.ensure_workload("llama_1b"), max_seq=512)
    L = gpu.lib()
    rng = np.random.default_rng(5)
    n = len(g["prompt"])
    prompts = [g["prompt"]] + [rng.integers(3, m.vocab, n + d).tolist() for d in (0, 3, 9)]
    steps = n - 1 + 24
    b = _batch(gpu, m, 4, 512)
    try:
        _begin(gpu, b, prompts)
        assert L.llamini_batch_step(b, steps) == 0, gpu.last_error()
        assert _tokens(gpu, b, 0, steps + 1) == g["tokens"][:steps + 1]
        got = _tokens(gpu, b, 2, steps + 1)
        alone = m.generate(np.array(prompts[2], np.uint32), steps + 1 - len(prompts[2])).tolist()
        assert got == alone[:steps + 1]
    finally:
        L.llamini_batch_free(b)
        m.close()
