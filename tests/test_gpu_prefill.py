"""Chunked prefill (llamini_set_prefill): prompt positions run 64 at a time
through the tensor-core GEMM with causal attention over the cache.

The greedy stream after a prefilled prompt must equal the reference's (golden
fixtures) and the one-position-at-a-time path's; the logits of the last prompt
position (the decode step that follows the prefill) stay within the 1e-3 bar of
the oracle -- for prompts of one chunk and of several chunks.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _gen(gpu, m, prompt, n, prefill):
    L = gpu.lib()
    assert L.llamini_set_prefill(prefill) == 0
    try:
        return m.generate(np.array(prompt, np.uint32), n).tolist()
    finally:
        L.llamini_set_prefill(-1)


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_tied", "tiny_gemma", "tiny_gpt2", "tiny_qwen2"])
def test_prefill_golden_streams(gpu, tiny, golden, name):
    g = golden["tokens"].get(name)
    m = gpu.Model(tiny.ensure(name))
    try:
        if g is not None:
            got = _gen(gpu, m, g["prompt"], 40, 1)
            assert got == g["tokens"][:len(got)], gpu.last_error()
        rng = np.random.default_rng(31)
        prompt = rng.integers(3, m.vocab, min(m.max_seq - 30, 100)).tolist()   # two chunks where the cache allows
        on = _gen(gpu, m, prompt, 20, 1)
        off = _gen(gpu, m, prompt, 20, 0)
        assert on == off, (on, off)
        assert gpu.lib().llamini_session_prefill(m.session()) == 1      # every format takes the GEMM
    finally:
        m.close()


@pytest.mark.parametrize("name,n_prompt", [("tiny_llama", 100), ("tiny_gemma", 40), ("tiny_gpt2", 60)])
def test_prefill_logits_vs_oracle(gpu, orc, tiny, name, n_prompt):
    path = tiny.ensure(name)
    m = gpu.Model(path)
    L = gpu.lib()
    try:
        rng = np.random.default_rng(37)
        prompt = rng.integers(3, m.vocab, n_prompt).astype(np.uint32)
        s = m.session()
        assert L.llamini_session_begin(s, gpu.ptr(prompt), n_prompt) == 0
        assert L.llamini_session_step(s, n_prompt) == 0, gpu.last_error()     # prefill, then the last position
        assert L.llamini_session_prefill(s) == 1
        lg = np.zeros(m.vocab, np.float32)
        assert L.llamini_session_logits(s, gpu.ptr(lg)) == 0, gpu.last_error()
        o = orc.oracle_model(path)
        want = None
        for p in range(n_prompt):
            want = o.forward(p, int(prompt[p]))
        assert rel_l2(lg, want) < TOL, rel_l2(lg, want)
    finally:
        m.close()


def test_prefill_workload_stream(gpu, synth, golden):
    """llama_1b: the 128-token golden prompt (two chunks) then 64 greedy tokens,
    identical to the reference's stream."""
    g = golden["tokens"]["llama_1b"]
    m = gpu.Model(synth.ensure_workload("llama_1b"), max_seq=512)
    try:
        got = _gen(gpu, m, g["prompt"], 64, 1)
        assert got == g["tokens"][:len(got)], gpu.last_error()
        assert gpu.lib().llamini_session_prefill(m.session()) == 1
    finally:
        m.close()


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_mixed", "tiny_gpt2", "tiny_tied", "tiny_gemma", "tiny_qwen2"])
def test_perplexity_chunked(gpu, orc, tiny, name):
    """compute_perplexity runs its positions 64 at a time (tensor-core GEMMs, the
    lm_head for every position, the log-softmax on the device) when the lm_head
    has a tensor-core plan, else one position at a time; both agree with each
    other and with a teacher-forced evaluation of the oracle's logits."""
    path = tiny.ensure(name)
    m = gpu.Model(path)
    L = gpu.lib()
    # the model's own greedy continuation of one token as the text: random ids
    # would give these random-weight models a loss beyond expf's range (an
    # infinite perplexity on every path)
    start = np.random.default_rng(41).integers(3, m.vocab, 1).astype(np.uint32)
    toks = np.asarray(m.generate(start, m.max_seq - 1), np.uint32)[:m.max_seq]
    try:
        assert L.llamini_set_prefill(0) == 0
        off = m.perplexity(toks)
        assert L.llamini_set_prefill(1) == 0
        on = m.perplexity(toks)
        short = m.perplexity(toks[:3])             # two positions: one partial chunk
    finally:
        L.llamini_set_prefill(-1)
    assert on > 0 and off > 0 and np.isfinite(on), (on, off, gpu.last_error())
    assert abs(on - off) / off < 1e-4, (on, off)
    o = orc.oracle_model(path, m.max_seq)
    nll = []
    for pos in range(len(toks) - 1):
        lg = o.forward(pos, int(toks[pos])).astype(np.float64)
        mx = lg.max()
        nll.append(-((lg[toks[pos + 1]] - mx) - np.log(np.exp(lg - mx).sum())))
    want = float(np.exp(np.mean(nll)))
    assert abs(on - want) / want < TOL, (on, want)
    want2 = float(np.exp(np.mean(nll[:2])))
    assert abs(short - want2) / want2 < TOL, (short, want2)


def test_perplexity_chunked_llama_1b(gpu, synth):
    """llama_1b, its greedy continuation of one seeded id, 300 positions (five
    chunks): the chunked path and the one-position-at-a-time path give the
    same perplexity."""
    m = gpu.Model(synth.ensure_workload("llama_1b"), max_seq=512)
    L = gpu.lib()
    toks = np.asarray(m.generate(synth.workload_prompt("llama_1b", 1), 299), np.uint32)
    try:
        assert L.llamini_set_prefill(0) == 0
        off = m.perplexity(toks)
        assert L.llamini_set_prefill(1) == 0
        on = m.perplexity(toks)
    finally:
        L.llamini_set_prefill(-1)
        m.close()
    assert on > 0 and off > 0 and np.isfinite(on), (on, off, gpu.last_error())
    assert abs(on - off) / off < 1e-4, (on, off)
