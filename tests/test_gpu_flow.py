"""The dataflow decode kernel (k_flow.cu), the default batch-1 step path of
LLaMA-family models whose matrices are Q4_K / Q6_K.

It computes every dot product with the per-op path's exact integer x fp16-pair
products but scales each 16-element group of the input by its own power of two
and applies RMSNorm's 1/rms after the dot product, so it is held to the oracle
(the reference's algorithm) at the 1e-3 relative-L2 bar, with greedy tokens
identical to the reference's own streams, not to the per-op path's bits.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _model_with(gpu, path, flag):
    old = os.environ.get("LLAMINI_DECODE_KERNEL")
    if flag is None:
        os.environ.pop("LLAMINI_DECODE_KERNEL", None)
    else:
        os.environ["LLAMINI_DECODE_KERNEL"] = flag
    try:
        m = gpu.Model(path)
        m.session()
    finally:
        if old is None:
            os.environ.pop("LLAMINI_DECODE_KERNEL", None)
        else:
            os.environ["LLAMINI_DECODE_KERNEL"] = old
    return m


@pytest.mark.parametrize("name,kind", [("tiny_llama", 2), ("tiny_tied", 2), ("tiny_gemma", 2), ("tiny_tp", 2),
                                       ("tiny_mixed", 0), ("tiny_qwen2", 0), ("tiny_gpt2", 0)])
def test_flow_kernel_selection(gpu, tiny, name, kind):
    m = _model_with(gpu, tiny.ensure(name), None)
    try:
        assert gpu.lib().llamini_session_kernel(m.session()) == kind, gpu.last_error()
    finally:
        m.close()


def test_flow_kernel_switch_off(gpu, tiny):
    a = _model_with(gpu, tiny.ensure("tiny_llama"), "0")
    b = _model_with(gpu, tiny.ensure("tiny_llama"), "1")
    try:
        assert gpu.lib().llamini_session_kernel(a.session()) == 0
        assert gpu.lib().llamini_session_kernel(b.session()) == 1
    finally:
        a.close()
        b.close()


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_tied", "tiny_gemma", "tiny_tp"])
def test_flow_logits_and_layers_vs_oracle(gpu, orc, tiny, golden, name):
    path = tiny.ensure(name)
    m = _model_with(gpu, path, None)
    o = orc.oracle_model(path)
    L = gpu.lib()
    s = m.session()
    assert L.llamini_session_kernel(s) == 2
    L.llamini_session_trace(s, 1)
    try:
        toks = golden["tokens"][name]["tokens"] if name in golden["tokens"] else list(range(3, 40))
        for pos, t in enumerate(toks[:16]):
            got = m.forward(pos, int(t))
            tr = np.zeros((m.n_layers, m.dim), np.float32)
            assert L.llamini_session_trace_read(s, gpu.ptr(tr)) == 0
            want, want_tr = o.forward(pos, int(t), trace=True)
            assert rel_l2(got, want) < TOL, (pos, rel_l2(got, want), gpu.last_error())
            for l in range(m.n_layers):
                assert rel_l2(tr[l], want_tr[l]) < TOL, (pos, l, rel_l2(tr[l], want_tr[l]))
    finally:
        L.llamini_session_trace(s, 0)
        m.close()


@pytest.mark.parametrize("name,n_gen", [("tiny_llama", 100), ("tiny_tp", 100), ("tiny_tied", 50), ("tiny_gemma", 50)])
def test_flow_long_stream_equals_oracle(gpu, orc, tiny, name, n_gen):
    """Greedy tokens after an 8-token prompt; 100 tokens take two kernel
    launches of up to 64 steps each, the step counters carried across them."""
    path = tiny.ensure(name)
    m = _model_with(gpu, path, None)
    try:
        assert gpu.lib().llamini_session_kernel(m.session()) == 2
        prompt = np.arange(3, 11, dtype=np.uint32)
        got = m.generate(prompt, n_gen)
        want = orc.oracle_model(path).generate(prompt, n_gen)
        assert got.tolist() == want.tolist(), gpu.last_error()
    finally:
        m.close()


def test_flow_deterministic(gpu, tiny):
    """Two sessions of one file: bit-identical logits (fixed reduction orders)."""
    path = tiny.ensure("tiny_llama")
    a = _model_with(gpu, path, None)
    b = _model_with(gpu, path, None)
    try:
        for pos, t in enumerate([5, 9, 400, 17, 3, 3, 200]):
            la, lb = a.forward(pos, t), b.forward(pos, t)
            assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)), pos
    finally:
        a.close()
        b.close()


def test_flow_fp16_cache_vs_oracle(gpu, orc, tiny):
    """fp16 KV cache on the flow kernel: logits near the f32 oracle (the
    cache's own rounding, ~2e-3, dominates)."""
    L = gpu.lib()
    L.llamini_set_kv_f16(1)
    try:
        path = tiny.ensure("tiny_llama")
        m = _model_with(gpu, path, None)
    finally:
        L.llamini_set_kv_f16(0)
    o = orc.oracle_model(path)
    try:
        assert L.llamini_session_kernel(m.session()) == 2
        for pos, t in enumerate([5, 9, 400, 17, 3, 3, 200, 11, 12]):
            got = m.forward(pos, t)
            want = o.forward(pos, t)
            assert rel_l2(got, want) < 1e-2, (pos, rel_l2(got, want))
    finally:
        m.close()


def test_flow_workload_tokens_and_logits(gpu, orc, synth, golden):
    """llama_1b: the first 64 greedy tokens equal the reference's golden stream
    (128-token prompt, chunked prefill, then the flow kernel), and the first
    positions' logits and residual stream are within 1e-3 of the oracle."""
    g = golden["tokens"]["llama_1b"]
    path = synth.ensure_workload("llama_1b")
    m = _model_with(gpu, path, None)
    try:
        assert gpu.lib().llamini_session_kernel(m.session()) == 2
        got = m.generate(np.array(g["prompt"], np.uint32), 64)
        assert got.tolist() == g["tokens"], gpu.last_error()
        o = orc.oracle_model(path)
        L = gpu.lib()
        s = m.session()
        L.llamini_session_trace(s, 1)
        try:
            for pos, t in enumerate(synth.workload_prompt("llama_1b", 4)):
                lg = m.forward(pos, int(t))
                tr = np.zeros((m.n_layers, m.dim), np.float32)
                assert L.llamini_session_trace_read(s, gpu.ptr(tr)) == 0
                want, want_tr = o.forward(pos, int(t), trace=True)
                assert rel_l2(lg, want) < TOL, (pos, rel_l2(lg, want))
                worst = max(rel_l2(tr[l], want_tr[l]) for l in range(m.n_layers))
                assert worst < TOL, (pos, worst)
        finally:
            L.llamini_session_trace(s, 0)
    finally:
        m.close()
