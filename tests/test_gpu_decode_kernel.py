"""The persistent decode kernel (k_decode.cu) against the per-op graph path.

Both paths compute every matrix tile, norm, attention split and merge with the
same arithmetic in the same order, so the greedy tokens, the logits and the
per-layer residual stream must be bit-identical -- not just within the 1e-3
bar the oracle comparisons use. A session uses the decode kernel when it is
created with LLAMINI_DECODE_KERNEL=1 and the per-op graphs with =0.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from conftest import same_bits

pytestmark = pytest.mark.gpu


def _session_with(gpu, path, flag):
    old = os.environ.get("LLAMINI_DECODE_KERNEL")
    os.environ["LLAMINI_DECODE_KERNEL"] = flag
    try:
        m = gpu.Model(path)
        m.session()
    finally:
        if old is None:
            del os.environ["LLAMINI_DECODE_KERNEL"]
        else:
            os.environ["LLAMINI_DECODE_KERNEL"] = old
    return m


def _pair(gpu, path):
    """Two independent loads of one file: decode kernel, then per-op graphs."""
    a = _session_with(gpu, path, "1")
    b = _session_with(gpu, path, "0")
    L = gpu.lib()
    assert L.llamini_session_kernel(a.session()) == 1, gpu.last_error()
    assert L.llamini_session_kernel(b.session()) == 0
    return a, b


def _trace_run(gpu, m, prompt, n):
    L = gpu.lib()
    s = m.session()
    L.llamini_session_trace(s, 1)
    out = []
    try:
        for pos, t in enumerate(prompt[:n]):
            lg = m.forward(pos, int(t))
            tr = np.zeros((m.n_layers, m.dim), np.float32)
            assert L.llamini_session_trace_read(s, gpu.ptr(tr)) == 0
            out.append((lg, tr))
    finally:
        L.llamini_session_trace(s, 0)
    return out


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_tied"])
def test_decode_kernel_bit_identical_to_per_op_path(gpu, tiny, golden, name):
    a, b = _pair(gpu, tiny.ensure(name))
    try:
        g = golden["tokens"][name]
        prompt = np.array(g["prompt"], np.uint32)
        # 64 generated tokens after the prompt: two launches of the decode
        # kernel (64 steps each at most), so the step counters carry over
        ta = a.generate(prompt, 64)
        tb = b.generate(prompt, 64)
        assert ta.tolist() == g["tokens"], gpu.last_error()
        assert tb.tolist() == g["tokens"]
        for (la, ra), (lb, rb) in zip(_trace_run(gpu, a, g["tokens"], 12), _trace_run(gpu, b, g["tokens"], 12)):
            assert same_bits(la, lb)
            assert same_bits(ra, rb)
    finally:
        a.close()
        b.close()


def test_decode_kernel_workload_bit_identical(gpu, synth, golden):
    """llama_1b (22 layers, Q4_K_M mix): the first 16 steps' logits and
    residuals, then 48 greedy tokens, identical on both paths."""
    a, b = _pair(gpu, synth.ensure_workload("llama_1b"))
    try:
        g = golden["tokens"]["llama_1b"]
        for (la, ra), (lb, rb) in zip(_trace_run(gpu, a, g["tokens"], 16), _trace_run(gpu, b, g["tokens"], 16)):
            assert same_bits(la, lb)
            assert same_bits(ra, rb)
        prompt = np.array(g["prompt"], np.uint32)
        ta = a.generate(prompt, 48)
        tb = b.generate(prompt, 48)
        assert ta.tolist() == tb.tolist() == g["tokens"][:len(ta)], gpu.last_error()
    finally:
        a.close()
        b.close()


def test_decode_kernel_fp16_cache_matches_per_op_path(gpu, tiny, golden):
    """fp16 KV cache: same bits on both paths as well."""
    L = gpu.lib()
    L.llamini_set_kv_f16(1)
    try:
        a, b = _pair(gpu, tiny.ensure("tiny_llama"))
    finally:
        L.llamini_set_kv_f16(0)
    try:
        prompt = np.array(golden["tokens"]["tiny_llama"]["prompt"], np.uint32)
        ta = a.generate(prompt, 40)
        tb = b.generate(prompt, 40)
        assert ta.tolist() == tb.tolist()
        for (la, ra), (lb, rb) in zip(_trace_run(gpu, a, ta, 10), _trace_run(gpu, b, tb, 10)):
            assert same_bits(la, lb)
            assert same_bits(ra, rb)
    finally:
        a.close()
        b.close()
