"""Whole-model parity on the GPU through the reference API.

For every small model (all formats, GQA, NORM/NEOX RoPE, biases, tied head,
GPT-2) and for the full-size LLaMA-1.1B and GPT-2-124M workloads:

* the greedy token stream equals the reference's (golden fixtures produced by
  the reference's own generate_autoregressive / gpt2_generate);
* the logits and the per-layer residual stream are within 1e-3 relative L2 of
  the CPU oracle on the same inputs;
* perplexity matches a teacher-forced evaluation of the oracle's logits.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3          # relative L2, activations and logits vs the oracle
TINY = ["tiny_llama", "tiny_mixed", "tiny_qwen2", "tiny_tied", "tiny_gpt2"]

_models = {}


def _model(gpu, path):
    if path not in _models:
        _models[path] = gpu.Model(path)
    return _models[path]


@pytest.mark.parametrize("name", TINY)
def test_tiny_tokens_equal_reference(gpu, tiny, golden, name):
    g = golden["tokens"][name]
    m = _model(gpu, tiny.ensure(name))
    got = m.generate(np.array(g["prompt"], np.uint32), 64)
    assert got.tolist() == g["tokens"], gpu.last_error()
    assert m.caches[0].cur_seq == len(g["tokens"]) - 1      # positions run, like the reference


@pytest.mark.parametrize("name", TINY)
def test_tiny_logits_and_layers_vs_oracle(gpu, orc, tiny, golden, name):
    path = tiny.ensure(name)
    m = _model(gpu, path)
    o = orc.oracle_model(path)
    s = m.session()
    L = gpu.lib()
    L.llamini_session_trace(s, 1)
    try:
        prompt = golden["tokens"][name]["prompt"]
        for pos, t in enumerate(prompt[:12]):
            got = m.forward(pos, t)
            tr = np.zeros((m.n_layers, m.dim), np.float32)
            assert L.llamini_session_trace_read(s, gpu.ptr(tr)) == 0
            want, want_tr = o.forward(pos, t, trace=True)
            assert rel_l2(got, want) < TOL, (pos, rel_l2(got, want))
            for l in range(m.n_layers):
                assert rel_l2(tr[l], want_tr[l]) < TOL, (pos, l, rel_l2(tr[l], want_tr[l]))
            if pos < 4:   # and directly against the reference's own logits
                ref = golden["logits"]["%s_%d" % (name, pos)]
                assert rel_l2(got, ref) < TOL
    finally:
        L.llamini_session_trace(s, 0)


@pytest.mark.parametrize("name", ["tiny_mixed", "tiny_gpt2", "tiny_llama"])
def test_tiny_perplexity(gpu, orc, tiny, name):
    path = tiny.ensure(name)
    m = _model(gpu, path)
    o = orc.oracle_model(path)
    toks = np.random.default_rng(8).integers(0, 500, 40).astype(np.uint32)
    ppl = m.perplexity(toks)
    nll = []
    for pos in range(len(toks) - 1):
        lg = o.forward(pos, int(toks[pos])).astype(np.float64)
        mx = lg.max()
        nll.append(-((lg[toks[pos + 1]] - mx) - np.log(np.exp(lg - mx).sum())))
    mean = float(np.mean(nll))
    if mean > 88.0:          # exp overflows f32: the reference's expf returns inf too
        assert ppl == float("inf")
    else:
        want = float(np.exp(mean))
        assert abs(ppl - want) / want < 1e-3, (ppl, want)
    assert m.perplexity(toks[:1]) == -1.0


def test_forward_step_matches_session_decode(gpu, tiny, golden):
    """forward_step's host logits and the device-resident loop agree."""
    m = _model(gpu, tiny.ensure("tiny_llama"))
    g = golden["tokens"]["tiny_llama"]
    toks = g["tokens"]
    L = gpu.lib()
    s = m.session()
    p = np.array(toks[:16], np.uint32)
    assert L.llamini_session_begin(s, gpu.ptr(p), 16) == 0
    assert L.llamini_session_step(s, 40) == 0
    out = np.zeros(64, np.uint32)
    n = L.llamini_session_tokens(s, gpu.ptr(out), 64)
    assert n == 41                       # 16 prompt tokens + 25 generated after 40 steps
    assert out[:n].tolist() == toks[:n]


def test_capacity_limit(gpu, tiny):
    m = _model(gpu, tiny.ensure("tiny_gpt2"))           # ctx 64
    s = m.session()
    L = gpu.lib()
    p = np.array([1, 2, 3], np.uint32)
    assert L.llamini_session_begin(s, gpu.ptr(p), 3) == 0
    assert L.llamini_session_step(s, 65) == -1
    assert "capacity" in gpu.last_error()
    gpu.lib().llamini_clear_error()


def test_reference_fake_model_tokens(gpu, orc, golden):
    """main.c:552-596's eager-f32 fake model through the unchanged caller code
    (ref_driver.c compiled against include/ and this library)."""
    d = orc.dropin()
    if d is None:
        pytest.skip("drop-in driver not built (make -C oracle dropin)")
    out = np.zeros(8, np.uint32)
    n = d.drv_fake_generate(orc.ptr(out))
    assert out[:n].tolist() == golden["kat"]["fake_generate"]


def test_reference_main_selftest(gpu, orc):
    """The reference's own main.c (--test) linked to this library."""
    exe = os.path.join(os.path.dirname(orc.__file__), "_ref", "llamini_b200")
    if not os.path.exists(exe):
        pytest.skip("drop-in main not built")
    import subprocess
    r = subprocess.run([exe, "--test"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert "1 3 4 2 0 0 0 0" in r.stdout
    assert "all malformed files correctly rejected" in r.stdout


@pytest.mark.parametrize("name,n_prompt", [("gpt2_124m", 64), ("llama_1b", 128)])
def test_workload_tokens_equal_reference(gpu, synth, golden, name, n_prompt):
    """Full-size workloads: the first 64 greedy tokens equal the reference's."""
    if name not in golden["tokens"]:
        pytest.skip("golden stream not generated")
    g = golden["tokens"][name]
    m = _model(gpu, synth.ensure_workload(name))
    got = m.generate(np.array(g["prompt"], np.uint32), 64)
    assert got.tolist() == g["tokens"]


@pytest.mark.parametrize("name", ["llama_1b", "gpt2_124m"])
def test_workload_logits_and_layers_vs_oracle(gpu, orc, synth, name):
    path = synth.ensure_workload(name)
    m = _model(gpu, path)
    o = orc.oracle_model(path)
    L = gpu.lib()
    s = m.session()
    L.llamini_session_trace(s, 1)
    try:
        prompt = synth.workload_prompt(name, 6)
        for pos, t in enumerate(prompt):
            got = m.forward(pos, int(t))
            tr = np.zeros((m.n_layers, m.dim), np.float32)
            assert L.llamini_session_trace_read(s, gpu.ptr(tr)) == 0
            want, want_tr = o.forward(pos, int(t), trace=True)
            assert rel_l2(got, want) < TOL, (pos, rel_l2(got, want))
            worst = max(rel_l2(tr[l], want_tr[l]) for l in range(m.n_layers))
            assert worst < TOL, (pos, worst)
    finally:
        L.llamini_session_trace(s, 0)
