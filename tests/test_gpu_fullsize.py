"""Full-size parity for the Qwen2-0.5B and LLaMA-7B-shape workloads.

* qwen2_05b (24 layers, dim 896, 14/2 heads, ffn 4864, vocab 151936, q/k/v
  biases, a Q5_0 attn_v in the Q4_K_M mix): after its 512-token prompt the
  first 64 greedy tokens equal the reference's own generate_autoregressive
  (tests/golden/tokens.json, made by tests/golden/make_golden.py
  --full-size-only from the reference's C).
* llama_7b (32 layers, dim 4096, 32 heads, ffn 11008): the same after a
  64-token prompt.
* For the first positions of each, the logits and every layer's residual
  stream are within 1e-3 relative L2 of the CPU oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3
_models = {}


def _model(gpu, path):
    if path not in _models:
        _models[path] = gpu.Model(path, max_seq=1024)
    return _models[path]


@pytest.mark.parametrize("name", ["qwen2_05b", "llama_7b"])
def test_fullsize_tokens_equal_reference(gpu, synth, golden, name):
    if name not in golden["tokens"]:
        pytest.skip("golden stream not generated (make_golden.py --full-size-only)")
    g = golden["tokens"][name]
    m = _model(gpu, synth.ensure_workload(name))
    got = m.generate(np.array(g["prompt"], np.uint32), len(g["tokens"]) - len(g["prompt"]))
    assert got.tolist() == g["tokens"]


@pytest.mark.parametrize("name,n_pos", [("qwen2_05b", 2), ("llama_7b", 1)])
def test_fullsize_logits_and_layers_vs_oracle(gpu, orc, synth, name, n_pos):
    path = synth.ensure_workload(name)
    m = _model(gpu, path)
    o = orc.oracle_model(path)
    L = gpu.lib()
    s = m.session()
    L.llamini_session_trace(s, 1)
    try:
        for pos, t in enumerate(synth.workload_prompt(name, n_pos)):
            got = m.forward(pos, int(t))
            tr = np.zeros((m.n_layers, m.dim), np.float32)
            assert L.llamini_session_trace_read(s, gpu.ptr(tr)) == 0
            want, want_tr = o.forward(pos, int(t), trace=True)
            assert rel_l2(got, want) < TOL, (pos, rel_l2(got, want))
            worst = max(rel_l2(tr[l], want_tr[l]) for l in range(m.n_layers))
            assert worst < TOL, (pos, worst)
    finally:
        L.llamini_session_trace(s, 0)
