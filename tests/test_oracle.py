"""The oracle is pinned before it is trusted: its decoders and ops against the
golden fixtures produced by the reference's own code, and (where the reference
was compiled here) against that code directly on the small models."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import rel_l2, same_bits

TYPES = [2, 3, 6, 8, 12, 13, 14, 1]   # Q4_0 Q4_1 Q5_0 Q8_0 Q4_K Q5_K Q6_K F16


@pytest.mark.parametrize("t", TYPES)
def test_oracle_dequant_matches_golden(orc, golden, synth, t):
    raw = golden["dequant"]["raw_%d" % t]
    want = golden["dequant"]["out_%d" % t]
    got = orc.dequant(t, raw, want.size)
    assert same_bits(got, want)


def test_oracle_f16_all_values(orc, golden):
    # every half bit pattern against numpy's IEEE conversion (NaN payloads aside)
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = orc.dequant(1, h.view(np.uint8), 65536)
    assert same_bits(got, ref)


def test_oracle_kats(orc, golden):
    L = orc.oracle()
    k = golden["kat"]
    x = np.array([1, 2, 3, 4], np.float32)
    o = np.zeros(4, np.float32)
    w = np.ones(4, np.float32)                 # held for the call: ptr() keeps no reference
    L.orc_rms_norm(orc.ptr(o), orc.ptr(x), orc.ptr(w), 4, np.float32(1e-8))
    assert np.array_equal(o, np.array(k["rms_norm"], np.float32))
    for neox, key in ((0, "rope_norm"), (1, "rope_neox")):
        v = np.ones(8, np.float32)
        L.orc_rope(orc.ptr(v), 5, 8, 4, np.float32(10000.0), neox)
        np.testing.assert_allclose(v, np.array(k[key], np.float32), rtol=0, atol=2e-7)
    # main.c:505-514 prints 19 22 43 50 for [[1,2],[3,4]] x [[5,6],[7,8]]
    assert k["matmul_2x2"] == [19.0, 22.0, 43.0, 50.0]
    assert k["fake_generate"] == [1, 3, 4, 2, 0, 0, 0, 0]


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_mixed", "tiny_qwen2", "tiny_tied", "tiny_gpt2"])
def test_oracle_tokens_match_reference_golden(orc, tiny, golden, name):
    g = golden["tokens"][name]
    m = orc.oracle_model(tiny.ensure(name))
    got = m.generate(np.array(g["prompt"], np.uint32), 64)
    assert got.tolist() == g["tokens"]


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_mixed", "tiny_qwen2", "tiny_tied", "tiny_gpt2"])
def test_oracle_logits_match_reference_golden(orc, tiny, golden, name):
    g = golden["tokens"][name]
    m = orc.oracle_model(tiny.ensure(name))
    for pos, t in enumerate(g["prompt"][:4]):
        got = m.forward(pos, t)
        want = golden["logits"]["%s_%d" % (name, pos)]
        assert rel_l2(got, want) < 1e-5, (pos, rel_l2(got, want))


def test_oracle_vs_reference_build(orc, tiny):
    ref = orc.reference()
    if ref is None:
        pytest.skip("reference sources not compiled on this machine")
    rng = np.random.default_rng(5)
    for name in ("tiny_llama", "tiny_qwen2", "tiny_gpt2", "tiny_gemma", "tiny_tp"):
        path = tiny.ensure(name)
        m = orc.oracle_model(path)
        assert ref.drv_open(path.encode(), 0) == 0
        v = ref.drv_vocab()
        for pos in range(6):
            t = int(rng.integers(0, v))
            want = np.zeros(v, np.float32)
            ref.drv_forward(pos, t, orc.ptr(want))
            assert rel_l2(m.forward(pos, t), want) < 1e-5
        ref.drv_close()


@pytest.mark.parametrize("name,n_prompt", [("gpt2_124m", 64), ("llama_1b", 128)])
def test_oracle_workload_tokens_match_reference_golden(orc, synth, golden, name, n_prompt):
    """Full-size workloads: the oracle's greedy stream equals the reference's
    (first 64 generated tokens)."""
    if name not in golden["tokens"]:
        pytest.skip("golden stream not generated")
    g = golden["tokens"][name]
    prompt = synth.workload_prompt(name, n_prompt)
    assert prompt.tolist() == g["prompt"]
    m = orc.oracle_model(synth.ensure_workload(name))
    got = m.generate(prompt, 64)
    assert got.tolist() == g["tokens"]
