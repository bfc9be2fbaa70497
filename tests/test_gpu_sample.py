"""sample_token (generate.c:25-60) on the device.

The device sampler takes u = rand() / (RAND_MAX + 1) from the host, so with the
same srand seed it sees the reference's draws in the reference's order, and it
replays the reference's f32 sums over the sorted nucleus whenever the nucleus
fits its shared-memory candidate list (8192 entries): then every pick is the
reference's. A flatter distribution (top_p 1, or a nucleus past 8192) is
resolved in double precision instead, where a pick can differ from the
reference's only when the reference's f32 rounding moves a boundary past u.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LIBC = C.CDLL("libc.so.6")
LIBC.rand.restype = C.c_int
LIBC.srand.argtypes = [C.c_uint]


def _u(seed: int) -> np.float32:
    """The reference's draw after srand(seed): (f32)rand() / ((f32)RAND_MAX + 1.0f)."""
    LIBC.srand(seed)
    return np.float32(LIBC.rand()) / (np.float32(2147483647.0) + np.float32(1.0))


@pytest.mark.parametrize("vocab,temp,top_p,scale,exact", [(32000, 0.8, 0.9, 3.0, True), (32000, 1.0, 0.5, 2.0, True),
                                                          (151936, 0.7, 0.95, 3.0, True), (50257, 1.0, 0.0, 2.0, True),
                                                          (8, 0.5, 0.8, 1.0, True), (1000, 1.0, 1.0, 1.0, True),
                                                          (32000, 1.5, 1.0, 6.0, False)])
def test_sampler_matches_reference_draws(gpu, orc, vocab, temp, top_p, scale, exact):
    ref = orc.reference()
    if ref is None:
        pytest.skip("reference build not present (make -C oracle ref)")
    L = gpu.lib()
    rng = np.random.default_rng(vocab + int(temp * 10))
    same = 0
    n = 40
    for trial in range(n):
        logits = (rng.standard_normal(vocab) * scale).astype(np.float32)
        logits[rng.integers(0, vocab, 3)] += np.float32(4.0)       # a few strong candidates
        seed = 1000 + trial
        LIBC.srand(seed)
        want = ref.sample_token(orc.ptr(logits), vocab, temp, top_p)
        got = L.llamini_sample_host(gpu.ptr(logits), vocab, temp, top_p, float(_u(seed)))
        assert got != 0xFFFFFFFF, gpu.last_error()
        assert got < vocab
        same += int(got == want)
    # a nucleus of the whole 32000-entry vocabulary: the double-precision
    # path; the reference's f32 running sums drift by ~1e-4 of the mass over
    # that many terms, a few elements' worth, so some draws land elsewhere
    assert same == n if exact else same >= int(0.8 * n), (same, n)


def test_sampler_ties_keep_index_order(gpu, orc):
    """Equal probabilities keep index order (the reference's qsort is glibc's
    merge sort, which is stable): with every logit equal and u just above k / V
    the pick is index k."""
    L = gpu.lib()
    V = 1000
    logits = np.zeros(V, np.float32)
    for k in (0, 1, 17, 999):
        u = np.float32((k + 0.5) / V)
        assert L.llamini_sample_host(gpu.ptr(logits), V, 1.0, 1.0, float(u)) == k


def test_sampler_small_top_p_takes_the_argmax(gpu):
    L = gpu.lib()
    rng = np.random.default_rng(5)
    logits = rng.standard_normal(32000).astype(np.float32)
    for u in (0.0, 0.3, 0.999):
        assert L.llamini_sample_host(gpu.ptr(logits), 32000, 1.0, 1e-9, u) == int(np.argmax(logits))


@pytest.mark.parametrize("name", ["tiny_llama", "tiny_gpt2"])
def test_sampled_generate_matches_reference(gpu, orc, tiny, name):
    """generate_autoregressive with temp 0.9, top_p 0.9 from srand(7): the device
    path's stream equals the reference's."""
    ref = orc.reference()
    if ref is None:
        pytest.skip("reference build not present (make -C oracle ref)")
    path = tiny.ensure(name)
    prompt = np.random.default_rng(7).integers(3, 500, 16).astype(np.uint32)
    assert ref.drv_open(path.encode(), 0) == 0
    want = np.zeros(len(prompt) + 48 + 1, np.uint32)
    n = ref.drv_generate_sampled(orc.ptr(prompt), len(prompt), orc.ptr(want), 48, 0xFFFFFFFF, 0.9, 0.9, 7)
    ref.drv_close()
    m = gpu.Model(path, max_seq=128)
    try:
        LIBC.srand(7)
        got = m.generate(prompt, 48, temp=0.9, top_p=0.9)
    finally:
        m.close()
    assert got.tolist() == want[:n].tolist()
