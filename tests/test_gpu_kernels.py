"""Kernel-level parity on the GPU, through the C-ABI.

* block decoders: bit-identical to the reference (golden fixtures made by the
  reference's own gguf.c, plus fresh random blocks checked against the oracle);
* fused dequant-GEMV: y = W x within 1e-4 relative L2 of the oracle's f32
  decode-then-dot, over the GEMV sweep's shapes and every block format;
* the host-pointer ops of model.h / tensor.h / generate.h against the oracle
  and the reference's unit-test values.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2, same_bits

pytestmark = pytest.mark.gpu

QTYPES = [2, 3, 6, 8, 12, 13, 14]
ALL_TYPES = QTYPES + [1]
GEMV_TOL = 1e-4          # relative L2, fused GEMV vs f32 decode-then-dot


@pytest.mark.parametrize("t", ALL_TYPES)
def test_dequant_golden_bit_exact(gpu, golden, t):
    raw = golden["dequant"]["raw_%d" % t]
    want = golden["dequant"]["out_%d" % t]
    got = np.zeros(want.size, np.float32)
    assert gpu.lib().llamini_dequant_host(t, gpu.ptr(raw), want.size, gpu.ptr(got)) == 0, gpu.last_error()
    assert same_bits(got, want)


@pytest.mark.parametrize("t", QTYPES)
def test_dequant_random_vs_oracle(gpu, orc, synth, t):
    be, _ = synth.BLOCK[t]
    rng = np.random.default_rng(31 + t)
    n = be * 4099                                     # odd block count, > 1 grid wave
    raw = synth.random_blocks(rng, t, n)
    got = np.zeros(n, np.float32)
    assert gpu.lib().llamini_dequant_host(t, gpu.ptr(raw), n, gpu.ptr(got)) == 0, gpu.last_error()
    assert same_bits(got, orc.dequant(t, raw, n))


def test_dequant_rejects_misaligned_count(gpu):
    out = np.zeros(300, np.float32)
    assert gpu.lib().llamini_dequant_host(12, gpu.ptr(np.zeros(200, np.uint8)), 300, gpu.ptr(out)) == -1


@pytest.mark.parametrize("name,row_len,rows", [("blk.0.attn_q.weight", 2048, (0, 64)),         # Q4_K
                                               ("blk.1.ffn_down.weight", 5632, (32, 96)),     # Q4_K
                                               ("blk.0.ffn_down.weight", 5632, (2000, 2048)),  # Q6_K
                                               ("output.weight", 2048, (31936, 32000))])      # Q6_K
def test_gguf_dequantize_rows_workload_vs_reference(gpu, orc, synth, name, row_len, rows):
    """gguf_dequantize_rows (gguf.c:602-605) through the drop-in C-ABI on the
    llama_1b file's quantized tensors: bit-identical to the reference build's
    own gguf_dequantize_rows on the same file and rows."""
    ref = orc.reference()
    if ref is None:
        pytest.skip("reference build not present (make -C oracle ref)")
    path = synth.ensure_workload("llama_1b")
    L = gpu.lib()
    gf = gpu.GGUFFile()
    assert L.gguf_open(path.encode(), C.byref(gf)) == 0
    try:
        ti = L.gguf_find_tensor(C.byref(gf), name.encode())
        assert ti
        r0, r1 = rows
        got = np.full((r1 - r0) * row_len, np.nan, np.float32)
        assert L.gguf_dequantize_rows(C.byref(gf), ti, r0, r1, row_len, gpu.ptr(got)) == 0, gpu.last_error()
        assert ref.drv_open_file(path.encode()) == 0
        want = np.zeros_like(got)
        assert ref.drv_dequant_rows(name.encode(), r0, r1, row_len, orc.ptr(want)) == 0
        assert same_bits(got, want)
    finally:
        L.gguf_close(C.byref(gf))


def _orc_linear(orc, t, raw, rows, cols, x):
    m = orc.OrcMat(t, rows, cols, raw.ctypes.data)
    y = np.zeros(rows, np.float32)
    orc.oracle().orc_linear(C.byref(m), orc.ptr(x), orc.ptr(y))
    return y


SWEEP = [(2048, 2048), (5632, 2048), (2048, 5632), (32000, 2048), (11008, 4096), (4096, 11008)]


@pytest.mark.parametrize("t", QTYPES)
@pytest.mark.parametrize("shape", SWEEP)
def test_gemv_sweep_vs_oracle(gpu, orc, synth, t, shape):
    """The isolated GEMV sweep: every shape x every format, batch 1 (seed 1)."""
    rows, cols = shape
    rng = np.random.default_rng(1)
    raw = synth.random_blocks(rng, t, rows * cols)
    x = rng.normal(0, 1, cols).astype(np.float32)
    y = np.zeros(rows, np.float32)
    assert gpu.lib().llamini_gemv_host(t, gpu.ptr(raw), rows, cols, gpu.ptr(x), 1, gpu.ptr(y)) == 0, gpu.last_error()
    want = _orc_linear(orc, t, raw, rows, cols, x)
    assert rel_l2(y, want) < GEMV_TOL, rel_l2(y, want)


@pytest.mark.parametrize("t", QTYPES + [1])
@pytest.mark.parametrize("batch", [3, 8, 64])
def test_gemv_batch_columns(gpu, orc, synth, t, batch):
    """Batch columns (the config's 1, 8 and 64, plus a batch that is not a
    multiple of 4): every column within the GEMV tolerance of the oracle (every
    block format and F16 through the tensor-core GEMM)."""
    rows, cols = (2048, 2048) if batch != 64 else (1000, 2048)
    rng = np.random.default_rng(1)
    raw = synth.random_blocks(rng, t, rows * cols) if t != 1 else \
        rng.normal(0, 0.05, rows * cols).astype(np.float16).view(np.uint8)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    y = np.full((batch, rows), np.nan, np.float32)
    assert gpu.lib().llamini_gemv_host(t, gpu.ptr(raw), rows, cols, gpu.ptr(x), batch, gpu.ptr(y)) == 0, gpu.last_error()
    for b in range(batch):
        assert rel_l2(y[b], _orc_linear(orc, t, raw, rows, cols, x[b])) < GEMV_TOL, (b, rel_l2(y[b], _orc_linear(orc, t, raw, rows, cols, x[b])))


@pytest.mark.parametrize("t", [12, 14, 8])
def test_gemv_batch_wide(gpu, orc, synth, t):
    """Batch 64 on the down-projection shape (K = 5632, split over CTAs)."""
    rows, cols, batch = 2048, 5632, 64
    rng = np.random.default_rng(2)
    raw = synth.random_blocks(rng, t, rows * cols)
    x = rng.normal(0, 1, (batch, cols)).astype(np.float32)
    y = np.full((batch, rows), np.nan, np.float32)
    assert gpu.lib().llamini_gemv_host(t, gpu.ptr(raw), rows, cols, gpu.ptr(x), batch, gpu.ptr(y)) == 0, gpu.last_error()
    for b in (0, 17, 63):
        assert rel_l2(y[b], _orc_linear(orc, t, raw, rows, cols, x[b])) < GEMV_TOL


@pytest.mark.parametrize("t", [0, 1])
def test_gemv_float_rows_odd_width(gpu, t):
    """F32/F16 rows of a width that is not a multiple of 32 (the eager path of
    the reference's fake model has rows of 16)."""
    rng = np.random.default_rng(3)
    rows, cols = 37, 16
    w = rng.normal(0, 1, (rows, cols)).astype(np.float32 if t == 0 else np.float16)
    x = rng.normal(0, 1, cols).astype(np.float32)
    y = np.zeros(rows, np.float32)
    assert gpu.lib().llamini_gemv_host(t, gpu.ptr(w), rows, cols, gpu.ptr(x), 1, gpu.ptr(y)) == 0
    np.testing.assert_allclose(y, w.astype(np.float32) @ x, rtol=1e-5, atol=1e-5)


# ---------------------------------------------------------------- host-pointer ops

def test_ops_reference_kats(gpu, golden):
    L, k = gpu.lib(), golden["kat"]
    x = np.array([1, 2, 3, 4], np.float32)
    o = np.zeros(4, np.float32)
    w = np.ones(4, np.float32)                 # held for the call: ptr() keeps no reference
    L.rms_norm(gpu.ptr(o), gpu.ptr(x), gpu.ptr(w), 4, 1e-8)
    np.testing.assert_allclose(o, k["rms_norm"], rtol=1e-6)
    for neox, key in ((0, "rope_norm"), (1, "rope_neox")):
        v = np.ones(8, np.float32)
        L.rope(gpu.ptr(v), 5, 8, 4, 10000.0, neox)
        np.testing.assert_allclose(v, k[key], rtol=0, atol=1e-6)
    s = (C.c_uint32 * 2)(2, 2)
    A, B, Cm = L.tensor_create(2, s), L.tensor_create(2, s), L.tensor_create(2, s)
    for i, v in enumerate((1, 2, 3, 4)):
        A.contents.data[i] = v
    for i, v in enumerate((5, 6, 7, 8)):
        B.contents.data[i] = v
    L.matmul(A, B, Cm)
    assert [Cm.contents.data[i] for i in range(4)] == k["matmul_2x2"]
    for t in (A, B, Cm):
        L.tensor_free(t)


def test_ops_vs_oracle(gpu, orc):
    L, O = gpu.lib(), orc.oracle()
    rng = np.random.default_rng(9)
    n = 5632
    g, u = rng.normal(0, 3, n).astype(np.float32), rng.normal(0, 1, n).astype(np.float32)
    for gelu in (0, 1):
        a, b = np.zeros(n, np.float32), np.zeros(n, np.float32)
        L.ffn_glu(gpu.ptr(a), gpu.ptr(g), gpu.ptr(u), n, gelu)
        O.orc_ffn_glu(orc.ptr(b), orc.ptr(g), orc.ptr(u), n, gelu)
        np.testing.assert_allclose(a, b, rtol=2e-6, atol=1e-6)
    x = rng.normal(0, 5, 2048).astype(np.float32)
    w = (1 + rng.normal(0, .05, 2048)).astype(np.float32)
    a, b = np.zeros(2048, np.float32), np.zeros(2048, np.float32)
    L.rms_norm(gpu.ptr(a), gpu.ptr(x), gpu.ptr(w), 2048, 1e-5)
    O.orc_rms_norm(orc.ptr(b), orc.ptr(x), orc.ptr(w), 2048, np.float32(1e-5))
    np.testing.assert_allclose(a, b, rtol=1e-5)
    for neox in (0, 1):
        for pos in (0, 1, 383, 2047):
            v1 = rng.normal(0, 1, 2048).astype(np.float32)
            v2 = v1.copy()
            L.rope(gpu.ptr(v1), pos, 2048, 64, 10000.0, neox)
            O.orc_rope(orc.ptr(v2), pos, 2048, 64, np.float32(10000.0), neox)
            np.testing.assert_allclose(v1, v2, rtol=0, atol=2e-5 * max(1, pos / 100))
    # greedy: first strict maximum, NaN and -0 rules of generate.c:3-9
    z = np.array([-0.0, 0.0, -1.0], np.float32)
    assert L.greedy_sample(gpu.ptr(z), 3) == 0
    z = np.array([np.nan, 5.0, 1.0], np.float32)
    assert L.greedy_sample(gpu.ptr(z), 3) == 0
    z = np.array([1.0, np.nan, 7.0, 7.0], np.float32)
    assert L.greedy_sample(gpu.ptr(z), 4) == 2
    lg = rng.normal(0, 1, 32000).astype(np.float32)
    lg[[100, 20000]] = 9.0
    assert L.greedy_sample(gpu.ptr(lg), 32000) == 100


def test_causal_mha_host_cache_vs_oracle(gpu, orc):
    """causal_mha over the caller's f32 cache, positions 0..pos, GQA 8:2."""
    L, O = gpu.lib(), orc.oracle()
    rng = np.random.default_rng(4)
    nh, nkv, hd, ms = 8, 2, 64, 64
    kc = gpu.KVCache()
    L.kv_cache_init(C.byref(kc), nkv * hd, ms)
    okc = np.zeros((ms, nkv * hd), np.float32)
    ovc = np.zeros((ms, nkv * hd), np.float32)
    for pos in range(20):
        q = rng.normal(0, 1, nh * hd).astype(np.float32)
        k = rng.normal(0, 1, nkv * hd).astype(np.float32)
        v = rng.normal(0, 1, nkv * hd).astype(np.float32)
        a, b = np.zeros(nh * hd, np.float32), np.zeros(nh * hd, np.float32)
        L.causal_mha(gpu.ptr(q), gpu.ptr(k), gpu.ptr(v), C.byref(kc), gpu.ptr(a), pos, nh, nkv, hd)
        O.orc_causal_mha(orc.ptr(q), orc.ptr(k), orc.ptr(v), orc.ptr(okc), orc.ptr(ovc), orc.ptr(b), pos, nh, nkv, hd)
        assert kc.cur_seq == pos + 1
        np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-5)
    libc = C.CDLL(None)
    libc.free.argtypes = [C.c_void_p]
    libc.free(C.cast(kc.key, C.c_void_p))
    libc.free(C.cast(kc.val, C.c_void_p))
