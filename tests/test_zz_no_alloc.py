"""llamini_causal_mha_noalloc: decode attention whose split partials live in a
fixed device array instead of a device allocation.

Compared with the existing entry causal_mha (model.h; the reference's
model.c:217-260 behaviour) and directly with the CPU oracle's causal_mha on the
same inputs, on calls made back to back, so a counter left non-zero or a stale
partial from the previous call would show up.
Collected last (file name) so it also runs after everything else in the suite.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2

TOL = 1e-5   # relative L2: both sides f32, different summation order


def _reference_entry(gpu, q, key, val, pos, nh, nkv, hd):
    """causal_mha over a host KVCache whose rows 0..pos-1 are key/val; row pos
    is passed as k/v (the function stores it, model.c:222-224)."""
    ms, kvd = key.shape
    kbuf = np.ascontiguousarray(key, np.float32).copy()
    vbuf = np.ascontiguousarray(val, np.float32).copy()
    kc = gpu.KVCache()
    kc.key = kbuf.ctypes.data_as(C.POINTER(C.c_float))
    kc.val = vbuf.ctypes.data_as(C.POINTER(C.c_float))
    kc.dim, kc.max_seq, kc.cur_seq = kvd, ms, pos
    out = np.zeros(nh * hd, np.float32)
    k = key[pos].copy()
    v = val[pos].copy()
    gpu.lib().causal_mha(gpu.ptr(q), gpu.ptr(k), gpu.ptr(v), C.byref(kc), gpu.ptr(out), pos, nh, nkv, hd)
    assert kc.cur_seq == pos + 1, gpu.last_error()
    return out


@pytest.mark.gpu
def test_noalloc_matches_causal_mha_on_consecutive_calls(gpu):
    import torch
    L = gpu.lib()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(11)
    stream = torch.cuda.current_stream(dev)
    cases = [(32, 8, 64, 1000),    # 16 position splits, GQA 4:1
             (32, 8, 64, 1500),    # 24 splits, same buffers
             (12, 12, 128, 37),    # one split: no partials
             (14, 2, 64, 4000)]    # 32 splits, GQA 7:1
    for nh, nkv, hd, pos in cases:
        ms = pos + 1
        q = rng.normal(0, 1, nh * hd).astype(np.float32)
        key = rng.normal(0, 1, (ms, nkv * hd)).astype(np.float32)
        val = rng.normal(0, 1, (ms, nkv * hd)).astype(np.float32)
        want = _reference_entry(gpu, q, key, val, pos, nh, nkv, hd)
        dq, dk, dv = (torch.from_numpy(a).to(dev) for a in (q, key, val))
        got = []
        for _ in range(2):     # two calls in a row on the same inputs
            dout = torch.full((nh * hd,), float("nan"), device=dev)
            rc = L.llamini_causal_mha_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dout.data_ptr(),
                                              pos, nh, nkv, hd, stream.cuda_stream)
            assert rc == 0, gpu.last_error()
            torch.cuda.synchronize(dev)
            got.append(dout.cpu().numpy())
        for g in got:
            assert np.isfinite(g).all()
            assert rel_l2(g, want) < TOL, (nh, nkv, hd, pos, rel_l2(g, want))
        # the merge runs in split order, so a repeat is bit-identical
        assert np.array_equal(got[0].view(np.uint32), got[1].view(np.uint32))


@pytest.mark.gpu
def test_noalloc_matches_oracle_including_reduced_split_counts(gpu, orc):
    """Directly against the CPU oracle's causal_mha (model.c:217-260), on shapes
    whose partials would overflow the fixed scratch at the natural split count,
    so the entry lowers the split count to fit: 64 heads of 128 at position
    3000 (31 splits instead of 32) and 256 heads of 256 at position 600 (3
    splits instead of 10), plus an ordinary 16-split case."""
    import torch
    L = gpu.lib()
    O = orc.oracle()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(12)
    stream = torch.cuda.current_stream(dev)
    for nh, nkv, hd, pos in [(64, 8, 128, 3000), (256, 16, 256, 600), (32, 8, 64, 1000)]:
        ms, kvd = pos + 1, nkv * hd
        q = rng.normal(0, 1, nh * hd).astype(np.float32)
        key = rng.normal(0, 1, (ms, kvd)).astype(np.float32)
        val = rng.normal(0, 1, (ms, kvd)).astype(np.float32)
        kc, vc = key.copy(), val.copy()
        k, v = key[pos].copy(), val[pos].copy()     # held: the oracle copies them into row pos
        want = np.zeros(nh * hd, np.float32)
        O.orc_causal_mha(orc.ptr(q), orc.ptr(k), orc.ptr(v), orc.ptr(kc), orc.ptr(vc), orc.ptr(want), pos, nh, nkv, hd)
        dq, dk, dv = (torch.from_numpy(a).to(dev) for a in (q, key, val))
        got = []
        for _ in range(2):
            dout = torch.full((nh * hd,), float("nan"), device=dev)
            rc = L.llamini_causal_mha_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dout.data_ptr(),
                                              pos, nh, nkv, hd, stream.cuda_stream)
            assert rc == 0, gpu.last_error()
            torch.cuda.synchronize(dev)
            got.append(dout.cpu().numpy())
        for g in got:
            assert np.isfinite(g).all()
            assert rel_l2(g, want) < TOL, (nh, nkv, hd, pos, rel_l2(g, want))
        assert np.array_equal(got[0].view(np.uint32), got[1].view(np.uint32))


@pytest.mark.gpu
def test_noalloc_rejects_sizes_beyond_its_scratch(gpu):
    import torch
    L = gpu.lib()
    dev = torch.device("cuda", 0)
    buf = torch.zeros(1 << 16, device=dev)
    p = buf.data_ptr()
    assert L.llamini_causal_mha_noalloc(p, p, p, p, 10, 512, 8, 64, None) == -1
    assert "scratch" in gpu.last_error()
    assert L.llamini_causal_mha_noalloc(p, p, p, p, 10, 8, 8, 512, None) == -1
    assert "scratch" in gpu.last_error()
    assert L.llamini_causal_mha_noalloc(p, p, p, p, 10, 6, 4, 64, None) == -1   # heads not a multiple of kv heads
    gpu.lib().llamini_clear_error()
