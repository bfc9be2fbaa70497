"""The C-ABI boundary without a GPU: the library loads, exports every function
declared in include/*.h, parses GGUF files on the host exactly like the
reference (including its hostile-file rejections, main.c:606-662), and fails
loudly -- never falls back to CPU -- when a compute call has no device."""
from __future__ import annotations

import ctypes as C
import os
import re
import struct
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    for h in os.listdir(os.path.join(ROOT, "include")):
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", text, flags=re.M):
            if not m.group(0).lstrip().startswith(("typedef", "#", "return")):
                names.add(m.group(1))
    return names


def test_exports_every_declared_function(lm):
    so = lm.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    declared = _declared_functions()
    assert len(declared) > 60
    missing = sorted(declared - exported)
    assert not missing, missing
    # and the Python binding covers exactly that set
    assert set(lm.SIGNATURES) == declared


def test_no_device_fails_loudly(lm):
    L = lm.lib()
    if L.llamini_device_count() > 0:
        pytest.skip("a GPU is present")
    x = np.ones(4, np.float32)
    out = np.full(4, 7.0, np.float32)
    assert L.llamini_dequant_host(12, lm.ptr(np.zeros(144, np.uint8)), 256, lm.ptr(np.zeros(256, np.float32))) == -1
    assert "no usable CUDA device" in lm.last_error()
    L.rms_norm(lm.ptr(out), lm.ptr(x), lm.ptr(x), 4, 1e-5)
    assert np.all(out == 7.0)          # untouched: no CPU fallback computed anything


def test_tp_join_argument_checks(lm):
    """Group membership is validated on the host: bad ranks fail with a
    message; a one-rank group needs no device."""
    L = lm.lib()
    assert L.llamini_tp_join(2, 2, None) == -1
    assert "rank 2 of 2" in lm.last_error()
    assert L.llamini_tp_join(0, 9, None) == -1
    assert L.llamini_tp_join(0, 0, None) == -1
    assert L.llamini_tp_join(0, 1, None) == 0
    assert L.llamini_tp_world() == 1 and L.llamini_tp_rank() == 0
    assert L.llamini_tp_leave() == 0                  # outside a group: nothing to leave, no device
    assert L.llamini_tp_world() == 1
    L.llamini_clear_error()


def _write(tmp_path, name, data: bytes) -> str:
    p = str(tmp_path / name)
    with open(p, "wb") as f:
        f.write(data)
    return p


def test_rejects_hostile_files(lm, tmp_path):
    """The three hostile files of main.c:606-662, plus truncation and version."""
    L = lm.lib()
    gf = lm.GGUFFile()
    bad_magic = b"XXXX" + b"\0" * 20
    huge = struct.pack("<IIQQ", 0x46554747, 3, 0x0000FFFFFFFFFFFF, 0)
    arr = struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + struct.pack("<Q", 1) + b"x" + \
        struct.pack("<IIQ", 9, 6, 1 << 62)
    v1 = struct.pack("<IIQQ", 0x46554747, 1, 0, 0)
    trunc = struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + struct.pack("<Q", 100) + b"ab"
    for i, data in enumerate((bad_magic, huge, arr, v1, trunc, b"")):
        assert L.gguf_open(_write(tmp_path, "bad%d.gguf" % i, data).encode(), C.byref(gf)) == -1
        if data:                      # parse failures reset the handle (gguf.c:224-230)
            assert gf.fd == -1 and not gf.data
    assert L.gguf_open(b"/nonexistent/file.gguf", C.byref(gf)) == -1


def test_parses_metadata_like_reference(lm, orc, tiny):
    """Metadata getters and tensor table agree with the reference build."""
    path = tiny.ensure("tiny_qwen2")
    L = lm.lib()
    gf = lm.GGUFFile()
    assert L.gguf_open(path.encode(), C.byref(gf)) == 0
    try:
        assert gf.hdr.version == 3 and gf.n_tensors == gf.hdr.n_tensors
        assert L.gguf_get_u32(C.byref(gf), b"qwen2.embedding_length", 0) == 192
        assert L.gguf_get_u32(C.byref(gf), b"missing.key", 77) == 77
        assert abs(L.gguf_get_f32(C.byref(gf), b"qwen2.rope.freq_base", 0.0) - 1e6) < 1
        assert L.gguf_meta_array_len(C.byref(gf), b"tokenizer.ggml.tokens", None) == 800
        cnt = C.c_uint64()
        arr = L.gguf_get_string_array(C.byref(gf), b"tokenizer.ggml.tokens", C.byref(cnt))
        assert cnt.value == 800
        strs = C.cast(arr, C.POINTER(C.c_char_p))
        assert strs[0] == b"<t0>" and strs[799] == b"<t799>"
        libc = C.CDLL(None)
        libc.free.argtypes = [C.c_void_p]
        for i in range(800):
            libc.free(C.cast(strs, C.POINTER(C.c_void_p))[i])
        libc.free(arr)
        ti = L.gguf_find_tensor(C.byref(gf), b"blk.1.attn_v.weight")
        assert ti and L.gguf_tensor_count(ti) == 192 * 64
        assert not L.gguf_find_tensor(C.byref(gf), b"nope")
        # unaligned row range is rejected before any device work (gguf.c:464)
        out = np.zeros(64, np.float32)
        assert L.gguf_dequantize_rows(C.byref(gf), ti, 0, 1, 33, lm.ptr(out)) == -1
        # F32 tensors are a plain copy and need no device
        tn = L.gguf_find_tensor(C.byref(gf), b"blk.0.attn_norm.weight")
        v = np.zeros(192, np.float32)
        assert L.gguf_dequantize_tensor(C.byref(gf), tn, lm.ptr(v), 192) == 0
        r = orc._synthetic().GGUFReader(path)
        assert np.array_equal(v, r.raw("blk.0.attn_norm.weight")[2].view(np.float32))
        # config from metadata (model.c:279-329)
        d = lm.LLaMAConfig(dim=1, n_layers=1, n_heads=1, n_heads_kv=1, ffn_dim=1, vocab_size=1, seq_len=4096,
                           rms_eps=1e-5, rope_freq_base=1e4)
        arch = C.c_char_p()
        c = L.llama_config_from_gguf(C.byref(gf), d, C.byref(arch))
        assert arch.value == b"qwen2"
        assert (c.dim, c.n_layers, c.n_heads, c.n_heads_kv, c.head_dim, c.ffn_dim, c.vocab_size) == \
            (192, 2, 6, 2, 32, 512, 800)
        assert c.rope_type == 1 and c.qkv_bias == 1 and c.seq_len == 128
        assert abs(c.rms_eps - 1e-6) < 1e-12
    finally:
        L.gguf_close(C.byref(gf))


def test_kv_cache_and_tensor_host_semantics(lm):
    L = lm.lib()
    kc = lm.KVCache()
    L.kv_cache_init(C.byref(kc), 512, 2048)      # main.c:533-541
    assert kc.dim == 512 and kc.max_seq == 2048 and kc.cur_seq == 0
    kc.cur_seq = 10
    L.kv_cache_reset(C.byref(kc))
    assert kc.cur_seq == 0
    libc = C.CDLL(None)
    libc.free.argtypes = [C.c_void_p]
    libc.free(C.cast(kc.key, C.c_void_p))
    libc.free(C.cast(kc.val, C.c_void_p))
    shape = (C.c_uint32 * 2)(3, 5)
    t = L.tensor_create(2, shape)
    assert t.contents.size == 15 and t.contents.data[14] == 0.0
    L.tensor_free(t)
