"""Tensor parallelism (llamini_tp_*): a LLaMA model split over two GPUs, one
process per GPU (heads and FFN columns sharded, embeddings / norms / lm_head
whole, the o-projection and ffn_down sums added across ranks over NVLink).

Both ranks must reproduce the oracle's greedy stream, and their logits must be
bit-identical to each other (every rank adds the ranks' partial sums in rank
order) and within the 1e-3 bar of the oracle's forward pass.
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

from conftest import ROOT, rel_l2

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, path, prompt, n_gen, q):
    import datetime
    import importlib.util
    import torch.distributed as dist
    import torch
    spec = importlib.util.spec_from_file_location("llamini_b200", os.path.join(ROOT, "llamini.cpp_b200", "__init__.py"))
    lm = importlib.util.module_from_spec(spec)
    sys.modules["llamini_b200"] = lm
    spec.loader.exec_module(lm)
    L = lm.lib()
    try:
        assert L.llamini_set_device(rank) == 0, lm.last_error()
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        h = np.zeros(64, np.uint8)
        assert L.llamini_tp_handle(lm.ptr(h)) == 0, lm.last_error()
        mine = torch.from_numpy(h)
        hs = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(hs, mine)
        allh = np.ascontiguousarray(np.concatenate([x.numpy() for x in hs]))
        assert L.llamini_tp_join(rank, world, lm.ptr(allh)) == 0, lm.last_error()
        assert L.llamini_tp_world() == world and L.llamini_tp_rank() == rank
        m = lm.Model(path)
        toks = m.generate(np.array(prompt, np.uint32), n_gen).tolist()
        lgs = np.stack([m.forward(p, int(toks[p])) for p in range(6)])
        err = lm.last_error()
        m.close()
        dist.barrier()
        q.put((rank, toks, lgs, err))
        dist.destroy_process_group()
    except Exception as e:                            # report, then leave: the parent fails the test
        q.put((rank, None, None, repr(e)))


def test_tp_two_ranks_match_oracle(orc, tiny):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    path = tiny.ensure("tiny_tp")
    rng = np.random.default_rng(21)
    prompt = rng.integers(3, 1000, 7).tolist()
    n_gen = 24
    # the oracle's greedy stream and logits (CPU)
    o = orc.oracle_model(path)
    toks = list(prompt)
    want = []
    for pos in range(len(prompt) + n_gen - 1):
        lg = o.forward(pos, toks[pos])
        if pos < 6:
            want.append(lg)
        if pos + 1 >= len(prompt):
            toks.append(int(np.argmax(lg)))
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, 2, port, path, prompt, n_gen, qq)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((qq.get(timeout=600) for _ in ps), key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    for rank, got, lgs, err in res:
        assert got is not None, (rank, err)
        assert got == toks, (rank, got, toks, err)
        for pos in range(6):
            assert rel_l2(lgs[pos], want[pos]) < TOL, (rank, pos, rel_l2(lgs[pos], want[pos]))
    assert np.array_equal(res[0][2].view(np.uint32), res[1][2].view(np.uint32))


def _rank_batch(rank, world, port, path, long_prompt, n_gen, prompts, steps, q):
    """One rank: a long-prompt generate (chunked prefill with the wide
    allreduce) and a batch of ragged prompts (prefill chunks, then lockstep
    steps) in the tensor-parallel group."""
    import datetime
    import importlib.util
    import ctypes as C
    import torch.distributed as dist
    import torch
    spec = importlib.util.spec_from_file_location("llamini_b200", os.path.join(ROOT, "llamini.cpp_b200", "__init__.py"))
    lm = importlib.util.module_from_spec(spec)
    sys.modules["llamini_b200"] = lm
    spec.loader.exec_module(lm)
    L = lm.lib()
    try:
        assert L.llamini_set_device(rank) == 0, lm.last_error()
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        h = np.zeros(64, np.uint8)
        assert L.llamini_tp_handle(lm.ptr(h)) == 0, lm.last_error()
        mine = torch.from_numpy(h)
        hs = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(hs, mine)
        allh = np.ascontiguousarray(np.concatenate([x.numpy() for x in hs]))
        assert L.llamini_tp_join(rank, world, lm.ptr(allh)) == 0, lm.last_error()
        m = lm.Model(path)
        long_toks = m.generate(np.array(long_prompt, np.uint32), n_gen).tolist()
        b = L.llamini_llama_batch(C.byref(m.model), len(prompts), m.max_seq)
        assert b, lm.last_error()
        flat = np.concatenate([np.asarray(p, np.uint32) for p in prompts])
        lens = np.array([len(p) for p in prompts], np.uint32)
        assert L.llamini_batch_begin(b, len(prompts), lm.ptr(flat), lm.ptr(lens)) == 0, lm.last_error()
        assert L.llamini_batch_step(b, steps) == 0, lm.last_error()
        btoks = []
        for s in range(len(prompts)):
            out = np.zeros(steps + 1, np.uint32)
            assert L.llamini_batch_tokens(b, s, lm.ptr(out), steps + 1) >= 0, lm.last_error()
            btoks.append(out.tolist())
        lg = np.zeros(m.vocab, np.float32)
        assert L.llamini_batch_logits(b, 0, lm.ptr(lg)) == 0, lm.last_error()
        L.llamini_batch_free(b)
        m.close()
        dist.barrier()
        q.put((rank, long_toks, btoks, lg, ""))
        dist.destroy_process_group()
    except Exception as e:                            # report, then leave: the parent fails the test
        q.put((rank, None, None, None, repr(e)))


def _oracle_stream(o, prompt, total):
    toks = list(prompt)
    lg = None
    for pos in range(total - 1):
        lg = o.forward(pos, toks[pos])
        if pos + 1 >= len(prompt):
            toks.append(int(np.argmax(lg)))
    return toks, lg


def test_tp_two_ranks_prefill_and_batch(orc, tiny):
    """Two ranks: a 70-token prompt (two prefill chunks whose o / down sums go
    through the wide allreduce) and a batch of three ragged prompts (prefill
    chunks of 21 positions x 3 sequences, then lockstep steps with the batch's
    columns allreduced) both reproduce the oracle's greedy streams; the ranks'
    tokens and logits are identical."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    path = tiny.ensure("tiny_tp")
    rng = np.random.default_rng(33)
    long_prompt = rng.integers(3, 1000, 70).tolist()
    n_gen = 16
    prompts = [rng.integers(3, 1000, n).tolist() for n in (24, 31, 27)]
    steps = 47
    o = orc.oracle_model(path)
    want_long, _ = _oracle_stream(o, long_prompt, len(long_prompt) + n_gen)
    want_b = []
    want_lg = None
    for i, p in enumerate(prompts):
        o = orc.oracle_model(path)
        t, lg = _oracle_stream(o, p, steps + 1)
        want_b.append(t)
        if i == 0:
            want_lg = lg
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_batch, args=(r, 2, port, path, long_prompt, n_gen, prompts, steps, qq))
          for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((qq.get(timeout=600) for _ in ps), key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    for rank, lt, bt, lg, err in res:
        assert lt is not None, (rank, err)
        assert lt == want_long, (rank, lt, want_long)
        assert bt == want_b, (rank, bt, want_b)
        assert rel_l2(lg, want_lg) < TOL, (rank, rel_l2(lg, want_lg))
    assert np.array_equal(res[0][3].view(np.uint32), res[1][3].view(np.uint32))


def _rank_fused(rank, world, port, path, prompt, n_gen, q):
    """One rank: the same stream and logits with the o / down reductions fused
    into the GEMVs (default) and as separate allreduce kernels
    (LLAMINI_TP_FUSED=0)."""
    import datetime
    import importlib.util
    import torch.distributed as dist
    import torch
    spec = importlib.util.spec_from_file_location("llamini_b200", os.path.join(ROOT, "llamini.cpp_b200", "__init__.py"))
    lm = importlib.util.module_from_spec(spec)
    sys.modules["llamini_b200"] = lm
    spec.loader.exec_module(lm)
    L = lm.lib()
    try:
        assert L.llamini_set_device(rank) == 0, lm.last_error()
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        h = np.zeros(64, np.uint8)
        assert L.llamini_tp_handle(lm.ptr(h)) == 0, lm.last_error()
        mine = torch.from_numpy(h)
        hs = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(hs, mine)
        allh = np.ascontiguousarray(np.concatenate([x.numpy() for x in hs]))
        assert L.llamini_tp_join(rank, world, lm.ptr(allh)) == 0, lm.last_error()
        res = []
        for mode in ("1", "0"):
            os.environ["LLAMINI_TP_FUSED"] = mode
            m = lm.Model(path)
            toks = m.generate(np.array(prompt, np.uint32), n_gen).tolist()
            lgs = np.stack([m.forward(p, int(toks[p])) for p in range(len(prompt) + 4)])
            m.close()
            res.append((toks, lgs))
            dist.barrier()
        q.put((rank, res, ""))
        dist.destroy_process_group()
    except Exception as e:                            # report, then leave: the parent fails the test
        q.put((rank, None, repr(e)))


def test_tp_fused_reduction_equals_separate(orc, tiny):
    """The reductions fused into the GEMVs (the o / ffn_down GEMV stores its
    partial rows into every rank's memory; the next GEMV waits for them and adds
    them in rank order) give bit-identical logits and the same stream as the
    separate allreduce kernels, and the oracle's stream."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    path = tiny.ensure("tiny_tp")
    prompt = np.random.default_rng(44).integers(3, 1000, 9).tolist()
    n_gen = 20
    want, _ = _oracle_stream(orc.oracle_model(path), prompt, len(prompt) + n_gen)
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_fused, args=(r, 2, port, path, prompt, n_gen, qq)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((qq.get(timeout=600) for _ in ps), key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    for rank, modes, err in res:
        assert modes is not None, (rank, err)
        (tf, lf), (ts, ls) = modes
        assert tf == want and ts == want, (rank, tf, ts, want)
        assert np.array_equal(lf.view(np.uint32), ls.view(np.uint32)), rank
    assert np.array_equal(res[0][1][0][1].view(np.uint32), res[1][1][0][1].view(np.uint32))


def _rank_dead_peer(rank, world, port, path, q):
    """Rank 1 joins and builds the session but never steps; rank 0 steps once:
    its first wait for rank 1's rows runs out (2 s), sets the session's error
    bit, and every later wait of that step returns at once."""
    import datetime
    import importlib.util
    import time
    import torch.distributed as dist
    import torch
    spec = importlib.util.spec_from_file_location("llamini_b200", os.path.join(ROOT, "llamini.cpp_b200", "__init__.py"))
    lm = importlib.util.module_from_spec(spec)
    sys.modules["llamini_b200"] = lm
    spec.loader.exec_module(lm)
    L = lm.lib()
    try:
        assert L.llamini_set_device(rank) == 0, lm.last_error()
        dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        h = np.zeros(64, np.uint8)
        assert L.llamini_tp_handle(lm.ptr(h)) == 0, lm.last_error()
        mine = torch.from_numpy(h)
        hs = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(hs, mine)
        allh = np.ascontiguousarray(np.concatenate([x.numpy() for x in hs]))
        assert L.llamini_tp_join(rank, world, lm.ptr(allh)) == 0, lm.last_error()
        m = lm.Model(path)
        s = m.session()
        prompt = np.array([5], np.uint32)
        assert L.llamini_session_begin(s, lm.ptr(prompt), 1) == 0, lm.last_error()
        dist.barrier()                                # both sessions exist; rank 1 stays idle
        res = None
        if rank == 0:
            out = np.zeros(4, np.uint32)
            t0 = time.time()
            assert L.llamini_session_step(s, 1) == 0, lm.last_error()   # enqueued
            rc = L.llamini_session_tokens(s, lm.ptr(out), 2)               # synchronises, reads the error bits
            dt = time.time() - t0
            err = lm.last_error()
            L.llamini_session_step(s, 1)
            rc2 = L.llamini_session_tokens(s, lm.ptr(out), 2)              # the bits stay set: refused
            res = (rc, dt, err, rc2)
        dist.barrier()                                # rank 1's buffer stays mapped until rank 0 is done
        m.close()
        assert L.llamini_tp_leave() == 0, lm.last_error()
        q.put((rank, res, ""))
        dist.destroy_process_group()
    except Exception as e:                            # report, then leave: the parent fails the test
        q.put((rank, None, repr(e)))


def test_tp_peer_that_never_arrives(tiny):
    """Failure detection without a GPU fault: a rank that never runs its step.
    The other rank's bounded wait (2 s) ends with the session's error bit, the
    remaining waits of the step fail at once (the step returns within seconds,
    not 2 s per reduction), and the session refuses further steps."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallelism needs two GPUs")
    path = tiny.ensure("tiny_tp")
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_dead_peer, args=(r, 2, port, path, qq)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted((qq.get(timeout=600) for _ in ps), key=lambda r: r[0])
    for p in ps:
        p.join(timeout=120)
    for rank, r, err in res:
        assert err == "", (rank, err)
    rc, dt, msg, rc2 = res[0][1]
    assert rc == -1 and rc2 == -1, (rc, rc2, msg)
    assert "tensor-parallel" in msg, msg
    assert 1.5 < dt < 20.0, dt
