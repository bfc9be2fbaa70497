"""The tensor-parallel shard plan (llamini_tp_plan, the plan tensor-parallel
LLaMA sessions are built with), on the CPU.

* The 7B shape (32 heads of 128, 32 kv heads, FFN 11008 = 43 super-blocks of
  256): for 2, 4 and 8 ranks the FFN cuts fall on super-block boundaries, cover
  the FFN exactly once, differ by at most one super-block per rank, and the
  o-proj cuts are whole heads on 256-column boundaries.
* Two gloo ranks on the tiny tensor-parallel model: each rank evaluates its
  shard of the o projection and of ffn_down with the oracle's dequantized
  weights (model.c:217-260 / generate.c:103-111 arithmetic in float64), the
  partial sums are added by an all-reduce, and the result equals the
  unsharded products.
"""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _plan(lm, W, R, heads, kv, hd, ffn):
    out = np.zeros(8, np.uint32)
    assert lm.lib().llamini_tp_plan(W, R, heads, kv, hd, ffn, lm.ptr(out)) == 0, lm.last_error()
    return out.tolist()


@pytest.mark.parametrize("W,sizes", [(2, [21, 22]), (4, [10, 11, 11, 11]), (8, [5, 5, 6, 5, 5, 6, 5, 6])])
def test_7b_shape_plan(lm, W, sizes):
    heads, kv, hd, ffn = 32, 32, 128, 11008
    plans = [_plan(lm, W, R, heads, kv, hd, ffn) for R in range(W)]
    # FFN: contiguous, on 256-column boundaries, covering [0, ffn) once
    assert plans[0][4] == 0 and plans[-1][5] == ffn
    for a, b in zip(plans, plans[1:]):
        assert a[5] == b[4]
    assert [(p[5] - p[4]) // 256 for p in plans] == sizes
    assert all(p[4] % 256 == 0 and p[5] % 256 == 0 for p in plans)
    # heads / kv heads / o-proj columns: whole heads, 256-column cuts (Q4_K blocks)
    for R, p in enumerate(plans):
        assert p[0:2] == [R * heads // W, (R + 1) * heads // W]
        assert p[2:4] == [R * kv // W, (R + 1) * kv // W]
        assert p[6:8] == [p[0] * hd, p[1] * hd]
        assert p[6] % 256 == 0 and p[7] % 256 == 0


def test_plan_rejects_shapes_that_do_not_split(lm):
    out = np.zeros(8, np.uint32)
    L = lm.lib()
    assert L.llamini_tp_plan(3, 0, 32, 32, 128, 11008, lm.ptr(out)) == -1        # heads % 3
    assert L.llamini_tp_plan(2, 0, 32, 32, 128, 11000, lm.ptr(out)) == -1        # ffn not 256-aligned
    assert L.llamini_tp_plan(8, 0, 32, 4, 128, 11008, lm.ptr(out)) == -1         # kv heads % 8
    assert L.llamini_tp_plan(2, 2, 32, 32, 128, 11008, lm.ptr(out)) == -1        # rank out of range


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, ws, port, out):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import conftest
    import oracle as O
    import tiny
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        lm = conftest._load_pkg()
        S = tiny.synthetic()
        path = tiny.ensure("tiny_tp")
        r = S.GGUFReader(path)
        dim, heads, kv = 512, 8, 4
        hd, ffn = dim // heads, 1536
        plan = _plan(lm, ws, rank, heads, kv, hd, ffn)

        def mat(name, rows, cols):
            t, ne, raw = r.raw(name)
            return O.dequant(t, raw, rows * cols).reshape(rows, cols).astype(np.float64)

        wo = mat("blk.0.attn_output.weight", dim, heads * hd)
        wd = mat("blk.0.ffn_down.weight", dim, ffn)
        rng = np.random.default_rng(3)                   # the same inputs on both ranks
        attn = rng.standard_normal(heads * hd)
        act = rng.standard_normal(ffn)
        part = np.concatenate([wo[:, plan[6]:plan[7]] @ attn[plan[6]:plan[7]],
                               wd[:, plan[4]:plan[5]] @ act[plan[4]:plan[5]]])
        t = torch.from_numpy(part)
        dist.all_reduce(t)                               # the two adds of generate.c:104, 111
        full = np.concatenate([wo @ attn, wd @ act])
        plans = [torch.zeros(8, dtype=torch.int64) for _ in range(ws)]
        dist.all_gather(plans, torch.tensor(plan, dtype=torch.int64))
        out.put((rank, float(np.max(np.abs(t.numpy() - full)) / np.max(np.abs(full))),
                 [p.tolist() for p in plans]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_sums_equal_unsharded(lm):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=240) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, plans in res:
        assert err < 1e-12, (rank, err)
        # the ranks' shards tile heads, kv heads, FFN and o-proj columns exactly
        assert [p[0] for p in plans] == [0, 4] and [p[1] for p in plans] == [4, 8]
        assert [p[2] for p in plans] == [0, 2] and [p[3] for p in plans] == [2, 4]
        assert [p[4] for p in plans] == [0, 768] and [p[5] for p in plans] == [768, 1536]
        assert [p[6] for p in plans] == [0, 256] and [p[7] for p in plans] == [256, 512]
