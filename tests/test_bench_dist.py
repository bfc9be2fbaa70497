"""Host logic of bench.py's multi-process runs, on two CPU ranks (gloo).

With --gpus N every rank decodes its own sequence (independent replicas, no
collective on the data path); the job is timed as the slowest rank, and the
reference arm runs on rank 0 alone.
"""
from __future__ import annotations

import importlib.util
import os
import socket

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("llamini_bench", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, ws, port, out):
    import torch.distributed as dist
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(ws), "LOCAL_RANK": str(rank)})
    b = _bench()
    d = b.init_dist(ws, rank, "gloo")
    # rank r timed (r + 1) ms for the steps and 10 - r s end to end
    t_max, e2e_max = b.max_over_ranks(d, [float(rank + 1), float(10 - rank)])
    rate = b.whole_job_rate(ws, 100, t_max)
    # the reference arm: only rank 0 does work (and prints); others return at once
    class A:
        steps, warmup = 1, 3
    ran = b.run_reference(A, ws, rank, rank) if rank != 0 else "skipped"
    out.put((rank, t_max, e2e_max, rate, ran))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_reduction_and_rate():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, t_max, e2e_max, rate, ran in res:
        assert t_max == 2.0 and e2e_max == 10.0          # max over both ranks, on every rank
        assert rate == pytest.approx(2 * 100 / 0.002)     # whole job: both ranks' tokens / slowest time
    assert res[1][4] is None                               # rank 1 runs no reference work


def test_single_rank_helpers():
    b = _bench()
    assert b.max_over_ranks(None, [1.5, float("nan")])[0] == 1.5
    assert b.whole_job_rate(1, 256, 1000.0) == pytest.approx(256.0)


def _rank_groups(rank, ws, port, out):
    import torch
    import torch.distributed as dist
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                       "WORLD_SIZE": str(ws), "LOCAL_RANK": str(rank)})
    b = _bench()
    d = b.init_dist(ws, rank, "gloo")
    T, DP, grp, r_in, B = b.tp_dp_split(ws, rank, 2)
    group = b.tp_dp_groups(d, ws, T)[grp]
    mine = torch.tensor([rank])
    got = [torch.zeros_like(mine) for _ in range(T)]
    dist.all_gather(got, mine, group=group)
    out.put((rank, (T, DP, grp, r_in, B), [int(x) for x in got]))
    dist.barrier()
    dist.destroy_process_group()


def test_four_ranks_tp_dp_groups():
    """The 7B batch-64 leg on 4 ranks with tensor-parallel groups of 2: groups
    {0, 1} and {2, 3}, 32 sequences each; a group's all_gather sees only its
    own ranks (the handle exchange of llamini_tp_join)."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank_groups, args=(r, 4, port, q)) for r in range(4)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, split, members in res:
        assert split == (2, 2, rank // 2, rank % 2, 32)
        assert members == [2 * (rank // 2), 2 * (rank // 2) + 1]
    b = _bench()
    assert b.tp_dp_split(8, 5) == (4, 2, 1, 1, 32)
    assert b.tp_dp_split(1, 0) == (1, 1, 0, 0, 64)
    with pytest.raises(SystemExit):
        b.tp_dp_split(6, 0, 4)
