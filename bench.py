"""Decode benchmark: llama_1b (LLaMA 1.1B shape, Q4_K_M mix), batch 1.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one greedy decode token of the workload (all 22 layers + lm_head +
argmax) at positions 127.., after a 128-token prompt. The weights (624 MB of
quantized blocks) exceed the 126 MB L2, so every step streams them from HBM.

  value   tok/s over exactly K device-timed steps (CUDA events on the library's
          stream, max over ranks), inputs already resident in GPU memory
  e2e     tok/s through generate_autoregressive (the reference's public call)
          from host buffers: a one-token prompt, 256 greedy tokens, wall clock
  roofline  the fused dequant-GEMV kernel at the step's largest launch shape
          (gate+up, 11264 x 2048 Q4_K = 12.98 MB/launch) timed with CUDA events
          over 22 distinct weight copies (286 MB > L2); peak = measured HBM copy
          bandwidth in MEASURED_PEAKS.json
  cpu_baseline  the reference's own C (oracle/_ref) on the host cores, a bounded
          sample of the same decode loop
  batch64 the batch-64 side of the metric: 64 independent llama_1b sequences
          (64 / N per GPU) after 128-token prompts, every weight matrix read once
          per step for the whole batch; tok/s of all sequences over K' timed steps

With --gpus N (torchrun) every rank decodes its own sequence (independent
replicas; the path has no cross-sequence exchange) and value sums the ranks.
--impl reference times the reference's CPU path on the same workload instead.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
WORKLOAD = "llama_1b"
N_PROMPT = 128
METRIC = "decode tok/s (llama_1b Q4_K_M, batch 1)"


def _load(name, path):
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, path)
    m = importlib.util.module_from_spec(spec)
    sys.modules[name] = m
    spec.loader.exec_module(m)
    return m


def pkg():
    return _load("llamini_b200", os.path.join(ROOT, "llamini.cpp_b200", "__init__.py"))


def synthetic():
    return _load("llamini_b200_synthetic", os.path.join(ROOT, "llamini.cpp_b200", "synthetic.py"))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling of SM clock and throttle reasons while running."""

    def __init__(self, index: int):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        q = "clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
            "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q,
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 6:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[2:]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(self.rows[0][1]) if self.rows[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(self.rows)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def init_dist(ws, local, backend):
    import torch
    import torch.distributed as dist
    if ws > 1 and not dist.is_initialized():
        import datetime
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600))
    return dist if ws > 1 else None


def max_over_ranks(dist, values):
    """Element-wise max over ranks of per-rank numbers (device times, wall
    times); the numbers themselves when there is one rank. NaN stays NaN."""
    if not dist:
        return [float(v) for v in values]
    import torch
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def whole_job_rate(ws, steps_per_rank, t_max_ms):
    """Tokens per second of the whole job: every rank decodes its own sequence
    for steps_per_rank steps; the job takes as long as the slowest rank."""
    return ws * steps_per_rank / (t_max_ms / 1e3)


def workload_path(rank, dist):
    S = synthetic()
    directory = os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200")
    if rank == 0:
        S.ensure_workload(WORKLOAD, directory)
    if dist:
        dist.barrier()
    return S.ensure_workload(WORKLOAD, directory)


# --------------------------------------------------------------------------- ours

GEMV_GATE_UP_TRAFFIC = 13059584


def kernel_roofline(lm, torch, stream, hbm_peak, peak_kind):
    """Dominant kernel: the fused GEMV at the gate+up launch shape of a layer."""
    S = synthetic()
    L = lm.lib()
    rows, cols, layers = 2 * 5632, 2048, 22
    raw = S.random_blocks(np.random.default_rng(0), S.Q4_K, rows * cols)
    nbytes = raw.size
    w = torch.empty((layers, nbytes + 16), dtype=torch.uint8, device="cuda")
    host = torch.from_numpy(raw)
    for i in range(layers):
        w[i, :nbytes].copy_(host)
    x = torch.randn(cols, device="cuda", dtype=torch.float32)
    y = torch.empty(rows, device="cuda", dtype=torch.float32)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(layers):                             # warm-up pass
            assert L.llamini_gemv_device(12, w[i].data_ptr(), rows, cols, x.data_ptr(), 1, y.data_ptr()) == 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        e0.record(stream)
        for _ in range(reps):
            for i in range(layers):
                L.llamini_gemv_device(12, w[i].data_ptr(), rows, cols, x.data_ptr(), 1, y.data_ptr())
        e1.record(stream)
    torch.cuda.synchronize()
    per_launch_s = e0.elapsed_time(e1) / 1e3 / (reps * layers)
    algo = nbytes + cols * 4 + rows * 4
    achieved = algo / per_launch_s / 1e9
    del w
    return {"kernel": "gemv_mma_kernel (Q4_K, 11264x2048, gate+up shape)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "algorithmic_bytes_per_launch": algo,
            "us_per_launch": round(per_launch_s * 1e6, 2),
            # dram__bytes_read.sum + dram__bytes_write.sum of this launch shape in one ncu
            # capture (profiles/gemv_mma_llama_1b_ncu.md): equal to the algorithmic bytes
            "traffic": GEMV_GATE_UP_TRAFFIC}


STEP_KERNEL_NAMES = {0: "per-op graph", 1: "decode_kernel (persistent, whole step)",
                     2: "flow_kernel (persistent dataflow, whole step)"}


def step_kernel_roofline(kind, step_bytes, t_ms, steps, hbm_peak, peak_kind, gemv_roof):
    """Roofline of the dominant kernel. With a persistent step kernel (kind 1
    or 2) that is the step itself: algorithmic bytes = all weights once + the
    KV cache read at the step's position, over the device time of the timed
    steps (one launch covers up to 64 steps, so launch duration = timed
    region)."""
    if kind == 0:
        return gemv_roof
    achieved = step_bytes / (t_ms / 1e3 / steps) / 1e9
    name = "flow_kernel" if kind == 2 else "decode_kernel"
    return {"kernel": name + " (22 layers + lm_head + argmax per step)", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": hbm_peak, "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "algorithmic_bytes_per_step": int(step_bytes),
            "us_per_step": round(t_ms * 1e3 / steps, 2), "traffic": None}


GLOBAL_BATCH = 64


def run_batch(args, lm, L, model, torch, stream, ws, rank, dist, hbm_peak):
    """Batched decode: 64 sequences in all (64 / N per rank, independent), each
    after its own 128-token prompt; K timed steps of every sequence. Returns this
    rank's device time and the per-step byte count, or None when skipped."""
    B = max(1, GLOBAL_BATCH // ws)
    max_seq = 512
    b = L.llamini_llama_batch(C.byref(model.model), B, max_seq)
    if not b:
        raise RuntimeError("batch: " + lm.last_error())
    try:
        rng = np.random.default_rng(1000 + rank)
        prompts = rng.integers(3, model.vocab, (B, args.prompt)).astype(np.uint32)
        lens = np.full(B, args.prompt, np.uint32)
        assert L.llamini_batch_begin(b, B, lm.ptr(prompts), lm.ptr(lens)) == 0, lm.last_error()
        assert L.llamini_batch_step(b, args.prompt - 1 + args.warmup) == 0, lm.last_error()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        pos0 = L.llamini_batch_pos(b)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        assert L.llamini_batch_step(b, args.batch_steps) == 0, lm.last_error()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        out = np.zeros(4, np.uint32)
        assert L.llamini_batch_tokens(b, 0, lm.ptr(out), 4) > 0
        weight_bytes = L.llamini_batch_weight_bytes(b)
        tc = L.llamini_batch_gemm_kind(b) == 1
    finally:
        L.llamini_batch_free(b)
    kv_per_pos = L.llamini_session_kv_bytes_per_pos(model.session())
    ctx_mean = pos0 + (args.batch_steps - 1) / 2 + 1
    return ms, weight_bytes + B * kv_per_pos * ctx_mean, B, tc


QWEN_PROMPT, QWEN_STEPS, QWEN_BATCH = 512, 512, 32


def run_qwen2(args, lm, L, torch, hbm_peak):
    """Qwen2-0.5B (24 layers, dim 896, 14/2 heads, ffn 4864, vocab 151936, q/k/v
    biases, Q5_0 attn_v in odd layers): a 512-token prompt through the chunked
    tcgen05 prefill, then 512 greedy decode steps at batch 1; and 32 independent
    sequences, each after its own 512-token prompt, 512 batched steps. Device
    time of the decode steps (rank 0 only)."""
    S = synthetic()
    path = S.ensure_workload("qwen2_05b", os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200"))
    m = lm.Model(path, max_seq=QWEN_PROMPT + QWEN_STEPS + 8)
    try:
        s = m.session()
        stream = torch.cuda.ExternalStream(L.llamini_stream())
        prompt = S.workload_prompt("qwen2_05b", QWEN_PROMPT)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        assert L.llamini_session_begin(s, lm.ptr(prompt), QWEN_PROMPT) == 0, lm.last_error()
        ev[0].record(stream)
        assert L.llamini_session_step(s, QWEN_PROMPT - 1) == 0, lm.last_error()
        ev[1].record(stream)
        assert L.llamini_session_step(s, QWEN_STEPS) == 0, lm.last_error()
        ev[2].record(stream)
        torch.cuda.synchronize()
        prefill_ms, decode_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
        wb = L.llamini_session_weight_bytes(s)
        kvp = L.llamini_session_kv_bytes_per_pos(s)
        step_bytes = wb + kvp * (QWEN_PROMPT + QWEN_STEPS / 2)
        b1 = {"value": round(QWEN_STEPS / (decode_ms / 1e3), 1), "unit": "tok/s", "batch": 1,
              "ms_per_step": round(decode_ms / QWEN_STEPS, 4),
              "weight_stream_gbs": round(step_bytes / (decode_ms / 1e3 / QWEN_STEPS) / 1e9, 1),
              "frac_of_hbm": round(step_bytes / (decode_ms / 1e3 / QWEN_STEPS) / 1e9 / hbm_peak, 4),
              "prefill": {"value": round((QWEN_PROMPT - 1) / (prefill_ms / 1e3), 1), "unit": "tok/s",
                          "positions": QWEN_PROMPT - 1, "path": "tcgen05 GEMM" if L.llamini_session_prefill(s) == 1
                          else "decode steps"}}
        B = QWEN_BATCH
        b = L.llamini_llama_batch(C.byref(m.model), B, QWEN_PROMPT + QWEN_STEPS + 8)
        if not b:
            raise RuntimeError("qwen2 batch: " + lm.last_error())
        try:
            rng = np.random.default_rng(3)
            prompts = rng.integers(3, m.vocab, (B, QWEN_PROMPT)).astype(np.uint32)
            lens = np.full(B, QWEN_PROMPT, np.uint32)
            assert L.llamini_batch_begin(b, B, lm.ptr(prompts), lm.ptr(lens)) == 0, lm.last_error()
            ev[0].record(stream)
            assert L.llamini_batch_step(b, QWEN_PROMPT - 1) == 0, lm.last_error()
            ev[1].record(stream)
            assert L.llamini_batch_step(b, QWEN_STEPS) == 0, lm.last_error()
            ev[2].record(stream)
            torch.cuda.synchronize()
            bp_ms, bd_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
            bwb = L.llamini_batch_weight_bytes(b)
        finally:
            L.llamini_batch_free(b)
        bbytes = bwb + B * kvp * (QWEN_PROMPT + QWEN_STEPS / 2)
        b32 = {"value": round(B * QWEN_STEPS / (bd_ms / 1e3), 1), "unit": "tok/s", "batch": B,
               "ms_per_step": round(bd_ms / QWEN_STEPS, 4),
               "frac_of_hbm": round(bbytes / (bd_ms / 1e3 / QWEN_STEPS) / 1e9 / hbm_peak, 4),
               "prompt_ms": round(bp_ms, 2),
               "prompt_positions_per_s": round(B * (QWEN_PROMPT - 1) / (bp_ms / 1e3), 1),
               "prompt_path": "prefill chunks of 2 positions x 32 sequences (tcgen05 GEMM)"}
    finally:
        m.close()
    return {"workload": "qwen2_05b: Qwen2 0.5B shape (24 layers, dim 896, 14/2 heads, ffn 4864, vocab 151936), "
                        "Q4_K_M mix with Q5_0 attn_v, seed 3; %d-token prompt, %d greedy decode steps" %
                        (QWEN_PROMPT, QWEN_STEPS), "batch1": b1, "batch32": b32}


GEMV_SWEEP = [(2048, 2048), (5632, 2048), (2048, 5632), (32000, 2048), (11008, 4096), (4096, 11008)]
GEMV_TYPES = [("Q4_0", 2), ("Q4_1", 3), ("Q5_0", 6), ("Q8_0", 8), ("Q4_K", 12), ("Q5_K", 13), ("Q6_K", 14)]


def run_gemv_sweep(lm, L, torch, stream, hbm_peak):
    """The isolated fused dequant-GEMV sweep: every shape x format x batch
    {1, 8, 64} (seed 1 blocks), y = W x through llamini_gemv_device. Each
    timing cycles over copies of W totalling more than the 126 MB L2, so every
    launch streams its weights from HBM. GB/s = (weight + x + y bytes) per
    launch / device time per launch."""
    S = synthetic()
    table = {}
    for tname, t in GEMV_TYPES:
        row = {}
        for rows, cols in GEMV_SWEEP:
            raw = S.random_blocks(np.random.default_rng(1), t, rows * cols)
            nb = raw.size
            copies = max(2, -(-(256 << 20) // nb))
            w = torch.empty((copies, nb + 16), dtype=torch.uint8, device="cuda")
            w[0, :nb].copy_(torch.from_numpy(raw))
            for i in range(1, copies):
                w[i].copy_(w[0])
            res = []
            for batch in (1, 8, 64):
                x = torch.randn(batch * cols, device="cuda", dtype=torch.float32)
                y = torch.empty(batch * rows, device="cuda", dtype=torch.float32)
                with torch.cuda.stream(stream):
                    for i in range(min(copies, 4)):
                        assert L.llamini_gemv_device(t, w[i].data_ptr(), rows, cols, x.data_ptr(), batch,
                                                     y.data_ptr()) == 0, lm.last_error()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for i in range(copies):
                        L.llamini_gemv_device(t, w[i].data_ptr(), rows, cols, x.data_ptr(), batch, y.data_ptr())
                    e1.record(stream)
                torch.cuda.synchronize()
                per = e0.elapsed_time(e1) / 1e3 / copies
                res.append(round((nb + batch * (cols + rows) * 4) / per / 1e9, 1))
            row["%dx%d" % (rows, cols)] = res
            del w
        table[tname] = row
    best = max(v for row in table.values() for r in row.values() for v in r)
    return {"unit": "GB/s", "columns": "batch 1, 8, 64", "peak": hbm_peak, "best_frac": round(best / hbm_peak, 4),
            "note": "weights cycled over copies > L2; bytes = weights + x + y per launch", "table": table}


TP_PROMPT = 1024


def run_tp7b(args, lm, L, torch, ws, rank, dist, hbm_peak):
    """LLaMA at 7B shape, batch 1, tensor parallel over every rank (unsharded at
    one GPU): a 1024-token prompt, then timed decode steps. Returns this rank's
    device time, weight bytes per step on this rank and the first timed position."""
    S = synthetic()
    directory = os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200")
    if rank == 0:
        S.ensure_workload("llama_7b", directory)
    if dist:
        dist.barrier()
    path = S.ensure_workload("llama_7b", directory)
    if ws > 1:
        h = np.zeros(64, np.uint8)
        assert L.llamini_tp_handle(lm.ptr(h)) == 0, lm.last_error()
        mine = torch.from_numpy(h).cuda()
        hs = [torch.zeros_like(mine) for _ in range(ws)]
        dist.all_gather(hs, mine)
        allh = np.ascontiguousarray(np.concatenate([x.cpu().numpy() for x in hs]))
        assert L.llamini_tp_join(rank, ws, lm.ptr(allh)) == 0, lm.last_error()
    m = lm.Model(path, max_seq=TP_PROMPT + args.warmup + args.tp_steps + 8)
    try:
        s = m.session()
        stream = torch.cuda.ExternalStream(L.llamini_stream())
        prompt = S.workload_prompt("llama_7b", TP_PROMPT)
        assert L.llamini_session_begin(s, lm.ptr(prompt), TP_PROMPT) == 0, lm.last_error()
        assert L.llamini_session_step(s, TP_PROMPT - 1 + args.warmup) == 0, lm.last_error()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        pos0 = L.llamini_session_pos(s)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        assert L.llamini_session_step(s, args.tp_steps) == 0, lm.last_error()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        # every rank's decoded tokens (the first 16 after the prompt) must be
        # bit-identical: a rank whose shard or sum went wrong decodes differently
        n_tok = TP_PROMPT + min(16, args.warmup + args.tp_steps)
        tk = np.zeros(n_tok, np.uint32)
        assert L.llamini_session_tokens(s, lm.ptr(tk), n_tok) >= n_tok, lm.last_error()
        mine = tk[TP_PROMPT:].astype(np.int64)
        if ws > 1:
            t_mine = torch.from_numpy(mine).cuda()
            t_all = [torch.zeros_like(t_mine) for _ in range(ws)]
            dist.all_gather(t_all, t_mine)
            per_rank = [x.cpu().numpy() for x in t_all]
        else:
            per_rank = [mine]
        identical = all(np.array_equal(per_rank[0], x) for x in per_rank)
        if not identical:
            raise SystemExit("tp_7b: ranks decoded different tokens: %s" % [x.tolist() for x in per_rank])
        # the reference's own greedy stream of this file (64-token prompt,
        # tests/golden/tokens.json, made by the reference's C): the sharded
        # decode must reproduce it token for token
        golden = None
        gpath = os.path.join(ROOT, "tests", "golden", "tokens.json")
        g = json.load(open(gpath)).get("llama_7b") if os.path.exists(gpath) else None
        if g is not None:
            gp = np.asarray(g["prompt"], np.uint32)
            n_g = len(g["tokens"])
            assert L.llamini_session_begin(s, lm.ptr(gp), len(gp)) == 0, lm.last_error()
            assert L.llamini_session_step(s, n_g - 1) == 0, lm.last_error()
            got = np.zeros(n_g, np.uint32)
            assert L.llamini_session_tokens(s, lm.ptr(got), n_g) >= n_g, lm.last_error()
            golden = bool(np.array_equal(got, np.asarray(g["tokens"], np.uint32)))
            if not golden:
                raise SystemExit("tp_7b: rank %d's stream differs from the reference's llama_7b golden stream" % rank)
        wb = L.llamini_session_weight_bytes(s)
        kvp = L.llamini_session_kv_bytes_per_pos(s)
    finally:
        m.close()
        if ws > 1:
            assert L.llamini_tp_leave() == 0, lm.last_error()
            dist.barrier()
    return ms, wb, kvp, pos0, per_rank[0].tolist(), golden


TPDP_BATCH = 64


def tp_dp_split(ws, rank, tp_size=0):
    """The 7B batch-64 leg's split of ws ranks: tensor-parallel groups of T
    consecutive ranks (T = tp_size, default min(ws, 4)), TPDP_BATCH sequences
    shared evenly by the ws / T groups. Returns (T, DP, group, rank in group,
    sequences per group)."""
    T = tp_size or min(ws, 4)
    if ws % T or TPDP_BATCH % (ws // T):
        raise SystemExit("tp_dp_7b_b64: %d ranks do not split into tensor-parallel groups of %d" % (ws, T))
    DP = ws // T
    return T, DP, rank // T, rank % T, TPDP_BATCH // DP


def tp_dp_groups(dist, ws, T):
    """Every rank creates every group's process group, in the same order."""
    return [dist.new_group(list(range(g * T, (g + 1) * T))) for g in range(ws // T)]


def run_tp_dp_7b(args, lm, L, torch, ws, rank, dist):
    """LLaMA at 7B shape, batch 64: tensor parallel over groups of T ranks
    (T = --b64-tp, default min(ws, 4)) and the 64 sequences split
    data-parallel over the ws / T groups. Each sequence has its own seeded
    1024-token prompt, run through the batch's prefill chunks; then warm-up
    and timed lockstep decode steps. Returns this rank's device time of the
    timed steps and of the prompt, and the split."""
    import ctypes as C
    T, DP, grp, r_in, B = tp_dp_split(ws, rank, args.b64_tp)
    S = synthetic()
    directory = os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200")
    if rank == 0:
        S.ensure_workload("llama_7b", directory)
    if dist:
        dist.barrier()
    path = S.ensure_workload("llama_7b", directory)
    group = None
    if dist and ws > 1:
        group = tp_dp_groups(dist, ws, T)[grp]
    if T > 1:
        h = np.zeros(64, np.uint8)
        assert L.llamini_tp_handle(lm.ptr(h)) == 0, lm.last_error()
        mine = torch.from_numpy(h).cuda()
        hs = [torch.zeros_like(mine) for _ in range(T)]
        dist.all_gather(hs, mine, group=group)
        allh = np.ascontiguousarray(np.concatenate([x.cpu().numpy() for x in hs]))
        assert L.llamini_tp_join(r_in, T, lm.ptr(allh)) == 0, lm.last_error()
    max_seq = TP_PROMPT + args.warmup + args.b64_steps + 2
    m = lm.Model(path, max_seq=max_seq)
    b = None
    try:
        b = L.llamini_llama_batch(C.byref(m.model), B, max_seq)
        assert b, lm.last_error()
        prompts = np.stack([np.random.default_rng(4000 + grp * B + i).integers(3, m.vocab, TP_PROMPT)
                            for i in range(B)]).astype(np.uint32)
        lens = np.full(B, TP_PROMPT, np.uint32)
        flat = np.ascontiguousarray(prompts.reshape(-1))
        assert L.llamini_batch_begin(b, B, lm.ptr(flat), lm.ptr(lens)) == 0, lm.last_error()
        stream = torch.cuda.ExternalStream(L.llamini_stream())
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        assert L.llamini_batch_step(b, TP_PROMPT - 1) == 0, lm.last_error()
        p1.record(stream)
        assert L.llamini_batch_step(b, args.warmup) == 0, lm.last_error()
        torch.cuda.synchronize()
        prompt_ms = p0.elapsed_time(p1)
        if dist:
            dist.barrier()
        pos0 = L.llamini_batch_pos(b)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        assert L.llamini_batch_step(b, args.b64_steps) == 0, lm.last_error()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        # the group's ranks must have decoded the same tokens (first sequence)
        n_tok = TP_PROMPT + 8
        tk = np.zeros(n_tok, np.uint32)
        assert L.llamini_batch_tokens(b, 0, lm.ptr(tk), n_tok) >= n_tok, lm.last_error()
        if T > 1:
            t_mine = torch.from_numpy(tk[TP_PROMPT:].astype(np.int64)).cuda()
            t_all = [torch.zeros_like(t_mine) for _ in range(T)]
            dist.all_gather(t_all, t_mine, group=group)
            if not all(torch.equal(t_all[0], x) for x in t_all):
                raise SystemExit("tp_dp_7b_b64: group %d's ranks decoded different tokens" % grp)
        wb = L.llamini_batch_weight_bytes(b)
        # f32 K and V rows of this rank's kv heads, all layers, per position per sequence
        kvp = 2 * 32 * (4096 // T) * 4
    finally:
        if b:
            L.llamini_batch_free(b)
        m.close()
        if T > 1:
            assert L.llamini_tp_leave() == 0, lm.last_error()
        if dist:
            dist.barrier()
    return ms, prompt_ms, T, DP, B, wb, kvp, pos0


def run_perplexity(lm, L, model, n_tok=1024):
    """compute_perplexity over n_tok seeded tokens (teacher forcing, generate.c:169-197):
    the chunked path (64 positions per tcgen05 GEMM pass, lm_head for every
    position, log-softmax on the device) against the one-position-at-a-time
    path, wall clock around the public call (tokens from host memory, the
    perplexity back)."""
    # the model's greedy continuation of one seeded id: seeded random ids give
    # this random-weight model a loss beyond expf's range on every path
    toks = np.asarray(model.generate(synthetic().workload_prompt(WORKLOAD, 1), n_tok - 1), np.uint32)[:n_tok]
    out = {}
    for name, flag in (("chunked", 1), ("steps", 0)):
        assert L.llamini_set_prefill(flag) == 0
        try:
            model.perplexity(toks[:80])                              # warm: buffers, graphs
            t = time.perf_counter()
            p = model.perplexity(toks)
            out[name] = (time.perf_counter() - t, p)
        finally:
            L.llamini_set_prefill(-1)
        assert p > 0, lm.last_error()
    (tc, pc), (ts, ps) = out["chunked"], out["steps"]
    return {"value": round((n_tok - 1) / tc, 1), "unit": "tok/s", "positions": n_tok - 1,
            "ms": round(tc * 1e3, 3), "ppl": round(pc, 6),
            "path": "tcgen05 GEMM, 64 positions per chunk, lm_head + log-softmax on the device",
            "steps_path": {"value": round((n_tok - 1) / ts, 1), "unit": "tok/s", "ppl": round(ps, 6)},
            "note": "compute_perplexity wall clock over the model's %d-token greedy continuation of a seeded id" % n_tok}


def profile_batch():
    """A profiler's workload: llama_1b batched decode of 64 sequences with 4-token
    prompts, 3 batch steps after the model upload, each the same launch sequence
    (embed, staging, 13 per layer, lm_head finish, token update)."""
    lm = pkg()
    L = lm.lib()
    path = synthetic().ensure_workload(WORKLOAD, os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200"))
    model = lm.Model(path, max_seq=512)
    try:
        b = L.llamini_llama_batch(C.byref(model.model), GLOBAL_BATCH, 512)
        if not b:
            raise RuntimeError("batch: " + lm.last_error())
        try:
            prompts = np.random.default_rng(1000).integers(3, model.vocab, (GLOBAL_BATCH, 4)).astype(np.uint32)
            lens = np.full(GLOBAL_BATCH, 4, np.uint32)
            assert L.llamini_batch_begin(b, GLOBAL_BATCH, lm.ptr(prompts), lm.ptr(lens)) == 0, lm.last_error()
            assert L.llamini_batch_step(b, 3) == 0, lm.last_error()
            out = np.zeros(4, np.uint32)
            assert L.llamini_batch_tokens(b, 0, lm.ptr(out), 4) > 0, lm.last_error()
        finally:
            L.llamini_batch_free(b)
    finally:
        model.close()
    print(json.dumps({"profile_batch": "ok", "sequences": GLOBAL_BATCH, "steps": 3}))


def profile_prefill(name):
    """A profiler's workload: one prompt of a named workload (qwen2_05b: 512
    tokens, llama_7b: 1024) through the chunked prefill (tcgen05 GEMMs, 64
    positions per chunk), run twice; prints the second run's device time."""
    import torch
    lm = pkg()
    L = lm.lib()
    n = {"qwen2_05b": QWEN_PROMPT, "llama_7b": TP_PROMPT}[name]
    S = synthetic()
    path = S.ensure_workload(name, os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200"))
    model = lm.Model(path, max_seq=n + 8)
    try:
        s = model.session()
        prompt = S.workload_prompt(name, n)
        stream = torch.cuda.ExternalStream(L.llamini_stream())
        ms = None
        for _ in range(2):
            assert L.llamini_session_begin(s, lm.ptr(prompt), n) == 0, lm.last_error()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            assert L.llamini_session_step(s, n - 1) == 0, lm.last_error()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
        assert L.llamini_session_prefill(s) == 1, "the prompt did not take the prefill path"
    finally:
        model.close()
    print(json.dumps({"profile_prefill": name, "positions": n - 1, "ms": round(ms, 3),
                      "positions_per_s": round((n - 1) / (ms / 1e3), 1)}))


def run_ours(args, ws, rank, local):
    import torch
    dist = init_dist(ws, local, "nccl")
    lm = pkg()
    L = lm.lib()
    torch.cuda.set_device(local)
    if L.llamini_set_device(local) != 0:
        raise RuntimeError(lm.last_error())
    path = workload_path(rank, dist)
    model = lm.Model(path, max_seq=2048)
    sess = model.session()
    stream = torch.cuda.ExternalStream(L.llamini_stream())
    n_prompt = args.prompt
    prompt = synthetic().workload_prompt(WORKLOAD, n_prompt)
    step_kind = L.llamini_session_kernel(sess)       # 0 per-op graphs, 1 / 2 persistent kernels
    weight_bytes = L.llamini_session_weight_bytes(sess)
    kv_per_pos = L.llamini_session_kv_bytes_per_pos(sess)
    if n_prompt + args.warmup + args.steps > model.max_seq:
        raise SystemExit("steps + warmup exceed the 2048-position cache")
    hbm_peak, peak_kind = peaks()

    # one untimed prompt pass builds the prefill buffers; the second one is timed
    assert L.llamini_session_begin(sess, lm.ptr(prompt), n_prompt) == 0, lm.last_error()
    assert L.llamini_session_step(sess, n_prompt - 1) == 0, lm.last_error()
    assert L.llamini_session_begin(sess, lm.ptr(prompt), n_prompt) == 0, lm.last_error()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record(stream)
    assert L.llamini_session_step(sess, n_prompt - 1) == 0, lm.last_error()   # prefill
    p1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = p0.elapsed_time(p1)
    prefill_path = L.llamini_session_prefill(sess)
    assert L.llamini_session_step(sess, args.warmup) == 0
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pos0 = L.llamini_session_pos(sess)
    with Clocks(local) as clk:
        time.sleep(0.3)
        e0.record(stream)
        assert L.llamini_session_step(sess, args.steps) == 0, lm.last_error()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        # e2e through the public call (host buffers), 256 tokens from a 1-token prompt
        e2e_tok, e2e_s = 256, float("nan")
        if not args.no_e2e:
            bos = np.array([1], np.uint32)
            model.generate(bos, 8)                             # warm
            t = time.perf_counter()
            out = model.generate(bos, e2e_tok)
            e2e_s = time.perf_counter() - t
            assert len(out) == e2e_tok + 1
        gemv_roof = None
        if rank == 0 and not args.no_kernel_roofline:
            gemv_roof = kernel_roofline(lm, torch, stream, hbm_peak, peak_kind)
        bt = None if args.no_batch else run_batch(args, lm, L, model, torch, stream, ws, rank, dist, hbm_peak)
    ppl = None if (rank != 0 or args.no_ppl) else run_perplexity(lm, L, model)
    model.close()
    tp7 = None if args.no_tp7b else run_tp7b(args, lm, L, torch, ws, rank, dist, hbm_peak)
    tpdp = None if args.no_b64_7b else run_tp_dp_7b(args, lm, L, torch, ws, rank, dist)
    qwen = None if (rank != 0 or args.no_qwen2) else run_qwen2(args, lm, L, torch, hbm_peak)
    sweep = None if (rank != 0 or args.no_sweep) else run_gemv_sweep(lm, L, torch,
                                                                     torch.cuda.ExternalStream(L.llamini_stream()),
                                                                     hbm_peak)
    t_max, e2e_max = max_over_ranks(dist, [ms, e2e_s])
    b_max = max_over_ranks(dist, [bt[0]])[0] if bt else None
    tp_max = max_over_ranks(dist, [tp7[0]])[0] if tp7 else None
    tpdp_max = max_over_ranks(dist, [tpdp[0], tpdp[1]]) if tpdp else None
    if rank == 0:
        steps = args.steps
        value = whole_job_rate(ws, steps, t_max)
        ctx_mean = pos0 + (steps - 1) / 2 + 1
        step_bytes = weight_bytes + kv_per_pos * ctx_mean
        step_s = t_max / 1e3 / steps
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": ws,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(t_max / steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": decode_workload(n_prompt, pos0, steps),
                       "global_batch": ws, "seq_len": pos0 + steps, "parallelism": "replicas x%d" % ws,
                       "l2": "weights %.0f MB > 126 MB L2, streamed every step" % (weight_bytes / 1e6)},
            "weight_stream_gbs": round(step_bytes / step_s / 1e9, 1),
            "step_roofline": {"bytes_per_step": int(step_bytes), "achieved_gbs": round(step_bytes / step_s / 1e9, 1),
                              "peak": hbm_peak, "frac": round(step_bytes / step_s / 1e9 / hbm_peak, 4)},
            "roofline": step_kernel_roofline(step_kind, step_bytes, t_max, steps, hbm_peak, peak_kind, gemv_roof),
            "gemv_roofline": gemv_roof,
            "e2e": None if args.no_e2e else {
                "value": round(ws * e2e_tok / e2e_max, 2), "unit": "tok/s",
                "h2d_bytes_per_step": round(4 / e2e_tok, 4), "d2h_bytes_per_step": 4,
                "call": "generate_autoregressive, 1-token prompt, 256 greedy tokens, wall clock"},
            # decode kernel: one embed launch + one launch per 64 steps per
            # session_step call; per-op graphs: embed, 5 per layer, lm_head, finish
            "prefill": {"value": round((n_prompt - 1) / (prefill_ms / 1e3), 1), "unit": "tok/s",
                        "positions": n_prompt - 1, "ms": round(prefill_ms, 3),
                        "path": "tcgen05 GEMM, 64 positions per chunk" if prefill_path == 1 else "decode steps",
                        "note": "the prompt before the timed decode (device time, second pass)"},
            "perplexity": ppl,
            "gpu_launches": (1 + (steps + 63) // 64) if step_kind else steps * (1 + 5 * 22 + 2),
            "step_kernel": STEP_KERNEL_NAMES.get(step_kind, str(step_kind)),
            "clocks": clk.summary(),
        }
        if bt:
            b_ms, b_bytes, b_per = bt[0], bt[1], bt[2]
            b_step_s = b_max / 1e3 / args.batch_steps
            line["batch64"] = {
                "value": round(whole_job_rate(ws * b_per, args.batch_steps, b_max), 1), "unit": "tok/s",
                "global_batch": ws * b_per, "per_gpu_batch": b_per, "steps": args.batch_steps,
                "ms_per_step": round(b_max / args.batch_steps, 4), "scaling": "strong",
                "workload": "llama_1b, %d independent sequences per GPU, %d-token prompts (seeded uniform ids), "
                            "timed decode steps after the prompt" % (b_per, args.prompt),
                "weight_stream_gbs": round(b_bytes / b_step_s / 1e9, 1),
                "frac_of_hbm": round(b_bytes / b_step_s / 1e9 / hbm_peak, 4),
                "gemm": "tcgen05 (tensor memory)" if bt[3] else "mma.sync",
                # per step, tensor-core GEMM: embed + staging; per layer the q/k/v GEMM and
                # finish, attention, staging, then o, gate+up and down GEMMs each followed by
                # a finish and a staging; lm_head GEMM + finish; token update. mma.sync GEMM:
                # embed; per layer 4 stagings, 4 GEMMs, 6 finishes, attention; lm_head
                # staging + GEMM + finish; token update
                "gpu_launches": args.batch_steps * ((2 + 22 * 13 + 3) if bt[3] else (1 + 22 * 15 + 3 + 1))}
        if tp7:
            t_step_s = tp_max / 1e3 / args.tp_steps
            tp_bytes = tp7[1] + tp7[2] * (tp7[3] + (args.tp_steps - 1) / 2 + 1)
            line["tp_7b"] = {
                "value": round(args.tp_steps / (tp_max / 1e3), 2), "unit": "tok/s", "tp": ws, "batch": 1,
                "steps": args.tp_steps, "ms_per_step": round(tp_max / args.tp_steps, 4), "scaling": "strong",
                "workload": "llama_7b: LLaMA 7B shape (32 layers, dim 4096, 32/32 heads, ffn 11008, vocab 32000), "
                            "Q4_K_M mix, seed 4; %d-token prompt, timed decode positions %d..%d; heads and FFN "
                            "columns split over %d rank(s), o-proj and ffn_down sums added over NVLink" %
                            (TP_PROMPT, tp7[3], tp7[3] + args.tp_steps - 1, ws),
                "per_gpu_bytes_per_step": int(tp_bytes),
                "per_gpu_stream_gbs": round(tp_bytes / t_step_s / 1e9, 1),
                "frac_of_hbm": round(tp_bytes / t_step_s / 1e9 / hbm_peak, 4),
                "tokens_after_prompt": tp7[4], "tokens_rank_identical": True,
                "reference_stream_match": tp7[5],
                # embed, 5 per layer (+ 2 allreduces per layer when split), lm_head, finish
                "gpu_launches": args.tp_steps * (1 + 32 * (5 + (2 if ws > 1 else 0)) + 2)}
        if tpdp:
            d_ms, d_pms = tpdp_max
            T, DP, B, wb, kvp, dpos0 = tpdp[2:]
            d_step_s = d_ms / 1e3 / args.b64_steps
            d_bytes = wb + kvp * B * (dpos0 + (args.b64_steps - 1) / 2 + 1)
            line["tp_dp_7b_b64"] = {
                "value": round(TPDP_BATCH * args.b64_steps / (d_ms / 1e3), 1), "unit": "tok/s",
                "tp": T, "dp": DP, "batch": TPDP_BATCH, "per_group_batch": B, "steps": args.b64_steps,
                "ms_per_step": round(d_ms / args.b64_steps, 4), "scaling": "strong",
                "workload": "llama_7b (7B shape, Q4_K_M mix, seed 4), 64 sequences with seeded 1024-token "
                            "prompts; timed lockstep decode positions %d..%d; tensor parallel over %d rank(s) "
                            "per group, %d group(s) with %d sequences each" %
                            (dpos0, dpos0 + args.b64_steps - 1, T, DP, B),
                "per_gpu_bytes_per_step": int(d_bytes),
                "per_gpu_stream_gbs": round(d_bytes / d_step_s / 1e9, 1),
                "prompt": {"value": round(TPDP_BATCH * (TP_PROMPT - 1) / (d_pms / 1e3), 1), "unit": "positions/s",
                           "ms": round(d_pms, 1),
                           "path": ("prefill chunks of %d positions x %d sequences (tcgen05 GEMM)" % (64 // B, B))
                           if B <= 32 else "lockstep batch steps (64 columns per weight pass either way)"},
                "tokens_rank_identical": True}
        if qwen:
            line["qwen2_05b"] = qwen
        if sweep:
            line["gemv_sweep"] = sweep
        if ws == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(path)
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def decode_workload(n_prompt, pos0, steps):
    """The batch-1 decode workload as both arms name it in `config`."""
    return ("llama_1b: LLaMA 1.1B shape (22 layers, dim 2048, 32/4 heads, ffn 5632, vocab 32000), Q4_K_M mix, "
            "seed 0; batch 1 per GPU; %d-token prompt, timed decode positions %d..%d" % (n_prompt, pos0,
                                                                                         pos0 + steps - 1))


# --------------------------------------------------------------------------- reference (CPU)

def _ref_lib():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    ref = O.reference()
    if ref is None:
        return None, O
    return ref, O


def cpu_baseline(path, budget_s=15.0):
    """The reference's own C on the host: a 4-token prompt, then greedy decode
    steps until ~budget_s of decode time (the lazy path is single-threaded)."""
    ref, O = _ref_lib()
    if ref is None:
        return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": "reference not built"}
    os.environ.setdefault("LLAMINI_THREADS", str(os.cpu_count()))
    assert ref.drv_open(path.encode(), 0) == 0
    prompt = synthetic().workload_prompt(WORKLOAD, 4)
    ref.drv_time_decode(0, int(prompt[0]), 1, None)
    for p in range(1, 4):
        ref.drv_time_decode(p, int(prompt[p]), 1, None)
    n, el, pos = 0, 0.0, 4
    tok = int(prompt[3])
    while el < budget_s and n < 64:
        el += ref.drv_time_decode(pos, tok, 1, None)
        pos += 1
        n += 1
    ref.drv_close()
    return {"value": round(n / el, 4), "unit": "tok/s", "cores": 1, "kind": "reference",
            "sample": "%d greedy decode steps of llama_1b at positions 4..%d after a 4-token prompt; "
                      "the reference's lazy Q4_K path is single-threaded (model.c:147-158)" % (n, pos - 1)}


def run_reference(args, ws, rank, local):
    if rank != 0:
        return
    ref, O = _ref_lib()
    if ref is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libllamini_ref.so was not built"}))
        return
    path = synthetic().ensure_workload(WORKLOAD)
    os.environ.setdefault("LLAMINI_THREADS", str(os.cpu_count()))
    assert ref.drv_open(path.encode(), 0) == 0
    # the GPU arm's context: the same prompt, fed token by token as the
    # reference's generate does (generate.c:141-150, untimed), then greedy-fed
    # decode steps from the prompt's last position
    n_prompt = args.prompt
    prompt = synthetic().workload_prompt(WORKLOAD, n_prompt)
    for p in range(n_prompt - 1):
        ref.drv_time_decode(p, int(prompt[p]), 1, None)
    out = np.zeros(1, np.uint32)
    pos, tok = n_prompt - 1, int(prompt[n_prompt - 1])
    for _ in range(args.warmup):
        ref.drv_time_decode(pos, tok, 1, O.ptr(out))
        tok, pos = int(out[0]), pos + 1
    # each step is one decode token; stop early (and say so) past ~240 s
    el, n = 0.0, 0
    while n < args.steps and el < 240.0:
        el += ref.drv_time_decode(pos, tok, 1, O.ptr(out))
        tok, pos = int(out[0]), pos + 1
        n += 1
    ref.drv_close()
    value = n / el
    sample = "%d of %d requested decode steps of llama_1b at positions %d..%d after the %d-token prompt (the GPU " \
             "arm's context, greedy-fed), single-threaded lazy Q4_K path (model.c:147-158)" % (
                 n, args.steps, pos - n, pos - 1, n_prompt)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": ws,
            "steps": n, "warmup": args.warmup, "ms_per_step": round(el / n * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": decode_workload(n_prompt, pos - n, n), "global_batch": 1, "seq_len": pos,
                       "parallelism": "replicas x1", "l2": "the reference reads its weights from the host "
                                                                 "memory map every step (no GPU)"},
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": 1, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the generate_autoregressive timing")
    ap.add_argument("--no-kernel-roofline", action="store_true", help="skip the isolated GEMV timing")
    ap.add_argument("--prompt", type=int, default=N_PROMPT, help="prompt length before the timed steps")
    ap.add_argument("--no-batch", action="store_true", help="skip the batch-64 decode timing")
    ap.add_argument("--no-ppl", action="store_true", help="skip the perplexity timing")
    ap.add_argument("--batch-steps", type=int, default=32, help="timed steps of the batch-64 leg")
    ap.add_argument("--no-tp7b", action="store_true", help="skip the 7B-shape tensor-parallel decode timing")
    ap.add_argument("--no-qwen2", action="store_true", help="skip the Qwen2-0.5B batch 1 / batch 32 legs")
    ap.add_argument("--no-sweep", action="store_true", help="skip the isolated GEMV sweep (6 shapes x 7 formats x 3 batches)")
    ap.add_argument("--tp-steps", type=int, default=64, help="timed decode steps of the 7B-shape leg")
    ap.add_argument("--no-b64-7b", action="store_true", help="skip the 7B-shape batch-64 TP x DP leg")
    ap.add_argument("--b64-steps", type=int, default=16, help="timed decode steps of the 7B batch-64 leg")
    ap.add_argument("--b64-tp", type=int, default=0, help="tensor-parallel group size of the 7B batch-64 leg "
                                                           "(default min(gpus, 4))")
    ap.add_argument("--profile-batch", action="store_true",
                    help="no bench line: only a short batch-64 run of llama_1b for profilers "
                         "(4-token prompts, 3 batch steps of identical launch sequences)")
    ap.add_argument("--profile-prefill", choices=["qwen2_05b", "llama_7b"],
                    help="no bench line: only one workload's prompt through the chunked prefill, twice")
    args = ap.parse_args()
    if args.profile_batch:
        profile_batch()
        return
    if args.profile_prefill:
        profile_prefill(args.profile_prefill)
        return
    if args.warmup < 3:
        args.warmup = 3
    ws, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank, local)
    else:
        run_ours(args, ws, rank, local)


if __name__ == "__main__":
    main()
