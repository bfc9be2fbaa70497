"""Per-op timeline of the batch-1 dataflow decode kernel (k_flow.cu).

Builds the profiling variant of the library (build.build(timeline=True):
%globaltimer stamps at eight points of every op of the last step of a launch,
into lib_timeline/), runs a LLaMA workload's decode on cuda:0 and prints, per
op kind of a layer (QKV, attention, O, gate/up, down), the median time of each
point after the previous op's last release, the latest CTA's release, and the
op-to-op period (last release to last release), averaged over the layers.

    python llamini.cpp_b200/flow_timeline.py [--workload llama_1b] [--prompt 128]

Stamps cost a few tens of nanoseconds each, so the periods read a little
longer than the uninstrumented kernel's.
"""
from __future__ import annotations

import argparse
import ctypes as C
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KINDS = ["qkv", "attn", "o", "gate/up", "down"]
POINTS = ["inputs ready", "staged", "tile in smem", "MMAs done", "epilogue has tile", "before release",
          "after release"]


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    m = importlib.util.module_from_spec(spec)
    sys.modules[name] = m
    spec.loader.exec_module(m)
    return m


def capture(workload: str, n_prompt: int, reps: int) -> np.ndarray:
    build = _load("llamini_b200_build", os.path.join(HERE, "build.py"))
    so = build.build(timeline=True)
    lm = _load("llamini_b200", os.path.join(HERE, "__init__.py"))
    syn = _load("llamini_b200_synthetic", os.path.join(HERE, "synthetic.py"))
    lm._lib = lm.load(so)
    L = lm._lib
    L.llamini_flow_timeline.argtypes = [C.c_int, C.c_void_p]
    L.llamini_flow_timeline.restype = C.c_int
    path = syn.ensure_workload(workload, os.environ.get("LLAMINI_WORKDIR", "/tmp/llamini_b200"))
    m = lm.Model(path, max_seq=2048)
    s = m.session()
    if L.llamini_session_kernel(s) != 2:
        raise SystemExit("the workload does not run on the dataflow kernel")
    prompt = syn.workload_prompt(workload, n_prompt)
    assert L.llamini_session_begin(s, lm.ptr(prompt), n_prompt) == 0, lm.last_error()
    assert L.llamini_session_step(s, n_prompt - 1 + 16) == 0, lm.last_error()
    out = []
    for _ in range(reps):
        assert L.llamini_flow_timeline(1, None) == 0
        assert L.llamini_session_step(s, 8) == 0, lm.last_error()
        buf = np.zeros(148 * 128 * 8, np.uint64)
        assert L.llamini_flow_timeline(0, lm.ptr(buf)) == 0
        out.append(buf.reshape(148, 128, 8).astype(np.int64))
    m.close()
    return np.stack(out)


def summarize(tl: np.ndarray, n_layers: int) -> str:
    t = tl[-1]
    n_ops = 5 * n_layers + 1
    sig = [t[:, op, 6][t[:, op, 6] > 0].max() if (t[:, op, 6] > 0).any() else 0 for op in range(n_ops)]
    lines = ["op kind   period | " + " | ".join(POINTS) + " | latest release | CTAs   (us after the previous "
             "op's last release; medians over CTAs, mean over layers)"]
    total = 0.0
    for k, name in enumerate(KINDS):
        rows = []
        for op in [o for o in range(1, n_ops - 1) if o % 5 == k]:
            base = sig[op - 1]
            r = t[:, op, :][t[:, op, 0] > 0] if k != 1 else t[:, op, :][t[:, op, 6] > 0]
            if len(r) == 0 or base == 0:
                continue
            med = [np.median(r[:, p] - base) / 1e3 if (r[:, p] > 0).all() else np.nan for p in range(7)]
            rows.append(med + [(r[:, 6].max() - base) / 1e3, len(r), (sig[op] - base) / 1e3])
        a = np.nanmean(np.array(rows, float), axis=0)
        total += a[9]
        lines.append("%-8s %7.2f | " % (name, a[9]) + " | ".join("%.2f" % v if v == v else "-" for v in a[:7]) +
                     " | %.2f | %d" % (a[7], a[8]))
    lines.append("per layer %.2f us" % total)
    return "\n".join(lines)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", default="llama_1b")
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--save", default="", help="also save the raw stamps (.npz)")
    args = ap.parse_args()
    tl = capture(args.workload, args.prompt, args.reps)
    if args.save:
        np.savez(args.save, tl=tl)
    n_layers = (int(((tl[-1][:, :, 0] > 0) | (tl[-1][:, :, 6] > 0)).any(axis=0).nonzero()[0].max()) + 1 - 1) // 5
    print(summarize(tl, n_layers))


if __name__ == "__main__":
    main()
