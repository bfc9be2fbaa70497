"""Regenerate the golden fixtures in tests/golden/ from the reference itself.

Runs the reference's own C (oracle/_ref/libllamini_ref.so, built by
`make -C oracle ref` from the reference sources) on seeded synthetic inputs and
stores what it returned:

  dequant.npz   per ggml type: raw blocks (random fields plus edge cases:
                zero, subnormal, negative, max, inf and NaN scales) and the f32
                values gguf_dequantize_rows produced for them
  kat.json      the reference's own unit-test inputs (main.c:505-596):
                rms_norm, rope NORM/NEOX, the fake-model generate tokens
  tokens.json   greedy token streams (temp 0, eos disabled) of the tiny models
                and of the llama_1b / gpt2_124m workloads
  logits.npz    full logits of the tiny models at a few positions

Usage: python tests/golden/make_golden.py [--skip-large | --full-size-only]
The llama_1b run takes a few minutes on the single-threaded lazy path;
--full-size-only adds the qwen2_05b (512-token prompt) and llama_7b (64-token
prompt) streams to tokens.json, which takes tens of minutes.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, HERE)

import oracle as O   # noqa: E402
import tiny          # noqa: E402

S = tiny.synthetic()
N_GEN = 64


def _edge_blocks(t: int) -> np.ndarray:
    """A few blocks of type t whose scale fields hit the f16 corner cases."""
    be, bb = S.BLOCK[t]
    rng = np.random.default_rng(100 + t)
    specials = [0x0000, 0x0001, 0x03FF, 0x0400, 0x8001, 0xBC00, 0x7BFF, 0xFBFF, 0x7C00, 0x7E01]
    blocks = S.random_blocks(rng, t, be * len(specials)).reshape(len(specials), bb)
    for i, h in enumerate(specials):
        lo, hi = h & 0xFF, h >> 8
        if t == S.Q6_K:
            blocks[i, 208], blocks[i, 209] = lo, hi
        else:
            blocks[i, 0], blocks[i, 1] = lo, hi
            if t in (S.Q4_1, S.Q4_K, S.Q5_K):          # second scale (m / dmin)
                h2 = specials[(i + 3) % len(specials)]
                blocks[i, 2], blocks[i, 3] = h2 & 0xFF, h2 >> 8
    if t == S.F16:
        return np.array(specials + [0x3C00, 0x0200], dtype=np.uint16).view(np.uint8)
    return blocks.reshape(-1)


def dequant_goldens(ref) -> dict:
    out = {}
    for t in S.QUANT_TYPES + [S.F16]:
        be, bb = S.BLOCK[t]
        rng = np.random.default_rng(200 + t)
        n_rand = be * 24 if be > 1 else 512
        raw = np.concatenate([S.random_blocks(rng, t, n_rand), _edge_blocks(t)])
        n = raw.size // bb * be
        spec = S.GGUFSpec([("general.architecture", 8, "none")], [S.TensorSpec("t", (n,), t)])
        with tempfile.TemporaryDirectory() as d:
            p = os.path.join(d, "one.gguf")
            S.write_gguf(p, spec, 0, payloads={"t": raw})
            assert ref.drv_open_file(p.encode()) == 0
            y = np.zeros(n, np.float32)
            assert ref.drv_dequant_rows(b"t", 0, 1, n, O.ptr(y)) == 0
            ref.drv_close()
        out["raw_%d" % t] = raw
        out["out_%d" % t] = y
    return out


def kats(ref) -> dict:
    k = {}
    x = np.array([1, 2, 3, 4], np.float32)
    w = np.ones(4, np.float32)
    o = np.zeros(4, np.float32)
    ref.drv_rms_norm(O.ptr(o), O.ptr(x), O.ptr(w), 4, np.float32(1e-8))
    k["rms_norm"] = o.tolist()
    for neox in (0, 1):
        v = np.ones(8, np.float32)
        ref.drv_rope(O.ptr(v), 5, 8, 4, np.float32(10000.0), neox)
        k["rope_neox" if neox else "rope_norm"] = v.tolist()
    toks = np.zeros(8, np.uint32)
    n = ref.drv_fake_generate(O.ptr(toks))
    k["fake_generate"] = toks[:n].tolist()
    k["matmul_2x2"] = [19.0, 22.0, 43.0, 50.0]
    return k


def streams(ref, names, prompts) -> tuple[dict, dict]:
    toks, logits = {}, {}
    for name, path, prompt in zip(names, [p for p, _ in prompts], [q for _, q in prompts]):
        assert ref.drv_open(path.encode(), 0) == 0, name
        out = np.zeros(len(prompt) + N_GEN + 1, np.uint32)
        n = ref.drv_generate(O.ptr(prompt), len(prompt), O.ptr(out), N_GEN, 0xFFFFFFFF)
        toks[name] = {"prompt": prompt.tolist(), "tokens": out[:n].tolist()}
        if name.startswith("tiny"):
            ref.drv_reset()
            v = ref.drv_vocab()
            for pos, t in enumerate(prompt[:4]):
                lg = np.zeros(v, np.float32)
                ref.drv_forward(pos, int(t), O.ptr(lg))
                logits["%s_%d" % (name, pos)] = lg
        ref.drv_close()
        print(name, "done", flush=True)
    return toks, logits


def main():
    ref = O.reference()
    if ref is None:
        sys.exit("reference not built: make -C oracle ref")
    np.savez_compressed(os.path.join(HERE, "dequant.npz"), **dequant_goldens(ref))
    with open(os.path.join(HERE, "kat.json"), "w") as f:
        json.dump(kats(ref), f, indent=1)
    names, prompts = [], []
    for name in tiny.specs():
        names.append(name)
        v = 1000
        prompts.append((tiny.ensure(name), np.random.default_rng(7).integers(3, 500, 16).astype(np.uint32)))
        del v
    if "--full-size-only" in sys.argv:
        # the full-size Qwen2-0.5B stream after its 512-token prompt and the
        # LLaMA-7B-shape stream after a 64-token prompt (tens of minutes on the
        # single-threaded lazy path), merged into the existing file
        names, prompts = [], []
        for name, n_prompt in (("qwen2_05b", 512), ("llama_7b", 64)):
            names.append(name)
            prompts.append((S.ensure_workload(name), S.workload_prompt(name, n_prompt)))
        toks, _ = streams(ref, names, prompts)
        path = os.path.join(HERE, "tokens.json")
        old = json.load(open(path))
        old.update(toks)
        with open(path, "w") as f:
            json.dump(old, f)
        return
    if "--skip-large" not in sys.argv:
        for name, n_prompt in (("gpt2_124m", 64), ("llama_1b", 128)):
            names.append(name)
            prompts.append((S.ensure_workload(name), S.workload_prompt(name, n_prompt)))
    toks, logits = streams(ref, names, prompts)
    path = os.path.join(HERE, "tokens.json")
    if "--skip-large" in sys.argv and os.path.exists(path):
        old = json.load(open(path))
        old.update(toks)
        toks = old
    with open(path, "w") as f:
        json.dump(toks, f)
    np.savez_compressed(os.path.join(HERE, "logits.npz"), **logits)


if __name__ == "__main__":
    main()
