"""Write the named-run fixtures: greedy token streams and logits of the CPU
oracle on the benchmark configurations, at their full shapes.

The oracle (oracle/mf_oracle.c) restates the reference's scalar CPU backend
and the LFM2 op order of
crates/executor-core/src/lfm2/executor/execution.rs:35-627 with the greedy
sample of `sample_epilogue` (:591-614).  Its thread pool splits only
independent outputs, so the streams do not depend on the thread count.

Run on any machine with the oracle built (no GPU, no reference checkout):

    python tests/golden/make_named_runs.py [--threads N] [config ...]

It takes about half an hour on eight cores (the 2,048-token prefill of the
1.2B-shaped model and the 2.6B-shaped prefix dominate).  The seeds below are
the ones bench.py uses, so the fixtures describe the benchmarked runs.

What it writes (tests/golden/named_runs/<name>.npz)
----------------------------------------------------
lfm2-350m   BASELINE config 3: weights seed 3, a 256-token uniform random
            prompt (rng 3003), then 128 greedy decode steps at batch 1.
lfm2-1.2b   BASELINE config 4: weights seed 0, the 2,048-token prompt of
            bench.py's rank 0 (rng 1000), then 256 greedy decode steps.
lfm2-2.6b   BASELINE config 5, a stated subset: weights seed 5, the 512-token
            prefix and the 512 x 64 suffixes of bench.py (rng 55); sequences
            SUBSET each fork the prefix, append their suffix and take 15
            greedy decode steps (16 greedy ids each).

Per run: `prompt` (or prefix/suffixes), `ids` (the greedy ids: the argmax of
the prompt's last row, then one per decode step), `margins` (the oracle's
top-1 minus top-2 logit at each greedy id, to explain a divergence should
one appear), and logits: the full prompt-row and final-step logit vectors for
configs 3 and 4; for config 5 the top-16 (index, value) pairs of each subset
sequence's suffix row plus its sum and sum of squares (float64).
"""
from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from runtime_b200 import lfm2 as M  # noqa: E402

OUT = os.path.join(HERE, "named_runs")

# Config 3.
C3_WEIGHT_SEED, C3_PROMPT_SEED, C3_PROMPT, C3_STEPS = 3, 3003, 256, 128
# Config 4 (bench.py: weights seed 0, prompt rng 1000 + rank).
C4_WEIGHT_SEED, C4_PROMPT_SEED, C4_PROMPT, C4_STEPS = 0, 1000, 2048, 256
# Config 5 (bench.py: weights seed 5, rng 55 draws the prefix, then the suffixes).
C5_WEIGHT_SEED, C5_TOKEN_SEED, C5_PREFIX, C5_SUFFIX, C5_SEQS = 5, 55, 512, 64, 512
C5_SUBSET = (0, 73, 146, 219, 292, 365, 438, 511)
C5_STEPS = 15


def margin(logits: np.ndarray) -> float:
    top = np.partition(logits.astype(np.float64), -2)[-2:]
    return float(top[1] - top[0])


def greedy(logits: np.ndarray) -> int:
    return int(np.argmax(logits))  # first maximum, as the oracle's argmax


def c3_inputs():
    cfg = M.PRESETS["lfm2-350m"].with_(max_tokens=C3_PROMPT + C3_STEPS + 8)
    prompt = np.random.default_rng(C3_PROMPT_SEED).integers(0, cfg.vocab, size=C3_PROMPT)
    return cfg, C3_WEIGHT_SEED, prompt


def c4_inputs():
    cfg = M.PRESETS["lfm2-1.2b"].with_(max_tokens=C4_PROMPT + C4_STEPS + 8)
    prompt = np.random.default_rng(C4_PROMPT_SEED).integers(0, cfg.vocab, size=C4_PROMPT)
    return cfg, C4_WEIGHT_SEED, prompt


def c5_inputs():
    cfg = M.PRESETS["lfm2-2.6b"].with_(max_tokens=C5_PREFIX + C5_SUFFIX + 64 + 8)
    rng = np.random.default_rng(C5_TOKEN_SEED)
    prefix = rng.integers(0, cfg.vocab, size=C5_PREFIX)
    suffixes = rng.integers(0, cfg.vocab, size=(C5_SEQS, C5_SUFFIX))
    return cfg, C5_WEIGHT_SEED, prefix, suffixes


def single_run(name, cfg, seed, prompt, steps, threads):
    t0 = time.time()
    ref = O.Lfm2Oracle(cfg, M.synthetic_weights(cfg, seed), threads=threads)
    first = ref.append(prompt, want_logits=True)
    print(f"{name}: prompt of {len(prompt)} in {time.time() - t0:.0f} s", flush=True)
    ids, margins = [greedy(first)], [margin(first)]
    last = first
    for i in range(steps):
        s, last = ref.append_argmax(ids[-1])
        assert int(s) == greedy(last)
        ids.append(int(s))
        margins.append(margin(last))
        if (i + 1) % 32 == 0:
            print(f"{name}: {i + 1}/{steps} steps, {time.time() - t0:.0f} s", flush=True)
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), prompt=prompt.astype(np.uint32),
                        ids=np.asarray(ids, np.int32), margins=np.asarray(margins, np.float64),
                        prompt_logits=first.astype(np.float32), final_logits=last.astype(np.float32),
                        weight_seed=np.int64(seed))
    print(f"{name}: done in {time.time() - t0:.0f} s; ids {ids[:12]}...; min margin {min(margins):.3g}",
          flush=True)


def batch_run(threads):
    t0 = time.time()
    cfg, seed, prefix, suffixes = c5_inputs()
    ref = O.Lfm2Oracle(cfg, M.synthetic_weights(cfg, seed), threads=threads)
    ref.append(prefix, want_logits=False)
    print(f"lfm2-2.6b: prefix in {time.time() - t0:.0f} s", flush=True)
    ids = np.zeros((len(C5_SUBSET), C5_STEPS + 1), np.int32)
    margins = np.zeros((len(C5_SUBSET), C5_STEPS + 1), np.float64)
    top_idx = np.zeros((len(C5_SUBSET), 16), np.int64)
    top_val = np.zeros((len(C5_SUBSET), 16), np.float32)
    sums = np.zeros((len(C5_SUBSET), 2), np.float64)
    for j, s in enumerate(C5_SUBSET):
        seq = ref.fork()
        lg = seq.append(suffixes[s], want_logits=True)
        order = np.argsort(-lg.astype(np.float64), kind="stable")[:16]
        top_idx[j], top_val[j] = order, lg[order]
        sums[j] = (lg.astype(np.float64).sum(), (lg.astype(np.float64) ** 2).sum())
        ids[j, 0], margins[j, 0] = greedy(lg), margin(lg)
        for i in range(C5_STEPS):
            smp, lg = seq.append_argmax(int(ids[j, i]))
            ids[j, i + 1], margins[j, i + 1] = int(smp), margin(lg)
        del seq
        print(f"lfm2-2.6b: sequence {s} done at {time.time() - t0:.0f} s: {ids[j][:8]}", flush=True)
    np.savez_compressed(os.path.join(OUT, "lfm2-2.6b.npz"), prefix=prefix.astype(np.uint32),
                        subset=np.asarray(C5_SUBSET, np.int64),
                        suffixes=suffixes[list(C5_SUBSET)].astype(np.uint32), ids=ids, margins=margins,
                        top_idx=top_idx, top_val=top_val, sums=sums, weight_seed=np.int64(seed))
    print(f"lfm2-2.6b: done in {time.time() - t0:.0f} s; min margin {margins.min():.3g}", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    ap.add_argument("configs", nargs="*", default=["lfm2-350m", "lfm2-1.2b", "lfm2-2.6b"])
    a = ap.parse_args()
    O.build()
    os.makedirs(OUT, exist_ok=True)
    for name in a.configs:
        if name == "lfm2-350m":
            cfg, seed, prompt = c3_inputs()
            single_run(name, cfg, seed, prompt, C3_STEPS, a.threads)
        elif name == "lfm2-1.2b":
            cfg, seed, prompt = c4_inputs()
            single_run(name, cfg, seed, prompt, C4_STEPS, a.threads)
        elif name == "lfm2-2.6b":
            batch_run(a.threads)
        else:
            raise SystemExit(f"unknown config {name}")


if __name__ == "__main__":
    main()
