#!/usr/bin/env python
"""Benchmark: greedy LFM2 decode through the B200 backend, with its roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the LFM2-1.2B-shaped model of the benchmark configurations:
hidden 2048, 16 layers = 10 gated short-conv + 6 GQA attention, 32 query /
8 KV heads, head_dim 64, FFN 8192, vocab 65536; NF4 attention/conv
projections, ternary FFN, INT8 tied embedding / LM head; random-init weights
and uniform-random prompt tokens, seeded):

* a 2048-token bulk prefill builds the prefix state (timed separately, as
  prefill tok/s);
* one bench STEP is one 256-token greedy decode at batch 1 from that prefix:
  the working state is restored from the prefix by a device copy (no
  allocation), then 256 captured decode steps run with the token ids kept on
  the device, as the reference's `append_argmax` loop does
  (crates/text-generation/src/lib.rs:304-460).
* `value` = decode tokens per second over all ranks (each rank is one full
  model replica decoding its own sequence: sequences shard with no
  collective, so scaling is weak).  The weights read per token (487 MB) are
  larger than L2 (126 MB), so no flush is needed between steps.
* `e2e` = the same steps through the C-ABI with host I/O as the reference's
  generation loop does it (crates/text-generation/src/lib.rs:304-460): each
  step's first token id host -> device, then every token's greedy id read
  device -> host before the next token is appended from the device-resident
  sample (`mf_lfm2_generate`, the reference loop on the C side).
* `roofline` = the decode step in the timed region: algorithmic bytes per
  token (every packed weight's codes + F32 group scales, the LM head, and the
  KV rows attention reads at the step's mean context) over the measured time
  per token, against the measured HBM copy bandwidth.  A token is one launch
  of the persistent decode kernel, so its average launch duration is the
  timed region over its tokens; `traffic` is that launch's DRAM bytes from
  ncu (the capture named in `traffic_source`).  `comparison` times the same
  steps through the opt-in persistent single-launch step.
* `packed_matmul_t{1,16,128,512}` = the packed matmul sweep of BASELINE
  config 2 (five (N, K) shapes x three formats, plus the ternary streams in
  the backend's LUT2 layout as `ternary_lut2_*`) at each token count, on
  rotating weight copies larger than L2: GB/s against HBM below 48 tokens
  (decode GEMV), useful TFLOP/s against the BF16 tensor peak from 48 tokens
  (tcgen05 GEMM).  `roofline_head` is the INT8 65536 x 2048 LM-head GEMV of
  the T=1 sweep.
* `config3` = BASELINE config 3 (LFM2-350M-shaped, dense F32 head) decode at
  batch 1 with its own roofline; `batched` = config 5 (512 sequences, 2.6B-
  shaped) with the bytes of a batched step (weights once + every sequence's
  KV rows).
* `cpu_baseline` = the CPU oracle (a C restatement of the reference's scalar
  backend) decoding the same model on all host cores and on one core, on a
  bounded sample, with the CPU model.

`--impl reference` times that CPU implementation alone (the reference's own
code is Rust and cannot be built on this machine).
"""
from __future__ import annotations

import argparse
import csv
import io
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "decode tok/s (batch 1, LFM2-1.2B-shaped)"
# mf_lfm2_generate's device control block: five u64, four 32-bit fields, 64 stop ids.
GEN_CTL_BYTES = 5 * 8 + 4 * 4 + 64 * 4
UNIT = "tok/s"
PREFILL = 2048
TOKENS_PER_STEP = 256
CONFIG = "lfm2-1.2b"
# 512 sequences share a 512-token prefix, each appends a
# 64-token suffix and decodes 64 greedy tokens; sequences shard over ranks.
BATCH_CONFIG = "lfm2-2.6b"
BATCH_SEQS, BATCH_PREFIX, BATCH_SUFFIX, BATCH_STEPS = 512, 512, 64, 64
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}
SWEEP_SHAPES = [(4608, 1024), (1024, 4608), (8192, 2048), (2048, 8192), (65536, 2048)]
SWEEP_TOKENS = (1, 16, 128, 512)
# BASELINE config 3 (LFM2-350M-shaped, ternary, dense F32 tied head): the
# named run's seeds (tests/golden/make_named_runs.py), 256-token prompt.
C3_CONFIG, C3_WEIGHT_SEED, C3_PROMPT_SEED, C3_PROMPT, C3_TOKENS = "lfm2-350m", 3, 3003, 256, 128
# DRAM traffic of one persistent decode launch (one token) of this workload,
# measured by ncu: dram__bytes_read.sum + dram__bytes_write.sum of one
# decode_persistent_kernel launch at the 2048-token prefix (the capture and
# its command: profiles/decode_persistent_lfm2-1.2b.md).  None until measured.
# DRAM bytes per decode token of the fused graph (ncu, one token, L2 warm):
# 523.0 MB read + 29.9 MB written, 1.02x the algorithmic 540.9 MB.
STEP_TRAFFIC = 552_898_304
STEP_TRAFFIC_SOURCE = "profiles/decode_traffic_lfm2-1.2b.md"


def parse(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--prefill", type=int, default=PREFILL)
    ap.add_argument("--tokens-per-step", type=int, default=TOKENS_PER_STEP)
    ap.add_argument("--e2e-steps", type=int, default=None, help="steps of the host-I/O leg (default: --steps)")
    ap.add_argument("--cpu-seconds", type=float, default=20.0, help="budget of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-pdl", action="store_true", help="launch every kernel without programmatic dependent launch")
    ap.add_argument("--no-batched", action="store_true", help="skip the batched multi-sequence leg (config 5)")
    ap.add_argument("--no-config3", action="store_true", help="skip the LFM2-350M-shaped decode leg (config 3)")
    ap.add_argument("--no-compare", action="store_true",
                    help="skip the separate-launch decode step timed for comparison")
    ap.add_argument("--batched-seqs", type=int, default=BATCH_SEQS, help="total sequences of the batched leg")
    ap.add_argument("--batched-steps", type=int, default=BATCH_STEPS, help="greedy tokens per sequence")
    ap.add_argument("--profile-batched", type=int, default=0, metavar="N",
                    help="after the batched leg's warm-up, run N batched decode steps between "
                         "cudaProfilerStart/Stop and exit")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="after the prefill warm-up, run one prefill between cudaProfilerStart/Stop and exit")
    ap.add_argument("--profile-gemm", action="store_true",
                    help="run one prefill-GEMM probe launch and one cuBLAS BF16 GEMM of the same shape "
                         "between cudaProfilerStart/Stop and exit")
    ap.add_argument("--persistent", action="store_true",
                    help="time the persistent one-launch decode step in the main leg (default: the fused graph)")
    ap.add_argument("--profile-gemv", action="store_true",
                    help="run one launch each of the one-token 65536 x 2048 GEMVs (ternary raw and LUT2, "
                         "INT8) between cudaProfilerStart/Stop and exit")
    ap.add_argument("--profile-decode", type=int, default=0, metavar="N",
                    help="for ncu --profile-from-start off: after the warm-up, decode N tokens "
                         "between cudaProfilerStart/Stop and exit (no timing)")
    a = ap.parse_args(argv)
    if a.warmup < 3 and a.impl == "ours":
        ap.error("--warmup must be at least 3")
    return a


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return dict(PEAKS_FALLBACK)


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


def bench_config(a, world: int) -> dict:
    return {"workload": f"{CONFIG}: {a.prefill}-token prefix, then {a.tokens_per_step} greedy "
                        f"decode tokens per step at batch 1",
            "model": CONFIG, "global_batch": world, "seq_len": a.prefill + a.tokens_per_step,
            "parallelism": f"sequence replicas x{world} (no collective)",
            "l2": "not flushed: 487 MB of weights read per token > 126 MB L2"}


def emit(obj):
    print(json.dumps(obj), flush=True)


# ---------------------------------------------------------------------------
# Clock sampling during the timed region
# ---------------------------------------------------------------------------
CLOCK_FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


class ClockSampler:
    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={CLOCK_FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.out = ""
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        rows = []
        for rec in csv.reader(io.StringIO(self.out or "")):
            rec = [r.strip() for r in rec]
            if len(rec) < 9:
                continue
            if self.uuid and rec[0] != self.uuid:
                continue
            rows.append(rec)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = sorted(float(r[1]) for r in rows if r[1].replace(".", "").isdigit())
        mx = max((float(r[2]) for r in rows if r[2].replace(".", "").isdigit()), default=None)
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU legs (oracle only as the timed baseline, never as the product)
# ---------------------------------------------------------------------------
def cpu_decode_sample(cfg, weights, threads: int, budget_s: float, max_tokens: int, warmup: int = 1):
    """Greedy decode on the CPU oracle from a short prompt; returns
    (tokens timed, seconds, prompt length)."""
    import numpy as np

    from oracle import oracle

    prompt_len = 16
    ref = oracle.Lfm2Oracle(cfg.with_(max_tokens=prompt_len + warmup + max_tokens + 1), weights,
                            threads=threads)
    rng = np.random.default_rng(7)
    logits = ref.append(rng.integers(0, cfg.vocab, size=prompt_len))
    tok = int(np.argmax(logits))
    for _ in range(warmup):
        s, _ = ref.append_argmax(tok)
        tok = int(s)
    n, t0 = 0, time.perf_counter()
    while n < max_tokens:
        s, _ = ref.append_argmax(tok)
        tok = int(s)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return n, time.perf_counter() - t0, prompt_len


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(a):
    """`--impl reference`: the CPU implementation of the path, all host threads."""
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    from runtime_b200 import lfm2 as M

    cfg = M.PRESETS[CONFIG]
    threads = os.cpu_count() or 1
    weights = M.synthetic_weights(cfg, 0)
    # Each step decodes one token; the run stops early once it has used its
    # time budget (150 s), and reports the tokens it timed.
    n, secs, plen = cpu_decode_sample(cfg, weights, threads, budget_s=150.0, max_tokens=a.steps,
                                      warmup=a.warmup)
    value = n / secs
    sample = (f"{n} greedy decode tokens at batch 1 after a {plen}-token prompt (context {plen}-"
              f"{plen + n + a.warmup}, not {a.prefill}+), {CONFIG} weights, C oracle restating backend-cpu, "
              f"{threads} threads of {cpu_model()}")
    emit({"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
          "steps": n, "warmup": a.warmup, "ms_per_step": 1e3 * secs / max(n, 1),
          "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
          "data": "synthetic (seeded random-init weights, uniform random token ids)",
          "config": bench_config(a, world),
          "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
          "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    return 0


# ---------------------------------------------------------------------------
# GPU legs
# ---------------------------------------------------------------------------
def matmul_sweep(be, torch, stream, pk, tokens: int) -> dict:
    """packed_linear at `tokens` rows per (format, N, K) through the handle
    tier: one CUDA graph per shape replays the op over
    rotating weight copies totalling more than 4x L2; mean CUDA-event time
    per op.  `gbs` = algorithmic bytes (codes + F32 scales + input + output
    rows) per second, `tflops` = useful 2*T*N*K flops per second; `frac` is
    against the measured HBM copy rate below 48 tokens (the decode GEMV) and
    against the measured BF16 tensor peak from 48 tokens (the tcgen05 GEMM)."""
    import numpy as np

    from runtime_b200 import formats as F

    out = {}
    rng = np.random.default_rng(11 + tokens)
    # "ternary_lut2": the same ternary streams repacked into the backend's
    # LUT2 layout, through packed_linear_lut2.
    for fmt in ("ternary", "ternary_lut2", "nf4", "int8"):
        lut2 = fmt == "ternary_lut2"
        op = be.packed_linear_lut2 if lut2 else be.packed_linear
        for n, k in SWEEP_SHAPES:
            codes, scales = F.synthetic_weight(rng, n, k, "ternary" if lut2 else fmt)
            wbytes = codes.nbytes + scales.nbytes
            copies = max(4, min(512, int(np.ceil(4 * 126e6 / wbytes))))
            bufs = [(be.upload_u8(codes), be.upload_f32(scales)) for _ in range(copies)]
            if lut2:
                repacked = [(be.repack_ternary_lut2(c), sc) for c, sc in bufs]
                for c, _ in bufs:
                    c.release()
                bufs = repacked
            bx = be.upload_f32(rng.normal(size=(tokens, k)).astype(np.float32))
            y = be.allocate_f32((tokens, n))
            op(y, bx, *bufs[0])   # sizes the backend's scratch before capture
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
                for c, sc in bufs:
                    op(y, bx, c, sc)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            reps = 3
            with torch.cuda.stream(stream):  # replay() launches on the current stream
                g.replay()
                e0.record(stream)
                for _ in range(reps):
                    g.replay()
                e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
            alg = wbytes + tokens * k * 4 + tokens * n * 4
            gbs = alg / us / 1e3
            tflops = 2.0 * tokens * n * k / us / 1e6
            rec = {"us": round(us, 2), "gbs": round(gbs, 1), "tflops": round(tflops, 2),
                   "bytes": int(alg), "flops": int(2 * tokens * n * k)}
            if tokens < 48:
                rec.update(bound="hbm", frac=round(gbs / pk["hbm_gbs"], 3))
            else:
                rec.update(bound="tensor", frac=round(tflops / pk["bf16_tflops"], 3))
            out[f"{fmt}_{n}x{k}"] = rec
            del g
            for c, sc in bufs:
                c.release()
                sc.release()
            bx.release()
            y.release()
    return out


def head_roofline(sweep, pk):
    """The INT8 65536 x 2048 LM-head GEMV of the T=1 sweep."""
    if not sweep or "int8_65536x2048" not in sweep:
        return None
    h = sweep["int8_65536x2048"]
    return {"bound": "hbm", "kernel": "packed_gemv_stream_kernel (INT8 65536 x 2048, one token)",
            "achieved": h["gbs"], "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": h["gbs"] / pk["hbm_gbs"],
            "us": h["us"], "peak_source": pk["source"]}


def dense_head_probe(be, torch, stream, pk) -> dict:
    """The config-3 tied LM head on its own: dense F32 65536 x 1024 at one
    token through `linear` (the streaming head kernel the decode step runs,
    without its argmax epilogue), one CUDA graph over rotating weight copies
    totalling more than 4x L2; mean CUDA-event time per launch.  Bytes =
    weights + input row + output row."""
    import numpy as np

    n, k = 65536, 1024
    rng = np.random.default_rng(23)
    w = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    copies = max(4, int(np.ceil(4 * 126e6 / w.nbytes)))
    bufs = [be.upload_f32(w) for _ in range(copies)]
    bx = be.upload_f32(rng.normal(size=(1, k)).astype(np.float32))
    y = be.allocate_f32((1, n))
    be.linear(y, bx, bufs[0])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
        for b in bufs:
            be.linear(y, bx, b)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    with torch.cuda.stream(stream):
        g.replay()
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
    alg = w.nbytes + 4 * k + 4 * n
    gbs = alg / us / 1e3
    del g
    for b in bufs + [bx, y]:
        b.release()
    return {"bound": "hbm", "kernel": "dense_head_argmax_kernel (F32 65536 x 1024, one token, logits only)",
            "us": round(us, 2), "bytes": int(alg), "achieved": round(gbs, 1), "peak": pk["hbm_gbs"],
            "unit": "GB/s", "frac": round(gbs / pk["hbm_gbs"], 3), "peak_source": pk["source"]}


def gemm_profile(be, torch):
    """For ncu: one launch of the prefill GEMM probe's op and one cuBLAS BF16
    GEMM of the same useful shape (T=2048, N=2x8192, K=2048) between
    cudaProfilerStart/Stop, so the tensor-pipe counters of the two can be
    compared launch for launch."""
    import numpy as np

    from runtime_b200 import formats as F

    rng = np.random.default_rng(17)
    t, n, k = 2048, 8192, 2048
    ca, sa = F.synthetic_weight(rng, n, k, "ternary")
    cb, sb = F.synthetic_weight(rng, n, k, "ternary")
    bufs = [be.upload_u8(ca), be.upload_f32(sa), be.upload_u8(cb), be.upload_f32(sb)]
    bx = be.upload_f32(rng.normal(size=(t, k)).astype(np.float32))
    out = be.allocate_f32((t, n))
    xa = torch.randn(t, k, device="cuda", dtype=torch.bfloat16)
    wb = torch.randn(k, 2 * n, device="cuda", dtype=torch.bfloat16)
    for _ in range(2):
        be.packed_swiglu_pair(out, bx, *bufs)
        yb = xa @ wb
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    be.packed_swiglu_pair(out, bx, *bufs)
    yb = xa @ wb
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    del yb
    for b in bufs + [bx, out]:
        b.release()


def gemv_profile(be, torch):
    """For ncu: the one-token 65536 x 2048 GEMVs of the sweep's largest
    shape (ternary raw, ternary in the LUT2 layout, INT8), one launch each
    after two warm-up calls, between cudaProfilerStart/Stop."""
    import numpy as np

    from runtime_b200 import formats as F

    rng = np.random.default_rng(19)
    n, k = 65536, 2048
    bx = be.upload_f32(rng.normal(size=(1, k)).astype(np.float32))
    y = be.allocate_f32((1, n))
    ops = []
    for fmt in ("ternary", "int8"):
        codes, scales = F.synthetic_weight(rng, n, k, fmt)
        bc, bs = be.upload_u8(codes), be.upload_f32(scales)
        ops.append((be.packed_linear, bc, bs))
        if fmt == "ternary":
            ops.append((be.packed_linear_lut2, be.repack_ternary_lut2(bc), bs))
    for _ in range(2):
        for op, c, sc in ops:
            op(y, bx, c, sc)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for op, c, sc in ops:
        op(y, bx, c, sc)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


def label_bytes(cfg, context: float) -> dict:
    """Algorithmic bytes per launch group of the fused decode step (the op
    labels of mf_lfm2_time_step): weights (codes + F32 scales, or dense
    F32) plus the input and output rows; attention reads K and V of every
    kv head at the given context."""
    from runtime_b200 import formats as F

    h, f, kvw = cfg.hidden, cfg.intermediate, cfg.kv_width

    def b(rows, cols, role):
        fmt = cfg.fmt(role)
        if fmt == "dense":
            return rows * cols * 4 + 4 * (rows + cols)
        return rows * cols // F.WEIGHTS_PER_BYTE[F.FORMATS[fmt]] + rows * (cols // 128) * 4 + 4 * (rows + cols)

    return {"ffn_gate_up": b(f, h, "w1") + b(f, h, "w3") - 4 * h,
            "ffn_down": b(h, f, "w2"),
            "conv_in_proj": b(3 * h, h, "conv_in"),
            "conv_out_proj": b(h, h, "conv_out"),
            "attn_qkv": b(h, h, "q") + b(kvw, h, "k") + b(kvw, h, "v") - 8 * h,
            "attention": 2 * kvw * 4 * context,
            "attn_o": b(h, h, "o"),
            "lm_head": b(cfg.vocab, h, "embedding")}


def step_kernel_profile(model, work, prefix, cfg, pk, tokens: int = 16) -> dict:
    """Per op label of the fused decode step: launches, device time and
    bytes per token from `tokens` greedy steps timed launch by launch
    (mf_lfm2_time_step: a CUDA event after every launch, so the spans are
    serialized per-launch times, not the graph's overlapped step)."""
    work.copy_from(prefix)
    agg = {}
    for _ in range(tokens):
        for name, us in work.time_step():
            a = agg.setdefault(name, [0, 0.0])
            a[0] += 1
            a[1] += us
    lb = label_bytes(cfg, prefix.length + tokens / 2)
    n_conv = sum(1 for k in cfg.layer_types if k == "conv")
    n_attn = len(cfg.layer_types) - n_conv
    per_token = {"ffn_gate_up": len(cfg.layer_types), "ffn_down": len(cfg.layer_types), "conv_in_proj": n_conv,
                 "conv_out_proj": n_conv, "attn_qkv": n_attn, "attention": n_attn, "attn_o": n_attn, "lm_head": 1}
    out = {}
    for name, (n, us) in agg.items():
        rec = {"launches_per_token": n / tokens, "us_per_token": round(us / tokens, 2),
               "us_per_launch": round(us / n, 3)}
        if name in lb:
            bpt = lb[name] * per_token[name]
            gbs = bpt / (us / tokens * 1e-6) / 1e9
            rec.update(bytes_per_token=int(bpt), achieved_gbs=round(gbs, 1), frac=round(gbs / pk["hbm_gbs"], 3))
        out[name] = rec
    return out


def dominant_entry(profile, pk, step_us=None):
    """The op label with the most device time per token in the step profile
    (serialized per-launch spans), with its bytes and fraction of HBM."""
    if not profile:
        return None
    cands = {k: v for k, v in profile.items() if "bytes_per_token" in v}
    if not cands:
        return None
    name, rec = max(cands.items(), key=lambda kv: kv[1]["us_per_token"])
    per_launch = rec["bytes_per_token"] / rec["launches_per_token"]
    out = {"label": name, "launches_per_token": rec["launches_per_token"], "us_per_launch": rec["us_per_launch"],
           "bytes_per_launch": int(per_launch), "achieved": rec["achieved_gbs"], "peak": pk["hbm_gbs"],
           "unit": "GB/s", "frac": rec["frac"], "timing": "CUDA events between launches (serialized spans)"}
    if step_us:
        # The label's share of the serialized spans applied to the measured
        # (overlapped) step: an estimate of its time inside the graph.
        total = sum(v["us_per_token"] for v in profile.values())
        est = step_us * rec["us_per_token"] / total / rec["launches_per_token"]
        out.update(apportioned_us_per_launch=round(est, 3),
                   apportioned_frac=round(per_launch / (est * 1e-6) / 1e9 / pk["hbm_gbs"], 3))
    return out


def gemm_tc_probe(be, torch, stream, pk) -> dict:
    """The prefill GEMM on the tensor cores, live: the config-4 FFN gate/up
    SwiGLU pair (ternary, 2 x 8192 x 2048) at 2,048 tokens through the handle
    tier (activation split + persistent tcgen05 GEMM), mean CUDA-event time of
    5 calls after 2 warm-up calls.  Useful flops 2*T*N*K per matrix (the
    tensor cores issue two BF16 MMAs per product: the ternary levels, exact
    in BF16, against the hi/lo split activation - `mma_passes`; executed
    flops are that many times the useful ones)."""
    import numpy as np

    from runtime_b200 import formats as F

    rng = np.random.default_rng(17)
    t, n, k = 2048, 8192, 2048
    ca, sa = F.synthetic_weight(rng, n, k, "ternary")
    cb, sb = F.synthetic_weight(rng, n, k, "ternary")
    bufs = [be.upload_u8(ca), be.upload_f32(sa), be.upload_u8(cb), be.upload_f32(sb)]
    bx = be.upload_f32(rng.normal(size=(t, k)).astype(np.float32))
    out = be.allocate_f32((t, n))
    for _ in range(2):
        be.packed_swiglu_pair(out, bx, *bufs)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record(stream)
    for _ in range(reps):
        be.packed_swiglu_pair(out, bx, *bufs)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / reps
    useful = 2 * 2.0 * t * n * k / (ms * 1e-3) / 1e12
    for b in bufs + [bx, out]:
        b.release()
    return {"op": "packed_swiglu_pair ternary 2x8192x2048, T=2048", "ms": round(ms, 3),
            "useful_tflops": round(useful, 1), "peak_bf16_tflops": pk["bf16_tflops"],
            "useful_frac": round(useful / pk["bf16_tflops"], 3), "peak_source": pk["source"],
            "mma_passes": 2, "executed_tflops": round(2 * useful, 1)}


def attention_tc_probe(be, torch, stream, pk) -> dict:
    """Prefill attention on the tensor cores, live: one config-4 attention
    layer's causal GQA over 2,048 new tokens (32 query heads, 8 kv heads,
    head_dim 64) through the handle tier (K/V append + attention), mean
    CUDA-event time of 5 calls after 2 warm-up calls, then the same calls on
    the F32 CUDA-core kernel (`mf_set_attention_tc(0)`).  Useful flops
    4 * q_heads * head_dim * T * (T + 1) / 2 (scores and weighted sum over
    the causal pairs); the tensor cores execute six BF16 MMAs per product
    (three-part operands)."""
    import numpy as np

    from runtime_b200 import _lib

    lib = _lib.load()
    qh, kvh, d, t = 32, 8, 64, 2048
    rng = np.random.default_rng(19)
    kvw = kvh * d
    bufs = [be.allocate_f32((t + 8, kvw)), be.allocate_f32((t + 8, kvw)),
            be.upload_f32(rng.normal(size=(t, qh * d)).astype(np.float32)),
            be.upload_f32(rng.normal(size=(t, kvw)).astype(np.float32)),
            be.upload_f32(rng.normal(size=(t, kvw)).astype(np.float32)), be.allocate_f32((t, qh * d))]
    kc, vc, q, k, v, out = bufs
    flops = 4.0 * qh * d * t * (t + 1) / 2
    res = {"op": "causal_gqa 32/8 heads x 64, T=2048 new tokens", "useful_gflop": round(flops / 1e9, 2)}
    try:
        for on, key in ((1, "tc"), (0, "f32")):
            lib.mf_set_attention_tc(on)
            for _ in range(2):
                be.causal_gqa(out, q, k, v, kc, vc, 0, (qh, kvh, d))
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(5):
                be.causal_gqa(out, q, k, v, kc, vc, 0, (qh, kvh, d))
            e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / 5
            res[f"{key}_us"] = round(us, 1)
            res[f"{key}_useful_tflops"] = round(flops / us / 1e6, 1)
    finally:
        lib.mf_set_attention_tc(1)
        for b in bufs:
            b.release()
    res["tc_executed_tflops"] = round(6 * res["tc_useful_tflops"], 1)
    res["peak_bf16_tflops"] = pk["bf16_tflops"]
    res["tc_executed_frac"] = round(res["tc_executed_tflops"] / pk["bf16_tflops"], 3)
    return res


def batched_leg(a, be, rank, world, dist, torch, stream, ev) -> dict:
    """Config 5 on this rank's share of the sequences (contiguous slice, no
    collective): one prefix state, a batch forked from it, the suffix append
    and the batched greedy decode, each timed with CUDA events (max over
    ranks).  Returns the whole-job figures."""
    import numpy as np

    from runtime_b200 import lfm2 as M
    from runtime_b200.sharding import shard

    mine = shard(a.batched_seqs, world, rank)
    seqs = len(mine)
    cfg = M.PRESETS[BATCH_CONFIG].with_(max_tokens=BATCH_PREFIX + BATCH_SUFFIX + a.batched_steps + 8)
    weights = M.synthetic_weights(cfg, 5)
    model = M.Lfm2Model(be, cfg, weights)
    rng = np.random.default_rng(55)
    prefix_tokens = rng.integers(0, cfg.vocab, size=BATCH_PREFIX)   # the same prefix on every rank
    suffixes = rng.integers(0, cfg.vocab, size=(a.batched_seqs, BATCH_SUFFIX))[mine.start:mine.stop]
    prefix = model.new_state()
    prefix.append(prefix_tokens, want_logits=False)
    batch = model.new_batch(max(seqs, 1))
    # warm-up: capture the step graph and size the workspace
    batch.fork(prefix)
    batch.append_argmax(suffixes)
    batch.decode(3)
    torch.cuda.synchronize()
    if a.profile_batched:
        torch.cuda.profiler.start()
        batch.decode(a.profile_batched)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        batch.close()
        prefix.close()
        model.close()
        return None
    if dist:
        dist.barrier()
    batch.fork(prefix)
    e0, e1, e2 = ev(), ev(), ev()
    e0.record(stream)
    batch.append_argmax(suffixes)
    e1.record(stream)
    batch.decode(a.batched_steps)
    e2.record(stream)
    e2.synchronize()
    suffix_ms, decode_ms = e0.elapsed_time(e1), e1.elapsed_time(e2)
    vals = torch.tensor([suffix_ms, decode_ms], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    suffix_ms, decode_ms = (float(v) for v in vals.tolist())
    kps = batch.kernels_per_step
    batch.close()
    prefix.close()
    model.close()
    total = a.batched_seqs
    # Bytes of one batched step on one rank: every weight once, plus every
    # sequence's KV rows at the steps' mean context.
    wb = M.weight_bytes(cfg)
    ctx = BATCH_PREFIX + BATCH_SUFFIX + a.batched_steps / 2
    step_bytes = wb["head"] + wb["layers"] + seqs * wb["kv_per_context_row"] * ctx
    step_s = decode_ms * 1e-3 / a.batched_steps
    return {
        "workload": f"{BATCH_CONFIG}: {total} sequences share a {BATCH_PREFIX}-token prefix, each appends a "
                    f"{BATCH_SUFFIX}-token suffix and decodes {a.batched_steps} greedy tokens; sequences "
                    f"sharded over {world} rank(s), {seqs} per rank",
        "decode_tok_s": total * a.batched_steps / (decode_ms * 1e-3),
        "decode_ms": decode_ms, "ms_per_step": decode_ms / a.batched_steps,
        "suffix_tok_s": total * BATCH_SUFFIX / (suffix_ms * 1e-3), "suffix_ms": suffix_ms,
        "sequences": total, "sequences_per_gpu": seqs, "kernels_per_step": kps,
        "scaling": "strong", "unit": UNIT,
        "roofline": {"bound": "hbm", "bytes_per_step_per_gpu": step_bytes,
                     "weight_bytes": wb["head"] + wb["layers"],
                     "kv_bytes": seqs * wb["kv_per_context_row"] * ctx,
                     "achieved": step_bytes / step_s / 1e9, "unit": "GB/s",
                     "peak": peaks()["hbm_gbs"], "frac": step_bytes / step_s / 1e9 / peaks()["hbm_gbs"]},
    }


def config3_leg(a, be, rank, torch, stream, ev, pk) -> dict:
    """BASELINE config 3 on this rank: the LFM2-350M-shaped ternary model with
    its dense F32 tied head (268 MB of the 349 MB read per token), a 256-token
    prompt, then 128-token greedy decode steps at batch 1 (the named run's
    seeds), timed like the main leg (3 warm-up steps, 5 timed)."""
    import numpy as np

    from runtime_b200 import lfm2 as M

    cfg = M.PRESETS[C3_CONFIG].with_(max_tokens=C3_PROMPT + C3_TOKENS + 16)
    model = M.Lfm2Model(be, cfg, M.synthetic_weights(cfg, C3_WEIGHT_SEED))
    prompt = np.random.default_rng(C3_PROMPT_SEED + rank).integers(0, cfg.vocab, size=C3_PROMPT)
    prefix = model.new_state()
    prefix.append(prompt[:-1], want_logits=False)
    prefix.append_argmax(int(prompt[-1]))
    work = model.new_state()
    for _ in range(3):
        work.copy_from(prefix)
        work.decode(C3_TOKENS)
    torch.cuda.synchronize()
    steps = 5
    e0, e1 = ev(), ev()
    e0.record(stream)
    for _ in range(steps):
        work.copy_from(prefix)
        work.decode(C3_TOKENS)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    wb = M.weight_bytes(cfg)
    per_token = wb["head"] + wb["layers"] + wb["kv_per_context_row"] * (C3_PROMPT + C3_TOKENS / 2)
    tok_s = steps * C3_TOKENS / (ms * 1e-3)
    active = work.persistent_active
    work.close()
    prefix.close()
    model.close()
    return {"workload": f"{C3_CONFIG}: {C3_PROMPT}-token prompt, then {C3_TOKENS} greedy decode tokens per step "
                        f"at batch 1 ({steps} timed steps after 3 warm-up)",
            "decode_tok_s": tok_s, "ms_per_token": ms / (steps * C3_TOKENS),
            "roofline": {"bound": "hbm", "bytes_per_token": per_token, "head_bytes": wb["head"],
                         "achieved": per_token * tok_s / 1e9, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": per_token * tok_s / 1e9 / pk["hbm_gbs"], "peak_source": pk["source"],
                         "kernel": "decode_persistent_kernel" if active else "separate launches"},
            "unit": UNIT}


def run_ours(a):
    import numpy as np
    import torch

    from runtime_b200 import lfm2 as M
    from runtime_b200.backend import CudaBackend

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    pk = peaks()
    cfg = M.PRESETS[CONFIG]
    # capacity: the prefix, one step's decode, and the profiled tokens
    cfg = cfg.with_(max_tokens=a.prefill + a.tokens_per_step + 16)
    weights = M.synthetic_weights(cfg, 0)   # same replica on every rank
    rng = np.random.default_rng(1000 + rank)  # each rank decodes its own sequence
    prompt = rng.integers(0, cfg.vocab, size=a.prefill)

    from runtime_b200 import _lib

    _lib.load().mf_set_pdl(0 if a.no_pdl else 1)
    be = CudaBackend(local)
    if a.profile_gemm:
        gemm_profile(be, torch)
        be.close()
        print("profiled one prefill GEMM launch and one cuBLAS BF16 GEMM")
        return 0
    if a.profile_gemv:
        gemv_profile(be, torch)
        be.close()
        print("profiled the one-token 65536 x 2048 GEMVs")
        return 0
    model = M.Lfm2Model(be, cfg, weights)
    if a.persistent:
        model.set_persistent(True)
    stream = torch.cuda.ExternalStream(be.stream)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    # Prefill: one warm-up pass, then three timed passes (the median is
    # reported).  Every pass starts from an empty state restored by device
    # copies into the same state object, so the timed passes allocate
    # nothing (its workspace was sized by the warm-up pass).
    pre_ms = []
    st, empty = model.new_state(), model.new_state()
    for i in range(4):
        st.copy_from(empty)
        torch.cuda.synchronize()
        e0, e1 = ev(), ev()
        e0.record(stream)
        st.append(prompt, want_logits=True)
        e1.record(stream)
        e1.synchronize()
        pre_ms.append(e0.elapsed_time(e1))
    st.close()
    empty.close()
    if a.profile_prefill:
        st = model.new_state()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        st.append(prompt, want_logits=True)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        if rank == 0:
            print(f"profiled one {a.prefill}-token prefill")
        st.close()
        model.close()
        be.close()
        if dist:
            dist.destroy_process_group()
        return 0

    # Prefix state: prompt[:-1] in bulk, then the last prompt token with argmax
    # (its greedy id is the first decode input, kept on the device).
    prefix = model.new_state()
    prefix.append(prompt[:-1], want_logits=False)
    prefix.append_argmax(int(prompt[-1]))
    work = model.new_state()

    def step():
        work.copy_from(prefix)
        work.decode(a.tokens_per_step)

    for _ in range(a.warmup):
        step()
    torch.cuda.synchronize()
    if a.profile_decode:
        work.copy_from(prefix)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        work.decode(a.profile_decode)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        if rank == 0:
            print(f"profiled {a.profile_decode} decode tokens ({model.kernels_per_decode_step} kernels each)")
        work.close()
        prefix.close()
        model.close()
        be.close()
        if dist:
            dist.destroy_process_group()
        return 0
    if dist:
        dist.barrier()
    uuid = str(torch.cuda.get_device_properties(local).uuid)
    uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    k0 = be.dispatch_counts()["kernels"]
    with ClockSampler(uuid) as clocks:
        torch.cuda.synchronize()
        e0, e1 = ev(), ev()
        e0.record(stream)
        for _ in range(a.steps):
            step()
        e1.record(stream)
        e1.synchronize()
    if dist:
        dist.barrier()
    launches = be.dispatch_counts()["kernels"] - k0
    ms = e0.elapsed_time(e1)

    # e2e through the C-ABI: the step's first id in, every greedy id out.
    # mf_lfm2_generate runs the loop on the device (stop ids, budget and
    # context checked after every step) and uploads and reads back its
    # control block once per call (GEN_CTL_BYTES each way).
    e2e_steps = a.e2e_steps or a.steps
    first = int(prefix.read_sampled())  # the first decode input, as the host sees it
    work.copy_from(prefix)
    work.generate(4, first_token=first)  # warm-up
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    f0, f1 = ev(), ev()
    f0.record(stream)
    for _ in range(e2e_steps):
        work.copy_from(prefix)
        # tokens_per_step appends: the step's input id and each new id are read back.
        work.generate(a.tokens_per_step + 1, first_token=first)
    f1.record(stream)
    f1.synchronize()
    e2e_wall = time.perf_counter() - t0
    e2e_ms = max(f0.elapsed_time(f1), e2e_wall * 1e3)

    # Per-op profile of decode steps at the prefix's context (roofline).
    work.copy_from(prefix)
    agg = {}
    n_prof = 8
    for _ in range(n_prof):
        prof = work.profile_step()
        for kname, v in prof.items():
            d = agg.setdefault(kname, {"launches": 0, "bytes": 0, "ms": 0.0, "ops": 0})
            for f in d:
                d[f] += v[f]
    kernels_per_token = model.kernels_per_decode_step   # of the timed (default) step
    # The same decode steps through the persistent single-launch step (one
    # CTA per SM for the whole token), for comparison.
    compare = None
    if not a.no_compare and rank == 0:
        model.set_persistent(True)
        sep = model.new_state()
        sep.copy_from(prefix)
        sep.decode(a.tokens_per_step)   # warm-up (captures its graphs)
        c0, c1 = ev(), ev()
        c0.record(stream)
        for _ in range(2):
            sep.copy_from(prefix)
            sep.decode(a.tokens_per_step)
        c1.record(stream)
        c1.synchronize()
        compare = {"persistent_tok_s": 2 * a.tokens_per_step / (c0.elapsed_time(c1) * 1e-3),
                   "persistent_active": sep.persistent_active,
                   "kernels_per_token": model.kernels_per_decode_step}
        sep.close()
        model.set_persistent(False)
    sweeps = {}
    if not a.no_sweep and rank == 0:
        for t in SWEEP_TOKENS:
            sweeps[f"packed_matmul_t{t}"] = matmul_sweep(be, torch, stream, pk, t)
    gemm = None if (a.no_sweep or rank != 0) else gemm_tc_probe(be, torch, stream, pk)
    attn = None if (a.no_sweep or rank != 0) else attention_tc_probe(be, torch, stream, pk)
    dense_head = None if (a.no_sweep or rank != 0) else dense_head_probe(be, torch, stream, pk)
    steps_profile = None if rank != 0 else step_kernel_profile(model, work, prefix, cfg, pk)
    c3 = None if (a.no_config3 or rank != 0) else config3_leg(a, be, rank, torch, stream, ev, pk)
    batched = None if a.no_batched else batched_leg(a, be, rank, world, dist, torch, stream, ev)
    if a.profile_batched:
        work.close()
        prefix.close()
        model.close()
        be.close()
        if dist:
            dist.destroy_process_group()
        return 0

    # max over ranks
    vals = torch.tensor([ms, e2e_ms, float(np.median(pre_ms[1:]))], dtype=torch.float64, device="cuda")
    if dist:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    ms, e2e_ms, pre_ms_max = (float(v) for v in vals.tolist())

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        threads = os.cpu_count() or 1
        n, secs, plen = cpu_decode_sample(cfg, weights, threads, budget_s=a.cpu_seconds, max_tokens=64)
        n1, secs1, _ = cpu_decode_sample(cfg, weights, 1, budget_s=a.cpu_seconds / 2, max_tokens=16)
        cpu = {"value": n / secs, "unit": UNIT, "cores": threads, "kind": "port", "cpu_model": cpu_model(),
               "sample": f"{n} greedy decode tokens at batch 1 after a {plen}-token prompt (context "
                         f"{plen}-{plen + n + 1}, shorter than the GPU's {a.prefill}+), same weights, "
                         f"C oracle restating backend-cpu, {threads} threads",
               "single_thread": {"value": n1 / secs1, "unit": UNIT, "cores": 1,
                                 "sample": f"{n1} greedy decode tokens, same prompt and weights, one thread "
                                           f"(the reference's CPU backend is single-threaded)"}}

    model_bytes = M.weight_bytes(cfg)
    if rank == 0:
        tokens = world * a.steps * a.tokens_per_step
        # One rank's tokens over its timed region; KV rows read at the mean context.
        step_bytes = (model_bytes["head"] + model_bytes["layers"]
                      + model_bytes["kv_per_context_row"] * (a.prefill + a.tokens_per_step / 2))
        us_per_token = 1e3 * ms / (a.steps * a.tokens_per_step)
        step_gbs = step_bytes / (us_per_token * 1e-6) / 1e9
        total_ms = sum(v["ms"] for v in agg.values())
        persistent = work.persistent_active
        kernel = ("decode_persistent_kernel (one launch per token)" if persistent else
                  f"decode step ({kernels_per_token} kernels per token in one CUDA graph)")
        t1 = sweeps.get("packed_matmul_t1")
        emit({
            "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms / a.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, uniform random token ids)",
            "config": bench_config(a, world),
            "e2e": {"value": tokens * e2e_steps / a.steps / (e2e_ms * 1e-3), "unit": UNIT,
                    "h2d_bytes_per_step": 4 + GEN_CTL_BYTES,
                    "d2h_bytes_per_step": 4 * (a.tokens_per_step + 1) + GEN_CTL_BYTES},
            "gpu_launches": int(launches),
            "pdl": not a.no_pdl,
            "kernels_per_token": kernels_per_token,
            "prefill": {"tokens": a.prefill, "ms": pre_ms_max,
                        "tok_s": world * a.prefill / (pre_ms_max * 1e-3)},
            # achieved = bytes_per_token / us_per_token; the dominant (only)
            # kernel of a token is the persistent launch, timed here as the
            # timed region over its launches.
            "roofline": {"bound": "hbm", "kernel": kernel,
                         "achieved": step_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": step_gbs / pk["hbm_gbs"], "peak_source": pk["source"],
                         "bytes_per_token": step_bytes, "us_per_token": us_per_token,
                         "weight_bytes_per_token": model_bytes["head"] + model_bytes["layers"],
                         "kv_bytes_per_token": model_bytes["kv_per_context_row"] * (a.prefill + a.tokens_per_step / 2),
                         "traffic": None if persistent else STEP_TRAFFIC,
                         "traffic_source": None if persistent else STEP_TRAFFIC_SOURCE,
                         "dominant": dominant_entry(steps_profile, pk, us_per_token)},
            "comparison": compare,
            "step_kernels": steps_profile,
            "roofline_head": head_roofline(t1, pk),
            "roofline_dense_head": dense_head,
            "op_by_op_profile_us_per_token": {kname: round(1e3 * v["ms"] / n_prof, 2) for kname, v in agg.items()},
            "op_by_op_profile_share": {kname: round(v["ms"] / total_ms, 4) for kname, v in agg.items() if total_ms},
            **sweeps,
            "prefill_gemm_tc": gemm,
            "prefill_attention_tc": attn,
            "config3": c3,
            "batched": batched,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
        })
    work.close()
    prefix.close()
    model.close()
    be.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None):
    a = parse(argv)
    if a.impl == "reference":
        return run_reference(a)
    return run_ours(a)


if __name__ == "__main__":
    sys.exit(main())
