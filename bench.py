"""Benchmark of the jax4j B200 engine's hot paths (one JSON line on rank 0).

Default workload (the metric's "Q8_0 dequant-GEMV GB/s"): y[8, 4096] = W x
with W a 4096 x 4096 weight drawn 0.02*N(0,1) by the engine's own counter PRNG
(PrngKey(0).split(2)[1]) and quantised Q8_0 on the device, x [8, 4096] ~ N(0,1)
(split(2)[0]). A step is one GEMV call; `value` is algorithmic bytes (GGUF weight bytes + x + y)
per second over all GPUs. The same run measures the metric's other workloads and reports each as
an entry of `secondary` (value, roofline, clocks, CPU baseline and end-to-end figure of its own):
q4_k_b1 and q4_k_b16 and rms_swiglu; --primary-only skips them.
Workloads selectable with --config:
  q4_k_b1, q4_k_b16   configs[2]: Q4_K decode GEMV, W [14336 x 4096], batch 1 / 16 (GB/s)
  q6_k_b1, q6_k_b16   Q6_K decode GEMV, W [4096 x 14336] (GB/s)
  rms_swiglu          configs[3]: the vmap-batched RMSNorm + SwiGLU value-and-gradient tape,
                      x [4096, 8192] per GPU (steps/s)
  mlp_adam            configs[0]: the compiled MLP valueAndGrad + Adam training step (steps/s)
  prefill_q4_0        configs[4] prefill projection x [16384, 4096] . W^T, W Q4_0 [14336 x 4096]
                      on the tcgen05 tensor cores (TFLOP/s)
  gemm_f32            the same shape as a dense f32 matmul, fp32-accurate 3-term mode (TFLOP/s)
  decoder_decode, decoder_prefill, conv*, aad*   see their tables below

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl engine|reference] [--config NAME]

N > 1 (launched by torchrun, one rank per GPU), weak scaling: for the GEMV each rank owns a
rows-per-GPU slab of a (rows N)-row weight and the GEMV epilogue stores its y slab into every
rank's buffer over NVLink (j4b_quant_matvec_allgather); for the tape each rank owns 4096 rows and
[dg, loss] are summed over NVLink peer memory (j4b_peer_allreduce); the GEMM and MLP workloads
run as independent replicas.

Timing: W untimed warm-up steps, then exactly K steps (replayed from a CUDA graph where the step
is graph-capturable), bracketed by a barrier and device synchronisation, timed with CUDA events
on the launching stream, max over ranks. The GEMV weights rotate over enough identical copies
(>= 2x L2) that every step streams its weight from HBM; the tape and GEMM inputs are larger than
L2. nvidia-smi samples clocks during the timed region.

--impl reference runs the oracle's restatement of the reference's CPU path (the reference is Java;
no JVM exists on the GPU box) on all host cores, with the same config dicts, metric and seeded
inputs (the oracle restates the engine's counter PRNG), rank 0 only.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import ctypes
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))

CONFIGS = {
    # name: (ggml type, rows per rank, cols, batch, label)
    "q8_0_b8": (8, 4096, 4096, 8, "BASELINE configs[1]: GGUF Q8_0 matmul x[8,4096] . W[4096x4096]"),
    "q4_k_b1": (12, 14336, 4096, 1, "BASELINE configs[2]: Q4_K decode GEMV B=1, W[14336x4096]"),
    "q4_k_b16": (12, 14336, 4096, 16, "BASELINE configs[2]: Q4_K decode GEMV B=16, W[14336x4096]"),
    "q6_k_b1": (14, 4096, 14336, 1, "Q6_K decode GEMV B=1, W[4096x14336] (ffn_down of GGUF Q4_K_M files)"),
    "q6_k_b16": (14, 4096, 14336, 16, "Q6_K decode GEMV B=16, W[4096x14336] (ffn_down of GGUF Q4_K_M files)"),
}
TAPE_CONFIGS = {
    # name: (rows per rank, cols, label)
    "rms_swiglu": (4096, 8192, "BASELINE configs[3]: vmap-batched JIT-fused RMSNorm+SwiGLU tape with "
                   "its grad, x[4096,8192], g[8192]"),
    "mlp_adam": (256, 784, "BASELINE configs[0]: JIT-compiled valueAndGrad of a 2-layer tanh MLP "
                 "784-512-10 with softmax cross-entropy, then one Adam step (lr 1e-3), batch 256"),
}
MLP_HIDDEN, MLP_CLASSES = 512, 10


def mlp_shapes(batch, d_in):
    ps = [(d_in, MLP_HIDDEN), (MLP_HIDDEN,), (MLP_HIDDEN, MLP_CLASSES), (MLP_CLASSES,)]
    return ps + ps + ps + [(1,), (batch, d_in), (batch, MLP_CLASSES)]


def mlp_inputs_host(batch, d_in, seed=0):
    """Glorot-uniform weights (u * 2a - a, a = sqrt(6 / (fan_in + fan_out))), zero biases, zero
    moments, step 0, x ~ N(0,1), one-hot labels floor(10 u)."""
    import numpy as np
    rng = np.random.default_rng(seed)
    a1 = math.sqrt(6.0 / (d_in + MLP_HIDDEN))
    a2 = math.sqrt(6.0 / (MLP_HIDDEN + MLP_CLASSES))
    w1 = (rng.random((d_in, MLP_HIDDEN)) * 2 * a1 - a1).astype(np.float32)
    w2 = (rng.random((MLP_HIDDEN, MLP_CLASSES)) * 2 * a2 - a2).astype(np.float32)
    b1, b2 = np.zeros(MLP_HIDDEN, np.float32), np.zeros(MLP_CLASSES, np.float32)
    params = [w1, b1, w2, b2]
    zeros = [np.zeros_like(p) for p in params]
    x = rng.standard_normal((batch, d_in)).astype(np.float32)
    labels = np.floor(10 * rng.random(batch)).astype(np.int64)
    onehot = np.eye(MLP_CLASSES, dtype=np.float32)[labels]
    return params + zeros + [z.copy() for z in zeros] + [np.zeros(1, np.float32), x, onehot]


def mlp_tape_fn():
    sys.path.insert(0, HERE)
    from jax4j_b200 import nn
    return nn.mlp_train_step(nn.FunctionalAdam(1e-3))


DECODER_CONFIGS = {
    # name: (batch, seq or cached tokens, label); d_model 4096, 32 heads x 128, FFN 14336, Q4_0
    "decoder_decode": (64, 2048, "BASELINE configs[4] decode: Llama-style block, Q4_0 weights, batch 64, "
                       "one new token per sequence against a 2048-token f16 KV cache"),
    "decoder_prefill": (8, 2048, "BASELINE configs[4] prefill: Llama-style block, Q4_0 weights, batch 8 x "
                        "seq 2048, causal attention, bf16 tensor-core projections"),
}
DEC_D, DEC_HEADS, DEC_FFN = 4096, 32, 14336
# default timed steps and warm-up per workload family (a GEMV call is microseconds, a prefill
# step tens of milliseconds)
DEFAULT_STEPS = {"gemv": (20000, 200), "tape": (20000, 200), "gemm": (100, 5), "decoder_decode": (200, 5),
                 "decoder_prefill": (10, 3), "aad": (20, 3), "aad_eager": (5, 3)}


def decoder_weight_bytes():
    d, f = DEC_D, DEC_FFN
    params = 3 * d * d + d * d + 2 * f * d + d * f
    return params // 32 * 18


def decoder_kv_bytes(batch, cached):
    return 2 * batch * DEC_HEADS * cached * 128 * 2


def decoder_prefill_flops(batch, seq):
    d, f = DEC_D, DEC_FFN
    proj = 2.0 * batch * seq * (3 * d * d + d * d + 2 * f * d + d * f)
    attn = 2.0 * 2.0 * batch * DEC_HEADS * (seq * (seq + 1) / 2) * 128  # causal q.k^T and p.v
    return proj + attn


GEMM_CONFIGS = {
    # name: (m, n, k, ggml type or None for dense f32, precision, label)
    "prefill_q4_0": (16384, 14336, 4096, 2, 1, "BASELINE configs[4] prefill projection: x[8*2048, 4096] . "
                     "W^T, W Q4_0 [14336 x 4096] (FFN up), bf16 tensor cores"),
    "gemm_f32": (16384, 14336, 4096, None, 2, "dense f32 matmul [16384, 4096] . [4096, 14336], "
                 "fp32-accurate 3-term bf16 split on tcgen05"),
}
TYPE_NAME = {8: "Q8_0", 12: "Q4_K", 14: "Q6_K", 2: "Q4_0", 42: "Q2_0"}
BLOCK = {8: (32, 34), 12: (256, 144), 14: (256, 210), 2: (32, 18), 42: (128, 34)}
METRIC = "Q4_K/Q8_0 dequant-GEMV GB/s vs HBM peak; fused-JIT tape steps/s at 1/2/4/8 B200"


def alg_bytes(qtype, rows, cols, batch):
    be, bb = BLOCK[qtype]
    return rows * cols // be * bb + batch * cols * 4 + batch * rows * 4


def measured_peaks():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU is busy."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sms, maxes, reasons = [], [], set()
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes),
                "reasons": sorted(reasons), "samples": len(sms)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ------------------------------------------------------------------------------------------------
# CPU side: the oracle restatement of the reference's CPU path (baseline and --impl reference)
# ------------------------------------------------------------------------------------------------

DEFAULT_CONFIG = "q8_0_b8"
# measured beside the default workload in the same run, each with its own roofline, clocks,
# CPU baseline and end-to-end figure
SECONDARY = ("q4_k_b1", "q4_k_b16", "rms_swiglu")

# Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of each workload's
# dominant kernel from one ncu capture of the same command, with the capture it comes from. A
# constant of this file, not a run-time measurement: the bench itself never runs under ncu.
TRAFFIC = {
    "q8_0_b8": (17995776, "ncu capture of one qgemv_stream_kernel launch (profiles/qgemv_q8_0_b8.md)"),
    "q4_k_b1": (33089280, "ncu capture of one qgemv_stream_kernel launch (profiles/qgemv_q4_k_b1.md)"),
    "q4_k_b16": (33368576, "ncu capture of one qgemv_stream_kernel launch (profiles/qgemv_q4_k_b16.md)"),
    "q6_k_b1": (48288000, "ncu capture of one qgemv_stream_kernel launch (profiles/qgemv_q6_k_b1.md)"),
    "rms_swiglu": (229038848, "ncu capture of one j4b_group0 launch (profiles/tape_rms_swiglu.md)"),
}


def gemv_config(name, world):
    """The workload's config dict, identical in the engine and the reference arm."""
    qtype, rows, cols, batch, label = CONFIGS[name]
    return {"workload": label, "quant": TYPE_NAME[qtype], "batch": batch, "rows_per_gpu": rows,
            "cols": cols, "bytes_per_step_per_gpu": alg_bytes(qtype, rows, cols, batch),
            "inputs": "PrngKey(0).split(2) -> (kx, kw): x = normal(kx) [batch, cols]; "
                      "W = 0.02 * normal(kw, counter + rank * rows * cols) [rows, cols], "
                      "quantised by the GGUF block encoder",
            "parallelism": "replica" if world == 1 else
            f"row-shard x{world}: each rank a {rows}-row slab, y all-gathered over NVLink peer stores "
            "fused into the GEMV epilogue (no NCCL call)"}


def tape_config(name, world):
    rows, cols, label = TAPE_CONFIGS[name]
    return {"workload": label, "rows_per_gpu": rows, "cols": cols,
            "bytes_per_step_per_gpu": tape_alg_bytes(rows, cols),
            "inputs": "PrngKey(0).split(2) -> (kx, kg): x = normal(kx, counter + rank * rows * cols) "
                      "[rows, cols]; g = 1 + 0.1 * normal(kg) [cols]",
            "parallelism": "replica" if world == 1 else
            f"data-parallel x{world}: rows per rank, [dg, loss] summed over NVLink peer memory "
            "(rank-ordered, no NCCL call)"}


def _keys():
    sys.path.insert(0, HERE)
    from jax4j_b200.prng import PrngKey
    return PrngKey.of(0).split(2)


def gemv_inputs_host(qtype, cols, batch, row0, nrows, rank=0, rows_per_rank=0):
    """Rows [row0, row0 + nrows) of the bench's weight and its x, drawn on the host by the
    oracle's restatement of the same counter PRNG the engine draws them with on the device."""
    import numpy as np
    from oracle import oracle as o
    kx, kw = _keys()
    x = o.random_normal(kx.seed, kx.counter, batch * cols).reshape(batch, cols)
    w = o.random_normal(kw.seed, kw.counter + (rank * rows_per_rank + row0) * cols, nrows * cols)
    w = (w * np.float32(0.02)).astype(np.float32).reshape(nrows, cols)
    return o.quantize(qtype, w), x


def tape_inputs_host(rows, cols, row0, nrows, rank=0):
    import numpy as np
    from oracle import oracle as o
    kx, kg = _keys()
    x = o.random_normal(kx.seed, kx.counter + (rank * rows + row0) * cols, nrows * cols).reshape(nrows, cols)
    g = (o.random_normal(kg.seed, kg.counter, cols) * np.float32(0.1) + np.float32(1.0)).astype(np.float32)
    return x, g


_CPU_INPUTS = {}  # the current sample's host inputs
_CALIBRATION = {}  # seconds per row of one thread, per workload shape


def cpu_matvec_rate(qtype, rows, cols, batch, threads, budget_s):
    """Times the oracle's float-sequential quantMatvec (reference loop style) on a bounded row
    sample of the bench's own weight (same PRNG keys), split over `threads` host threads.
    Returns (GB/s of algorithmic bytes, sample text, seconds)."""
    sys.path.insert(0, HERE)
    from oracle import oracle as o
    rb = o.quant_row_bytes(qtype, cols)
    ckey = ("gemv-row-s", qtype, cols, batch)
    if ckey not in _CALIBRATION:  # one thread, 16 rows
        blob16, x = gemv_inputs_host(qtype, cols, batch, 0, 16)
        t0 = time.perf_counter()
        o.quant_matvec(qtype, blob16, 16, cols, x)
        _CALIBRATION[ckey] = (time.perf_counter() - t0) / 16
    per_row = _CALIBRATION[ckey]
    sample_rows = max(threads, min(rows, int(budget_s * threads / max(per_row, 1e-9))))
    key = ("gemv", qtype, rows, cols, batch, sample_rows)
    if key not in _CPU_INPUTS:
        _CPU_INPUTS.clear()
        _CPU_INPUTS[key] = gemv_inputs_host(qtype, cols, batch, 0, sample_rows)
    blob, x = _CPU_INPUTS[key]
    chunks = [(i * sample_rows // threads, (i + 1) * sample_rows // threads) for i in range(threads)]

    def work(c):
        r0, r1 = c
        if r1 > r0:
            o.quant_matvec(qtype, blob[r0 * rb:r1 * rb], r1 - r0, cols, x)

    t0 = time.perf_counter()
    if threads == 1:
        work(chunks[0])
    else:
        with concurrent.futures.ThreadPoolExecutor(threads) as ex:
            list(ex.map(work, chunks))
    dt = time.perf_counter() - t0
    nbytes = alg_bytes(qtype, sample_rows, cols, batch)
    sample = (f"{sample_rows} of {rows} rows x {cols} cols, batch {batch}, "
              f"{TYPE_NAME[qtype]} float-sequential oracle port, {threads} thread(s)")
    return nbytes / dt / 1e9, sample, dt


def tape_alg_bytes(rows, cols):
    """Read x and g, write dx, dg and the loss (f32)."""
    return 4 * (2 * rows * cols + 2 * cols + 1)


def cpu_tape_rate(rows, cols, threads, budget_s):
    """Times the oracle's call-by-call replay of the tape (the reference CPU backend's
    primitives, single-threaded each) on a bounded row sample of the bench's own x (same PRNG
    keys), split over `threads` host threads (row chunks; their column sums and losses combine).
    Returns (steps/s of the full workload, sample text, seconds)."""
    sys.path.insert(0, HERE)
    from jax4j_b200 import jit as J, nn
    from oracle.backend import run_tape
    ckey = ("tape-row-s", cols)
    if ckey not in _CALIBRATION:  # one thread, 8 rows
        x8, g = tape_inputs_host(rows, cols, 0, 8)
        t8 = J.trace(nn.rms_swiglu_value_and_grad, [(8, cols), (cols,)])
        t0 = time.perf_counter()
        run_tape(t8, [x8, g])
        _CALIBRATION[ckey] = (time.perf_counter() - t0) / 8
    per_row = _CALIBRATION[ckey]
    sample_rows = max(threads, min(rows, int(budget_s * threads / max(per_row, 1e-9))))
    chunk = -(-sample_rows // threads)
    sample_rows = chunk * threads
    key = ("tape", rows, cols, sample_rows)
    if key not in _CPU_INPUTS:
        _CPU_INPUTS.clear()
        _CPU_INPUTS[key] = tape_inputs_host(rows, cols, 0, sample_rows)
    x, g = _CPU_INPUTS[key]
    tape = J.trace(nn.rms_swiglu_value_and_grad, [(chunk, cols), (cols,)])

    def work(i):
        return run_tape(tape, [x[i * chunk:(i + 1) * chunk], g])

    t0 = time.perf_counter()
    if threads == 1:
        work(0)
    else:
        with concurrent.futures.ThreadPoolExecutor(threads) as ex:
            list(ex.map(work, range(threads)))
    dt = time.perf_counter() - t0
    steps_per_s = sample_rows / rows / dt
    sample = (f"{sample_rows} of {rows} rows x {cols} cols ({threads} chunk(s) of {chunk} rows), "
              f"oracle replay of the same tape (CpuBackend primitives), {threads} thread(s)")
    return steps_per_s, sample, dt


def gemv_kernel_name(batch):
    return "qgemv_stream_kernel" if batch <= 16 else "qgemm_fused_kernel"


def cpu_mlp_rate(batch, d_in, budget_s):
    """Times the oracle's call-by-call replay of the MLP training-step tape (single-threaded C
    primitives, the reference CPU backend's loops). Returns (steps/s, sample, seconds)."""
    sys.path.insert(0, HERE)
    from jax4j_b200 import jit as J
    from oracle.backend import run_tape
    inputs = mlp_inputs_host(batch, d_in)
    tape = J.trace(mlp_tape_fn(), [a.shape for a in inputs])
    n, t0 = 0, time.perf_counter()
    while True:
        run_tape(tape, inputs)
        n += 1
        if time.perf_counter() - t0 >= budget_s or n >= 50:
            break
    dt = (time.perf_counter() - t0) / n
    return 1.0 / dt, f"{n} full training step(s), oracle replay of the same tape, 1 thread", dt


def run_reference_tape(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    rows, cols, label = TAPE_CONFIGS[args.config]
    if args.config == "mlp_adam":
        budget = max(0.5, min(10.0, 90.0 / max(args.steps + args.warmup, 1)))
        rates, sample = [], ""
        for _ in range(args.warmup):
            cpu_mlp_rate(rows, cols, budget)
        for _ in range(args.steps):
            r, sample, _ = cpu_mlp_rate(rows, cols, budget)
            rates.append(r)
        value = statistics.median(rates)
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "steps/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 / value, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": label, "batch": rows, "d_in": cols},
            "cpu_baseline": {"value": round(value, 5), "unit": "steps/s", "cores": 1, "kind": "port",
                             "sample": sample + " (the step is one dependent chain; the port is single-threaded)"},
            "e2e": {"value": round(value, 5), "unit": "steps/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    return run_reference_workloads(args)


def reference_entry(name, K, W, threads, budget, world):
    """The reference arm's result for one GEMV / tape workload: the oracle port of the
    reference's CPU path on `threads` host threads, K bounded samples after W warm-up ones."""
    is_tape = name in TAPE_CONFIGS
    if is_tape:
        rows, cols, _ = TAPE_CONFIGS[name]
        rate = lambda: cpu_tape_rate(rows, cols, threads, budget)  # noqa: E731
        unit, cfg = "steps/s", tape_config(name, world)
    else:
        qtype, rows, cols, batch, _ = CONFIGS[name]
        rate = lambda: cpu_matvec_rate(qtype, rows, cols, batch, threads, budget)  # noqa: E731
        unit, cfg = "GB/s", gemv_config(name, world)
    for _ in range(W):
        rate()
    rates, times, sample = [], [], ""
    for _ in range(K):
        r, sample, dt = rate()
        rates.append(r)
        times.append((1.0 / r) if is_tape else dt)
    value = statistics.median(rates)
    digits = 5 if is_tape else 3
    return {"name": name, "value": round(value, digits), "unit": unit, "steps": K, "warmup": W,
            "ms_per_step": round(1e3 * statistics.median(times), 3), "higher_is_better": True,
            "config": cfg,
            "cpu_baseline": {"value": round(value, digits), "unit": unit, "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, digits), "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def run_reference_workloads(args):
    """Reference arm of the GEMV / tape workloads: rank 0 alone; the same config dicts and the
    same seeded inputs as the engine arm, the default run with the same secondary workloads."""
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    names = [args.config] + (list(SECONDARY) if args.config == DEFAULT_CONFIG and not args.primary_only else [])
    total = (args.steps + args.warmup) * len(names)
    budget = max(0.002, min(2.0, 60.0 / max(total, 1)))  # whole run within a few minutes
    entries = [reference_entry(n, args.steps, args.warmup, threads, budget, world) for n in names]
    e = entries[0]
    line = {"impl": "reference", "metric": METRIC, "value": e["value"], "unit": e["unit"],
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": e["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": e["config"], "cpu_baseline": e["cpu_baseline"], "e2e": e["e2e"]}
    if len(entries) > 1:
        line["secondary"] = entries[1:]
    print(json.dumps(line), flush=True)
    return 0


def cpu_gemm_rate(m, n, k, qtype, threads, budget_s):
    """Times the oracle's i-p-j float matmul (CpuBackend.java:188-216; for a quantised weight the
    dequantised rows, as the reference would multiply them) on a bounded sample of output rows
    split over `threads` host threads. Returns (TFLOP/s, sample text, seconds)."""
    import numpy as np
    sys.path.insert(0, HERE)
    from oracle import oracle as o
    rng = np.random.default_rng(0)
    bt = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    x = rng.standard_normal((64, k)).astype(np.float32)
    t0 = time.perf_counter()
    o.matmul(x[:1], bt)
    per_row = time.perf_counter() - t0
    rows = max(threads, min(64, int(budget_s * threads / max(per_row, 1e-9))))
    chunks = [(i * rows // threads, (i + 1) * rows // threads) for i in range(threads)]

    def work(c):
        if c[1] > c[0]:
            o.matmul(x[c[0]:c[1]], bt)

    t0 = time.perf_counter()
    with concurrent.futures.ThreadPoolExecutor(threads) as ex:
        list(ex.map(work, chunks))
    dt = time.perf_counter() - t0
    tflops = 2.0 * rows * n * k / dt / 1e12
    kind = "dequantised " + TYPE_NAME[qtype] if qtype else "f32"
    return tflops, f"{rows} of {m} output rows x {n} cols, K {k}, {kind} weight, oracle i-p-j float matmul, {threads} thread(s)", dt


def run_reference_gemm(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    m, n, k, qtype, prec, label = GEMM_CONFIGS[args.config]
    threads = os.cpu_count() or 1
    budget = max(0.2, min(5.0, 90.0 / max(args.steps + args.warmup, 1)))
    for _ in range(args.warmup):
        cpu_gemm_rate(m, n, k, qtype, threads, budget)
    rates, sample = [], ""
    for _ in range(args.steps):
        r, sample, _ = cpu_gemm_rate(m, n, k, qtype, threads, budget)
        rates.append(r)
    value = statistics.median(rates)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(2.0 * m * n * k / (value * 1e12) * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": label, "m": m, "n": n, "k": k},
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference(args):
    if args.config in CONV_CONFIGS:
        return run_reference_conv(args)
    if args.config in AAD_CONFIGS:
        return run_reference_aad(args)
    if args.config in DECODER_CONFIGS:
        return run_reference_decoder(args)
    if args.config in TAPE_CONFIGS:
        return run_reference_tape(args)
    if args.config in GEMM_CONFIGS:
        return run_reference_gemm(args)
    return run_reference_workloads(args)


# ------------------------------------------------------------------------------------------------
# engine arm
# ------------------------------------------------------------------------------------------------

def run_engine_mlp(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from jax4j_b200 import jit as J
    from jax4j_b200 import _lib
    from jax4j_b200.backend import B200Backend, TapeHandle, torch_stream

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    be = B200Backend(local)
    batch, d_in, label = TAPE_CONFIGS[args.config]
    host = mlp_inputs_host(batch, d_in, seed=rank)
    tape = J.trace(mlp_tape_fn(), [a.shape for a in host])
    handle = TapeHandle(be, tape)
    st = handle.stats()
    # two buffer sets: step i reads set i % 2 (params, moments, step) and writes set (i + 1) % 2,
    # so consecutive replays are a real training loop
    state = [[be.upload(a, a.shape) for a in host[:13]] for _ in range(2)]
    x = be.upload(host[13], host[13].shape)
    onehot = be.upload(host[14], host[14].shape)
    loss = torch.empty(4, dtype=torch.float32, device=torch.device("cuda", local))
    nbytes = sum(a.nbytes for a in host)

    def step(i, stream):
        src, dst = state[i % 2], state[(i + 1) % 2]
        handle.launch([b.ptr for b in src] + [x.ptr, onehot.ptr],
                      [loss.data_ptr()] + [b.ptr for b in dst], stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    K, W = args.steps, max(3, args.warmup)
    K += K % 2  # even: the graph ends on the starting buffer set

    def capture(n):
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step(0, torch_stream())
            step(1, torch_stream())
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            for i in range(n):
                step(i, torch_stream())
        return g

    warm, main = capture(W + W % 2), capture(K)
    warm.replay()
    main.replay()  # the first replay of a graph also uploads it: keep that out of the timed one
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        main.replay()
        end.record()
        barrier()
    clk = clocks.summary()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=torch.device("cuda", local))
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_us = ms * 1e3 / K
    value = world * K / (ms * 1e-3)
    peak, peak_kind = measured_peaks()
    # minimum bytes of a step (x, one-hot, params, moments read; params, moments written; loss)
    min_bytes = (host[13].nbytes + host[14].nbytes + 3 * sum(a.nbytes for a in host[:4])
                 + 3 * sum(a.nbytes for a in host[:4]) + 4)

    # end to end: x and the one-hot labels from pinned host memory, the loss back, every step
    xh = torch.from_numpy(host[13]).pin_memory()
    oh = torch.from_numpy(host[14]).pin_memory()
    lh = torch.empty(1, dtype=torch.float32).pin_memory()
    s = torch_stream()
    e_steps = max(2, min(K, 200))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e_steps):
        _lib.call("j4b_h2d", x.ptr, ctypes.c_void_p(xh.data_ptr()), xh.numel() * 4, s)
        _lib.call("j4b_h2d", onehot.ptr, ctypes.c_void_p(oh.data_ptr()), oh.numel() * 4, s)
        step(i, s)
        _lib.call("j4b_d2h", ctypes.c_void_p(lh.data_ptr()), loss.data_ptr(), 4, s)
    e1.record()
    barrier()
    e2e = world * e_steps / (e0.elapsed_time(e1) * 1e-3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, sample, _ = cpu_mlp_rate(batch, d_in, 10.0)
        cpu = {"value": round(rate, 5), "unit": "steps/s", "cores": 1, "kind": "port",
               "sample": sample + f" (host has {os.cpu_count()} cores)"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "steps/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(ms / K, 6), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": label, "batch": batch, "d_in": d_in, "hidden": MLP_HIDDEN,
                       "classes": MLP_CLASSES,
                       "tape": {"calls": st["calls"], "kernels": st["groups"], "folds": st["folds"],
                                "eager_steps": st["eager_steps"], "launches": st["launches"]},
                       "l2": "working set (5.7 MB) is L2-resident: a latency-bound step",
                       "parallelism": "replica" if world == 1 else f"{world} independent replicas",
                       "timing": "CUDA graph of K training steps (ping-pong parameter buffers), CUDA events"},
            "roofline": {"bound": "hbm", "achieved": round(min_bytes / (step_us * 1e-6) / 1e9, 1),
                         "peak": peak, "unit": "GB/s",
                         "frac": round(min_bytes / (step_us * 1e-6) / 1e9 / peak, 4), "traffic": None,
                         "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs",
                         "kernel": "the whole step (tape kernels + GEMMs)", "kernel_avg_us": round(step_us, 3),
                         "note": "latency-bound; min bytes / step time"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 2), "unit": "steps/s",
                    "h2d_bytes_per_step": host[13].nbytes + host[14].nbytes, "d2h_bytes_per_step": 4},
            "gpu_launches": K * st["launches"],
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                       "reasons": clk["reasons"], "samples": clk["samples"]},
        }
        print(json.dumps(line), flush=True)
    del main, warm
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_engine_tape(args):
    if args.config == "mlp_adam":
        return run_engine_mlp(args)
    return run_engine_workloads(args)


class EngineCtx:
    """Per-process engine state shared by the workloads one bench run measures: the device,
    the process group (N > 1), the backend and, created on first use, the peer-memory group."""

    def __init__(self):
        import torch
        import torch.distributed as dist
        sys.path.insert(0, HERE)
        from jax4j_b200.backend import B200Backend
        self.world, self.rank, self.local = dist_env()
        torch.cuda.set_device(self.local)
        if self.world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
        self.be = B200Backend(self.local)
        self.dev = torch.device("cuda", self.local)
        self._peers = None

    def peers(self):
        if self._peers is None:
            from jax4j_b200.peers import PeerGroup
            self._peers = PeerGroup(self.local, self.rank, self.world)
        return self._peers

    def barrier(self):
        import torch
        import torch.distributed as dist
        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(self, ms):
        import torch
        import torch.distributed as dist
        if self.world > 1:
            t = torch.tensor([ms], device=self.dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def close(self):
        import torch.distributed as dist
        if self.world > 1:
            if self._peers is not None:
                status = self._peers.status()
                self._peers.close()
                if status and self.rank == 0:
                    print("peer collective wait gave up", file=sys.stderr)
            dist.barrier()
            dist.destroy_process_group()


def timed_graph(ctx, step, K, W):
    """Captures W warm-up and K timed steps in CUDA graphs, soaks ~0.5 s so clocks reach their
    loaded state, then times the K-step graph with CUDA events on the launching stream between
    barriers (max over ranks) while nvidia-smi samples the clocks. Returns (ms, clocks)."""
    import torch

    def capture(n):
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step(0)  # warm the path on the capture stream
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            for i in range(n):
                step(i)
        return g

    warm, main = capture(W), capture(K)
    main.replay()  # the first replay of a graph also uploads it: keep that out of the timed one
    warm.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    soak_t0 = time.perf_counter()
    with ClockSampler(ctx.local) as clocks:
        while time.perf_counter() - soak_t0 < 0.5:
            warm.replay()
            torch.cuda.synchronize()
        ctx.barrier()
        start.record()
        main.replay()
        end.record()
        ctx.barrier()
        tail = time.perf_counter()  # keep sampling briefly so short timed regions get samples
        while time.perf_counter() - tail < 0.3:
            warm.replay()
            torch.cuda.synchronize()
    ms = ctx.max_over_ranks(start.elapsed_time(end))
    del main, warm
    return ms, clocks.summary()


def roofline_entry(achieved, kernel, kernel_avg_us, traffic_key):
    peak, peak_kind = measured_peaks()
    traffic, traffic_src = TRAFFIC.get(traffic_key, (None, "no ncu capture"))
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_source": traffic_src,
            "peak_source": f"{peak_kind} MEASURED_PEAKS.json hbm_gbs" if peak_kind == "measured" else "fallback 6.65 TB/s",
            "kernel": kernel, "kernel_avg_us": round(kernel_avg_us, 3)}


def clocks_entry(clk):
    return {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
            "samples": clk["samples"]}


def measure_gemv(ctx, name, K, W, cpu_budget):
    """One GEMV workload (CONFIGS[name]); returns its result entry (rank 0) or None."""
    import numpy as np
    import torch
    from jax4j_b200 import _lib
    from jax4j_b200.backend import torch_stream
    from jax4j_b200.prng import PrngKey
    be, world, rank = ctx.be, ctx.world, ctx.rank
    qtype, rows, cols, batch, label = CONFIGS[name]
    per_call = alg_bytes(qtype, rows, cols, batch)

    # ---- synthetic inputs, generated on the device by the engine (the keys of gemv_inputs_host) ----
    kx, kw = PrngKey.of(0).split(2)
    x = be.random_normal(kx.seed, kx.counter, (batch, cols))
    w32 = be.scalar("MUL", be.random_normal(kw.seed, kw.counter + rank * rows * cols, (rows, cols)), 0.02)
    blob = be.quantize(w32, qtype)
    l2 = torch.cuda.get_device_properties(ctx.dev).L2_cache_size
    copies = max(2, math.ceil(2 * l2 / blob.numel()))
    weights = [be.upload_quantized(blob, qtype, (rows, cols)) for _ in range(copies)]
    del w32, blob
    y = torch.empty(batch * rows, dtype=torch.float32, device=ctx.dev)
    y_all = torch.empty(world * batch * rows, dtype=torch.float32, device=ctx.dev) if world > 1 else None
    peers = ctx.peers() if world > 1 else None
    torch.cuda.synchronize()

    def gemv(i):
        _lib.call("j4b_quant_matvec", ctypes.c_void_p(weights[i % copies].handle), x.ptr, 0,
                  y.data_ptr(), batch, torch_stream())

    def step(i):
        if world > 1:  # the GEMV's epilogue stores into every rank's buffer over NVLink
            peers.allgather_matvec(weights[i % copies], x.ptr, y_all.data_ptr(), batch, torch_stream())
        else:
            gemv(i)

    from jax4j_b200 import diagnostics
    before = diagnostics()["dispatches"]
    step(0)  # one eager call: the engine's kernel launches per step
    launches = diagnostics()["dispatches"] - before
    ms, clk = timed_graph(ctx, step, K, W)
    kernel_ms = timed_graph(ctx, gemv, K, W)[0] if world > 1 else ms
    value = world * per_call * K / (ms * 1e-3) / 1e9
    kernel_avg_us = kernel_ms * 1e3 / K

    # ---- end to end through the public API: pinned host x in, y out, every step ----
    # host buffers in and out every step through the C ABI: j4b_quant_matvec_host (one GPU) or
    # j4b_quant_matvec_allgather_host (N GPUs), recorded per weight as a plan and replayed;
    # pinned buffers cross PCIe inside the kernels
    x_host = torch.from_numpy(np.ascontiguousarray(be.download(x))).pin_memory()
    y_host = torch.empty(world * batch * rows, dtype=torch.float32).pin_memory()
    e2e_steps = max(K, 200)
    stream = torch_stream()

    # a decode loop records each weight's host-buffer call once and replays it every step
    if world > 1:
        plans = [peers.allgather_matvec_host_plan(wq, x_host, y_host, batch, stream) for wq in weights]
    else:
        plans = [be.quant_matvec_host_plan(wq, x_host, y_host) for wq in weights]

    def e2e_step(i):
        plans[i % copies].run(stream)

    for i in range(3):  # warm the path
        e2e_step(i)
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record()
    for i in range(e2e_steps):
        e2e_step(i)
    e1.record()
    host_issue_s = time.perf_counter() - t0
    ctx.barrier()
    e_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * per_call * e2e_steps / (e_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and cpu_budget > 0:
        rate, sample, _ = cpu_matvec_rate(qtype, rows, cols, batch, 1, cpu_budget)
        cpu = {"value": round(rate, 4), "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": sample + f" (host has {os.cpu_count()} cores)"}
    del weights, plans
    if rank != 0:
        return None
    return {
        "name": name, "value": round(value, 2), "unit": "GB/s", "steps": K, "warmup": W,
        "ms_per_step": round(ms / K, 6), "higher_is_better": True,
        "config": gemv_config(name, world),
        "method": {"compute": "quant codes -> exact fp16 mma.sync operands, x split fp16 hi+lo, fp32 accumulate",
                   "l2": f"weights rotate over {copies} copies ({copies * per_call / 1e6:.0f} MB > 2x L2)",
                   "timing": "CUDA graph of K GEMV calls, CUDA events, max over ranks"},
        "roofline": roofline_entry(per_call / (kernel_avg_us * 1e-6) / 1e9, gemv_kernel_name(batch),
                                   kernel_avg_us, name),
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s",
                "h2d_bytes_per_step": batch * cols * 4, "d2h_bytes_per_step": world * batch * rows * 4,
                "call": "j4b_quant_matvec_host_run (a plan of j4b_quant_matvec_host" +
                        (")" if world == 1 else " over the peer group: j4b_quant_matvec_allgather_host)"),
                "host_issue_us_per_step": round(host_issue_s * 1e6 / e2e_steps, 2),
                "device_us_per_step": round(e_ms * 1e3 / e2e_steps, 2)},
        "gpu_launches": K * launches,
        "clocks": clocks_entry(clk),
    }


def measure_tape(ctx, name, K, W, cpu_budget):
    """The vmap-batched RMSNorm + SwiGLU value-and-gradient tape (TAPE_CONFIGS[name])."""
    import numpy as np
    import torch
    from jax4j_b200 import jit as J, nn
    from jax4j_b200 import _lib
    from jax4j_b200.backend import TapeHandle, torch_stream
    from jax4j_b200.prng import PrngKey
    be, world, rank = ctx.be, ctx.world, ctx.rank
    rows, cols, label = TAPE_CONFIGS[name]
    per_step = tape_alg_bytes(rows, cols)

    # ---- synthetic inputs on the device: x ~ N(0,1) [rows, cols] per rank, g = 1 + 0.1 N(0,1)
    kx, kg = PrngKey.of(0).split(2)
    x = be.random_normal(kx.seed, kx.counter + rank * rows * cols, (rows, cols))
    g = be.scalar("ADD", be.scalar("MUL", be.random_normal(kg.seed, kg.counter, (cols,)), 0.1), 1.0)

    # the tape: value and gradient of the mean of y^2 over the global batch (each rank's mean
    # scaled by 1/world, so the all-reduced sums are the global loss and dg)
    tape = J.trace(nn.rms_swiglu_value_and_grad_dp(world), [(rows, cols), (cols,)])
    handle = TapeHandle(be, tape)
    # dg and the loss share one buffer (loss right after dg, 16-byte aligned): one all-reduce
    red_len = cols + 4
    reduced = torch.empty(red_len, dtype=torch.float32, device=ctx.dev)
    dg, loss = reduced[:cols], reduced[cols:cols + 1]
    dx = torch.empty(rows * cols, dtype=torch.float32, device=ctx.dev)
    launches = handle.stats()["launches"]
    peers = ctx.peers() if world > 1 else None

    def step(i, xp=None, gp=None, s=None):
        s = torch_stream() if s is None else s
        handle.launch([x.ptr if xp is None else xp, g.ptr if gp is None else gp],
                      [loss.data_ptr(), dx.data_ptr(), dg.data_ptr()], s)
        if world > 1:  # rank-ordered sum over NVLink peer memory, in place (no NCCL call)
            peers.allreduce(reduced.data_ptr(), red_len, reduced.data_ptr(), s)

    ms, clk = timed_graph(ctx, step, K, W)
    step_us = ms * 1e3 / K
    value = world * K / (ms * 1e-3)

    # ---- end to end through the public API: pinned host x, g -> device, tape, loss -> host
    x_host = torch.from_numpy(np.ascontiguousarray(be.download(x))).pin_memory()
    g_host = torch.from_numpy(np.ascontiguousarray(be.download(g))).pin_memory()
    loss_host = torch.empty(1, dtype=torch.float32).pin_memory()
    xin, gin = be.full(0.0, (rows, cols)), be.full(0.0, (cols,))
    e2e_steps = max(3, min(K, 50))
    stream = torch_stream()
    ctx.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(e2e_steps):
        _lib.call("j4b_h2d", xin.ptr, ctypes.c_void_p(x_host.data_ptr()), x_host.numel() * 4, stream)
        _lib.call("j4b_h2d", gin.ptr, ctypes.c_void_p(g_host.data_ptr()), g_host.numel() * 4, stream)
        step(i, xin.ptr, gin.ptr, stream)
        _lib.call("j4b_d2h", ctypes.c_void_p(loss_host.data_ptr()), loss.data_ptr(), 4, stream)
    e1.record()
    ctx.barrier()
    e_ms = ctx.max_over_ranks(e0.elapsed_time(e1))
    e2e_value = world * e2e_steps / (e_ms * 1e-3)

    cpu = None
    if rank == 0 and world == 1 and cpu_budget > 0:
        rate, sample, _ = cpu_tape_rate(rows, cols, 1, cpu_budget)
        cpu = {"value": round(rate, 5), "unit": "steps/s", "cores": 1, "kind": "port",
               "sample": sample + f" (host has {os.cpu_count()} cores)"}
    if rank != 0:
        return None
    st = handle.stats()
    return {
        "name": name, "value": round(value, 2), "unit": "steps/s", "steps": K, "warmup": W,
        "ms_per_step": round(ms / K, 6), "higher_is_better": True,
        "config": tape_config(name, world),
        "method": {"tape": {"calls": st["calls"], "kernels": st["groups"], "folds": st["folds"],
                            "eager_steps": st["eager_steps"]},
                   "l2": f"inputs larger than L2 (x {rows * cols * 4 / 1e6:.0f} MB read, dx {rows * cols * 4 / 1e6:.0f} MB written per step)",
                   "timing": "CUDA graph of K tape replays, CUDA events, max over ranks"},
        "roofline": roofline_entry(per_step / (step_us * 1e-6) / 1e9,
                                   "j4b_group0 + j4b_group0_fold (the whole step)", step_us, name),
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_value, 3), "unit": "steps/s",
                "h2d_bytes_per_step": (rows * cols + cols) * 4, "d2h_bytes_per_step": 4},
        "gpu_launches": K * launches,
        "clocks": clocks_entry(clk),
    }


def engine_line(entry, world, secondary=None):
    """The contract's JSON line from a primary result entry (+ the secondary workloads)."""
    line = {"metric": METRIC, "value": entry["value"], "unit": entry["unit"], "n_gpus": world,
            "steps": entry["steps"], "warmup": entry["warmup"], "ms_per_step": entry["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": entry["config"], "method": entry["method"],
            "roofline": entry["roofline"], "cpu_baseline": entry["cpu_baseline"], "e2e": entry["e2e"],
            "gpu_launches": entry["gpu_launches"] + sum(s["gpu_launches"] for s in secondary or []),
            "clocks": entry["clocks"]}
    if secondary is not None:
        line["secondary"] = secondary
    return line


def run_engine_workloads(args):
    """GEMV and RMSNorm+SwiGLU tape workloads. The default run measures BASELINE configs[1]
    (q8_0_b8) as the line's value and the other headline workloads as `secondary` entries."""
    ctx = EngineCtx()
    names = [args.config] + (list(SECONDARY) if args.config == DEFAULT_CONFIG and not args.primary_only else [])
    entries = []
    for i, name in enumerate(names):
        budget = 0.0 if args.no_cpu_baseline else (10.0 if i == 0 else 6.0)
        if name in TAPE_CONFIGS:
            entries.append(measure_tape(ctx, name, args.steps, max(3, args.warmup), budget))
        else:
            entries.append(measure_gemv(ctx, name, args.steps, max(3, args.warmup), budget))
    if ctx.rank == 0:
        print(json.dumps(engine_line(entries[0], ctx.world, entries[1:] if len(entries) > 1 else None)), flush=True)
    ctx.close()
    return 0


def run_engine_gemm(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from jax4j_b200 import _lib
    from jax4j_b200.backend import B200Backend, torch_stream
    from jax4j_b200.prng import PrngKey

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    be = B200Backend(local)
    m, n, k, qtype, prec, label = GEMM_CONFIGS[args.config]
    flops = 2.0 * m * n * k
    dev = torch.device("cuda", local)
    kx, kw = PrngKey.of(0).split(2)
    x = be.random_normal(kx.seed, kx.counter + rank * m * k, (m, k))
    if qtype is not None:
        w32 = be.scalar("MUL", be.random_normal(kw.seed, kw.counter, (n, k)), 0.02)
        w = be.upload_quantized(be.quantize(w32, qtype), qtype, (n, k))
        del w32
    else:
        b = be.scalar("MUL", be.random_normal(kw.seed, kw.counter, (k, n)), 0.02)
    y = torch.empty(m * n, dtype=torch.float32, device=dev)

    def step(stream):
        if qtype is not None:
            _lib.call("j4b_quant_gemm", ctypes.c_void_p(w.handle), x.ptr, y.data_ptr(), m, prec, stream)
        else:
            _lib.call("j4b_matmul", x.ptr, b.ptr, y.data_ptr(), 1, m, k, n, prec, stream)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    K, W = args.steps, max(3, args.warmup)
    s = torch_stream()
    for _ in range(W):
        step(s)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for _ in range(K):
            step(s)
        end.record()
        barrier()
    clk = clocks.summary()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_ms = ms / K
    value = world * flops * K / (ms * 1e-3) / 1e12
    achieved = flops / (step_ms * 1e-3) / 1e12
    peaks_path = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(peaks_path):
        pk = json.load(open(peaks_path))
        peak, peak_src = float(pk["bf16_tflops_sustained"]), "measured MEASURED_PEAKS.json bf16_tflops_sustained"
    else:
        peak, peak_src = 1400.0, "fallback 1.4 PFLOP/s sustained"

    # end to end: x from pinned host memory every step, y back to the host
    x_host = torch.from_numpy(np.ascontiguousarray(be.download(x))).pin_memory()
    y_host = torch.empty(m * n, dtype=torch.float32).pin_memory()
    e_steps = max(2, min(K, 5))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        _lib.call("j4b_h2d", x.ptr, ctypes.c_void_p(x_host.data_ptr()), x_host.numel() * 4, s)
        step(s)
        _lib.call("j4b_d2h", ctypes.c_void_p(y_host.data_ptr()), y.data_ptr(), y_host.numel() * 4, s)
    e1.record()
    barrier()
    e_ms = e0.elapsed_time(e1)
    e2e = world * flops * e_steps / (e_ms * 1e-3) / 1e12

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, sample, _ = cpu_gemm_rate(m, n, k, qtype, 1, 10.0)
        cpu = {"value": round(rate, 6), "unit": "TFLOP/s", "cores": 1, "kind": "port",
               "sample": sample + f" (host has {os.cpu_count()} cores)"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if prec == 1 else "f32 (3-term bf16)",
            "data": "synthetic",
            "config": {"workload": label, "m": m, "n": n, "k": k, "precision": prec,
                       "l2": "operands larger than L2 (x 268 MB, y 940 MB)",
                       "parallelism": "replica" if world == 1 else f"{world} independent replicas",
                       "timing": "K back-to-back calls (operand decode/conversion included), CUDA events"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_src,
                         "kernel": ("qgemm_fused_kernel + x conversion (the whole call; the weight decoded "
                                    "inside the GEMM)" if qtype is not None
                                    else "tc_gemm_kernel + operand conversion (the whole call)"),
                         "kernel_avg_us": round(step_ms * 1e3, 1)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": m * k * 4,
                    "d2h_bytes_per_step": m * n * 4},
            "gpu_launches": K * 3,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                       "reasons": clk["reasons"], "samples": clk["samples"]},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------------------------
# convolution (ComputeBackend.conv2d)
# ------------------------------------------------------------------------------------------------

CONV_CONFIGS = {
    # name: (batch, ConvSpec ints (in_c, in_h, in_w, out_c, kernel, stride, pad), precision, label)
    "conv_resnet": (64, (64, 56, 56, 64, 3, 1, 1), 0, "conv2d forward, ResNet-style 3x3 layer: x [64, 64x56x56], "
                    "W [64, 64x3x3], stride 1, pad 1, fp32-accurate (3-term bf16 split on tcgen05)"),
}
CONV_METRIC = "conv2d TFLOP/s (2 x batch x outC x outH x outW x inC x k x k)"


def run_reference_conv(args):
    """The CPU conv2d (oracle restatement of CpuBackend.conv2d) on all host threads, one image per
    task, over a sample of the batch per step."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    sys.path.insert(0, HERE)
    from oracle import oracle as O
    batch, ints, prec, label = CONV_CONFIGS[args.config]
    c, h, w_, o, k, st, pd = ints
    oh, ow = (h + 2 * pd - k) // st + 1, (w_ + 2 * pd - k) // st + 1
    flops_img = 2.0 * o * oh * ow * c * k * k
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    sample = min(batch, threads)
    x = rng.standard_normal((sample, c * h * w_)).astype(np.float32)
    wt = (rng.standard_normal((o, c * k * k)) * 0.05).astype(np.float32)
    K, W = args.steps, max(3, args.warmup)
    times = []
    with ThreadPoolExecutor(threads) as ex:
        for i in range(K + 1):
            t0 = time.perf_counter()
            list(ex.map(lambda j: O.conv2d(x[j:j + 1], wt, ints), range(sample)))
            if i:
                times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    v = flops_img * sample / sec / 1e12
    print(json.dumps({"metric": CONV_METRIC, "value": round(v, 6), "unit": "TFLOP/s", "n_gpus": world, "steps": K,
                      "warmup": W, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak",
                      "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
                      "config": {"workload": label, "images_per_step": sample},
                      "cpu_baseline": {"value": round(v, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                                       "sample": f"{sample} images per step, one per thread"},
                      "e2e": {"value": round(v, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)
    return 0


def run_engine_conv(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from jax4j_b200.backend import B200Backend
    from jax4j_b200.prng import PrngKey
    from jax4j_b200.tensor import ConvSpec

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    be = B200Backend(local)
    batch, ints, prec, label = CONV_CONFIGS[args.config]
    spec = ConvSpec(*ints)
    flops = 2.0 * batch * spec.out_channels * spec.out_height * spec.out_width * spec.weight_size
    kx, kw = PrngKey.of(0).split(2)
    x = be.random_normal(kx.seed, kx.counter + rank * batch * spec.input_size, spec.input_shape(batch))
    w = be.scalar("MUL", be.random_normal(kw.seed, kw.counter, spec.weight_shape()), 0.05)
    dev = torch.device("cuda", local)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    K, W = args.steps, max(3, args.warmup)
    for _ in range(W):
        y = be.conv2d(x, w, spec, prec)
        del y
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for _ in range(K):
            y = be.conv2d(x, w, spec, prec)
        end.record()
        barrier()
    clk = clocks.summary()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_ms = ms / K
    value = world * flops * K / (ms * 1e-3) / 1e12
    peaks_path = os.path.join(HERE, "MEASURED_PEAKS.json")
    pk = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {}
    peak = float(pk.get("bf16_tflops_sustained", 1400.0))
    # end to end through the public call: x from pinned host memory, y back to the host, every step
    x_host = torch.from_numpy(np.ascontiguousarray(be.download(x))).pin_memory()
    y_host = torch.empty(tuple(y.shape), dtype=torch.float32).pin_memory()
    e_steps = max(2, min(K, 5))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        x.tensor.view(-1).copy_(x_host.view(-1), non_blocking=True)
        yy = be.conv2d(x, w, spec, prec)
        y_host.view(-1).copy_(yy.tensor.view(-1), non_blocking=True)
    e1.record()
    barrier()
    e2e = world * flops * e_steps / (e0.elapsed_time(e1) * 1e-3) / 1e12
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        xs = be.download(x)[:2]
        t0 = time.perf_counter()
        O.conv2d(xs, be.download(w), ints)
        sec = time.perf_counter() - t0
        cpu = {"value": round(flops / batch * 2 / sec / 1e12, 6), "unit": "TFLOP/s", "cores": 1, "kind": "port",
               "sample": f"2 of {batch} images, oracle restatement of CpuBackend.conv2d, 1 thread"}
    if rank == 0:
        achieved = flops / (step_ms * 1e-3) / 1e12
        line = {
            "metric": CONV_METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32 (3-term bf16)" if prec != 1 else "bf16", "data": "synthetic",
            "config": {"workload": label, "batch": batch, "spec": list(ints),
                       "l2": "patch matrix 462 MB > L2 per call",
                       "parallelism": "replica" if world == 1 else f"{world} independent replicas",
                       "timing": "K back-to-back calls (patch gather, tcgen05 GEMM, permute), CUDA events"},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_source": "measured MEASURED_PEAKS.json bf16_tflops_sustained",
                         "kernel": "conv2d call (im2col + tc_gemm + permute)", "kernel_avg_us": round(step_ms * 1e3, 1)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 3), "unit": "TFLOP/s", "h2d_bytes_per_step": batch * spec.input_size * 4,
                    "d2h_bytes_per_step": batch * spec.output_size * 4},
            "gpu_launches": None,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                       "reasons": clk["reasons"], "samples": clk["samples"]},
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------------------------
# scalar-AAD Monte-Carlo replay (the AadEngine SPI's CUDA engines)
# ------------------------------------------------------------------------------------------------

AAD_CONFIGS = {
    # name: (engine, paths per step, label)
    "aad_asian": ("cuda", 1 << 24, "scalar-AAD replay, engine cuda (generated kernel), FLOAT32: 64-step "
                  "arithmetic Asian call under GBM (408 nodes, 64 normal draws), value + 5 adjoints"),
    "aad_asian_interp": ("cuda-interp", 1 << 24, "scalar-AAD replay, engine cuda-interp (fixed interpreter), "
                         "FLOAT32: 64-step arithmetic Asian call under GBM, value + 5 adjoints"),
    "aad_asian_eager": ("cuda-eager", 1 << 21, "scalar-AAD replay, engine cuda-eager (one launch per node), "
                        "FLOAT32: 64-step arithmetic Asian call under GBM, value + 5 adjoints"),
}
AAD_STEPS = 64


def asian_tape(steps=AAD_STEPS):
    """Arithmetic-average Asian call under geometric Brownian motion (log-Euler steps):
    exp(-r T) max(mean_t S_t - K, 0); inputs S0, K, sigma, r, T."""
    from jax4j_b200.aad import AadRecorder

    def body(rec):
        s0, k, sig, r, t = (rec.input(n, v) for n, v in
                            (("S0", 100.0), ("K", 100.0), ("sigma", 0.2), ("r", 0.05), ("T", 1.0)))
        dt = t / steps
        drift = (r - sig * sig * 0.5) * dt
        vol = sig * dt.sqrt()
        s, total = s0, rec.constant(0.0)
        for _ in range(steps):
            s = s * (drift + vol * rec.randn()).exp()
            total = total + s
        rec.output(((total / steps - k).max(0.0)) * (r.neg() * t).exp())
    return AadRecorder.record(body)


def cpu_aad_rate(tape, budget_s, threads):
    """The CPU engine's replay (oracle restatement of ScalarReplay, double precision) on
    `threads` host threads over a sample sized to ~budget_s: paths/s."""
    sys.path.insert(0, HERE)
    from oracle import oracle
    args = (tape.ops, tape.arg_a, tape.arg_b, tape.constants, tape.recorded_inputs(), tape.input_nodes,
            tape.output_nodes, tape.rand_stream_count())
    n = 2000 * threads
    t0 = time.perf_counter()
    oracle.aad_replay(*args, n, 0, 42, True, threads)
    probe = time.perf_counter() - t0
    n = max(n, int(n * budget_s / max(probe, 1e-6)))
    t0 = time.perf_counter()
    oracle.aad_replay(*args, n, 0, 42, True, threads)
    return n / (time.perf_counter() - t0), n


def aad_inst_per_path(cfg):
    """Warp instructions per path of the engine's kernel from the committed ncu summary."""
    path = os.path.join(HERE, "profiles", f"{cfg}.md")
    if not os.path.exists(path):
        return None
    m = re.search(r"warp_instructions_per_path:\s*([0-9.]+)", open(path).read())
    return float(m.group(1)) if m else None


def run_reference_aad(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    engine, _, label = AAD_CONFIGS[args.config]
    tape = asian_tape()
    threads = os.cpu_count() or 1
    K, W = args.steps, max(3, args.warmup)
    rate, n = cpu_aad_rate(tape, 2.0, threads)  # warm-up + sizing
    times = []
    for _ in range(K):
        t0 = time.perf_counter()
        sys.path.insert(0, HERE)
        from oracle import oracle
        oracle.aad_replay(tape.ops, tape.arg_a, tape.arg_b, tape.constants, tape.recorded_inputs(),
                          tape.input_nodes, tape.output_nodes, 1, n, 0, 42, True, threads)
        times.append(time.perf_counter() - t0)
    sec = sum(times) / len(times)
    v = n / sec
    line = {"metric": AAD_METRIC, "value": round(v, 1), "unit": "paths/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic", "impl": "reference",
            "config": {"workload": label.replace("FLOAT32", "FLOAT64 CPU"), "paths_per_step": n},
            "cpu_baseline": {"value": round(v, 1), "unit": "paths/s", "cores": threads, "kind": "port",
                             "sample": f"{n} paths per step, oracle restatement of ScalarReplay on {threads} threads"},
            "e2e": {"value": round(v, 1), "unit": "paths/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


AAD_METRIC = "scalar-AAD Monte-Carlo replay paths/s (value + adjoints of every input)"


def run_engine_aad(args):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from jax4j_b200.aad import AadEngines, AadOptions, Precision
    from jax4j_b200.backend import torch_stream

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    engine, P, label = AAD_CONFIGS[args.config]
    tape = asian_tape()
    exe = AadEngines.require(engine, AadOptions(Precision.FLOAT32), local).compile(tape, AadOptions(Precision.FLOAT32))
    dev = torch.device("cuda", local)
    ins = torch.tensor(exe.inputs, dtype=torch.float64, device=dev)
    sums = torch.zeros(exe.channels, dtype=torch.float64, device=dev)
    s = torch_stream()
    K, W = args.steps, max(3, args.warmup)
    base = rank * (K + W + 8) * P  # disjoint scenario ranges per rank

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(W):
        exe.launch(ins.data_ptr(), P, base + i * P, 42, sums.data_ptr(), s)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for i in range(K):
            exe.launch(ins.data_ptr(), P, base + (W + i) * P, 42, sums.data_ptr(), s)
        end.record()
        barrier()
    clk = clocks.summary()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_ms = ms / K
    value = world * P * K / (ms * 1e-3)

    # end to end through the public call: host inputs up, host sums back, every step
    e_steps = max(2, min(K, 5))
    barrier()
    t0 = time.perf_counter()
    for i in range(e_steps):
        r = exe.replay(P, base + i * P, 43)
    e_sec = time.perf_counter() - t0
    e2e = world * P * e_steps / e_sec
    launches_per_step = 1 if engine != "cuda-eager" else None
    if engine == "cuda-eager":
        active = int(tape.active.sum())
        n_rev = sum(1 for i in range(tape.size()) if tape.active[i] and tape.op(i) > 3)
        chunks = -(-P // exe.threads_or_slot)
        launches_per_step = chunks * (tape.size() + 2 + 1 + n_rev + tape.input_count())
        del active

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, n = cpu_aad_rate(tape, 10.0, threads)
        cpu = {"value": round(rate, 1), "unit": "paths/s", "cores": threads, "kind": "port",
               "sample": f"{n} paths of the same tape, oracle restatement of ScalarReplay (double) on "
                         f"{threads} threads"}
    ipp = aad_inst_per_path(args.config)
    if rank == 0:
        clock_hz = (clk["sm_mhz"] or 1965.0) * 1e6
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        peak_issue = sms * 4 * clock_hz / 1e9  # warp instructions per second, 4 schedulers per SM
        achieved = ipp * P / (step_ms * 1e-3) / 1e9 if ipp else None
        line = {
            "metric": AAD_METRIC, "value": round(value, 1), "unit": "paths/s", "n_gpus": world,
            "steps": K, "warmup": W, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (f64 accumulation)", "data": "synthetic",
            "config": {"workload": label, "engine": engine, "paths_per_step": P, "nodes": tape.size(),
                       "value_check": round(r.value(), 6), "delta_S0": round(r.gradient("S0"), 6),
                       "l2": "no memory-resident inputs: draws are generated in-kernel from (path, seed)",
                       "parallelism": "replica" if world == 1 else f"{world} ranks, disjoint scenario ranges",
                       "timing": "K back-to-back launches on device buffers, CUDA events, max over ranks"},
            "roofline": {"bound": "issue", "achieved": round(achieved, 1) if achieved else None,
                         "peak": round(peak_issue, 1), "unit": "G warp-instructions/s",
                         "frac": round(achieved / peak_issue, 4) if achieved else None, "traffic": None,
                         "peak_source": f"{sms} SMs x 4 schedulers x measured median SM clock",
                         "kernel": {"cuda": "aad_replay (generated)", "cuda-interp": "aad_interp_kernel",
                                    "cuda-eager": "aad_eager_forward/reverse/reduce"}[engine],
                         "kernel_avg_us": round(step_ms * 1e3, 1)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 1), "unit": "paths/s", "h2d_bytes_per_step": 8 * tape.input_count(),
                    "d2h_bytes_per_step": 8 * exe.channels},
            "gpu_launches": K * launches_per_step,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                       "reasons": clk["reasons"], "samples": clk["samples"]},
        }
        print(json.dumps(line), flush=True)
    exe.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------------------------------------
# decoder block
# ------------------------------------------------------------------------------------------------

def cpu_decoder_rate(mode, blobs, g_attn, g_ffn, budget_s, threads):
    """Times the float64 oracle block (oracle/decoder.py) on a bounded sample: decode of one of the
    sequences against a 2048-token cache, or prefill of one 64-token sequence, with numpy's BLAS
    limited to `threads`. Returns (rate in the workload's unit, sample text, seconds per step)."""
    from threadpoolctl import threadpool_limits
    with threadpool_limits(threads):
        return _cpu_decoder_rate(mode, blobs, g_attn, g_ffn, budget_s)


def _cpu_decoder_rate(mode, blobs, g_attn, g_ffn, budget_s):
    import numpy as np
    sys.path.insert(0, HERE)
    from oracle.decoder import Block
    ref = Block(blobs, DEC_D, DEC_HEADS, DEC_FFN, g_attn, g_ffn)
    rng = np.random.default_rng(0)
    if mode == "decoder_decode":
        cached = 2048
        k = rng.standard_normal((1, DEC_HEADS, cached, 128)).astype(np.float16)
        v = rng.standard_normal((1, DEC_HEADS, cached, 128)).astype(np.float16)
        x = rng.standard_normal((1, DEC_D)).astype(np.float32)
        n, t0 = 0, time.perf_counter()
        while True:
            ref.decode(x, k, v, cached - 1)
            n += 1
            dt = time.perf_counter() - t0
            if dt >= budget_s:
                break
        per = decoder_weight_bytes() + decoder_kv_bytes(1, cached)
        return per * n / dt / 1e9, (f"{n} decode step(s) of 1 of 64 sequences (2048 cached tokens), float64 "
                                    "numpy oracle block"), dt / n
    seq = 64
    x = rng.standard_normal((seq, DEC_D)).astype(np.float32)
    n, t0 = 0, time.perf_counter()
    while True:
        ref.prefill(x, 1, seq)
        n += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s:
            break
    return (decoder_prefill_flops(1, seq) * n / dt / 1e12,
            f"{n} prefill(s) of one 64-token sequence, float64 numpy oracle block", dt / n)


def run_reference_decoder(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    import numpy as np
    sys.path.insert(0, HERE)
    from oracle import oracle as o
    batch, seq, label = DECODER_CONFIGS[args.config]
    # host-drawn weights with the oracle's encoder (no GPU on this arm)
    rng = np.random.default_rng(1)
    shapes = {"wqkv": (3 * DEC_D, DEC_D), "wo": (DEC_D, DEC_D), "wgu": (2 * DEC_FFN, DEC_D), "wd": (DEC_D, DEC_FFN)}
    blobs = {name: o.quantize(2, (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float32))
             for name, shape in shapes.items()}
    g_attn = (1 + 0.1 * rng.standard_normal(DEC_D)).astype(np.float32)
    g_ffn = (1 + 0.1 * rng.standard_normal(DEC_D)).astype(np.float32)
    threads = os.cpu_count() or 1
    budget = max(0.5, min(10.0, 90.0 / max(args.steps + args.warmup, 1)))
    for _ in range(min(args.warmup, 1)):
        cpu_decoder_rate(args.config, blobs, g_attn, g_ffn, budget, threads)
    rates, times, sample = [], [], ""
    for _ in range(min(args.steps, 5)):
        r, sample, dt = cpu_decoder_rate(args.config, blobs, g_attn, g_ffn, budget, threads)
        rates.append(r)
        times.append(dt)
    value = statistics.median(rates)
    unit = "GB/s" if args.config == "decoder_decode" else "TFLOP/s"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * statistics.median(times), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": label, "batch": batch, "seq": seq, "d_model": DEC_D, "heads": DEC_HEADS,
                   "ffn": DEC_FFN},
        "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_engine_decoder(args):
    import numpy as np
    import torch
    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from jax4j_b200 import _lib
    from jax4j_b200.backend import B200Backend, torch_stream
    from jax4j_b200.decoder import HEAD_DIM, DecoderBlock, DecoderWeights, KVCache
    from jax4j_b200.prng import PrngKey

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    be = B200Backend(local)
    batch, seq, label = DECODER_CONFIGS[args.config]
    if args.batch:
        batch, label = args.batch, label + f" (batch overridden to {args.batch})"
    decode = args.config == "decoder_decode"
    dev = torch.device("cuda", local)
    want_cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    # world > 1: tensor parallel, rank r holds heads and FFN rows [r/n, (r+1)/n) (strong scaling)
    w = DecoderWeights.random(be, DEC_D, DEC_HEADS, DEC_FFN, PrngKey.of(1), keep_blobs=want_cpu,
                              world=world, rank=rank)
    block = DecoderBlock(be, w)
    kx, kc = PrngKey.of(0).split(2)
    hl = w.heads
    cache = KVCache(be, batch, hl, seq)
    if decode:
        tokens = batch
        # cached keys/values of slots 0 .. seq - 2 ~ N(0, 1), drawn per sequence by the engine's
        # PRNG over all heads (so every world size sees the same cache), this rank's heads kept
        per = DEC_HEADS * seq * HEAD_DIM
        for b in range(batch):
            for dst in (cache.k, cache.v):
                r = be.random_normal(kc.seed, kc.counter + (2 * b + (dst is cache.v)) * per, (DEC_HEADS, seq, HEAD_DIM))
                dst[b] = r.tensor.view(DEC_HEADS, seq, HEAD_DIM)[rank * hl:(rank + 1) * hl].half()
        cache.k[:, :, seq - 1:] = 0
        cache.v[:, :, seq - 1:] = 0
        pos = seq - 1
        step_bytes = decoder_weight_bytes() + decoder_kv_bytes(batch, seq) + 2 * batch * DEC_D * 4
    else:
        tokens = batch * seq
        flops = decoder_prefill_flops(batch, seq)
    x = be.random_normal(kx.seed, kx.counter, (tokens, DEC_D))
    torch.cuda.synchronize()

    def step():
        return block.decode(x, cache, pos) if decode else block.prefill(x, cache, seq, 1)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    K, W = args.steps, max(3, args.warmup)
    for _ in range(W):
        step()
    barrier()
    graph = None
    if decode and world == 1:
        # decode steps replay from a CUDA graph (no host work between the ~12 launches of a step)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(K):
                step()
        graph.replay()  # the first replay of a graph also uploads it: keep that out of the timed one
        torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        if graph is not None:
            graph.replay()
        else:
            for _ in range(K):
                step()
        end.record()
        barrier()
    clk = clocks.summary()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_ms = ms / K
    peaks_path = os.path.join(HERE, "MEASURED_PEAKS.json")
    pk = json.load(open(peaks_path)) if os.path.exists(peaks_path) else {}

    # dominant kernel alone
    s = torch_stream()
    if decode:
        q = torch.randn(batch * DEC_HEADS * HEAD_DIM, device=dev)
        att = torch.empty(batch * DEC_D, device=dev)
        reps = 20
        for _ in range(3):
            _lib.call("j4b_attention_decode", q.data_ptr(), cache.k.data_ptr(), cache.v.data_ptr(), batch,
                      hl, HEAD_DIM, seq, seq, att.data_ptr(), s)
        torch.cuda.synchronize()
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record()
        for _ in range(reps):
            _lib.call("j4b_attention_decode", q.data_ptr(), cache.k.data_ptr(), cache.v.data_ptr(), batch,
                      hl, HEAD_DIM, seq, seq, att.data_ptr(), s)
        k1.record()
        torch.cuda.synchronize()
        kern_us = k0.elapsed_time(k1) * 1e3 / reps
        kv = decoder_kv_bytes(batch, seq) // world + 2 * batch * hl * HEAD_DIM * 4
        peak = float(pk.get("hbm_gbs", 6650.0))
        roof = {"bound": "hbm", "achieved": round(kv / (kern_us * 1e-6) / 1e9, 1), "peak": peak, "unit": "GB/s",
                "frac": round(kv / (kern_us * 1e-6) / 1e9 / peak, 4), "traffic": None,
                "peak_source": "measured MEASURED_PEAKS.json hbm_gbs" if pk else "fallback",
                "kernel": f"attn_decode_kernel ({batch} x {hl} heads x {seq} cached tokens of f16 K and V per launch)",
                "kernel_avg_us": round(kern_us, 1)}
        value = step_bytes / (step_ms * 1e-3) / 1e9  # the whole block's bytes: strong scaling
        unit = "GB/s"
    else:
        peak = float(pk.get("bf16_tflops_sustained", 1400.0))
        achieved = flops / (step_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4), "traffic": None,
                "peak_source": "measured MEASURED_PEAKS.json bf16_tflops_sustained" if pk else "fallback 1.4 PFLOP/s",
                "kernel": "the whole prefill step (qgemm_fused_kernel projections hold ~97% of its flops)",
                "kernel_avg_us": round(step_ms * 1e3, 1)}
        value = flops / (step_ms * 1e-3) / 1e12
        unit = "TFLOP/s"

    # end to end through the public API: x from pinned host memory, the block output back
    x_host = torch.from_numpy(np.ascontiguousarray(be.download(x))).pin_memory()
    y_host = torch.empty(tokens * DEC_D, dtype=torch.float32).pin_memory()
    e_steps = max(2, min(K, 20 if decode else 3))
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        _lib.call("j4b_h2d", x.ptr, ctypes.c_void_p(x_host.data_ptr()), x_host.numel() * 4, s)
        y = step()
        _lib.call("j4b_d2h", ctypes.c_void_p(y_host.data_ptr()), y.ptr, y_host.numel() * 4, s)
    e1.record()
    barrier()
    e_s = e0.elapsed_time(e1) * 1e-3
    e2e = (step_bytes / 1e9 if decode else flops / 1e12) * e_steps / e_s

    cpu = None
    if want_cpu:
        blobs = {k2: v2.cpu().numpy() for k2, v2 in w.blobs.items()}
        rate, sample, _ = cpu_decoder_rate(args.config, blobs, be.download(w.g_attn), be.download(w.g_ffn), 10.0, 1)
        cpu = {"value": round(rate, 6), "unit": unit, "cores": 1, "kind": "port",
               "sample": sample + f", 1 BLAS thread (host has {os.cpu_count()} cores)"}
    if rank == 0:
        cfg = {"workload": label, "batch": batch, "seq" if not decode else "cached_tokens": seq, "d_model": DEC_D,
               "heads": DEC_HEADS, "head_dim": HEAD_DIM, "ffn": DEC_FFN, "quant": "Q4_0",
               "parallelism": "single GPU" if world == 1 else
               f"tensor parallel tp{world}: heads and FFN rows sharded, 2 NCCL all-reduces of [tokens, d] per step",
               "l2": "weights 137 MB and KV cache 2.1 GB exceed L2" if decode else "activations exceed L2"}
        if decode:
            cfg["tokens_per_s"] = round(world * batch / (step_ms * 1e-3), 1)
            cfg["bytes_per_step"] = step_bytes
            cfg["timing"] = ("CUDA graph of K decode steps, CUDA events" if world == 1 else
                             "K eager decode steps (NCCL all-reduces between), CUDA events, max over ranks")
        else:
            cfg["flop_per_step"] = flops
            cfg["timing"] = "K back-to-back prefill steps, CUDA events"
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": unit, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(step_ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32 (Q4_0 weights, f16 KV)" if decode else "bf16 (Q4_0 weights, f16 attention)",
            "data": "synthetic", "config": cfg, "roofline": roof, "cpu_baseline": cpu,
            "e2e": {"value": round(e2e, 3), "unit": unit, "h2d_bytes_per_step": tokens * DEC_D * 4,
                    "d2h_bytes_per_step": tokens * DEC_D * 4},
            "gpu_launches": K * (21 if decode else 19),
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"],
                       "samples": clk["samples"]},
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_engine(args):
    if args.config in CONV_CONFIGS:
        return run_engine_conv(args)
    if args.config in AAD_CONFIGS:
        return run_engine_aad(args)
    if args.config in DECODER_CONFIGS:
        return run_engine_decoder(args)
    if args.config in TAPE_CONFIGS:
        return run_engine_tape(args)
    if args.config in GEMM_CONFIGS:
        return run_engine_gemm(args)
    return run_engine_workloads(args)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None, help="timed steps (default per workload)")
    p.add_argument("--warmup", type=int, default=None, help="warm-up steps (default per workload)")
    p.add_argument("--impl", choices=["engine", "reference"], default="engine")
    p.add_argument("--config", choices=sorted(CONFIGS) + sorted(TAPE_CONFIGS) + sorted(GEMM_CONFIGS)
                   + sorted(DECODER_CONFIGS) + sorted(AAD_CONFIGS) + sorted(CONV_CONFIGS), default=DEFAULT_CONFIG)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--primary-only", action="store_true",
                   help="default config: measure q8_0_b8 alone, without the secondary workloads")
    p.add_argument("--batch", type=int, default=None,
                   help="decoder workloads only: override the batch (e.g. a smaller case for profiling)")
    args = p.parse_args()
    family = ("tape" if args.config in TAPE_CONFIGS else "gemm" if args.config in GEMM_CONFIGS
              else args.config if args.config in DECODER_CONFIGS
              else ("aad_eager" if args.config == "aad_asian_eager" else "aad") if args.config in AAD_CONFIGS
              else "gemm" if args.config in CONV_CONFIGS
              else "gemv")
    steps, warmup = DEFAULT_STEPS[family]
    args.steps = steps if args.steps is None else args.steps
    args.warmup = warmup if args.warmup is None else args.warmup
    if args.impl == "reference":
        return run_reference(args)
    return run_engine(args)


if __name__ == "__main__":
    sys.exit(main())
