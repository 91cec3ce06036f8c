#!/usr/bin/env python
"""Benchmark of the int4 / int8 weight-only dequant-matvec hot path on B200.

Workload (one step): one decode token through LAYERS=32 resident int4 MLP
pairs, each layer's output feeding the next layer's input: up [4096 x 11008]
then down [11008 x 4096], group-64 scales, M=1 activation row, fp32
accumulation (x0 -> up_0 -> h -> down_0 -> x1 -> up_1 -> ...). 32 distinct
weight copies (1.63 GB) are streamed per step, so every matvec reads HBM, not
L2 (126 MB).

  value    algorithmic GB/s over the device-timed region (CUDA events, max over
           ranks), bytes per matvec = codes + scales + x + out (each once). The
           step is 64 single-call matvec launches (tq_matmul_dev: the tensor-core
           kernel cmv_kernel<4,1,true>, one launch per matvec) in one CUDA graph.
  e2e      the same bytes through the C-ABI MatVec entry point (tq_matvec) with
           host buffers, one call per matvec as the Go MatVec makes them: every
           call copies x host->device and out device->host, and each call's
           output is the next call's input
  roofline the matvec kernel's achieved GB/s: algorithmic bytes of one launch
           over its mean device time (CUDA events on the launching stream around
           the step's 64 launches), against the measured HBM copy bandwidth
  chain    the same dependent workload as ONE launch of the chain kernel
           (tq_chain_run), for comparison
  cpu_baseline  the CPU oracle (AVX2 restatement of quant4_simd.go with the
           reference's worker split) on the host cores, bounded sample

`--impl reference` times the reference's CPU implementation of the path (the
oracle's AVX2 restatement; the Go reference cannot be built here) on the same
config. Under torchrun (N>1) every rank streams its own copy of the workload
(replicas, weak scaling); the kernels exchange nothing.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "int8/int4 dequant-matvec HBM GB/s (% of peak); decode tokens/s at 1/2/4/8 GPU"
K_UP, N_UP = 4096, 11008
LAYERS = 32
FALLBACK_HBM_GBS = 6650.0
WORKLOAD = ("int4 g64 MLP pair (up 4096x11008 + down 11008x4096), M=1, fp32 accumulate; "
            "32 resident layer copies streamed per step, each layer's output the next one's input")


def algo_bytes(bits: int, rows: int, cols: int, m: int) -> int:
    """Codes + scales + x + out, each counted once."""
    codes = rows * cols if bits == 8 else rows * cols // 2
    scales = cols * 4 if bits == 8 else ((rows + 63) // 64) * cols * 4
    return codes + scales + 4 * m * rows + 4 * m * cols


def pair_bytes(m: int = 1) -> int:
    return algo_bytes(4, K_UP, N_UP, m) + algo_bytes(4, N_UP, K_UP, m)


def load_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def load_traffic():
    """Per-launch DRAM bytes (read + write) of the matvec kernel from the
    committed ncu summary of the same workload (its
    `traffic_bytes_per_launch:` line), or None."""
    import re
    path = os.path.join(ROOT, "profiles", "tmv_int4_m1_mlp_pair.md")
    try:
        with open(path) as f:
            m = re.search(r"traffic_bytes_per_launch:\s*(\d+)", f.read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, index: int, period: float = 0.01):
        self.index, self.period = index, period
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for b, name in self.REASONS.items():
                    if bits & b:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml"}


# ---------------------------------------------------------------------------
# CPU side (oracle): the reference's algorithm on the host cores
# ---------------------------------------------------------------------------

def cpu_pairs(npairs: int, seed: int = 1):
    from oracle import oracle as O
    pairs = []
    for l in range(npairs):
        up = O.quantize4(O.synth((K_UP, N_UP), seed, 2 * l, 0.02))
        down = O.quantize4(O.synth((N_UP, K_UP), seed, 2 * l + 1, 0.02))
        pairs.append((up, down))
    x_up = O.synth((K_UP,), seed, 1000, 1.0)
    x_down = O.synth((N_UP,), seed, 1001, 1.0)
    return pairs, x_up, x_down


def cpu_pair_pass(pairs, x_up, x_down, l):
    from oracle import oracle as O
    (qu, su), (qd, sd) = pairs[l % len(pairs)]
    O.q4_matmul(qu, su, K_UP, N_UP, x_up, O.AVX2)
    O.q4_matmul(qd, sd, N_UP, K_UP, x_down, O.AVX2)


def cpu_baseline(seconds: float = 8.0):
    """Oracle AVX2 MatVec on all host threads, 2 alternating pairs (100 MB,
    beyond the last-level cache), run for about `seconds`."""
    from oracle import oracle as O
    threads = O.set_threads(0)
    pairs, xu, xd = cpu_pairs(2)
    for l in range(2):
        cpu_pair_pass(pairs, xu, xd, l)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        cpu_pair_pass(pairs, xu, xd, n)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": round(pair_bytes() * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} MLP-pair passes (up+down, M=1) over 2 alternating resident pairs (101.7 MB), "
                      f"{dt:.1f} s, oracle AVX2 restatement of quant4_simd.go with the reference worker split"}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    from oracle import oracle as O
    threads = O.set_threads(0)
    pairs, xu, xd = cpu_pairs(2)
    for w in range(max(args.warmup, 1)):
        cpu_pair_pass(pairs, xu, xd, w)
    t0 = time.perf_counter()
    for s in range(args.steps):
        cpu_pair_pass(pairs, xu, xd, s)
    dt = time.perf_counter() - t0
    value = pair_bytes() * args.steps / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Irwin-Hall normal: weights std 0.02, activations std 1)",
        "config": bench_config(),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "each step = one MLP pair (up+down, M=1), alternating between 2 resident "
                                   "pairs (101.7 MB); the Go reference cannot be built here (no Go "
                                   "toolchain), so its AVX2 kernel runs as the oracle's C restatement"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# Side measurements of the other kernel configs (device time per call, CUDA
# graph of back-to-back calls over enough distinct weight copies to exceed L2).
# A config is one matrix shape, or the MLP pair (up then down, the down call
# reading the up call's output).
SIDE_CONFIGS = [
    # name, bits, [(rows, cols), ...], m
    ("C1 int8 4096x4096 M=1", 8, [(4096, 4096)], 1),
    ("C2 int4 MLP pair M=4", 4, [(K_UP, N_UP), (N_UP, K_UP)], 4),
    ("C2 int4 MLP pair M=8", 4, [(K_UP, N_UP), (N_UP, K_UP)], 8),
    ("C3 int4 4096x4096 M=64 (tf32)", 4, [(4096, 4096)], 64),
]


def side_cpu_baseline(bits, shapes, m, seconds=1.5):
    """The oracle's AVX2 MatVec on all host threads over the config's shapes
    (m rows = m MatVec calls, as quant.go:77 is applied per row)."""
    from oracle import oracle as O
    threads = O.set_threads(0)
    mats = []
    for i, (r, c) in enumerate(shapes):
        w = O.synth((r, c), 7, 300 + i, 0.02)
        mats.append(((O.quantize8 if bits == 8 else O.quantize4)(w), r, c))
    xs = [O.synth((m, r), 7, 299, 1.0) for _, r, _ in mats]
    fn = O.q8_matmul if bits == 8 else O.q4_matmul
    per = sum(algo_bytes(bits, r, c, m) for _, r, c in mats)

    def one():
        for ((q, sc), r, c), x in zip(mats, xs):
            fn(q, sc, r, c, x, O.AVX2)

    one()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        one()
        n += 1
    dt = time.perf_counter() - t0
    rec = {"value": round(per * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
           "sample": f"{n} passes over the config's matrices ({m} rows each), {dt:.2f} s, oracle AVX2 "
                     f"restatement of quant_simd.go / quant4_simd.go with the reference worker split"}
    if m >= 16:
        flops = sum(2.0 * m * r * c for _, r, c in mats)
        rec["TFLOP/s"] = round(flops * n / dt / 1e12, 4)
    return rec


def measure_side_configs(L, Q, torch, stream, peak, only=None, cpu=False):
    out = {}
    sp = ctypes.c_void_p(stream.cuda_stream)
    for name, bits, shapes, m in SIDE_CONFIGS:
        if only and not name.startswith(only + " "):
            continue
        per = sum(algo_bytes(bits, r, c, m) for r, c in shapes)
        code_bytes = sum(r * c // (1 if bits == 8 else 2) for r, c in shapes)
        copies = max(2, int(160e6 // code_bytes) + 1)  # > L2 in total
        hs = []
        for i in range(copies):
            for j, (r, c) in enumerate(shapes):
                w = torch.empty(r, c, device="cuda")
                Q.synth_dev(w, 7, 100 + len(shapes) * i + j, 0.02)
                hs.append(Q.quantize_dev(w, bits))
                del w
        bufs = [torch.empty(m, shapes[0][0], device="cuda")] + [torch.empty(m, c, device="cuda") for _, c in shapes]
        Q.synth_dev(bufs[0], 7, 99, 1.0)
        ptr = [ctypes.c_void_p(b.data_ptr()) for b in bufs]
        torch.cuda.synchronize()

        def calls():
            for i in range(copies):
                for j in range(len(shapes)):
                    L.tq_matmul_dev(hs[len(shapes) * i + j], ptr[j], ptr[j + 1], m, sp)

        with torch.cuda.stream(stream):
            for i in range(copies):
                for j in range(len(shapes)):
                    _check_rc(L, L.tq_matmul_dev(hs[len(shapes) * i + j], ptr[j], ptr[j + 1], m, sp))
        torch.cuda.synchronize()
        reps = 4
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(reps):
                calls()
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * copies)  # per pass over the config's shapes
        rec = {"us_per_pass": round(us, 3), "GB/s": round(per / us / 1e3, 1),
               "frac_hbm": round(per / us / 1e3 / peak, 4), "algorithmic_bytes": per,
               "weight_copies": copies, "calls_per_pass": len(shapes)}
        if m >= 16:
            rec["TFLOP/s"] = round(sum(2.0 * m * r * c for r, c in shapes) / us / 1e6, 2)
        del g
        for h in hs:
            Q.free(h)
        if cpu:
            rec["cpu_baseline"] = side_cpu_baseline(bits, shapes, m)
        out[name] = rec
    return out


GPT2_PROMPT, GPT2_GEN = 128, 256


def measure_gpt2(cpu: bool):
    """GPT-2-small int8 greedy decode (128-token prompt, 256 tokens): device
    time of the fp32 prefill and of the 255 decode steps (one CUDA graph per
    token). With cpu=True also the oracle's decode rate on the host cores over
    a bounded 32-token sample."""
    from tensai_b200.decode import GPT2_SMALL, Gpt2, synth_tokens
    prompt = synth_tokens(GPT2_PROMPT, GPT2_SMALL["vocab"], 1)
    with Gpt2(GPT2_SMALL, 1) as m:
        m.generate(prompt, 16)  # warm-up: kernel set-up and the step graph
        m.generate(prompt, GPT2_GEN)
        pre_ms, dec_ms = m.last_times_ms
    rec = {"decode_tok_s": round((GPT2_GEN - 1) / (dec_ms * 1e-3), 1), "ms_per_token": round(dec_ms / (GPT2_GEN - 1), 4),
           "prefill_ms": round(pre_ms, 3), "prompt": GPT2_PROMPT, "generated": GPT2_GEN,
           "algorithmic_bytes_per_token": "124,064,836 + 73,728 x cached positions",
           "weights": "random-init N(0, 0.02), int8 QuantizeMatrix decode weights, fp32 prefill"}
    if cpu:
        from oracle import oracle as O
        secs = [0.0, 0.0]
        O.gpt2_generate(O.GPT2_SMALL, 1, 0.02, prompt, 33, seconds=secs)
        rec["cpu_baseline"] = {"decode_tok_s": round(32 / secs[1], 2), "cores": O.set_threads(0), "kind": "port",
                               "sample": "32 decode steps after the 128-token prompt, oracle restatement of the "
                                         "-q8 loop (AVX2 int8 MatVec, float64 attention)"}
    return rec


def measure_quant_load(cpu: bool):
    """Quantize-on-load of every Qwen2.5-7B int4 matrix (per layer q|k|v
    3584x4608, o 3584x3584, gate|up 3584x37888, down 18944x3584; the lm head
    3584x152064) from device-resident BF16 Linear weights [out, in]
    (tq_quantize4_linear_dev: the loader's transpose and widening fused into
    QuantizeMatrix4). Wall time of the 197 calls with a final synchronize,
    allocation of the handles included. With cpu=True also the oracle's
    QuantizeMatrix4 on the host for one layer's four matrices, extrapolated
    to the model by parameters."""
    import torch
    from tensai_b200 import quant as Q
    d, kv, f, v = 3584, 512, 18944, 152064
    shapes = [(d + 2 * kv, d), (d, d), (2 * f, d), (d, f)] * 28 + [(v, d)]  # [out, in]
    params = sum(a * b for a, b in shapes)
    buf = torch.empty(max(a * b for a, b in shapes), device="cuda", dtype=torch.bfloat16)
    buf.normal_(0.0, 0.02)
    torch.cuda.synchronize()
    hs = [Q.quantize_linear_dev(buf[: a * b].view(a, b), 4) for a, b in shapes[:4]]  # warm-up (kernel set-up)
    torch.cuda.synchronize()
    for h in hs:
        Q.free(h)
    t0 = time.perf_counter()
    hs = [Q.quantize_linear_dev(buf[: a * b].view(a, b), 4) for a, b in shapes]
    torch.cuda.synchronize()
    secs = time.perf_counter() - t0
    for h in hs:
        Q.free(h)
    del buf
    torch.cuda.empty_cache()
    rec = {"seconds": round(secs, 4), "params": params, "bf16_GB_read": round(2 * params / 1e9, 3),
           "GB/s_of_bf16": round(2 * params / secs / 1e9, 1),
           "what": "197 int4 matrices of the 7B shape from device BF16 [out, in] weights: transpose, widening and "
                   "QuantizeMatrix4 in one kernel, plus the K-packed copy; handle allocation included"}
    if cpu:
        from oracle import oracle as O
        threads = O.set_threads(0)
        sample = shapes[:4]
        t = 0.0
        for a, b in sample:
            w = O.synth((b, a), 5, a, 0.02)  # the transposed f32 matrix the loader quantizes
            t1 = time.perf_counter()
            O.quantize4(w)
            t += time.perf_counter() - t1
        sp = sum(a * b for a, b in sample)
        rec["cpu_baseline"] = {"seconds": round(t * params / sp, 2), "cores": threads, "kind": "port",
                               "sample": f"one layer's four matrices ({sp} parameters, {t:.2f} s) through the oracle's "
                                         "QuantizeMatrix4 on all host threads (the reference's runs on one), "
                                         "extrapolated to the model by parameters; the BF16 widening and "
                                         "transpose not counted"}
    return rec


QWEN_PROMPT, QWEN_GEN = 2048, 512
QWEN_BYTES_PER_TOKEN = 3_977_035_776  # int4 codes + scales streamed per token (all layers + lm head)


def measure_qwen(rank: int, world: int, peak: float, cpu: bool = False):
    """Qwen2.5-7B-shaped int4 greedy decode, tensor parallel over the job's
    GPUs (one rank per GPU): the 2048-token prompt through the decode step,
    then 512 tokens. Decode tokens/s from the device time of the 511 later
    steps, max over ranks. Every rank must call this (collective)."""
    import torch
    import torch.distributed as dist

    from tensai_b200.decode import QWEN_7B, Qwen, broadcast_nccl_id, synth_tokens
    prompt = synth_tokens(QWEN_PROMPT, QWEN_7B["vocab"], 1)
    nid = broadcast_nccl_id(dist) if world > 1 else None
    with Qwen(QWEN_7B, 1, 0.02, rank, world, nid) as m:
        exchange = m.exchange
        toks = m.generate(prompt, QWEN_GEN)
        pre_ms, dec_ms = m.last_times_ms
        # the same run with the prompt in 64-row chunks on the tf32 matmul
        # (tq_qwen_set_prefill); every rank takes the same branch
        btoks, bpre_ms, bwhy = None, 0.0, ""
        try:
            m.set_prefill(64)
            ok = 1
        except Exception as e:  # a shard layout the batched prefill does not take
            ok, bwhy = 0, str(e)
        flag = torch.tensor([ok], device="cuda", dtype=torch.int32)
        if world > 1:
            dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()):
            btoks = m.generate(prompt, QWEN_GEN)
            bpre_ms = m.last_times_ms[0]
        elif not bwhy:
            bwhy = "another rank's shard layout does not take the batched prefill"
    t = torch.tensor([pre_ms, dec_ms, bpre_ms], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    pre_ms, dec_ms, bpre_ms = float(t[0]), float(t[1]), float(t[2])
    tok_s = (QWEN_GEN - 1) / (dec_ms * 1e-3)
    bound = world * peak * 1e9 / QWEN_BYTES_PER_TOKEN
    rec = {"tp": world, "exchange": exchange, "decode_tok_s": round(tok_s, 2), "ms_per_token": round(dec_ms / (QWEN_GEN - 1), 4),
            "prompt_ms": round(pre_ms, 1), "prompt_tok_s": round(QWEN_PROMPT / (pre_ms * 1e-3), 1),
            "roofline": {"bound": "aggregate hbm", "tok_s_bound": round(bound, 1), "frac": round(tok_s / bound, 4),
                         "bytes_per_token": QWEN_BYTES_PER_TOKEN, "peak_gbs_per_gpu": peak},
            "first_tokens": [int(x) for x in toks[:8]]}
    if btoks is not None:
        same = np.asarray(btoks) == np.asarray(toks)
        rec["batched_prefill"] = {"rows": 64, "prompt_ms": round(bpre_ms, 1),
                                  "prompt_tok_s": round(QWEN_PROMPT / (bpre_ms * 1e-3), 1),
                                  "ids_equal_to_token_by_token": int(same.sum()), "of": len(same),
                                  "first_equal_in_a_row": int(np.argmin(same)) if not same.all() else len(same)}
    else:
        rec["batched_prefill"] = {"unavailable": bwhy}
    golden = os.path.join(ROOT, "tests", "golden", "qwen7b_decode_golden_2048_512.npz")
    if os.path.exists(golden):  # the oracle's greedy ids for this prompt and seed (TP does not change them)
        g = np.load(golden)
        if np.array_equal(g["prompt"], prompt):
            rec["tokens_match_golden"] = bool(np.array_equal(np.asarray(toks[:len(g["tokens"])]), g["tokens"]))
    if cpu and rank == 0:
        # the oracle's -q4 step on this box's cores at the mean decode position
        # of the run (prompt + half the generated tokens), a few steps timed
        from oracle import oracle as O
        threads = O.set_threads(0)
        pos0, n = QWEN_PROMPT + QWEN_GEN // 2, 3
        secs, build = O.qwen_time_steps(QWEN_7B, pos0, n)
        rec["cpu_baseline"] = {"decode_tok_s": round(n / secs, 3), "cores": threads, "kind": "port",
                               "sample": f"{n} decode steps at cached positions {pos0}..{pos0 + n - 1} of the 7B shape "
                                         f"({secs:.2f} s), oracle restatement of the -q4 step (AVX2 int4 MatVec, "
                                         "float64 attention) with filler weights; tokens/s extrapolated from the "
                                         "per-step time at the run's mean context"}
    return rec


def _check_rc(L, rc):
    if rc:
        raise RuntimeError(L.tq_last_error().decode())


def bench_config():
    return {"workload": WORKLOAD.replace("32 resident", f"{LAYERS} resident"), "weights": "int4 group-64 (QuantizeMatrix4 layout)", "m": 1,
            "layers_per_step": LAYERS, "bytes_per_step": pair_bytes() * LAYERS,
            "l2": f"inputs larger than L2: {pair_bytes() * LAYERS / 1e9:.2f} GB of weights streamed per step",
            "launch": "one CUDA graph replay per step"}


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------

def run_gpu(args, rank: int, world: int):
    import torch
    import torch.distributed as dist

    from tensai_b200 import _lib
    from tensai_b200 import quant as Q

    dev = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(dev)
    L = _lib.load()
    _lib.check(L.tq_set_device(dev))
    if args.kernel is not None:
        _lib.check(L.tq_set_matvec_kernel(args.kernel))

    # Resident weights: generated and quantized on the device.
    handles = []
    tmp = torch.empty(K_UP * N_UP, device="cuda", dtype=torch.float32)
    for l in range(LAYERS):
        for j, (r, c) in enumerate(((K_UP, N_UP), (N_UP, K_UP))):
            w = tmp.view(r, c)
            Q.synth_dev(w, 1, 2 * l + j, 0.02)
            handles.append(Q.quantize_dev(w, 4))
    torch.cuda.synchronize()
    del tmp
    # x0 -> up_0 -> h -> down_0 -> xa -> up_1 -> h -> ... (the step's dataflow)
    x0 = torch.empty(K_UP, device="cuda")
    Q.synth_dev(x0, 1, 1000, 1.0)
    h = torch.empty(N_UP, device="cuda")
    xa = torch.empty(K_UP, device="cuda")
    ops = []
    for l in range(LAYERS):
        ops.append({"handle": handles[2 * l], "x": x0 if l == 0 else xa, "out": h})
        ops.append({"handle": handles[2 * l + 1], "x": h, "out": xa})
    chain = Q.Chain(ops)

    stream = torch.cuda.Stream()
    sp = ctypes.c_void_p(stream.cuda_stream)
    mm = L.tq_matmul_dev

    def chain_step():
        chain.run(stream)

    def single_step():
        for o in ops:
            rc = mm(o["handle"], ctypes.c_void_p(o["x"].data_ptr()), ctypes.c_void_p(o["out"].data_ptr()), 1, sp)
            if rc:
                _lib.check(rc)

    def capture(fn):
        with torch.cuda.stream(stream):
            fn()  # kernel set-up and the stream's scratch, outside the capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        torch.cuda.synchronize()
        return g

    def timed(g, steps, sample_clocks=False):
        for _ in range(max(args.warmup, 3)):
            g.replay()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        with ClockSampler(dev) if sample_clocks else _Null() as clocks:
            with torch.cuda.stream(stream):
                start.record(stream)
                for _ in range(steps):
                    g.replay()
                end.record(stream)
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = start.elapsed_time(end)
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return ms, float(t.item()), clocks

    g_chain = capture(chain_step)
    ms_chain, ms_chain_max, _ = timed(g_chain, args.steps)
    del g_chain
    g_single = capture(single_step)
    ms, ms_max, clocks = timed(g_single, args.steps, sample_clocks=True)
    del g_single
    # the chain (column-owner CTAs) adds each column in its own fixed order: the
    # single calls' final activations agree with it to the matvec bar
    out_single = xa.clone()
    with torch.cuda.stream(stream):
        chain_step()
    torch.cuda.synchronize()
    # 64 random layers grow the activations past float32 in places (+-Inf in
    # both paths alike); compare the finite entries and count the others
    fin = torch.isfinite(out_single) & torch.isfinite(xa)
    a, b = xa[fin].double(), out_single[fin].double()
    chain_rel = float((a - b).norm() / b.norm().clamp_min(1e-30)) if fin.any() else None
    chain_nonfinite = int((~fin).sum())
    chain_same_nonfinite = bool(torch.equal(torch.isfinite(out_single), torch.isfinite(xa)))

    bytes_step = pair_bytes() * LAYERS
    value = bytes_step * world * args.steps / (ms_max * 1e-3) / 1e9

    # End to end through the C-ABI MatVec (host buffers, synchronous calls),
    # each call's output the next call's input.
    hx0 = x0.cpu().numpy().copy()
    hh = np.empty(N_UP, np.float32)
    hxa = np.empty(K_UP, np.float32)
    pv = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    e2e_steps = max(1, min(args.steps, 20))

    def e2e_step():
        for l in range(LAYERS):
            _lib.check(L.tq_matvec(handles[2 * l], pv(hx0 if l == 0 else hxa), K_UP, pv(hh), N_UP))
            _lib.check(L.tq_matvec(handles[2 * l + 1], pv(hh), N_UP, pv(hxa), K_UP))

    e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    e2e_t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_value = bytes_step * world * e2e_steps / float(e2e_t.item()) / 1e9
    e2e_same = bool(np.array_equal(hxa, out_single.cpu().numpy()))

    side = None
    if rank == 0 and args.side_config:
        side = measure_side_configs(L, Q, torch, stream, load_peak()[0], args.side_config)
    elif rank == 0 and not args.no_side_configs:
        side = measure_side_configs(L, Q, torch, stream, load_peak()[0], cpu=world == 1 and not args.no_cpu_baseline)
        side["C4 GPT-2-small int8 greedy decode"] = measure_gpt2(world == 1 and not args.no_cpu_baseline)
        side["F2 Qwen2.5-7B int4 quantize-on-load from BF16"] = measure_quant_load(world == 1 and not args.no_cpu_baseline)
    qwen = None
    if not args.no_side_configs and not args.side_config:
        try:
            qwen = measure_qwen(rank, world, load_peak()[0], cpu=world == 1 and not args.no_cpu_baseline)  # collective
        except Exception as e:  # reported in the line; the headline stands on its own
            qwen = {"tp": world, "error": str(e)[:300]}
        if side is not None:
            side[f"C5 Qwen2.5-7B int4 greedy decode TP={world}"] = qwen
    if rank == 0:
        peak, peak_src = load_peak()
        call_us = ms / (args.steps * 2 * LAYERS) * 1e3  # one launch per matvec on this rank
        achieved = pair_bytes() / 2 / (call_us * 1e-6) / 1e9
        traffic = load_traffic()
        chain_us = ms_chain / (args.steps * 2 * LAYERS) * 1e3
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded Irwin-Hall normal: weights std 0.02, activations std 1)",
            "config": bench_config(),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "frac_of_8tbs": round(achieved / 8000.0, 4),
                         "traffic": traffic,
                         "kernel": "cmv_kernel<4,1,true> (int4 matvec on the tensor cores by mma.sync u8 x s8 "
                                   "over the K-packed codes, M=1, one launch per matvec)",
                         "call_us_mean": round(call_us, 3),
                         "algorithmic_bytes_per_launch": pair_bytes() / 2},
            "e2e": {"value": round(e2e_value, 3), "unit": "GB/s",
                    "h2d_bytes_per_step": LAYERS * 4 * (K_UP + N_UP),
                    "d2h_bytes_per_step": LAYERS * 4 * (N_UP + K_UP),
                    "api": "tq_matvec (host x/out, synchronous), the MatVec drop-in, one call per matvec",
                    "steps": e2e_steps, "same_bits_as_device_calls": e2e_same},
            "chain": {"value": round(bytes_step * args.steps / (ms_chain_max * 1e-3) / 1e9, 3), "unit": "GB/s",
                      "us_per_matvec": round(chain_us, 3),
                      "frac": round(pair_bytes() / 2 / (chain_us * 1e-6) / 1e9 / peak, 4),
                      "kernel": "chain4_kernel: the step's 64 dependent matvecs in one launch (tq_chain_run), "
                                "column-owner CTAs",
                      "rel_l2_vs_single_calls_after_64": chain_rel,
                      "non_finite_entries_after_64": chain_nonfinite,
                      "same_non_finite_entries": chain_same_nonfinite},
            "gpu_launches": args.steps * 2 * LAYERS,
            "clocks": clocks.summary(),
        }
        if side:
            line["side_configs"] = side
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
        print(json.dumps(line), flush=True)
    chain.free()
    for hd in handles:
        Q.free(hd)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        pass


def main():
    global LAYERS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="resident MLP pairs per step (default 32 = 1.63 GB; small values for profiling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-side-configs", action="store_true")
    ap.add_argument("--side-config", default=None,
                    help="run only this kernel side config (C1, C2, C3) after the headline, e.g. for profiling")
    ap.add_argument("--kernel", type=int, default=None,
                    help="matvec kernel for M <= 15 (tq_set_matvec_kernel); default: the library's")
    args = ap.parse_args()
    args.steps = max(args.steps, 1)
    LAYERS = max(1, args.layers)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        run_gpu(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
