#!/usr/bin/env python
"""Benchmark of the cooperative-matrix GEMM / flash-attention path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl lvb|reference]

One step = one call of the hot path over one batch of synthetic input, already resident in
HBM. The default workload is BASELINE config 2, the fp16 GEMM M=N=K=8192 (fp32 accumulate,
fp16 C) on one GPU; with N GPUs (torchrun, one rank per GPU) every rank runs its own
8192-row shard of A against a replicated B (rows of A are independent: weak scaling, no
collective on the data path). Rank 0 prints one JSON line: whole-job TFLOP/s over the max
of the ranks' device times, plus roofline, end-to-end (host buffers, copies inside the
timed region), CPU baseline and SM clocks sampled during the timed region.

The same line carries the rest of the metric, each timed in its own region with its own
roofline and clock record (skipped with --no-extras):
  * "attention": C4 (fp16, B4 H32 S4096 causal) and C5 (bf16 GQA, B8 Hq64 Hkv8 S16384
    causal) — one problem each, its (batch, KV head) units sharded over the N ranks (strong
    scaling; at N = 1 the whole problem on one GPU);
  * "split": C3 (int8 8192^3) with the rows of A and C sharded in 128-row blocks over the
    N ranks (strong scaling), and at N > 1 the NCCL all-gather of C timed apart;
  * "cublas": torch.matmul on the headline GEMM's operands, a library figure beside ours.

``--impl reference`` times the reference's CPU path stand-in (the oracle port: host
float32 BLAS, or exact float64 BLAS for int8, or blockwise float32 attention) on the host
cores — Lava's own path (Lava→SPIR-V on lavapipe, host Julia BLAS) needs Julia and a
graphics stack, which this box does not have.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "lava.jl_b200"
for _p in (str(REPO), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "GEMM / attention TFLOPS (and % dense tensor peak) at 1/2/4/8 B200"

WORKLOADS = {
    # name: (kind, config, shape per GPU)
    "gemm_f16": dict(kind="gemm", cfg="C2", M=8192, N=8192, K=8192, ab="Float16", out="Float16",
                     seed=1, dtype="f16"),
    "gemm_f16_512": dict(kind="gemm", cfg="C1", M=512, N=512, K=512, ab="Float16", out="Float32",
                         seed=0, dtype="f16"),
    "gemm_i8": dict(kind="gemm", cfg="C3", M=8192, N=8192, K=8192, ab="Int8", out="Int32",
                    seed=2, dtype="int8"),
    # one rank's share of C3 row-sharded over 8 GPUs (the `split` key's per-GPU problem at N=8)
    "gemm_i8_shard8": dict(kind="gemm", cfg="C3-shard-of-8", M=1024, N=8192, K=8192,
                           ab="Int8", out="Int32", seed=2, dtype="int8"),
    "gemm_bf16": dict(kind="gemm", cfg="C5-gemm", M=65536, N=8192, K=8192, ab="BFloat16",
                      out="BFloat16", seed=5, dtype="bf16"),
    # C2 with the fused epilogue C = gelu(A·B + bias + R) (bias per column, R fp16 M×N)
    "gemm_f16_fused": dict(kind="gemm", cfg="C2+epilogue", M=8192, N=8192, K=8192,
                           ab="Float16", out="Float16", seed=1, dtype="f16", epilogue="gelu"),
    # C2 with both operands MN-contiguous (A column-major, B row-major): read MN-major
    "gemm_f16_mn": dict(kind="gemm", cfg="C2-transposed", M=8192, N=8192, K=8192,
                        ab="Float16", out="Float16", seed=1, dtype="f16", a_rowmajor=False,
                        b_rowmajor=True),
    "attn_f16": dict(kind="attn", cfg="C4", B=4, Hq=32, Hkv=32, S=4096, D=128, ab="Float16",
                     causal=True, seed=3, dtype="f16"),
    "attn_bf16": dict(kind="attn", cfg="C5-attn", B=8, Hq=64, Hkv=8, S=16384, D=128,
                      ab="BFloat16", causal=True, seed=4, dtype="bf16"),
    # HBM-bound shapes (roofline in GB/s against the measured copy bandwidth):
    # decoding one token per sequence against C5's KV cache (the cache resident on the GPU)
    "attn_decode_bf16": dict(kind="attn", cfg="C5-decode", B=8, Hq=64, Hkv=8, S=16384, Sq=1,
                             D=128, ab="BFloat16", causal=True, seed=4, dtype="bf16",
                             bound="hbm", resident_kv=True),
    # int8 matrix-vector product (dot4x8), A 16384x16384 row-major (268 MB)
    "gemv_i8": dict(kind="gemm", cfg="dot4x8-GEMV", M=16384, N=1, K=16384, ab="Int8",
                    out="Int32", seed=2, dtype="int8", bound="hbm"),
}


def work_units(w) -> float:
    if w["kind"] == "gemm":
        return 2.0 * w["M"] * w["N"] * w["K"]
    Sq, S = w.get("Sq", w["S"]), w["S"]
    if Sq == S:
        f = 4.0 * w["B"] * w["Hq"] * S * S * w["D"]
        return f / 2 if w["causal"] else f
    # query i sees keys j <= i + (S - Sq): the exact count of visible (query, key) pairs
    pairs = sum(min(S, i + S - Sq + 1) for i in range(Sq)) if w["causal"] else Sq * S
    return 4.0 * w["B"] * w["Hq"] * pairs * w["D"]


ESIZE = {"Float16": 2, "BFloat16": 2, "Float32": 4, "Int8": 1, "Int32": 4}


def algo_bytes(w) -> float:
    """Bytes the op must move at least once: its operands and its result."""
    if w["kind"] == "gemm":
        e, o = ESIZE[w["ab"]], ESIZE[w["out"]]
        return (w["M"] * w["K"] + w["K"] * w["N"]) * e + w["M"] * w["N"] * o
    Sq = w.get("Sq", w["S"])
    e = ESIZE[w["ab"]]
    return (2 * w["B"] * w["Hq"] * Sq + 2 * w["B"] * w["Hkv"] * w["S"]) * w["D"] * e


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic(workload: str):
    """dram bytes per launch of the dominant kernel from the committed ncu summary."""
    f = REPO / "profiles" / f"{workload}_ncu.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


# ----------------------------------------------------------------------------------------
# clocks during the timed region (NVML polled from a thread; nvidia-smi fields)
# ----------------------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown", 0x1: "gpu_idle",
               0x2: "applications_clocks_setting", 0x100: "display_clock_setting"}

    def __init__(self, torch_device_index: int, period_s: float = 0.01):
        self.period = period_s
        self.samples = []
        self.err = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml as nv
            import torch
            nv.nvmlInit()
            uuid = "GPU-" + str(torch.cuda.get_device_properties(torch_device_index).uuid)
            try:
                self.h = nv.nvmlDeviceGetHandleByUUID(uuid)
            except Exception:  # noqa: BLE001 — older bindings want bytes
                self.h = nv.nvmlDeviceGetHandleByUUID(uuid.encode())
            self.nv = nv
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(self.h, nv.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001
            self.err = f"nvml unavailable: {e}"

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((sm, rs, pw))
            except Exception as e:  # noqa: BLE001
                self.err = str(e)
                return
            time.sleep(self.period)

    def start(self):
        if self.err is None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join()
        if self.err and not self.samples:
            return {"error": self.err}
        sms = [s[0] for s in self.samples]
        mask = 0
        for s in self.samples:
            mask |= s[1]
        reasons = sorted({n for b, n in self.REASONS.items() if mask & b and n != "gpu_idle"})
        return {"sm_mhz": statistics.median(sms) if sms else None, "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(sms),
                "power_w_max": max((s[2] for s in self.samples), default=None),
                "source": "nvml (nvidia-smi clocks.sm / clocks_event_reasons)"}


# ----------------------------------------------------------------------------------------
# CPU baseline (oracle port on the host cores) — also the reference arm
# ----------------------------------------------------------------------------------------
def blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:  # noqa: BLE001
        return os.cpu_count() or 1


def cpu_step_factory(w, target_s: float):
    """A callable doing one bounded sample of the workload on the CPU, its work units, and a
    description of the sample. The sample is sized so one call takes about target_s."""
    import numpy as np
    g = np.random.default_rng(w["seed"])
    if w["kind"] == "gemm":
        N, K = w["N"], w["K"]
        integer = w["ab"] == "Int8"
        B = (g.integers(-128, 128, size=(K, N)).astype(np.float64) if integer
             else g.uniform(-1, 1, size=(K, N)).astype(np.float16).astype(np.float32))
        rows = 64
        while True:
            A = (g.integers(-128, 128, size=(rows, K)).astype(np.float64) if integer
                 else g.uniform(-1, 1, size=(rows, K)).astype(np.float16).astype(np.float32))
            t0 = time.perf_counter()
            A @ B
            dt = time.perf_counter() - t0
            if dt >= target_s / 2 or rows >= w["M"]:
                break
            rows = min(w["M"], rows * 2)
        how = ("exact int8 GEMM as float64 BLAS (integer partial sums < 2^53)" if integer
               else "float32 BLAS sgemm on fp16-rounded inputs")
        sample = f"{rows} of {w['M']} rows of A: ({rows}x{K}) @ ({K}x{N}), {how}"
        if w.get("epilogue"):
            from oracle.gemm import ACTIVATIONS
            act = ACTIVATIONS[w["epilogue"]]
            bias = g.uniform(-1, 1, size=N).astype(np.float32)
            R = g.uniform(-1, 1, size=(rows, N)).astype(np.float32)
            sample += f", then {w['epilogue']}(. + bias + R) in float32"
            return (lambda: act(A @ B + bias + R)), 2.0 * rows * N * K, sample
        return (lambda: A @ B), 2.0 * rows * N * K, sample
    # attention: whole (b, h) units at full sequence length
    from oracle.attention import attention_blockwise
    S, D = w["S"], w["D"]
    Sq = w.get("Sq", S)
    q = g.standard_normal((Sq, D), dtype=np.float32)
    k = g.standard_normal((S, D), dtype=np.float32)
    v = g.standard_normal((S, D), dtype=np.float32)
    units = 1
    per = work_units(w) / (w["B"] * w["Hq"])
    t0 = time.perf_counter()
    attention_blockwise(q, k, v, w["causal"], D ** -0.5, block=512)
    dt = time.perf_counter() - t0
    units = max(1, min(int(target_s / max(dt, 1e-3)), w["B"] * w["Hq"]))

    def step():
        for _ in range(units):
            attention_blockwise(q, k, v, w["causal"], D ** -0.5, block=512)
    sample = (f"{units} of {w['B'] * w['Hq']} (batch, head) units at Sq={Sq}, Skv={S}, D={D}, "
              "blockwise float32 online softmax on host BLAS")
    return step, units * per, sample


def cpu_baseline(w, budget_s: float = 12.0):
    step, units, sample = cpu_step_factory(w, target_s=min(3.0, budget_s / 4))
    step()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 2:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    best = min(times)
    unit = "TOPS" if w["ab"] == "Int8" else "TFLOP/s"
    return {"value": units / best / 1e12, "unit": unit, "cores": blas_threads(), "kind": "port",
            "sample": sample + f"; best of {len(times)} runs", "host_cpus": os.cpu_count()}


def run_reference(args, w):
    # Every host core, whatever the launcher set: torchrun exports OMP_NUM_THREADS=1, which
    # would leave the host BLAS on one thread (and shrink the time-sized sample) at N > 1.
    # The BLAS reads its thread count when numpy loads it, and threadpoolctl acts only on
    # libraries already loaded: set both, in that order.
    ncpu = str(os.cpu_count() or 1)
    for var in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[var] = ncpu
    import numpy  # noqa: F401  (loads the BLAS with the thread count above)
    try:
        from threadpoolctl import threadpool_limits
        limits = threadpool_limits(limits=int(ncpu), user_api="blas")
    except Exception:  # noqa: BLE001
        limits = None
    step, units, sample = cpu_step_factory(w, target_s=1.0)
    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    threads = blas_threads()
    if limits is not None:
        limits.restore_original_limits()
    tot = sum(times)
    value = units * len(times) / tot / 1e12
    unit = "TOPS" if w["ab"] == "Int8" else "TFLOP/s"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": tot / len(times) * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic (seeded)",
        "config": config_of(w, args.gpus), "device": "host CPU",
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port",
                         "sample": sample, "host_cpus": os.cpu_count()},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("Lava's own path (Julia -> SPIR-V on lavapipe, host Julia BLAS) is unavailable "
                 "on this box (no Julia, no graphics stack); the oracle port stands in"),
    }
    print(json.dumps(line), flush=True)


def config_of(w, n):
    c = {"workload": f"{w['cfg']} " + (
        f"{w['ab']} GEMM M={w['M']} N={w['N']} K={w['K']} per GPU, {w['out']} C, "
        f"A {'row' if w.get('a_rowmajor', True) else 'column'}-major, "
        f"B {'row' if w.get('b_rowmajor', False) else 'column'}-major, C row-major"
        + (f", fused epilogue {w['epilogue']}(A·B + bias[n] + R), bias/R {w['out']}"
           if w.get("epilogue") else "") if w["kind"] == "gemm" else
        f"{w['ab']} attention fwd B={w['B']} Hq={w['Hq']} Hkv={w['Hkv']} "
        f"Sq={w.get('Sq', w['S'])} Skv={w['S']} D={w['D']} causal={w['causal']} per GPU")}
    c["parallelism"] = (f"row-shard x{n} (independent shards, no collective)" if w["kind"] == "gemm"
                        else f"(batch, kv-head) shard x{n}") if n > 1 else "single GPU"
    c["l2"] = "inputs larger than L2 (126 MB): working set re-read every step from HBM"
    return c


# ----------------------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------------------
def make_gemm(torch, lvb, w, rank):
    gen = torch.Generator(device="cuda").manual_seed(w["seed"] * 1000 + rank)
    M, N, K = w["M"], w["N"], w["K"]
    tdt = {"Float16": torch.float16, "BFloat16": torch.bfloat16, "Int8": torch.int8}[w["ab"]]
    odt = {"Float16": torch.float16, "BFloat16": torch.bfloat16, "Float32": torch.float32,
           "Int32": torch.int32}[w["out"]]
    a_rm, b_rm = w.get("a_rowmajor", True), w.get("b_rowmajor", False)
    # storage shapes: A (M,K) row-major or (K,M) column-major; B (N,K) column-major or (K,N)
    a_shape = (M, K) if a_rm else (K, M)
    b_shape = (K, N) if b_rm else (N, K)
    if tdt == torch.int8:
        As = torch.randint(-128, 128, a_shape, generator=gen, device="cuda", dtype=torch.int16).to(tdt)
        Bs = torch.randint(-128, 128, b_shape, generator=gen, device="cuda", dtype=torch.int16).to(tdt)
    else:
        As = (torch.rand(a_shape, generator=gen, device="cuda") * 2 - 1).to(tdt)
        Bs = (torch.rand(b_shape, generator=gen, device="cuda") * 2 - 1).to(tdt)
    view_a = (lambda t: t) if a_rm else (lambda t: t.t())
    view_b = (lambda t: t) if b_rm else (lambda t: t.t())
    # C row-major: a rank's row block of the job's C is one contiguous slab, so the optional
    # all-gather concatenates shards without a reshuffle (the kernel stores it as Cᵀ = BᵀAᵀ).
    Cs = torch.empty((M, N), dtype=odt, device="cuda")
    ins, outs = [As, Bs], [Cs]
    act = w.get("epilogue")
    if act:
        bias = (torch.rand((N,), generator=gen, device="cuda") * 2 - 1).to(odt)
        R = (torch.rand((M, N), generator=gen, device="cuda") * 2 - 1).to(odt)
        ins += [bias, R]

    def call(d_ins, d_outs, stream=None):
        if act:
            lvb.gemm(d_outs[0], view_a(d_ins[0]), view_b(d_ins[1]), stream=stream,
                     bias=d_ins[2], residual=d_ins[3], activation=act)
        else:
            lvb.gemm(d_outs[0], view_a(d_ins[0]), view_b(d_ins[1]), stream=stream)

    # the timed step: the same call, described once (lvb.prepare_gemm: one foreign call per
    # launch); e2e goes through lvb.gemm every step
    if act:
        prepared = lvb.prepare_gemm(Cs, view_a(As), view_b(Bs), bias=ins[2], residual=ins[3],
                                    activation=act)
    else:
        prepared = lvb.prepare_gemm(Cs, view_a(As), view_b(Bs))

    def step(stream=None):
        prepared(stream)

    def compute(d_ins, d_outs, stream):
        call(d_ins, d_outs, stream)
    step.plain = lambda: call(ins, outs)
    return step, compute, ins, outs


def make_attn(torch, lvb, w, rank):
    gen = torch.Generator(device="cuda").manual_seed(w["seed"] * 1000 + rank)
    tdt = {"Float16": torch.float16, "BFloat16": torch.bfloat16}[w["ab"]]
    Bn, Hq, Hkv, S, D = w["B"], w["Hq"], w["Hkv"], w["S"], w["D"]
    Sq = w.get("Sq", S)
    Q = torch.randn((Bn, Hq, Sq, D), generator=gen, device="cuda").to(tdt)
    K = torch.randn((Bn, Hkv, S, D), generator=gen, device="cuda").to(tdt)
    V = torch.randn((Bn, Hkv, S, D), generator=gen, device="cuda").to(tdt)
    O = torch.empty_like(Q)

    def step():
        lvb.attention(O, Q, K, V, causal=w["causal"])

    if w.get("resident_kv"):
        # decoding: the KV cache is the serving loop's state on the GPU; a step's inputs are
        # the new query rows and its result the output rows
        def compute(d_ins, d_outs, stream):
            lvb.attention(d_outs[0], d_ins[0], K, V, causal=w["causal"], stream=stream)
        return step, compute, [Q], [O]

    def compute(d_ins, d_outs, stream):
        lvb.attention(d_outs[0], d_ins[0], d_ins[1], d_ins[2], causal=w["causal"], stream=stream)
    return step, compute, [Q, K, V], [O]


def run_e2e(torch, compute, ins, outs, steps):
    """Steps through the public API with host buffers: every step copies its inputs from
    pinned host memory, runs the op and copies the result back to pinned host memory.
    Two device buffer sets and three streams (copy-in, compute, copy-out) let step i+1's
    upload, step i's compute and step i-1's download overlap, as a serving loop would.
    Returns ms per step (device events around the whole sequence)."""
    h_ins = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in ins]
    for h, t in zip(h_ins, ins):
        h.copy_(t)
    sets = [([torch.empty_like(t) for t in ins], [torch.empty_like(t) for t in outs],
             [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in outs])
            for _ in range(2)]
    s_in, s_mm, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_mm = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]

    def one(i):
        k = i % 2
        d_in, d_out, h_out = sets[k]
        with torch.cuda.stream(s_in):
            if i >= 2:
                s_in.wait_event(ev_mm[k])          # set k's inputs consumed by step i-2
            for d, h in zip(d_in, h_ins):
                d.copy_(h, non_blocking=True)
            ev_in[k].record(s_in)
        with torch.cuda.stream(s_mm):
            s_mm.wait_event(ev_in[k])
            if i >= 2:
                s_mm.wait_event(ev_out[k])         # set k's outputs downloaded by step i-2
            compute(d_in, d_out, s_mm)
            ev_mm[k].record(s_mm)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_mm[k])
            for h, d in zip(h_out, d_out):
                h.copy_(d, non_blocking=True)
            ev_out[k].record(s_out)

    for i in range(2):
        one(i)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(s_in)
    for i in range(steps):
        one(i)
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_mm)
    t1.record(s_out)
    t1.synchronize()
    return t0.elapsed_time(t1) / steps


# ----------------------------------------------------------------------------------------
# The rest of the metric on the same line: attention (C4, C5) and the north star's split
# problem (C3 row-sharded over the ranks, one problem in total), each timed on its own
# ----------------------------------------------------------------------------------------
def timed_region(torch, step, steps, warmup, stream, local, sync, max_over_ranks):
    """Warm-up, then `steps` calls between CUDA events on `stream` with SM clocks sampled;
    returns (this rank's ms per step, max over ranks, clock record)."""
    for _ in range(warmup):
        step()
    sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    sampler.start()
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    e1.synchronize()
    clocks = sampler.stop()
    ms_local = e0.elapsed_time(e1) / steps
    sync()
    return ms_local, max_over_ranks(ms_local), clocks


def tensor_roofline(flop_local, ms_local, steps, peaks, src, scale=1.0):
    """Roofline of one timed region against the measured bf16 GEMM (x2 for int8): the
    sustained figure for regions of a second or more, the burst figure otherwise."""
    timed_s = ms_local * steps / 1e3
    kind = "sustained" if timed_s >= 1.0 else "burst"
    burst = peaks["bf16_tflops"] * scale
    peak = (peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"]) * scale
            if kind == "sustained" else burst)
    achieved = flop_local / (ms_local * 1e-3) / 1e12
    return {"bound": "tensor", "achieved": achieved, "peak": peak,
            "unit": "TOPS" if scale != 1.0 else "TFLOP/s", "frac": achieved / peak,
            "peak_kind": kind, "frac_of_burst": achieved / burst, "timed_region_s": timed_s,
            "peak_source": f"{src} bf16_tflops{'_sustained' if kind == 'sustained' else ''}"
                           f"{' x2 (int8 dense rate)' if scale != 1.0 else ''}"}


def attention_shard(torch, lvb, name, world, rank):
    """This rank's share of attention config `name`, sharded by (batch, KV head) units (a
    unit carries its group of query heads: no K/V is duplicated): n units laid out as a batch
    of n with Hkv = 1, Hq = group — the same work items as the whole problem's."""
    from lvb.dist import attention_units
    w = {"C4": WORKLOADS["attn_f16"], "C5": WORKLOADS["attn_bf16"]}[name]
    Bn, Hq, Hkv, S, D = w["B"], w["Hq"], w["Hkv"], w["S"], w["D"]
    g = Hq // Hkv
    units = attention_units(Bn, Hkv, world, rank)
    n = len(units)
    tdt = torch.float16 if w["ab"] == "Float16" else torch.bfloat16
    gen = torch.Generator(device="cuda").manual_seed(w["seed"] * 1000 + rank)
    Q = torch.randn((n, g, S, D), generator=gen, device="cuda").to(tdt)
    K = torch.randn((n, 1, S, D), generator=gen, device="cuda").to(tdt)
    V = torch.randn((n, 1, S, D), generator=gen, device="cuda").to(tdt)
    O = torch.empty_like(Q)
    flop_local = 4.0 * n * g * S * S * D / 2
    flop_total = work_units(w)
    plan = lvb.attention_plan(n, g, 1, S, S, D, lvb.F16 if w["ab"] == "Float16" else lvb.BF16,
                              True, sm_count=torch.cuda.get_device_properties(0).multi_processor_count)

    # One foreign call per step (the descriptor is built once): at N = 8 a rank's share is
    # ~70 us of kernel time, and eight ranks share the host's cores.
    step = lvb.prepare_attention(O, Q, K, V, causal=True)
    return w, step, flop_local, flop_total, plan.launches, (Q, K, V, O), n


def measure_extras(args, torch, lvb, world, rank, local, stream, sync, max_over_ranks):
    """Secondary keys of the bench line (see the module docstring)."""
    peaks, src = measured_peaks()
    out = {}
    # ---- attention: C4 and C5, the one problem sharded by (batch, KV head) over the ranks ----
    att = {}
    for name in ("C4", "C5"):
        w, step, fl, ft, launches, keep, n = attention_shard(torch, lvb, name, world, rank)
        steps = args.steps if name == "C4" else max(3, min(args.steps, 20))
        ms_l, ms, clocks = timed_region(torch, step, steps, args.warmup, stream, local, sync,
                                        max_over_ranks)
        st = lvb.device_status()
        assert st[0] == 0, f"device status {st} after attention {name}"
        att[name] = {
            "workload": config_of(w, 1)["workload"].replace(" per GPU", ""),
            "value": ft / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "steps": steps, "units_per_rank": n, "flop_per_step": ft,
            "parallelism": (f"(batch, kv-head) units sharded over {world} ranks, one problem"
                            if world > 1 else "single GPU"),
            "scaling": "strong" if world > 1 else None,
            "roofline": dict(tensor_roofline(fl, ms_l, steps, peaks, src),
                             traffic=profile_traffic("attn_f16" if name == "C4" else "attn_bf16")
                             if world == 1 else None),
            "clocks": clocks, "gpu_launches": steps * launches}
        del keep
        torch.cuda.empty_cache()
    out["attention"] = att
    # ---- C3 int8 8192^3 row-sharded (128-row blocks) over the ranks, then the all-gather ----
    from lvb.dist import gemm_rows, allgather_rows
    w = WORKLOADS["gemm_i8"]
    M, N, K = w["M"], w["N"], w["K"]
    r0, rn = gemm_rows(M, world, rank)
    gen = torch.Generator(device="cuda").manual_seed(w["seed"] * 1000 + rank)
    A = torch.randint(-128, 128, (max(rn, 1), K), generator=gen, device="cuda",
                      dtype=torch.int16).to(torch.int8)[:rn]
    g2 = torch.Generator(device="cuda").manual_seed(w["seed"])   # B replicated: same on all
    Bm = torch.randint(-128, 128, (N, K), generator=g2, device="cuda", dtype=torch.int16).to(torch.int8)
    Cm = torch.empty((rn, N), dtype=torch.int32, device="cuda")
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    plan = lvb.gemm_plan(max(rn, 1), N, K, lvb.I8, lvb.I32, c_rowmajor=True, sm_count=sms)

    # One foreign call per step (prepared once): a 1024-row shard is ~47 us of kernel time.
    gcall = lvb.prepare_gemm(Cm, A, Bm.t()) if rn else None

    def gstep():
        if gcall is not None:
            gcall()
    ms_l, ms, clocks = timed_region(torch, gstep, args.steps, args.warmup, stream, local, sync,
                                    max_over_ranks)
    st = lvb.device_status()
    assert st[0] == 0, f"device status {st} after the split GEMM"
    split = {
        "workload": f"C3 Int8 GEMM M={M} N={N} K={K} Int32 C (row-major), rows of A and C "
                    f"sharded in 128-row blocks over the ranks ({rn} rows on rank {rank}), "
                    "B replicated",
        "value": 2.0 * M * N * K / (ms * 1e-3) / 1e12, "unit": "TOPS", "ms_per_step": ms,
        "steps": args.steps, "rows_per_rank": rn, "scaling": "strong" if world > 1 else None,
        "tiles_per_rank": plan.tiles, "ctas": plan.ctas, "cta_pair": plan.cta_pair,
        "roofline": tensor_roofline(2.0 * rn * N * K, ms_l, args.steps, peaks, src, scale=2.0),
        "clocks": clocks, "gpu_launches": args.steps * plan.launches, "allgather": None}
    if world > 1:
        for _ in range(2):
            full = allgather_rows(Cm, total=M)
        sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record(stream)
        for _ in range(reps):
            full = allgather_rows(Cm, total=M)
        e1.record(stream)
        e1.synchronize()
        ag_ms = max_over_ranks(e0.elapsed_time(e1) / reps)
        nbytes = full.numel() * full.element_size()
        split["allgather"] = {
            "ms": ag_ms, "bytes": nbytes,
            "busbw_GBs": nbytes * (world - 1) / world / (ag_ms * 1e-3) / 1e9,
            "algbw_GBs": nbytes / (ag_ms * 1e-3) / 1e9,
            "how": "torch.distributed all_gather_into_tensor of the int32 C row blocks (NCCL "
                   "over NVLink/NVSwitch), timed apart from the GEMM"}
        split["value_with_allgather"] = 2.0 * M * N * K / ((ms + ag_ms) * 1e-3) / 1e12
        del full
        sync()
    out["split"] = split
    del A, Bm, Cm
    torch.cuda.empty_cache()
    return out


def host_path_breakdown(torch, step, stream, n=2000, graph_calls=100):
    def per_call_us(fn, calls):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(calls):
            fn()
        e1.record(stream)
        e1.synchronize()
        return e0.elapsed_time(e1) * 1e3 / calls
    out = {"lvb_gemm_us": per_call_us(step.plain, n), "prepared_us": per_call_us(step, n)}
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=side):
            for _ in range(graph_calls):
                step(side)
    torch.cuda.synchronize()
    out["graph_replay_us"] = per_call_us(g.replay, 20) / graph_calls
    out["how"] = ("device time per call over back-to-back calls: lvb.gemm (descriptor built "
                  "in Python each call), lvb.prepare_gemm (one foreign call), and a CUDA graph "
                  f"of {graph_calls} captured prepared calls (~ the kernel's own time)")
    del g
    return out


def cublas_sanity(torch, w, ins, steps, warmup, stream):
    """torch.matmul (cuBLAS) on the headline GEMM's operands in the same kind of timed
    region: a library figure beside the kernel's, not part of `value`."""
    if w["kind"] != "gemm" or w.get("epilogue") or w["ab"] == "Int8":
        return None
    A, B = ins[0], ins[1]
    a = A if w.get("a_rowmajor", True) else A.t()
    b = B.t() if not w.get("b_rowmajor", False) else B
    out = torch.empty((a.shape[0], b.shape[1]), dtype=a.dtype, device="cuda")
    for _ in range(warmup):
        torch.matmul(a, b, out=out)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        torch.matmul(a, b, out=out)
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del out
    return {"value": work_units(w) / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "steps": steps, "how": "torch.matmul (cuBLAS) on the same operands, same steps"}


def run_gpu(args, w):
    import torch
    import torch.distributed as dist
    import importlib.util
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))

    spec = importlib.util.spec_from_file_location("lvb_build", PKG / "build.py")
    b = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(b)
    if rank == 0:
        b.build()
    if world > 1:
        dist.barrier(device_ids=[local])
    import lvb

    step, compute, ins, outs = (make_gemm if w["kind"] == "gemm" else make_attn)(torch, lvb, w, rank)
    units = work_units(w)
    # kernel launches of this library per step, from the library's own plan for the call
    sms = torch.cuda.get_device_properties(local).multi_processor_count
    dt_of = {"Float16": lvb.F16, "BFloat16": lvb.BF16, "Int8": lvb.I8, "Float32": lvb.F32,
             "Int32": lvb.I32}
    if w["kind"] == "gemm":
        launches_per_step = lvb.gemm_plan(
            w["M"], w["N"], w["K"], dt_of[w["ab"]], dt_of[w["out"]], c_rowmajor=True,
            sm_count=sms, a_rowmajor=w.get("a_rowmajor", True),
            b_rowmajor=w.get("b_rowmajor", False)).launches
    else:
        launches_per_step = lvb.attention_plan(
            w["B"], w["Hq"], w["Hkv"], w.get("Sq", w["S"]), w["S"], w["D"], dt_of[w["ab"]],
            w["causal"], sm_count=sms).launches
    stream = torch.cuda.current_stream()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing ----
    for _ in range(args.warmup):
        step()
    st = lvb.device_status()
    assert st[0] == 0, f"device status {st} after warm-up"
    barrier()
    sampler = ClockSampler(local)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.start()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    clocks = sampler.stop()
    ms_local = e0.elapsed_time(e1) / args.steps
    barrier()
    st = lvb.device_status()
    assert st[0] == 0, f"device status {st} after the timed region"
    ms = max_over_ranks(ms_local)
    value = units * world / (ms * 1e-3) / 1e12

    # ---- end to end through the public API with host buffers ----
    e2e_steps = 0 if args.no_e2e else max(3, min(args.steps, 20))
    e2e_ms = float("nan")
    if e2e_steps:
        barrier()
        e2e_ms = max_over_ranks(run_e2e(torch, compute, ins, outs, e2e_steps))
        barrier()
    h2d = sum(t.numel() * t.element_size() for t in ins)
    d2h = sum(t.numel() * t.element_size() for t in outs)

    # ---- optional NCCL all-gather of the outputs (timed separately, not in `value`) ----
    allgather = None
    if args.allgather and world > 1:
        from lvb.dist import allgather_rows
        shard = outs[0].reshape(outs[0].shape[0], -1)
        for _ in range(2):
            full = allgather_rows(shard)
        barrier()
        e0.record(stream)
        for _ in range(5):
            full = allgather_rows(shard)
        e1.record(stream)
        e1.synchronize()
        ag_ms = max_over_ranks(e0.elapsed_time(e1) / 5)
        nbytes = full.numel() * full.element_size()
        allgather = {"ms": ag_ms, "bytes": nbytes,
                     "busbw_GBs": nbytes * (world - 1) / world / (ag_ms * 1e-3) / 1e9,
                     "how": "torch.distributed all_gather_into_tensor (NCCL over NVLink)"}
        del full
        barrier()

    # ---- fused epilogue: the same result as GEMM + a separate elementwise pass ----
    unfused = None
    if w.get("epilogue") and rank == 0:
        import torch.nn.functional as F
        A_, B_, bias_, R_ = ins
        C_ = outs[0]
        view_a = (lambda t: t) if w.get("a_rowmajor", True) else (lambda t: t.t())
        view_b = (lambda t: t) if w.get("b_rowmajor", False) else (lambda t: t.t())
        tanh = w["epilogue"] == "gelu"

        def two_pass():
            lvb.gemm(C_, view_a(A_), view_b(B_))
            C_.copy_(F.gelu(C_.float() + bias_.float() + R_.float(),
                            approximate="tanh" if tanh else "none"))
        n_un = max(3, min(args.steps, 200))
        for _ in range(3):
            two_pass()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(n_un):
            two_pass()
        e1.record(stream)
        e1.synchronize()
        un_ms = e0.elapsed_time(e1) / n_un
        unfused = {"ms_per_step": un_ms, "steps": n_un, "fused_ms_per_step": ms_local,
                   "how": "lvb_gemm without epilogue, then torch elementwise "
                          f"{w['epilogue']}(C + bias + R) as a second pass over C"}

    # host path of a small GEMM: per-call device time through lvb.gemm (Python wrapper each
    # call), through the prepared call (the timed step), and replayed from a CUDA graph of
    # captured calls (about the kernel's own time)
    per_call = None
    if w["kind"] == "gemm" and w["M"] * w["N"] * w["K"] <= 1 << 30 and args.extras == "all":
        per_call = host_path_breakdown(torch, step, stream)

    cublas = None
    if not args.no_extras:
        cublas = cublas_sanity(torch, w, ins, args.steps, args.warmup, stream)
    extras = None
    if args.extras == "all" and args.workload == "gemm_f16":
        torch.cuda.empty_cache()
        extras = measure_extras(args, torch, lvb, world, rank, local, stream, barrier,
                                max_over_ranks)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w)

    if rank == 0:
        peaks, src = measured_peaks()
        # A timed region of a second or more of back-to-back launches is the condition the
        # sustained figure was measured under (cuBLAS back to back for seconds, power-capped);
        # shorter regions compare against the burst figure.
        timed_s = ms_local * args.steps / 1e3
        kind = "sustained" if timed_s >= 1.0 else "burst"
        burst = peaks["bf16_tflops"]
        peak = peaks.get("bf16_tflops_sustained", burst) if kind == "sustained" else burst
        unit = "TOPS" if w["ab"] == "Int8" else "TFLOP/s"
        scale = 1.0
        hbm_src = src
        if w["ab"] == "Int8":
            # no measured int8 peak: dense int8 is twice dense bf16 on this part
            scale = 2.0
            src += " (2x bf16: int8 dense rate)"
        peak, burst = peak * scale, burst * scale
        achieved = units / (ms_local * 1e-3) / 1e12
        traffic = profile_traffic(args.workload)
        hbm = w.get("bound") == "hbm"
        if hbm:
            # memory-bound shape: algorithmic bytes per launch over the launch time, against
            # the measured copy bandwidth
            hbm_peak = peaks.get("hbm_gbs", 6650.0)
            gbs = algo_bytes(w) / (ms_local * 1e-3) / 1e9
        line = {
            "impl": "lvb", "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": w["dtype"], "data": "synthetic: torch.Generator on the GPU (seed = the "
            "config's seed x 1000 + rank), not the configs' numpy PCG64 streams (the parity "
            f"tests use those); shapes and distributions of BASELINE {w['cfg']}",
            "config": config_of(w, world),
            "roofline": ({"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s",
                          "frac": gbs / hbm_peak, "traffic": traffic,
                          "algorithmic_bytes": algo_bytes(w), "timed_region_s": timed_s,
                          "tensor_frac_of_burst": achieved / burst,
                          "peak_source": f"{hbm_src} hbm_gbs (MEASURED_PEAKS.json)"
                                         if hbm_src.startswith("measured") else f"{hbm_src} (6.65 TB/s)"}
                         if hbm else
                         {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": unit,
                          "frac": achieved / peak, "traffic": traffic,
                          "peak_kind": kind, "timed_region_s": timed_s,
                          "frac_of_burst": achieved / burst,
                          "peak_source": f"{src} bf16_tflops{'_sustained' if kind == 'sustained' else ''}"
                                         " (MEASURED_PEAKS.json)" if src.startswith("measured")
                                         else f"{src} (1.59 burst / 1.40 sustained PFLOP/s)"}),
            "e2e": None if args.no_e2e else {"value": units * world / (e2e_ms * 1e-3) / 1e12, "unit": unit,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms, "steps": e2e_steps,
                    "path": "lvb Python binding -> liblvb C ABI; pinned host buffers; every "
                            "step: H2D of its inputs, the op, D2H of its output, on copy-in / "
                            "compute / copy-out streams over two device buffer sets"
                            + ("; the KV cache stays resident on the GPU (decoding state)"
                               if w.get("resident_kv") else "")},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": args.steps * launches_per_step,
            "allgather": allgather,
        }
        if unfused:
            line["unfused_comparison"] = unfused
        if cublas:
            line["cublas"] = cublas
        if per_call:
            line["per_call"] = per_call
        if extras:
            line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="gemm_f16", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="lvb", choices=["lvb", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--allgather", action="store_true",
                    help="also time an NCCL all-gather of the outputs (N > 1), reported apart")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end leg (used for short profiling runs)")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the attention / split-GEMM / cuBLAS keys of the default line")
    ap.add_argument("--extras", default="all", choices=["all", "none", "cublas"],
                    help="which of those keys to measure (cublas: only the cuBLAS figure; "
                         "--no-extras is 'none')")
    args = ap.parse_args()
    if args.no_extras:
        args.extras = "none"
    args.no_extras = args.extras == "none"
    w = WORKLOADS[args.workload]
    if args.steps is None:
        # about 2 s of timed device work at the expected rate
        args.steps = {"gemm_f16": 2000, "gemm_f16_512": 2000, "gemm_i8": 3000,
                      "gemm_bf16": 250, "attn_f16": 2000, "attn_bf16": 40,
                      "gemm_f16_fused": 2000, "gemm_f16_mn": 2000,
                      "attn_decode_bf16": 10000, "gemv_i8": 20000,
                      "gemm_i8_shard8": 20000}[args.workload]
        if args.impl == "reference":
            args.steps = 5
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        run_reference(args, w)
        return 0
    run_gpu(args, w)
    return 0


if __name__ == "__main__":
    sys.exit(main())
