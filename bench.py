#!/usr/bin/env python
"""Benchmark of the fused TDA forward (BASELINE.json metric: "fused TDA fwd
TFLOP/s & % bf16 tensor peak, S=8K D=128, at 1/2/4/8 B200").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tda|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...   (N > 1)

Workload (default): threshold differential attention, bf16, q1,q2,k1,k2,v of
shape (8, 32, 8192, 128) from seeded N(0,1), beta=1, lambda=0.5, p=2,
normalize=True, causal.  The 256 (batch, head) slices are split over the N
ranks (contiguous blocks, no collective on the data path); the total problem
is fixed, so scaling is strong.

One step = the key-norm pre-pass for k1 and k2 plus the fused forward kernel,
on inputs resident in HBM (2.7 GB of inputs, larger than the 126 MB L2, so no
flush is needed between steps).  FLOPs are the dense causal algorithmic count
3*B*H*S^2*D (QK1, QK2 and one PV), never the executed count.

Prints one JSON line on rank 0.  ``--impl reference`` times the CPU restatement
of the reference (oracle/) on the host cores instead; ``--impl reference-triton``
times the reference module's own Triton kernel on the GPU (N=1, from
baseline/_ref, installed by baseline/install_reference.sh).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fused TDA fwd TFLOP/s & % bf16 tensor peak, S=8K D=128, at 1/2/4/8 B200"

WORKLOADS = {
    # name: (op, B, H, S, D, beta, lambda, p, normalize)
    "diff8k": ("diff", 8, 32, 8192, 128, 1.0, 0.5, 2.0, True),
    "rect8k": ("rect", 8, 32, 8192, 128, 1.0, 0.0, 2.0, True),
    "rect4k": ("rect", 4, 32, 4096, 128, 1.0, 0.0, 2.0, True),
    "diff32k": ("diff", 1, 16, 32768, 128, 1.5, 0.8, 2.0, True),
    # one rank's share of BASELINE config 4 on 8 GPUs (2 of its 16 heads), timed on one GPU
    "diff32k_share8": ("diff", 1, 2, 32768, 128, 1.5, 0.8, 2.0, True),
    # one rank's share of the headline on 8 GPUs (32 of its 256 (batch, head) slices)
    "diff8k_share8": ("diff", 1, 32, 8192, 128, 1.0, 0.5, 2.0, True),
    "rect8k_share8": ("rect", 1, 32, 8192, 128, 1.0, 0.0, 2.0, True),
    # beta = 0 with normalize: P is nonzero wherever cos > 0 (about half the
    # entries), the dense worst case for the transform
    "diff8k_dense": ("diff", 8, 32, 8192, 128, 0.0, 0.5, 2.0, True),
    "rect8k_dense": ("rect", 8, 32, 8192, 128, 0.0, 0.0, 2.0, True),
    # small cases for profiler captures (inputs 168 / 201 MB, above the L2
    # size; a few hundred microseconds per launch); not bench lines.  The
    # *_s8k cases keep the full sequence length (CTAs of up to 64 key tiles).
    "diff2k": ("diff", 2, 32, 2048, 128, 1.0, 0.5, 2.0, True),
    "rect2k": ("rect", 4, 32, 2048, 128, 1.0, 0.0, 2.0, True),
    "diff_s8k": ("diff", 2, 8, 8192, 128, 1.0, 0.5, 2.0, True),
    "rect_s8k": ("rect", 4, 8, 8192, 128, 1.0, 0.0, 2.0, True),
    # BASELINE config 5's shape (parameter sweep), beta=1 p=2 normalized; with --dtype f32 the
    # exact-fp32 CUDA-core path
    "sweep2k": ("rect", 2, 16, 2048, 64, 1.0, 0.0, 2.0, True),
}

# dram__bytes_read.sum + dram__bytes_write.sum of one main-kernel launch,
# from one ncu capture of this bench's workload (a single-pass capture of those
# two metrics on the full-size launch)
MEASURED_TRAFFIC = {"diff8k": 3263129344, "rect8k": 2142068736}

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def flops_of(op, bh, S, D):
    return (3.0 if op == "diff" else 2.0) * bh * float(S) ** 2 * D


def bwd_flops_of(op, bh, S, D):
    """Dense causal algorithmic backward FLOPs: per branch five GEMMs of
    2*S*S*D/2 per (batch, head) (recomputed S, dP = dout V^T, dV = P^T dout,
    dQ = dA K, dK = dA^T Q), twice for the differential form."""
    return (10.0 if op == "diff" else 5.0) * bh * float(S) ** 2 * D


def describe(name):
    op, B, H, S, D, beta, lam, p, norm = WORKLOADS[name]
    lam_s = f" lambda={lam}" if op == "diff" else ""
    return f"{op} bf16 ({B},{H},{S},{D}) beta={beta}{lam_s} p={p} normalize={norm} causal"


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons during the
    timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id = gpu_id
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, val in zip(names, parts[4:8]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def gpu_smi_id(dev_index):
    import torch
    try:
        u = torch.cuda.get_device_properties(dev_index).uuid
        s = str(u)
        return s if s.startswith("GPU-") else "GPU-" + s
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            return vis.split(",")[dev_index]
        return str(dev_index)


# ------------------------------------------------------------- CPU baseline
def _use_all_cores():
    """Give numpy's BLAS every host core (torchrun sets OMP_NUM_THREADS=1).
    Returns the thread count in effect."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=n)
        return max((i.get("num_threads", 1) for i in threadpool_info()), default=n)
    except Exception:
        return n


def cpu_baseline(name, budget_s=10.0):
    """The oracle's fp32 formula (the reference's algorithm restated on CPU)
    on whole (batch, head) slices of the workload, one after another until the
    time budget is spent.  Returns (TFLOP/s, cores, sample description)."""
    import numpy as np
    from oracle import tda_oracle as O
    cores = _use_all_cores()
    op, B, H, S, D, beta, lam, p, norm = WORKLOADS[name]
    rng = np.random.Generator(np.random.PCG64(1234))
    n = 5 if op == "diff" else 3
    done = 0
    elapsed = 0.0  # compute time only (input generation excluded)
    while elapsed < budget_s:
        xs = [O.bf16_round(rng.standard_normal((1, 1, S, D), dtype=np.float32)) for _ in range(n)]
        t = time.perf_counter()
        if op == "diff":
            O.diff_fwd(*xs, beta, lam, p, norm, dtype=np.float32)
        else:
            O.rect_fwd(*xs, beta, p, norm, dtype=np.float32)
        elapsed += time.perf_counter() - t
        done += 1
    tf = flops_of(op, done, S, D) / elapsed / 1e12
    sample = f"{done} of {B * H} (batch,head) slices, all {S} rows, numpy fp32 formula"
    return tf, cores, sample, elapsed


def run_reference(args, rank, world):
    """--impl reference: the reference's algorithm on the host cores (the
    CPU restatement in oracle/, since the reference itself is Triton-only)."""
    if rank != 0:
        return 0
    import numpy as np
    from oracle import tda_oracle as O
    name = args.config
    op, B, H, S, D, beta, lam, p, norm = WORKLOADS[name]
    cores = _use_all_cores()
    rng = np.random.Generator(np.random.PCG64(4321))
    n = 5 if op == "diff" else 3
    xs = [O.bf16_round(rng.standard_normal((1, 1, S, D), dtype=np.float32)) for _ in range(n)]
    rows = np.arange(S - args.ref_rows, S)  # the last rows: each sees ~S keys

    def step():
        if op == "diff":
            O.diff_fwd(*xs, beta, lam, p, norm, dtype=np.float32, rows=rows)
        else:
            O.rect_fwd(*xs, beta, p, norm, dtype=np.float32, rows=rows)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    gemms = 3.0 if op == "diff" else 2.0
    step_flops = gemms * 2.0 * D * float(np.sum(rows + 1))  # causal algorithmic work of the sampled rows
    val = step_flops * args.steps / el / 1e12
    sample = f"1 (batch,head) slice, last {args.ref_rows} of {S} query rows, numpy fp32 formula"
    line = {
        "metric": METRIC, "value": val, "unit": "TFLOP/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": describe(name), "sample": sample},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_triton(args, rank, local, world):
    """--impl reference-triton: the unmodified reference module
    (``triton_threshold_attention.py``, installed into baseline/_ref by
    baseline/install_reference.sh) on this GPU, through its public functions,
    on the same inputs as the tda arm.  The reference upcasts to fp32 and runs
    its Triton kernel (TF32 dots, the whole S x S score map: ``T.py:66``) once
    per branch; the normalized rectified form is the reference called on
    F.normalize(q), F.normalize(k), as each branch of ``T.py:505-512`` does.
    N = 1 only (the reference has no multi-GPU path)."""
    if world > 1:
        if rank == 0:
            print(json.dumps({"impl": "reference-triton", "unavailable": "runs at N=1 only"}), flush=True)
        return 0
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref_dir, "triton_threshold_attention.py")):
        print(json.dumps({"impl": "reference-triton",
                          "unavailable": "baseline/_ref holds no reference install (baseline/install_reference.sh)"}),
              flush=True)
        return 0
    import torch
    import torch.nn.functional as F
    from tda_b200.shard import shard_range
    sys.path.insert(0, ref_dir)
    import triton_threshold_attention as ref

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    name = args.config
    op, B, H, S, D, beta, lam, p, norm = WORKLOADS[name]
    xs = make_inputs(name, shard_range(B * H, 1, 0), dev, "bhsd", args.dtype)
    bt = torch.tensor(beta)
    if op == "diff":
        lt = torch.tensor(lam, device=dev)

        def step():
            return ref.differential_threshold_rela_triton(*xs, bt, lt, p, norm)
    else:
        q, k, v = xs

        def step():
            if norm:
                return ref.threshold_rela_triton(F.normalize(q, dim=-1), F.normalize(k, dim=-1), v, bt, p)
            return ref.threshold_rela_triton(q, k, v, bt, p)

    timed = step
    if args.backward:
        # the reference's autograd backward (its ThresholdRelaFunction.backward
        # kernels, T.py:118-324 / :405-469, plus F.normalize's and the combine's
        # gradients) for the same upstream gradient as the tda arm's --backward
        xs_g = [x.detach().requires_grad_(True) for x in xs]
        if op == "diff":
            out = ref.differential_threshold_rela_triton(*xs_g, bt, lt, p, norm)
        elif norm:
            out = ref.threshold_rela_triton(F.normalize(xs_g[0], dim=-1), F.normalize(xs_g[1], dim=-1), xs_g[2], bt, p)
        else:
            out = ref.threshold_rela_triton(*xs_g, bt, p)
        g = torch.Generator(device=dev).manual_seed(777)
        dout = torch.randn(out.shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16).to(out.dtype)

        def timed():
            torch.autograd.backward(out, dout, retain_graph=True)

    for _ in range(args.warmup):
        timed()
    torch.cuda.synchronize()
    clocks = ClockSampler(gpu_smi_id(local))
    clocks.start()
    time.sleep(0.4)  # let the sampler start before the timed region
    ms = []
    for _ in range(args.steps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        timed()
        b.record()
        torch.cuda.synchronize()
        ms.append(a.elapsed_time(b))
    clk = clocks.stop()
    total = sum(ms)
    flops = bwd_flops_of(op, B * H, S, D) if args.backward else flops_of(op, B * H, S, D)
    val = flops * args.steps / (total * 1e-3) / 1e12
    line = {
        "metric": f"TDA backward TFLOP/s ({name})" if args.backward else METRIC, "value": val, "unit": "TFLOP/s",
        "impl": "reference-triton", "pass": "backward" if args.backward else "forward", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 (TF32 dots)",
        "data": "synthetic",
        "config": {"workload": describe(name) + (", fp32 inputs" if args.dtype == "f32" else ""),
                   "how": "reference public API, CUDA events per step on the current stream; FLOPs are the "
                          "same dense causal algorithmic count as the tda arm",
                   "flops_per_step": flops},
        "ms_per_step_min": min(ms),
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------- backward
def run_tda_backward(args, rank, local, world):
    """--backward: the backward pass (tda_rect_bwd per branch) of the workload,
    device-resident inputs and upstream gradient; value = algorithmic backward
    TFLOP/s (five GEMMs of 2*S*S*D/2 per branch and (batch, head))."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from tda_b200 import _lib
    from tda_b200.shard import max_over_ranks, shard_range

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    name = args.config
    op, B, H, S, D, beta, lam, p, norm = WORKLOADS[name]
    shard = shard_range(B * H, world, rank)
    f32 = args.dtype == "f32"
    kind = _lib.TDA_F32 if f32 else _lib.TDA_BF16
    xs = make_inputs(name, shard, dev, "bhsd", args.dtype)
    g = torch.Generator(device=dev).manual_seed(777 + shard.start)
    dout = torch.randn(xs[0].shape, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16).to(xs[0].dtype)
    n_bh = shard.size
    lib = _lib.load()
    grads = [torch.empty(xs[0].shape, dtype=torch.float32, device=dev) for _ in range(5)]
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    ptr = [x.data_ptr() for x in xs]
    lamc = min(max(lam, 0.0), 1.0)
    ws_n = lib.tda_bwd_workspace_size(kind, n_bh, S, D, int(norm))
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)
    from tda_b200 import ops
    status = ops._status_word(dev)

    def bwd(qp, kp, gq, gk, scale, acc):
        _lib.check(lib.tda_rect_bwd(qp, kp, ptr[-1], dout.data_ptr(), kind, gq.data_ptr(), gk.data_ptr(),
                                    grads[4].data_ptr(), n_bh, S, D, beta, p, int(norm), scale, acc,
                                    ws.data_ptr(), ws_n, status.data_ptr(), sp))

    def step():
        if op == "diff":
            bwd(ptr[0], ptr[2], grads[0], grads[2], 1.0, 0)
            bwd(ptr[1], ptr[3], grads[1], grads[3], -lamc, 1)
        else:
            bwd(ptr[0], ptr[1], grads[0], grads[1], 1.0, 0)

    for _ in range(args.warmup):
        step()
    barrier()
    clocks = ClockSampler(gpu_smi_id(local)) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.4)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    clk = clocks.stop() if clocks else None
    ms = max_over_ranks(e0.elapsed_time(e1), dev)
    fl = bwd_flops_of(op, B * H, S, D)
    value = fl * args.steps / (ms / 1e3) / 1e12
    peaks, peak_src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    peak_note = f"bf16_tflops (burst) of {peak_src}"
    if f32:
        peak = 148 * 128 * 2 * 1.965e9 / 1e12
        peak_note = "nominal FFMA peak, 148 SMs x 128 lanes x 2 x 1.965 GHz"
    ops.check_status(dev)
    achieved = bwd_flops_of(op, n_bh, S, D) * args.steps / (e0.elapsed_time(e1) / 1e3) / 1e12
    if rank == 0:
        line = {
            "metric": f"TDA backward TFLOP/s ({name})", "value": value, "unit": "TFLOP/s", "impl": "tda",
            "pass": "backward", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32" if f32 else "bf16", "data": "synthetic",
            "config": {"workload": describe(name) + (", fp32 inputs (CUDA-core path)" if f32 else "") + " backward", "batch": B, "heads": H, "seq_len": S,
                       "head_dim": D, "flops_per_step": fl,
                       "executed_flops_per_step_dense": fl * 8.0 / 5.0,
                       "kernels": "tda_bwd_dq_kernel + tda_bwd_dkv_kernel per branch" if f32 else
                       "key / query tables + tda_tc_bwd_dq_kernel + tda_tc_bwd_dkv_kernel per branch"},
            "roofline": {"bound": "fp32-fma" if f32 else "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None, "peak_source": peak_note},
            "cpu_baseline": None, "e2e": None,
            "gpu_launches": (2 if f32 else 4) * (2 if op == "diff" else 1) * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


# ------------------------------------------------------------------- GPU arm
def make_inputs(name, shard, device, layout="bhsd", dtype="bf16"):
    """Seeded N(0,1) inputs per (tensor, flattened head): identical data for a
    given head whatever the number of ranks.  layout "bshd" stores each tensor
    as (1, S, heads, D) and returns the (1, heads, S, D) transposed view, the
    layout of a fused QKV projection that the strided entry points read in
    place; dtype "f32" / "f16" keeps the same values in fp32 / fp16."""
    import torch
    op, B, H, S, D, beta, lam, p, norm = WORKLOADS[name]
    n = 5 if op == "diff" else 3
    tdt = {"f32": torch.float32, "f16": torch.float16}.get(dtype, torch.bfloat16)
    xs = []
    for t in range(n):
        if layout == "bshd":
            x = torch.empty((1, S, shard.size, D), dtype=tdt, device=device).transpose(1, 2)
        else:
            x = torch.empty((1, shard.size, S, D), dtype=tdt, device=device)
        for i, bh in enumerate(range(shard.start, shard.stop)):
            g = torch.Generator(device=device).manual_seed(1_000_003 * (t + 1) + bh)
            x[0, i] = torch.randn((S, D), generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
        xs.append(x)
    return xs


def run_tda(args, rank, local, world):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import tda_b200
    from tda_b200 import _lib, ops
    from tda_b200.shard import max_over_ranks, shard_range

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    name = args.config
    op, B, H, S, D, beta, lam, p, norm = WORKLOADS[name]
    shard = shard_range(B * H, world, rank)
    xs = make_inputs(name, shard, dev, args.layout, args.dtype)
    n_bh = shard.size
    lib = _lib.load()
    status = ops._status_word(dev)
    S_pad = (S + 127) // 128 * 128
    f32 = args.dtype == "f32"
    f16 = args.dtype == "f16"  # fp16 operands on the tensor cores: the call runs its own key pre-pass
    strided = args.layout == "bshd"
    out = torch.empty((1, n_bh, S, D), dtype=torch.float32 if f32 else (torch.float16 if f16 else torch.bfloat16),
                      device=dev)
    rk = [torch.zeros(n_bh * S_pad // 16 * 17, dtype=torch.float32, device=dev) for _ in range(2)]  # key tables
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    ptr = [x.data_ptr() for x in xs]

    # the fp32 path computes the norms inside its kernel; the strided entries
    # run their key-norm pre-pass inside the call (timed with the main kernel)
    separate_norms = norm and not f32 and not f16 and not strided
    # the strided entries take the key-table workspace; fp32 at head_dim 64 takes
    # the TF32 split copies of its tensor-core path (other fp32 head dims: none)
    ws_kind = _lib.TDA_F32 if f32 else (_lib.TDA_F16 if f16 else _lib.TDA_BF16)
    ws_n = (lib.tda_workspace_size(int(op == "diff"), ws_kind, n_bh, S, D, int(norm))
            if (strided or f32 or f16) else 0)
    ws = torch.empty(max(ws_n, 1), dtype=torch.uint8, device=dev)
    strides = (ctypes.c_int64 * (3 * len(xs)))(*[st for x in xs for st in x.stride()[:3]])

    def launch_norms():
        # the key tables of k (rect) or of k1 and k2 (diff, one launch)
        if separate_norms:
            if op == "diff":
                _lib.check(lib.tda_key_inv_norms_pair(ptr[2], ptr[3], _lib.TDA_BF16, n_bh, S, D, rk[0].data_ptr(),
                                                      rk[1].data_ptr(), sp))
            else:
                _lib.check(lib.tda_key_inv_norms(ptr[1], _lib.TDA_BF16, n_bh, S, D, rk[0].data_ptr(), sp))

    def launch_main():
        if f16:
            if op == "diff":
                _lib.check(lib.tda_diff_fwd(*ptr, out.data_ptr(), _lib.TDA_F16, _lib.TDA_F16, n_bh, S, D, beta, lam,
                                            p, int(norm), ws.data_ptr() if ws_n else None, ws_n,
                                            status.data_ptr(), sp))
            else:
                _lib.check(lib.tda_rect_fwd(*ptr, out.data_ptr(), _lib.TDA_F16, _lib.TDA_F16, n_bh, S, D, beta, p,
                                            int(norm), ws.data_ptr() if ws_n else None, ws_n, status.data_ptr(),
                                            sp))
        elif f32:
            if op == "diff":
                _lib.check(lib.tda_diff_fwd(*ptr, out.data_ptr(), _lib.TDA_F32, _lib.TDA_F32, n_bh, S, D, beta, lam,
                                            p, int(norm), ws.data_ptr() if ws_n else None, ws_n,
                                            status.data_ptr(), sp))
            else:
                _lib.check(lib.tda_rect_fwd(*ptr, out.data_ptr(), _lib.TDA_F32, _lib.TDA_F32, n_bh, S, D, beta, p,
                                            int(norm), ws.data_ptr() if ws_n else None, ws_n, status.data_ptr(),
                                            sp))
        elif strided:
            fn = lib.tda_diff_fwd_strided if op == "diff" else lib.tda_rect_fwd_strided
            extra = (beta, lam, p) if op == "diff" else (beta, p)
            _lib.check(fn(*ptr, ctypes.cast(strides, ctypes.c_void_p), out.data_ptr(), _lib.TDA_BF16, 1, n_bh, S,
                          D, *extra, int(norm), ws.data_ptr(), ws_n, status.data_ptr(), sp))
        elif op == "diff":
            _lib.check(lib.tda_diff_fwd_tc(ptr[0], ptr[1], ptr[2], ptr[3], ptr[4], out.data_ptr(), _lib.TDA_BF16,
                                           n_bh, S, D, beta, lam, p, int(norm), rk[0].data_ptr(),
                                           rk[1].data_ptr(), status.data_ptr(), sp))
        else:
            _lib.check(lib.tda_rect_fwd_tc(ptr[0], ptr[1], ptr[2], out.data_ptr(), _lib.TDA_BF16, n_bh, S, D, beta,
                                           p, int(norm), rk[0].data_ptr(), status.data_ptr(), sp))

    n_br = 2 if op == "diff" else 1
    tf32 = f32 and D in (64, 128)  # fp32 on the tensor cores: one split pre-pass launch and the forward
    launches_per_step = 2 if tf32 else int(norm and not f32) + 1

    for _ in range(args.warmup):
        launch_norms()
        launch_main()
    barrier()
    ops.check_status(dev)

    clocks = ClockSampler(gpu_smi_id(local)) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.4)  # let the sampler start before the timed region
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    barrier()
    for i in range(args.steps):
        ev[i][0].record(stream)
        launch_norms()
        ev[i][1].record(stream)
        launch_main()
        ev[i][2].record(stream)
    barrier()
    clk = clocks.stop() if clocks else None
    ops.check_status(dev)
    # executed tensor-core work of the main kernel, counted in one more
    # (untimed) launch: the 16-key P.V slabs it multiplied against those a
    # dense P.V would multiply (bf16 / fp16 tensor-core path)
    pv_slabs = None
    if not f32:
        cnt = torch.zeros(2, dtype=torch.int64, device=dev)
        _lib.check(lib.tda_debug_stats(cnt.data_ptr()))
        try:
            launch_norms()
            launch_main()
            torch.cuda.synchronize(dev)
        finally:
            _lib.check(lib.tda_debug_stats(None))
        issued, dense = (int(x) for x in cnt.tolist())
        if dense > 0:
            pv_slabs = (issued, dense)
    total_ms = ev[0][0].elapsed_time(ev[-1][2])
    main_ms = [ev[i][1].elapsed_time(ev[i][2]) for i in range(args.steps)]
    norm_ms = [ev[i][0].elapsed_time(ev[i][1]) for i in range(args.steps)]
    total_ms_max = max_over_ranks(total_ms, dev)
    main_avg = statistics.mean(main_ms)
    main_avg_max = max_over_ranks(main_avg, dev)

    flops_total = flops_of(op, B * H, S, D)
    value = flops_total * args.steps / (total_ms_max / 1e3) / 1e12
    peaks, peak_src = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    peak_note = f"bf16_tflops (burst) of {peak_src}"
    if tf32:
        # three TF32 products per fp32 product at the TF32 rate, half the bf16 rate on B200
        peak = peak / 2.0 / 3.0
        peak_note = f"bf16_tflops (burst) of {peak_src} / 2 (TF32 rate) / 3 (products per fp32 product)"
    elif f32:
        # FFMA: 148 SMs x 128 FMA lanes x 2 FLOP x 1.965 GHz (nominal; no measured fp32 figure)
        peak = 148 * 128 * 2 * 1.965e9 / 1e12
        peak_note = "nominal FFMA peak, 148 SMs x 128 lanes x 2 x 1.965 GHz"
    achieved = flops_of(op, n_bh, S, D) / (main_avg / 1e3) / 1e12  # this rank's launch
    executed = None
    if pv_slabs:
        # tensor-core work the main kernel ran on this rank: every QK product of
        # the (query tile, key tile) pairs it processed (dense / 8 of them, 8
        # 16-key slabs per tile) and the hi + lo products of each P.V slab it
        # multiplied (P is split into two bf16 / fp16 parts)
        issued, dense = pv_slabs
        n_qk = 2 if op == "diff" else 1
        kt = 128  # query / key tile edge of the tensor-core kernels
        ex = dense // 8 * n_qk * 2 * kt * kt * D + issued * 2 * 2 * kt * 16 * D
        executed = {"pv_slabs_issued": issued, "pv_slabs_dense": dense, "pv_issued_frac": issued / dense,
                    "tflops": ex / (main_avg / 1e3) / 1e12, "frac_of_peak": ex / (main_avg / 1e3) / 1e12 / peak,
                    "how": "one extra untimed launch with tda_debug_stats counters; all QK products of the "
                           "processed tiles plus hi + lo products of the multiplied P.V slabs, over the "
                           "timed mean main-kernel time"}

    # ---- end to end through the public API with pinned host buffers
    # host copies keep the device layout (the storage of a bshd view)
    stor = [x.transpose(1, 2) if strided else x for x in xs]
    host_in = [x.cpu().pin_memory() for x in stor]
    host_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    h2d = sum(x.numel() * x.element_size() for x in host_in)
    d2h = host_out.numel() * host_out.element_size()
    betat, lamt = torch.tensor(beta), torch.tensor(lam)

    # (batch, head) slices are independent, so the step streams chunks of
    # heads: host->device copy of chunk c+1 (copy engine), the public API on
    # chunk c (compute stream) and device->host copy of chunk c-1 (second copy
    # engine) overlap.  Every byte of every input and of the output crosses
    # PCIe inside the timed region.
    dev_in = [torch.empty_like(x) for x in stor]
    # a chunk of heads of a bshd tensor is not one block of memory: copy it whole
    n_chunks = 1 if strided else min(n_bh, 8)
    bounds = [(c * n_bh // n_chunks, (c + 1) * n_bh // n_chunks) for c in range(n_chunks)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    def e2e_step():
        start = torch.cuda.Event()
        start.record(stream)
        s_in.wait_event(start)
        s_out.wait_event(start)
        ready = []
        with torch.cuda.stream(s_in):
            for a, b in bounds:
                for hbuf, dbuf in zip(host_in, dev_in):
                    if strided:
                        dbuf.copy_(hbuf, non_blocking=True)
                    else:
                        dbuf[:, a:b].copy_(hbuf[:, a:b], non_blocking=True)
                e = torch.cuda.Event()
                e.record(s_in)
                ready.append(e)
        for (a, b), e in zip(bounds, ready):
            stream.wait_event(e)
            d = [x.transpose(1, 2) if strided else x[:, a:b] for x in dev_in]
            if op == "diff":
                o = tda_b200.differential_threshold_rela_triton(*d, betat, lamt, p, norm)
            else:
                o = tda_b200.threshold_rela_triton(*d, betat, p, norm)
            done = torch.cuda.Event()
            done.record(stream)
            s_out.wait_event(done)
            o.record_stream(s_out)
            with torch.cuda.stream(s_out):
                host_out[:, a:b].copy_(o, non_blocking=True)
        end = torch.cuda.Event()
        end.record(s_out)
        stream.wait_event(end)

    e2e_steps = max(1, min(args.steps, 5))
    e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    ops.check_status(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), dev)
    e2e_val = flops_total * e2e_steps / (e2e_ms / 1e3) / 1e12

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tf, cores, sample, _ = cpu_baseline(name, args.cpu_budget)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}

    n_inputs = 5 if op == "diff" else 3
    in_bytes = n_inputs * B * H * S * D * (4 if f32 else 2) // world
    l2_note = (f"inputs {in_bytes / 1e9:.2f} GB per GPU > 126 MB L2; no flush" if in_bytes > 126e6 else
               f"inputs {in_bytes / 1e6:.0f} MB per GPU, not above the 126 MB L2")
    if rank == 0:
        traffic = None if (f32 or strided) else MEASURED_TRAFFIC.get(name)
        if traffic is not None and world > 1:
            # measured at N = 1; a launch's DRAM bytes are proportional to the (batch, head) slices it covers
            traffic = traffic * n_bh / (B * H)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "TFLOP/s",
            "impl": "tda",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms_max / args.steps,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32" if f32 else ("f16" if f16 else "bf16"),
            "data": "synthetic",
            "pct_bf16_peak": None if f32 else value / world / peak,
            "config": {
                "workload": describe(name) + ((", fp32 inputs (tensor cores, three TF32 products per product; "
                                               "main_kernel_ms includes the split pre-pass)") if tf32 else
                                              (", fp32 inputs (CUDA-core path)" if f32 else
                                               (", fp16 inputs (tensor cores, fp16 operands; main_kernel_ms "
                                                "includes the key pre-pass)" if f16 else "")))
                + (", (B, S, H, D) storage read in place through the strided entry (main_kernel_ms includes "
                   "its key-norm pre-pass)" if strided else ""),
                "layout": args.layout,
                "batch": B, "heads": H, "seq_len": S, "head_dim": D,
                "parallelism": f"(batch x head) shards over {world} GPU(s), no collective on the data path",
                "flops_per_step": flops_total,
                "l2": l2_note,
                "key_norm_ms_per_step": statistics.mean(norm_ms),
                "main_kernel_ms": main_avg,
                "main_kernel_ms_max_rank": main_avg_max,
            },
            "roofline": {
                "bound": "tensor" if (tf32 or not f32) else "fp32-fma",
                "achieved": achieved,
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "peak_source": peak_note,
            },
            "executed": executed,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "TFLOP/s",
                    "how": f"public API on {n_chunks} chunks of (batch, head) slices per rank; pinned-host "
                           "inputs in and output out, copies overlapped with compute on two copy streams",
                    "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["tda", "reference", "reference-triton"], default="tda",
                    help="reference: the reference's algorithm on the host cores (the driver's reference arm); "
                         "reference-triton: the reference module's own Triton kernel on this GPU (N=1)")
    ap.add_argument("--config", choices=sorted(WORKLOADS), default="diff8k")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU-baseline work")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layout", choices=["bhsd", "bshd"], default="bhsd",
                    help="bshd: (B, S, H, D) storage passed as transposed views (strided entry points)")
    ap.add_argument("--dtype", choices=["bf16", "f32", "f16"], default="bf16",
                    help="f32: fp32 inputs (tensor cores at head_dim 64 / 128, else CUDA cores); f16: fp16 inputs "
                         "on the tensor cores")
    ap.add_argument("--backward", action="store_true",
                    help="time the backward pass of the workload instead of the forward")
    ap.add_argument("--ref-rows", type=int, default=256, help="query rows per reference-arm step")
    args = ap.parse_args()
    from tda_b200.shard import env_rank_world
    rank, local, world = env_rank_world()
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.impl == "reference-triton":
        return run_reference_triton(args, rank, local, world)
    if args.backward:
        return run_tda_backward(args, rank, local, world)
    return run_tda(args, rank, local, world)


if __name__ == "__main__":
    sys.exit(main())
