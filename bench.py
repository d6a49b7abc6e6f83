"""Benchmark: attention forward TFLOPS (4*B*H*N^2*d / t) on 1..8 B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 3]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1, one rank per GPU)

Workload (the configuration its 1/2/4/8-GPU metric and
its 60%-of-peak target are quoted on): B=64 H=64 N=1024 d=64, bf16 Q/K/V ~ N(0,1)
(seeded, synthetic), scale 1/8, non-causal. The 4096 B*H slices are split over
the ranks with no collective (strong scaling: total work fixed).

One step = one kernel launch over this rank's slices, inputs resident in HBM.
`value` = total FLOPs of all ranks / max-over-ranks device time.
`e2e`   = the same metric through the public host-buffer API (blackflash_b200.blackflash_host):
          Q/K/V in pinned host memory, O returned in host memory, every step; the
          copies of one slice group overlap the kernel of the previous one.
`--impl reference` times the reference's CPU path (torch fp32 math attention,
reference tests/test_blackflash.py:16-19) on the host cores, rank 0 only.

Inputs (3 x 512 MiB at N=1) exceed the 126 MB L2, so no flush is needed between
steps; the JSON says so.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

CONFIGS = {
    # name: (B, H, N, d, dist)
    "1": (2, 2, 512, 64, "normal"),
    "2": (4, 8, 1024, 64, "normal"),
    "3": (64, 64, 1024, 64, "normal"),
    "4": (8, 16, 8192, 64, "peaked"),
    # long sequence: sequence-sharded over the ranks, KV rotated ring-style over NCCL, LSE merge
    "5": (1, 32, 65536, 64, "normal"),
    # profiling case: same per-slice shape as config 3, 1/4 of the slices (1.6 GB device memory)
    "prof": (16, 64, 1024, 64, "normal"),
    # one rank's share of config 3 at 8 GPUs (512 slices), run on one GPU
    "r8": (8, 64, 1024, 64, "normal"),
    # head dimension 128 (extension; the reference kernel is d = 64 only)
    "d128": (16, 16, 4096, 128, "normal"),
    # attention backward (extension), d = 64: a main case and a small profiling case
    "bwd": (16, 16, 4096, 64, "normal"),
    "bwdprof": (4, 16, 2048, 64, "normal"),
}
METRIC = "attention fwd TFLOPS (4BHN^2d/t)"

# DRAM bytes (read + write) per launch of the main kernel for config 3 at N=1. Measured by
# ncu on a quarter-size case (profiles/fa_fwd_sm100_b16h64n1024.md: 402.7 MB read +
# 114.5 MB written for 1024 slices) and scaled by 4; traffic is linear in the slice count
# because every slice is independent.
TRAFFIC_BYTES = {"3": 4 * (402.700032e6 + 114.543360e6)}


def flops(B, H, N, d):
    return 4.0 * B * H * N * N * d


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"bf16_tflops": p.get("bf16_tflops"), "bf16_tflops_sustained": p.get("bf16_tflops_sustained"),
                "hbm_gbs": p.get("hbm_gbs"), "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle sampling in the background (200 ms period)."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []  # (host_time, sm_mhz, max_mhz, reasons)
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                sm, mx = float(parts[2]), float(parts[3])
            except ValueError:
                continue
            reasons = [n for n, v in zip(names, parts[6:10]) if v.lower() == "active"]
            self.samples.append((time.time(), sm, mx, reasons))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self, t0: float, t1: float):
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        window = "timed"
        if not inside:  # timed region shorter than the sampling period: use the loaded samples around it
            inside = [s for s in self.samples if t0 - 1.0 <= s[0] <= t1 + 0.5]
            window = "timed+-1s"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "window": "none"}
        reasons = sorted({r for s in inside for r in s[3]})
        return {"sm_mhz": statistics.median(s[1] for s in inside), "sm_max_mhz": max(s[2] for s in inside),
                "reasons": reasons, "samples": len(inside), "window": window}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_reference_sample(B, H, N, d, dist, budget_s: float, seed: int = 0):
    """Reference CPU path (torch fp32 math, tests/test_blackflash.py:16-19) on a bounded
    sample of the workload: whole (b,h) slices, and for long sequences a block of at
    most 2048 query rows per slice against all N keys. Returns
    (TFLOPS, sample description, seconds, threads)."""
    from blackflash_b200.inputs import make_qkv
    from oracle import oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    chunk = 4 if N <= 8192 else 1
    rows = min(N, 2048)
    q, k, v = make_qkv(1, chunk, N, d, dist=dist, seed=seed)
    q = q[:, :, :rows].contiguous()
    oracle.torch_math(q, k, v, 1.0 / math.sqrt(d))  # warm-up
    done, t0 = 0, time.perf_counter()
    while True:
        oracle.torch_math(q, k, v, 1.0 / math.sqrt(d))
        done += chunk
        el = time.perf_counter() - t0
        if el >= budget_s or done >= B * H:
            break
    sample = f"{done} of {B*H} (b,h) slices" + (f", {rows} of {N} query rows each" if rows < N else "")
    return 4.0 * done * rows * N * d / el / 1e12, sample, el, torch.get_num_threads()


def workload_desc(B, H, N, d, dist):
    """The workload string both arms print (the same for the same configuration)."""
    return f"B={B} H={H} N={N} d={d} {dist}, non-causal, scale 1/sqrt({d})"


# Reference-arm steps run the whole workload when it takes at most this many seconds
# on the host (config 3: ~3 s on 16 cores); larger configs time a bounded sample.
REF_FULL_MAX_FLOP = 4.0 * 64 * 64 * 1024 * 1024 * 64


def run_reference(args, cfg_name):
    """The reference's CPU path (torch fp32 math, tests/test_blackflash.py:16-19) on all
    host threads, rank 0 only. For configs up to config 3's size every step computes the
    whole workload (every (b,h) slice), so ms_per_step is a measured step time; larger
    configs time a bounded sample of slices per step and say so."""
    world, rank, _ = dist_env()
    if rank != 0:
        return  # rank 0 alone runs the CPU reference
    from blackflash_b200.inputs import make_qkv
    from oracle import oracle
    B, H, N, d, dist = CONFIGS[cfg_name]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    scale = 1.0 / math.sqrt(d)
    full = flops(B, H, N, d) <= REF_FULL_MAX_FLOP
    if full:
        q, k, v = (t.reshape(B * H, N, d) for t in make_qkv(B, H, N, d, dist=dist, seed=1000))
        chunk = 4

        def step():
            for s0 in range(0, B * H, chunk):
                oracle.torch_math(q[s0:s0 + chunk], k[s0:s0 + chunk], v[s0:s0 + chunk], scale)
            return flops(B, H, N, d)
        sample = f"whole workload every step: all {B*H} (b,h) slices, torch fp32 CPU math, {chunk} slices per call"
    else:
        budget = args.ref_step_seconds

        def step():
            tf, _, el, _ = cpu_reference_sample(B, H, N, d, dist, budget_s=budget)
            return tf * 1e12 * el
        sample = (f"bounded sample per step (about {budget:.0f} s of whole slices, at most 2048 query rows each); "
                  f"TFLOPS = sampled FLOPs / time")
    for _ in range(args.warmup if full else 1):
        step()
    t_total, f_total = 0.0, 0.0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        f_total += step()
        t_total += time.perf_counter() - t0
    value = f_total / t_total / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_total / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_desc(B, H, N, d, dist), "global_batch": B, "seq_len": N,
                   "parallelism": "cpu host cores (rank 0 only)"},
        "cpu_baseline": {"value": value, "unit": "TFLOPS", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_bwd(args, cfg_name):
    """Backward configs (one GPU): `attention_backward` on inputs resident in HBM, after one
    forward for O and lse (outside the timed region). FLOPs are counted as 2.5x the forward's."""
    from blackflash_b200 import attention_backward, forward_lse
    from blackflash_b200.inputs import make_qkv

    world, rank, local = dist_env()
    if world != 1:
        raise SystemExit("backward configs run on one GPU")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    B, H, N, d, dist = CONFIGS[cfg_name]
    q, k, v = make_qkv(B, H, N, d, dist=dist, seed=1000, device=dev)
    g = torch.Generator(device=dev).manual_seed(7)
    do = torch.randn(q.shape, generator=g, device=dev).to(torch.bfloat16)
    scale = 1.0 / math.sqrt(d)
    O, lse, _ = forward_lse(q, k, v, scale)
    for _ in range(args.warmup):
        attention_backward(q, k, v, O, do, lse, scale)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0 = time.time()
    e0.record(stream)
    for _ in range(args.steps):
        attention_backward(q, k, v, O, do, lse, scale)
    e1.record(stream)
    torch.cuda.synchronize()
    h1 = time.time()
    sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    f = 2.5 * flops(B, H, N, d)
    value = f / (ms * 1e-3) / 1e12
    peaks = load_peaks()
    line = {
        "metric": "attention bwd TFLOPS (2.5*4BHN^2d/t)", "value": value, "unit": "TFLOPS", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"backward B={B} H={H} N={N} d={d} {dist}, non-causal, scale 1/sqrt({d})",
                   "global_batch": B, "seq_len": N, "parallelism": "single GPU",
                   "l2": "inputs larger than L2" if 5 * q.numel() * 2 > 126e6 else "inputs fit in L2"},
        "roofline": {"bound": "tensor", "achieved": value, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": value / peaks["bf16_tflops"], "traffic": None,
                     "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)",
                     "kernel": "fa_bwd_kernel (+ bwd_prep_kernel, bwd_dq_kernel, dq memset)"},
        "cpu_baseline": None,
        "clocks": sampler.summary(h0, h1),
        "gpu_launches": args.steps * 3,
    }
    print(json.dumps(line), flush=True)


def cudnn_comparator(q, k, v, scale, f_launch, steps=10):
    """The vendor library on the same device and the same inputs: torch SDPA restricted to
    its cuDNN backend, timed with CUDA events after the main timed region (not part of
    `value`). Returns TFLOPS, or the reason it could not run."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from torch.nn.functional import scaled_dot_product_attention as sdpa
    try:
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            for _ in range(3):
                out = sdpa(q, k, v, scale=scale)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                out = sdpa(q, k, v, scale=scale)
            e1.record()
            torch.cuda.synchronize()
        del out
    except RuntimeError as e:
        return {"unavailable": str(e).splitlines()[0][:200]}
    ms = e0.elapsed_time(e1) / steps
    return {"value": f_launch / (ms * 1e-3) / 1e12, "unit": "TFLOPS", "ms_per_launch": ms,
            "what": "torch SDPA, cuDNN backend only, same inputs and device, CUDA events"}


def run_ours(args, cfg_name):
    import torch.distributed as dist_mod

    from blackflash_b200 import _lib
    from blackflash_b200.inputs import make_qkv
    from blackflash_b200.shard import slice_range

    world, rank, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist_mod.init_process_group("nccl", device_id=dev)

    B, H, N, d, dist = CONFIGS[cfg_name]
    total = B * H
    s0, s1 = slice_range(total, world, rank)
    my = s1 - s0
    q, k, v = make_qkv(1, my, N, d, dist=dist, seed=1000 + rank, device=dev)
    O = torch.empty_like(q)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    scale = 1.0 / math.sqrt(d)

    def step():
        rc = lib.blackflash_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), O.data_ptr(), None, None, 1, my, N, d,
                                scale, stream.cuda_stream)
        if rc != 0:
            raise RuntimeError(lib.blackflash_last_error().decode())

    def barrier():
        if world > 1:
            dist_mod.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist_mod.all_reduce(t, op=dist_mod.ReduceOp.MAX)
        return float(t.item())

    w0, w1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0.record(stream)
    for _ in range(args.warmup):
        step()
    w1.record(stream)
    torch.cuda.synchronize()
    warm_ms = max(w0.elapsed_time(w1) / args.warmup, 1e-3)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    # Untimed steps that keep the GPU loaded while the sampler settles, for at least
    # ~20 ms, so the timed steps start at the clocks of a busy GPU.
    for _ in range(max(args.warmup, math.ceil(20.0 / warm_ms))):
        step()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    h1 = time.time()
    barrier()
    ms_local = ev0.elapsed_time(ev1)
    sampler.stop()
    ms_total = max_over_ranks(ms_local)
    ms_step = ms_total / args.steps
    f_total = flops(B, H, N, d)
    f_rank = flops(1, my, N, d)
    value = f_total / (ms_step * 1e-3) / 1e12
    clocks = sampler.summary(h0, h1)

    # ---- end to end through the public API with host buffers: blackflash_host takes pinned
    # host Q/K/V and returns O in host memory, overlapping the copies with the kernel.
    from blackflash_b200 import blackflash_host
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty(O.shape, dtype=O.dtype, pin_memory=True)
    e2e_steps = max(1, min(args.steps, args.e2e_steps))

    def e2e_step():
        blackflash_host(qh, kh, vh, scale, device=dev, out=oh)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()  # the caller's stream waits for the copies and the kernel of the call
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    e2e_value = f_total / (e2e_ms * 1e-3) / 1e12
    bytes_in = 3 * q.numel() * q.element_size()
    bytes_out = O.numel() * O.element_size()

    comparators = None
    if world == 1 and not args.no_comparators:
        comparators = {"cudnn_sdpa": cudnn_comparator(q, k, v, scale, f_rank)}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tf, desc, el, threads = cpu_reference_sample(B, H, N, d, dist, budget_s=args.cpu_seconds)
        cpu = {"value": tf, "unit": "TFLOPS", "cores": threads, "kind": "port",
               "sample": f"{desc} of the same workload, torch fp32 CPU math "
                         f"(reference tests/test_blackflash.py:16-19), {el:.1f} s"}

    if rank == 0:
        peaks = load_peaks()
        per_gpu_achieved = f_rank / (ms_local / args.steps * 1e-3) / 1e12  # rank 0's kernel rate
        peak = peaks["bf16_tflops"]
        traffic = TRAFFIC_BYTES.get(cfg_name)
        if traffic is not None:
            traffic *= my / total  # per launch on this rank: traffic is linear in the slice count
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload_desc(B, H, N, d, dist),
                       "global_batch": B, "seq_len": N, "parallelism": f"bxh{world} (no collective)",
                       "l2": "inputs larger than L2 (no flush)", "slices_per_rank": my},
            "roofline": {"bound": "tensor", "achieved": per_gpu_achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": per_gpu_achieved / peak if peak else None, "traffic": traffic,
                         "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)",
                         "kernel": "fa_fwd_sm100_kernel" if d == 64 else "fa_fwd_d128_kernel", "flops_per_launch": f_rank},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": "TFLOPS", "h2d_bytes_per_step": bytes_in,
                    "d2h_bytes_per_step": bytes_out, "ms_per_step": e2e_ms},
            "gpu_launches": args.steps,
        }
        if comparators is not None:
            line["comparators"] = comparators
        print(json.dumps(line), flush=True)
    if world > 1:
        dist_mod.destroy_process_group()


SP_DESC = {
    "ring": "ring{world}: KV rotated both ways round the ring by NCCL send/recv, two blocks per step in one kernel, LSE merge per step",
    "ring1": "ring{world}: KV rotated one way by NCCL send/recv, one block per step, LSE merge per step",
    "ipc": "ring{world}: KV rotated both ways by peer copies over CUDA IPC (copy engines, NVLink), GPU-side flags, C++ driver, LSE merge per step",
    "allgather": "sp{world}: NCCL all-gather of K/V overlapping the own-block kernel, one gathered-block kernel, one LSE merge",
}


def sp_launches(mode: str, w: int) -> int:
    """Our kernels per step (partials, merges, the bf16 cast)."""
    if mode == "allgather":
        return 4 if w > 1 else 2
    if mode == "ipc" and w > 1:
        nl, nr = w // 2, (w + 1) // 2 - 1
        compute = 1 + 3 * nl + nr + 1                               # partials, flag waits, merges, cast
        copies = (3 * nl - 1) + (3 * nr - 1 if nr > 0 else 0)      # flag waits and sets of the two push streams
        signals = nl + nr + 2                                       # slot-free flag sets
        return compute + copies + signals
    if mode == "ring" and w > 2:
        return 1 + 2 * (w // 2) + 1
    return 2 * w


def run_ring(args, cfg_name):
    """Config 5: the sequence is split over the ranks and KV rotates round the ring
    (NCCL send/recv into local buffers, overlapping the kernels; LSE merge per step).
    --sp-mode ring (default) rotates both ways, two blocks per step in one launch;
    ring1 is the one-way ring; allgather replaces the rotation by one all-gather."""
    import torch.distributed as dist_mod

    from blackflash_b200.inputs import make_qkv
    from blackflash_b200.ring import allgather_attention, close_ipc_rings, ipc_ring_attention, ring_attention

    if args.sp_mode == "allgather":
        sp = allgather_attention
    elif args.sp_mode == "ipc":
        sp = ipc_ring_attention
    else:
        def sp(q_, k_, v_, scale_):
            return ring_attention(q_, k_, v_, scale_, bidirectional=(args.sp_mode == "ring"))
    world, rank, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist_mod.init_process_group("nccl", device_id=dev)
    B, H, N, d, dist = CONFIGS[cfg_name]
    if N % world:
        raise SystemExit("N must divide evenly over the ranks")
    n_loc = N // world
    q, k, v = (t.reshape(B * H, n_loc, d) for t in make_qkv(B, H, n_loc, d, dist=dist, seed=2000 + rank, device=dev))
    scale = 1.0 / math.sqrt(d)
    stream = torch.cuda.current_stream(dev)

    def step():
        return sp(q, k, v, scale)

    def barrier():
        if world > 1:
            dist_mod.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist_mod.all_reduce(t, op=dist_mod.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    h0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    h1 = time.time()
    barrier()
    sampler.stop()
    ms_step = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    f_total = flops(B, H, N, d)
    value = f_total / (ms_step * 1e-3) / 1e12

    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)

    def e2e_step():
        o = sp(qh.to(dev, non_blocking=True), kh.to(dev, non_blocking=True),
                           vh.to(dev, non_blocking=True), scale)
        oh.copy_(o, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tf, desc, el, threads = cpu_reference_sample(B, H, N, d, dist, budget_s=args.cpu_seconds)
        cpu = {"value": tf, "unit": "TFLOPS", "cores": threads, "kind": "port",
               "sample": f"{desc} of the same workload, torch fp32 CPU math, {el:.1f} s"}
    if rank == 0:
        peaks = load_peaks()
        per_gpu = value / world
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOPS", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"B={B} H={H} N={N} d={d} {dist}, non-causal, sequence-parallel",
                       "global_batch": B, "seq_len": N, "parallelism": SP_DESC[args.sp_mode].format(world=world),
                       "l2": "inputs larger than L2 (no flush)"},
            "roofline": {"bound": "tensor", "achieved": per_gpu, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": per_gpu / peaks["bf16_tflops"], "traffic": None,
                         "peak_source": f"{peaks['source']} bf16 burst (MEASURED_PEAKS.json)",
                         "kernel": "fa_fwd_sm100_kernel (fp32 partial mode)"},
            "cpu_baseline": cpu,
            "clocks": sampler.summary(h0, h1),
            "e2e": {"value": f_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOPS",
                    "h2d_bytes_per_step": 3 * q.numel() * 2, "d2h_bytes_per_step": q.numel() * 2,
                    "ms_per_step": e2e_ms},
            "gpu_launches": args.steps * sp_launches(args.sp_mode, world),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        if args.sp_mode == "ipc":
            close_ipc_rings()
        dist_mod.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="3")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-step-seconds", type=float, default=2.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-comparators", action="store_true", help="skip the cuDNN SDPA comparison")
    ap.add_argument("--sp-mode", choices=["ring", "ring1", "allgather", "ipc"], default="ring",
                    help="sequence-parallel schedule of config 5")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args, args.config)
    elif args.config == "5":
        run_ring(args, args.config)
    elif args.config in ("bwd", "bwdprof"):
        run_bwd(args, args.config)
    else:
        run_ours(args, args.config)


if __name__ == "__main__":
    main()
