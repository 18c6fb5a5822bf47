"""Benchmark of the AdaAttn attention-forward hot path on B200.

Workload: dense BF16 causal attention, B8 H32 N4096 D128 (Q, K, V iid
N(0,1)/sqrt(D), seeded), precision forced to BF16 and rank to dense -- the
peak-throughput configuration. One step = one attention forward over one
batch, inputs resident in HBM (805 MB > L2, so no flush is needed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Multi-GPU (torchrun, one process per GPU): weak scaling by (batch x head)
shards -- every rank processes its own B8 H32 slice of a job N times larger,
no collective inside the timed attention; an NCCL all-gather of outputs is
timed separately afterwards. Rank 0 prints one JSON line.

--impl reference times the reference algorithm's CPU implementation (the
oracle's restatement of AdaAttention._compute_dense_attention) on the host
cores, on a bounded sample of the same workload per step.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = ("attn fwd TFLOP/s & % TC peak at B8 H32 N4096 D128; tokens/s at 1/2/4/8 B200")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
PROFILE = os.path.join(ROOT, "profiles", "fmha_tc_bf16_dense_bf16.md")


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def profiled_traffic():
    """DRAM bytes per launch of the attention kernel from the committed ncu
    summary (a line 'dram_bytes_per_launch_full = <int>'), else None."""
    if not os.path.exists(PROFILE):
        return None
    for line in open(PROFILE):
        if line.strip().startswith("dram_bytes_per_launch_full"):
            try:
                return int(float(line.split("=")[1].split()[0]))
            except (ValueError, IndexError):
                return None
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index: int, period: float = 0.05):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            if not uuid.startswith("GPU-"):
                uuid = "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid.encode())
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None
        self.period = period

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_sample(workload, seconds: float = 10.0, max_reps: int = 50):
    """Time the oracle's dense BF16 attention on a slice of the workload.

    Sample: batch row 0, `heads` heads, full sequence; repeated until about
    `seconds` of CPU work. Returns (TFLOP/s, threads, description)."""
    import oracle as O
    from adaattn_b200.workloads import make_qkv
    torch.set_num_threads(os.cpu_count() or 1)
    heads = 4
    w = workload.scaled(batch=1, heads=heads)
    q, k, v = make_qkv(w, seed=0)
    flops = w.dense_flops()
    times = []
    t_start = time.perf_counter()
    while len(times) < max_reps:
        t0 = time.perf_counter()
        O.dense_attention(q, k, v, O.BF16, 1.0 / math.sqrt(w.head_dim), w.causal)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > seconds and len(times) >= 2:
            break
    t = statistics.median(times)
    desc = (f"oracle dense BF16 (torch CPU, the reference's arithmetic) on batch row 0, "
            f"{heads} of {workload.heads} heads, N={w.seq}; median of {len(times)} runs, "
            f"{t * 1e3:.1f} ms each; throughput scales to the full workload "
            f"(slices are independent)")
    return flops / t / 1e12, torch.get_num_threads(), desc


def run_reference(args, workload):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    seconds = max(1.0, min(10.0, 120.0 / max(1, args.steps + args.warmup)))
    vals = []
    cores = None
    desc = ""
    for i in range(args.warmup + args.steps):
        v, cores, desc = cpu_sample(workload, seconds=seconds, max_reps=3)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    flops = workload.dense_flops()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": flops / (value * 1e12) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1)/sqrt(D) bf16",
        "config": workload_config(workload, args.gpus),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": desc + ("; the host cores of one node, so the same value at "
                                           "every GPU count" if args.gpus > 1 else "")},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "tokens_per_s": workload.tokens / (flops / (value * 1e12)),
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(w, n):
    return {"workload": f"dense_bf16 causal attention B{w.batch} H{w.heads} N{w.seq} "
                        f"D{w.head_dim}, precision forced BF16, rank forced dense",
            "batch_per_gpu": w.batch, "global_batch": w.batch * n, "heads": w.heads,
            "seq_len": w.seq, "head_dim": w.head_dim, "causal": w.causal,
            "parallelism": f"(batch x head) shards, {n} GPU(s), no collective in attention",
            "l2": "inputs 805 MB per GPU > 126 MB L2 (no flush needed)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="profiling only: smaller batch than the B8 workload")
    ap.add_argument("--heads", type=int, default=None,
                    help="profiling only: fewer heads than the H32 workload")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    from adaattn_b200.workloads import WORKLOADS, make_qkv
    workload = WORKLOADS["dense_bf16"].scaled(batch=args.batch, heads=args.heads)
    if args.impl == "reference":
        return run_reference(args, workload)

    import torch.distributed as dist
    from adaattn_b200 import PrecisionMode, attention_forward, attention_forward_host
    from adaattn_b200.core import host_buffer_bytes
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    w = workload
    scale = 1.0 / math.sqrt(w.head_dim)
    q, k, v = make_qkv(w, seed=1000 + rank, device=str(dev))
    out = torch.empty(w.batch, w.seq, w.heads, w.head_dim, dtype=w.dtype, device=dev)
    out_v = out.transpose(1, 2)

    def step():
        attention_forward(q, k, v, scale=scale, causal=w.causal,
                          static_precision=PrecisionMode.BF16, out=out_v)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        start.record()
        for _ in range(args.steps):
            step()
        stop.record()
        barrier()
    ms_total = start.elapsed_time(stop)
    t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_per_step = ms_total / args.steps
    flops = w.dense_flops()
    value = world * flops * args.steps / (ms_total * 1e-3) / 1e12
    tokens_per_s = world * w.tokens * args.steps / (ms_total * 1e-3)

    # NCCL all-gather of the outputs (outside the timed attention region).
    allgather_ms = None
    if world > 1:
        gathered = torch.empty(world, *out.shape, dtype=out.dtype, device=dev)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        dist.all_gather_into_tensor(gathered, out)
        e1.record()
        barrier()
        ag = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        dist.all_reduce(ag, op=dist.ReduceOp.MAX)
        allgather_ms = float(ag.item())
        del gathered

    # End to end through the public API with host buffers: every step copies
    # q, k, v from pinned host memory and the output back, inside the timed
    # region. ada_attn_fwd_host streams chunks of (b, h) slices so the copies in,
    # the forward and the copies out overlap.
    e2e_steps = max(1, min(args.e2e_steps, args.steps))
    hq, hk, hv = (x.contiguous().cpu().pin_memory() for x in (q, k, v))
    hout = torch.empty(hq.shape, dtype=out.dtype).pin_memory()
    stage = torch.empty(host_buffer_bytes(hq, hk, hv, scale=scale, static_precision=PrecisionMode.BF16),
                        dtype=torch.uint8, device=dev)

    def e2e_step():
        attention_forward_host(hq, hk, hv, scale=scale, causal=w.causal,
                               static_precision=PrecisionMode.BF16, out=hout, device=dev,
                               buffer=stage)

    e2e_step()
    barrier()
    start.record()
    for _ in range(e2e_steps):
        e2e_step()
    stop.record()
    barrier()
    e2e_ms = torch.tensor([start.elapsed_time(stop)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    e2e_value = world * flops * e2e_steps / (e2e_ms * 1e-3) / 1e12
    h2d = sum(x.numel() * x.element_size() for x in (q, k, v))
    d2h = out.numel() * out.element_size()

    if world > 1:
        dist.barrier()
    if rank == 0:
        peaks, src = load_peaks()
        peak = float(peaks["bf16_tflops"])
        achieved = flops / (ms_per_step * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: seeded N(0,1)/sqrt(D) bf16",
            "config": workload_config(w, world),
            "tokens_per_s": tokens_per_s,
            "pct_of_bf16_peak": 100.0 * achieved / peak,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"{src} bf16_tflops (burst)",
                         "traffic": profiled_traffic(),
                         "algorithmic_flops_per_launch": flops},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "ms_per_step": e2e_ms / e2e_steps},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
        }
        if allgather_ms is not None:
            line["allgather_outputs_ms"] = allgather_ms
        if not args.no_cpu_baseline and world == 1:  # the host-core baseline is an N=1 figure
            v_cpu, cores, desc = cpu_sample(w)
            line["cpu_baseline"] = {"value": v_cpu, "unit": "TFLOP/s", "cores": cores,
                                    "kind": "port", "sample": desc}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
