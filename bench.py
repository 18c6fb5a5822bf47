"""Benchmark of the AdaAttn attention-forward hot path on B200.

Workload: dense BF16 causal attention, B8 H32 N4096 D128 (Q, K, V iid
N(0,1)/sqrt(D), seeded), precision forced to BF16 and rank to dense -- the
peak-throughput configuration. One step = one attention forward over one
batch, inputs resident in HBM (805 MB > L2, so no flush is needed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Multi-GPU (torchrun, one process per GPU): strong scaling by (batch x head)
shards -- the 256 (b, h) units of the one B8 H32 job are split into
contiguous ranges, one per rank, with no collective inside the timed
attention; the NCCL all-gather of the outputs is timed separately afterwards
(``--scaling weak`` gives every rank its own B8 H32 job instead). The time of
a step is the maximum over ranks; rank 0 prints one JSON line, with every
rank's kernel time. A second leg times the GPT-2-small-shaped decoder with
AdaAttention in every layer, its batch of 16 split over the ranks. On one
GPU a third leg times the E4M3 variant of the same attention workload beside
a dense FP8 GEMM peak measured in the same process.

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


SAMPLE_HEADS = 4  # heads of batch row 0 in one host-core sample


def cpu_sample(workload, seconds: float = 10.0, max_reps: int = 50):
    """Time the oracle's dense BF16 attention on a slice of the workload.

    Sample: batch row 0, SAMPLE_HEADS heads, full sequence; repeated until
    about `seconds` of CPU work. Returns (TFLOP/s, threads, description)."""
    import oracle as O
    from adaattn_b200.workloads import make_qkv
    torch.set_num_threads(os.cpu_count() or 1)
    heads = SAMPLE_HEADS
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
    sample_heads = SAMPLE_HEADS
    sample_flops = workload.scaled(batch=1, heads=sample_heads).dense_flops()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": flops / (value * 1e12) * 1e3, "higher_is_better": True,
        "scaling": "strong" if args.scaling == "strong" else "weak", "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1)/sqrt(D) bf16",
        "config": workload_config(workload, args.gpus, args.scaling),
        # Each step times a slice of the workload; ms_per_step is that slice's
        # measured time scaled to the full job by its share of the FLOPs
        # ((b, h) slices are independent and equally costly).
        "extrapolated": True,
        "slice": f"batch row 0, {sample_heads} of {workload.heads} heads, N={workload.seq}, "
                 f"{sample_flops / flops:.5f} of the job's FLOPs",
        "measured_ms_per_slice": sample_flops / (value * 1e12) * 1e3,
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": desc + ("; the host cores of one node, so the same value at "
                                           "every GPU count" if args.gpus > 1 else "")},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "tokens_per_s": workload.tokens / (flops / (value * 1e12)),
    }
    print(json.dumps(line), flush=True)
    return 0


def workload_config(w, n, scaling):
    units = w.batch * w.heads
    if scaling == "strong":
        par = (f"(batch x head) shards: the {units} (b, h) units of one job split over {n} "
               f"GPU(s), contiguous ranges, no collective in attention; outputs all-gathered "
               f"over NCCL afterwards, timed separately")
        batch = w.batch
    else:
        par = (f"(batch x head) shards, weak scaling: each of {n} GPU(s) processes its own "
               f"B{w.batch} H{w.heads} job; no collective in attention")
        batch = w.batch * n
    return {"workload": f"dense_bf16 causal attention B{w.batch} H{w.heads} N{w.seq} "
                        f"D{w.head_dim}, precision forced BF16, rank forced dense",
            "global_batch": batch, "heads": w.heads, "seq_len": w.seq, "head_dim": w.head_dim,
            "causal": w.causal, "parallelism": par,
            "l2": "inputs 805 MB per job > 126 MB L2 (no flush needed)"}


def gpt2_leg(dev, world, rank, barrier, steps=10):
    """GPT-2-small-shaped decoder with AdaAttention in every layer (12 layers,
    E768, H12, FF3072, seq 1024, batch 16, weights N(0, 0.02), bf16): forward
    tokens/s, the batch split over the ranks (replicated weights, no
    collective in the forward), each step one replay of the forward captured
    in a CUDA graph."""
    from adaattn_b200 import AdaAttention
    from adaattn_b200.host_model import AdaptiveTransformer
    from adaattn_b200.shard import shard_range
    from adaattn_b200.workloads import GPT2_SMALL as c, make_token_ids
    torch.manual_seed(0)
    model = AdaptiveTransformer(vocab_size=c["vocab"], embed_dim=c["embed_dim"],
                                num_heads=c["num_heads"], num_layers=c["num_layers"],
                                ff_dim=c["ff_dim"], max_seq_len=c["seq"], dropout=0.0)
    model.init_gpt2_weights(std=0.02)
    for m in model.modules():
        if isinstance(m, AdaAttention):
            m.config.enable_nan_check = False
    model = model.to(dev).to(torch.bfloat16).eval()
    ids = make_token_ids(c["batch"], c["seq"], c["vocab"], seed=0, device=str(dev))
    lo, hi = shard_range(c["batch"], rank, world)
    local = ids[lo:hi]

    def step():
        with torch.no_grad():
            return model(local)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    # One forward captured in a CUDA graph (no host synchronisation inside:
    # decisions, statistics and workspaces live on the device) and replayed:
    # at a few sequences per GPU the eager forward is bound by the host's
    # launch sequence, not by the GPU.
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    try:
        with torch.cuda.stream(side):
            step()
            with torch.cuda.graph(graph, stream=side):
                step()
        run = graph.replay
    except Exception:  # capture refused: time the eager forward instead
        graph = None
        run = step
    torch.cuda.current_stream(dev).wait_stream(side)
    torch.cuda.synchronize()
    for _ in range(3):
        run()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        run()
    e1.record()
    barrier()
    ms = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item()) / steps
    stats = model.get_attention_statistics()[0]
    used_graph = graph is not None
    del run, graph
    del model
    return {"workload": f"gpt2_small decoder B{c['batch']} N{c['seq']} E{c['embed_dim']} "
                        f"H{c['num_heads']} L{c['num_layers']} bf16, batch split over {world} GPU(s)",
            "tokens_per_s": c["batch"] * c["seq"] / (ms * 1e-3), "ms_per_forward": ms,
            "sequences_per_gpu": hi - lo, "steps": steps, "cuda_graph": used_graph,
            "attention_precision_layer0": stats["precision_distribution"]}


def fp8_leg(dev, w, steps=20):
    """The E4M3 variant on the same workload (static precision FP8, E4M3
    quantisation of q, k, v included in every step), beside a dense FP8 GEMM
    peak measured in this process (cuBLASLt e4m3 x e4m3 -> bf16, 8192^3,
    best of 10): the denominator for the E4M3 kernel's tensor-core fraction."""
    from adaattn_b200 import PrecisionMode, attention_forward
    from adaattn_b200.workloads import make_qkv
    n = 8192
    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    one = torch.ones((), device=dev)
    peak = None
    try:
        for _ in range(3):
            torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        best = float("inf")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _ in range(10):
            e0.record()
            torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        peak = 2.0 * n ** 3 / (best * 1e-3) / 1e12
    except Exception as e:  # no FP8 GEMM in this torch build
        peak_err = (str(e).splitlines() or [type(e).__name__])[0][:120]
    del a, b
    q, k, v = make_qkv(w, seed=1000, device=str(dev))
    out = torch.empty(q.shape, dtype=w.dtype, device=dev)
    scale = 1.0 / math.sqrt(w.head_dim)

    def step():
        attention_forward(q, k, v, scale=scale, causal=w.causal, static_precision=PrecisionMode.FP8,
                          out=out)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    tflops = w.dense_flops() / (ms * 1e-3) / 1e12
    res = {"workload": f"dense causal attention B{w.batch} H{w.heads} N{w.seq} D{w.head_dim}, "
                       "precision forced FP8 (E4M3 operands, per-tile scales; quantisation in the step)",
           "ms_per_step": ms, "tflops": tflops, "steps": steps}
    if peak is not None:
        res["fp8_gemm_peak_tflops"] = peak
        res["frac_of_fp8_peak"] = tflops / peak
    else:
        res["fp8_gemm_peak_tflops"] = None
        res["fp8_peak_unavailable"] = peak_err
    del q, k, v, out
    torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong: one B8 H32 job split over the GPUs (default); weak: a job per GPU")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gpt2", action="store_true", help="skip the GPT-2-small leg")
    ap.add_argument("--no-fp8", action="store_true", help="skip the E4M3 leg")
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
    from adaattn_b200.shard import gather_slices, local_slices, shard_range
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    w = workload
    scale = 1.0 / math.sqrt(w.head_dim)
    strong = args.scaling == "strong"
    if strong:
        # every rank draws the same job and keeps its contiguous range of (b, h) units
        qf, kf, vf = make_qkv(w, seed=1000, device=str(dev))
        q, k, v = (local_slices(x, rank, world).contiguous() for x in (qf, kf, vf))
        del qf, kf, vf
        u0, u1 = shard_range(w.batch * w.heads, rank, world)
        units_total = w.batch * w.heads
    else:
        q, k, v = make_qkv(w, seed=1000 + rank, device=str(dev))
        u0, u1 = 0, w.batch * w.heads
        units_total = world * w.batch * w.heads
    torch.cuda.empty_cache()
    out = torch.empty(q.shape, dtype=w.dtype, device=dev)

    def step():
        attention_forward(q, k, v, scale=scale, causal=w.causal,
                          static_precision=PrecisionMode.BF16, out=out)

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
    ms_rank = start.elapsed_time(stop)
    per_rank = torch.tensor([ms_rank / args.steps], device=dev, dtype=torch.float64)
    if world > 1:
        gathered_ms = [torch.empty_like(per_rank) for _ in range(world)]
        dist.all_gather(gathered_ms, per_rank)
        per_rank_ms = [float(x.item()) for x in gathered_ms]
    else:
        per_rank_ms = [float(per_rank.item())]
    ms_per_step = max(per_rank_ms)
    unit_flops = w.dense_flops() / (w.batch * w.heads)   # every (b, h) unit costs the same
    job_flops = unit_flops * units_total
    value = job_flops / (ms_per_step * 1e-3) / 1e12
    tokens_per_s = (units_total // w.heads) * w.seq / (ms_per_step * 1e-3)

    # NCCL all-gather of the outputs (outside the timed attention region);
    # the first call sets up NCCL's connections and is not timed.
    allgather_ms = None
    if world > 1:
        def gather():
            if strong:
                return gather_slices(out, w.batch, w.heads)
            full = torch.empty(world, *out.shape, dtype=out.dtype, device=dev)
            dist.all_gather_into_tensor(full, out)
            return full
        del_full = gather()
        del del_full
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        full = gather()
        e1.record()
        barrier()
        ag = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        dist.all_reduce(ag, op=dist.ReduceOp.MAX)
        allgather_ms = float(ag.item())
        del full

    # End to end through the public API with host buffers: every step copies
    # this rank's q, k, v from pinned host memory and the output back, inside
    # the timed region. ada_attn_fwd_host streams chunks of (b, h) slices so
    # the copies in, the forward and the copies out overlap.
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
    e2e_value = job_flops * e2e_steps / (e2e_ms * 1e-3) / 1e12
    h2d = sum(x.numel() * x.element_size() for x in (q, k, v))
    d2h = out.numel() * out.element_size()
    del hq, hk, hv, hout, stage, q, k, v, out
    torch.cuda.empty_cache()

    gpt2 = None if args.no_gpt2 else gpt2_leg(dev, world, rank, barrier)
    fp8 = None
    if world == 1 and not args.no_fp8:
        try:
            fp8 = fp8_leg(dev, workload)
        except Exception as e:  # a failure here must not cost the headline line
            fp8 = {"error": (str(e).splitlines() or [type(e).__name__])[0][:200]}

    if world > 1:
        dist.barrier()
    if rank == 0:
        peaks, src = load_peaks()
        peak = float(peaks["bf16_tflops"])
        # roofline of one GPU's kernel: its own units over its own time
        local_flops = unit_flops * (u1 - u0)
        achieved = local_flops / (per_rank_ms[0] * 1e-3) / 1e12
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic: seeded N(0,1)/sqrt(D) bf16",
            "config": workload_config(w, world, args.scaling),
            "tokens_per_s": tokens_per_s,
            "pct_of_bf16_peak": 100.0 * achieved / peak,
            "per_rank_ms": per_rank_ms,
            "units_per_rank": [shard_range(w.batch * w.heads, r, world) for r in range(world)]
            if strong else None,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_source": f"{src} bf16_tflops (burst)",
                         "traffic": profiled_traffic() if world == 1 else None,
                         "algorithmic_flops_per_launch": local_flops},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                    "ms_per_step": e2e_ms / e2e_steps,
                    "note": "per rank: its own (b, h) units through ada_attn_fwd_host"},
            "gpu_launches": args.steps,
            "clocks": clk.summary(),
        }
        if allgather_ms is not None:
            line["allgather_outputs_ms"] = allgather_ms
        if gpt2 is not None:
            line["gpt2_small"] = gpt2
        if fp8 is not None:
            line["fp8_e4m3"] = fp8
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
