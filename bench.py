#!/usr/bin/env python
"""Routed-attention throughput on B200 (the BASELINE.json metric).

Default workload: preset ``a1``
SharedDictionaryAttention forward in fp16, batch 8 x seq 512 per GPU
(x ~ N(0,1) from a seeded generator, weights from torch.manual_seed(0)).
A "step" is one module forward over one batch; ``value`` is routed tokens/s
summed over all ranks with inputs resident in HBM, ``e2e`` is the same
through the public module call with pinned host input/output copied inside
the timed region.  One JSON line is printed by rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|4]
  python bench.py --impl reference ...   # the reference algorithm on host cores

Multi-GPU runs are launched with torchrun (one rank per GPU, NCCL); each
rank processes its own batch (weak scaling) and the slowest rank's device
time is reported.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "routed-attention tokens/sec"
# Larger than the 126 MB L2; its ~80 us of device time also keeps the GPU
# busy while the host enqueues the timed step after it.
L2_FLUSH_BYTES = 512 << 20

CONFIGS = {
    # a1 forward, fp16, B8 T512
    2: dict(preset="a1", dtype=torch.float16, batch=8, seq=512, mode="fwd",
            workload="a1 SharedDictionaryAttention forward, fp16, B8 T512 per GPU"),
    # a1-r512-d1536 forward, bf16, 4 x 8192 per GPU
    4: dict(preset="a1-r512-d1536", dtype=torch.bfloat16, batch=4, seq=8192, mode="fwd",
            workload="a1-r512-d1536 SharedDictionaryAttention forward, bf16, B4 T8192 per GPU"),
}


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--no-graph", action="store_true", help="time eager launches instead of a CUDA graph")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    return p.parse_args(argv)


# ----------------------------------------------------------------------------- distributed
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Polls NVML (SM clock, throttle reasons) every ~2 ms while timing runs."""

    REASONS = {
        "hw_slowdown": 0x8,
        "hw_thermal_slowdown": 0x40,
        "sw_thermal_slowdown": 0x20,
        "sw_power_cap": 0x4,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int) -> None:
        self.index = index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[self.index]) if visible else self.index
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._nvml = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as exc:  # sampling is best effort; recorded in the output
            self.error = str(exc)
        return self

    def _run(self):
        nv = self._nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM), get_reasons(self._h)))
            except Exception:
                pass
            time.sleep(0.002)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "error": self.error}
        reasons = sorted({name for _, bits in self.samples for name, bit in self.REASONS.items() if bits & bit})
        return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


# ----------------------------------------------------------------------------- workload
def build_module(cfg, device):
    from double_attention_b200 import SharedDictionaryAttention, experiment_config

    torch.manual_seed(0)
    module = SharedDictionaryAttention(experiment_config(cfg["preset"]))
    return module.to(device=device, dtype=cfg["dtype"]).eval()


def make_input(cfg, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(cfg["batch"], cfg["seq"], 512, generator=g).to(cfg["dtype"])


def time_steps(fn, steps: int, flush: torch.Tensor, stream) -> list[float]:
    """Per-step device time (ms) with CUDA events on `stream`, L2 flushed before each step."""
    times = []
    for _ in range(steps):
        flush.zero_()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        fn()
        end.record(stream)
        times.append((start, end))
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in times]


def kernel_rooflines(module, cfg, x, flush, stream, reps: int = 20):
    """Live duration of the route and attention kernels at this workload."""
    from double_attention_b200 import ops

    c = module.config
    b, t = cfg["batch"], cfg["seq"]
    with torch.no_grad():
        views = ops.dictionary_views(module.bank.raw_key, module.bank.raw_value, c.eps, cfg["dtype"])
        w = torch.cat((module.query.weight, module.key.weight), 0)
        proj = ops.qk_projection(x, w)
        beta = module.beta
        value = module.value(x).to(torch.bfloat16)
        routed = ops.route_projected(proj, views, beta, c, b, t)
        scales = ops.score_scale_from_log(module.log_score_scales)

        def route():
            ops._route_forward(proj, b * t, 2 * c.qk_branches, c.routing_dim, views, beta, c.eps,
                               c.normalize_routing_input, c.normalize_routing_output)

        def attention():
            ops.routed_attention_mixed(routed, value, scales, None, c)

        out = {}
        for name, fn in (("route_fwd", route), ("attention_fwd", attention)):
            for _ in range(3):
                fn()
            ms = statistics.mean(time_steps(fn, reps, flush, stream))
            out[name] = ms
    rows = 2 * b * t * c.qk_branches
    flops = {
        "route_fwd": 4.0 * c.routing_dim * c.dictionary_size * rows,
        # causal: T^2/2 key pairs, 2 flop per MAC, R-wide scores + D-wide values
        "attention_fwd": b * t * t * (c.outer_maps * c.routing_dim + c.model_dim),
    }
    return out, flops


def load_peaks():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def load_traffic(kernel: str, workload_key: str):
    path = REPO / "profiles" / "ncu_traffic.json"
    if not path.exists():
        return None
    try:
        return json.loads(path.read_text()).get(workload_key, {}).get(kernel)
    except (ValueError, AttributeError):
        return None


def count_kernel_launches(module, x) -> int:
    from double_attention_b200 import _lib

    counted = {"da_dict_norm_fwd", "da_route_fwd", "da_attn_fwd", "da_gemm", "da_col_norm_max"}
    n = 0
    orig = _lib.call

    def counting(name, *args):
        nonlocal n
        if name in counted:
            n += 1
        return orig(name, *args)

    import double_attention_b200.ops as ops_mod

    ops_mod.call = counting
    try:
        with torch.no_grad():
            module(x)
        torch.cuda.synchronize()
    finally:
        ops_mod.call = orig
    return n


def cpu_reference(cfg, seconds: float, steps: int | None = None, warmup: int = 0):
    """The reference algorithm (the CPU oracle restatement) on host cores."""
    import oracle
    from double_attention_b200 import SharedDictionaryAttention, experiment_config

    torch.manual_seed(0)
    module = SharedDictionaryAttention(experiment_config(cfg["preset"]))
    params = {k: v.detach().float() for k, v in module.state_dict().items()}
    x = make_input(cfg, seed=1).float()
    threads = torch.get_num_threads()
    sample_batch = cfg["batch"]
    if cfg["seq"] > 2048:  # bound the sample: one sequence, scaled by tokens
        sample_batch = 1
    xs = x[:sample_batch]
    with torch.no_grad():
        for _ in range(max(1, warmup)):
            oracle.attention_forward(params, xs, module.config)
        times = []
        t_end = time.perf_counter() + seconds
        while (steps is None and time.perf_counter() < t_end) or (steps is not None and len(times) < steps):
            t0 = time.perf_counter()
            oracle.attention_forward(params, xs, module.config)
            times.append(time.perf_counter() - t0)
            if steps is None and len(times) >= 1000:
                break
    sec = statistics.median(times)
    tokens = sample_batch * cfg["seq"]
    return tokens / sec, threads, len(times), sample_batch, sec


# ----------------------------------------------------------------------------- arms
def run_reference(args, cfg, world, rank):
    if rank != 0:
        return
    tps, threads, n, sb, sec = cpu_reference(cfg, args.cpu_seconds, steps=args.steps, warmup=args.warmup)
    sample = (f"{n} steps of the fp32 CPU oracle forward on {sb}x{cfg['seq']} tokens "
              f"(median {sec * 1e3:.1f} ms/step), tokens/s of that sample")
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": tps,
        "unit": "tokens/s",
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": sec * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic",
        "config": {"workload": cfg["workload"], "preset": cfg["preset"], "batch_per_gpu": cfg["batch"],
                   "seq_len": cfg["seq"], "parallelism": f"dp{args.gpus}", "device": "host cpu"},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args, cfg, world, rank, local):
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    module = build_module(cfg, device)
    x_host = make_input(cfg, seed=1 + rank).pin_memory()
    x = x_host.to(device)
    y_host = torch.empty(cfg["batch"], cfg["seq"], 512, dtype=cfg["dtype"]).pin_memory()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    tokens = cfg["batch"] * cfg["seq"]

    # --- device-resident step, captured in a CUDA graph when possible
    graph = None
    with torch.no_grad():
        for _ in range(max(3, args.warmup)):
            y = module(x)
        torch.cuda.synchronize()
        if not args.no_graph:
            try:
                side = torch.cuda.Stream(device)
                side.wait_stream(stream)
                with torch.cuda.stream(side):
                    module(x)
                stream.wait_stream(side)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    y_graph = module(x)
                graph.replay()
                torch.cuda.synchronize()
            except Exception as exc:  # graph capture is an optimisation only
                print(f"[bench] CUDA graph capture failed ({exc}); timing eager launches", file=sys.stderr)
                graph = None

        def step():
            if graph is not None:
                graph.replay()
            else:
                module(x)

        for _ in range(args.warmup):
            step()
        barrier(world)
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            time.sleep(0.05)  # let the sampler take its first readings
            times = time_steps(step, args.steps, flush, stream)
        barrier(world)
        torch.cuda.synchronize()
    ms = max_over_ranks(sum(times) / len(times), world)
    value = tokens * world / (ms / 1e3)

    # --- end to end through the public API: pinned host in, pinned host out
    with torch.no_grad():
        def e2e_step():
            xd = x_host.to(device, non_blocking=True)
            yd = module(xd)
            y_host.copy_(yd, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        barrier(world)
        torch.cuda.synchronize()
        e2e_times = time_steps(e2e_step, args.steps, flush, stream)
        barrier(world)
    e2e_ms = max_over_ranks(sum(e2e_times) / len(e2e_times), world)
    e2e_value = tokens * world / (e2e_ms / 1e3)
    h2d = x_host.numel() * x_host.element_size()
    d2h = y_host.numel() * y_host.element_size()

    launches = count_kernel_launches(module, x)

    # --- roofline of the dominant kernel (rank 0 only; timed alone, L2 flushed)
    roofline = cpu_base = None
    if rank == 0:
        durations, flops = kernel_rooflines(module, cfg, x, flush, stream)
        top = max(durations, key=durations.get)
        peak_tf, _hbm, peak_kind = load_peaks()
        achieved = flops[top] / (durations[top] / 1e3) / 1e12
        roofline = {
            "kernel": top, "bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
            "frac": achieved / peak_tf, "peak_source": f"{peak_kind} bf16 dense (burst)",
            "flops_per_launch": flops[top], "ms_per_launch": durations[top],
            "traffic": load_traffic(top, f"config{args.config}"),
            "other_kernels": {k: {"ms": v, "tflops": flops[k] / (v / 1e3) / 1e12} for k, v in durations.items()
                              if k != top},
        }
        if world == 1:
            tps, threads, n, sb, sec = cpu_reference(cfg, args.cpu_seconds)
            cpu_base = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                        "sample": f"{n} fp32 CPU oracle forwards of {sb}x{cfg['seq']} tokens in "
                                  f"~{args.cpu_seconds:.0f} s (median {sec * 1e3:.1f} ms)"}

    clock_summary = clocks.summary()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "fp16" if cfg["dtype"] == torch.float16 else "bf16",
            "data": "synthetic",
            "config": {
                "workload": cfg["workload"], "preset": cfg["preset"], "batch_per_gpu": cfg["batch"],
                "global_batch": cfg["batch"] * world, "seq_len": cfg["seq"], "mode": cfg["mode"],
                "parallelism": f"dp{world}", "l2": "flushed before every timed step (512 MiB write)",
                "cuda_graph": graph is not None,
            },
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms},
            "roofline": roofline,
            "cpu_baseline": cpu_base,
            "clocks": clock_summary,
            "gpu_launches": launches * args.steps,
        }
        print(json.dumps(line), flush=True)


def main(argv=None) -> int:
    args = parse_args(argv)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, cfg, world, rank)
        return 0
    world, rank, local = init_dist()
    try:
        run_b200(args, cfg, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
