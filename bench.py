#!/usr/bin/env python
"""Routed-attention throughput on B200 (the BASELINE.json metric).

Default workload (the largest single-GPU module
configuration and the forward+backward half of the metric): preset ``qk4-s4``
SharedDictionaryAttention forward+backward in bf16, global batch 16 x seq 2048
split over the GPUs, dY ~ N(0,1).
Other workloads (``--config``):
  2  a1 SharedDictionaryAttention forward, fp16, batch 8 x seq 512 per GPU
  4  a1-r512-d1536 forward, bf16, batch 4 x 8192 per GPU
  5  DoubleAttentionLM training step (a1, 6 layers, one bank, FFN 1536, vocab 2048, T 1024),
     bf16 autocast, AdamW, global batch 256 data-parallel with NCCL gradient averaging
Inputs are synthetic: x ~ N(0,1) and dY ~ N(0,1) from seeded generators,
token ids uniform in [0, 2048), weights from torch.manual_seed(0).

A "step" is one pass of the workload over one batch; ``value`` is routed
tokens/s summed over all ranks with inputs resident in HBM, ``e2e`` is the
same through the public module call with pinned host inputs copied in and
the result copied out inside the timed region (for the module workloads
the copies are double-buffered on two copy streams, as a prefetching input
pipeline runs them, and the region spans all timed steps).  One JSON line
is printed by rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5]
  python bench.py --impl reference ...   # the reference algorithm on host cores

Multi-GPU runs are launched with torchrun (one rank per GPU, NCCL); the
slowest rank's device time is reported.
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

import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "routed-attention tokens/sec"
# Larger than the 126 MB L2; its device time also keeps the GPU busy while
# the host enqueues the timed step after it.
L2_FLUSH_BYTES = 512 << 20

CONFIGS = {
    # a1 forward, fp16, B8 T512 per GPU
    2: dict(kind="module", preset="a1", dtype=torch.float16, batch=8, seq=512, mode="fwd", scaling="weak",
            workload="a1 SharedDictionaryAttention forward, fp16, B8 T512 per GPU",
            operands="fp16 projection and route operands; the probability-value products of the route and the "
                     "attention take bf16 operands (V and the value dictionary in bf16), fp32 accumulation"),
    # qk4-s4 forward+backward, bf16, B16 T2048 split over the GPUs
    3: dict(kind="module", preset="qk4-s4", dtype=torch.bfloat16, batch=16, seq=2048, mode="fwdbwd",
            scaling="strong",
            workload="qk4-s4 SharedDictionaryAttention forward+backward, bf16, global B16 T2048, dY ~ N(0,1)"),
    # a1-r512-d1536 forward, bf16, 4 x 8192 per GPU
    4: dict(kind="module", preset="a1-r512-d1536", dtype=torch.bfloat16, batch=4, seq=8192, mode="fwd",
            scaling="weak", workload="a1-r512-d1536 SharedDictionaryAttention forward, bf16, B4 T8192 per GPU"),
    # LM training step, global batch 256 split over the GPUs
    5: dict(kind="lm", preset="a1", dtype=torch.bfloat16, batch=256, seq=1024, mode="train", scaling="strong",
            layers=6, ffn=1536, vocab=2048,
            workload="DoubleAttentionLM a1 6 layers train step (AdamW), bf16 autocast, global B256 T1024"),
}

# kernels whose live duration is measured for the roofline, per mode
ROOFLINE_KERNELS = {
    "fwd": ("route", "attention"),
    "fwdbwd": ("route", "attention", "route_bwd", "attention_bwd"),
    "train": ("route", "attention", "route_bwd", "attention_bwd"),
}


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=None, help="timed steps (default per config)")
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--config", type=int, default=3, choices=sorted(CONFIGS))
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--no-graph", action="store_true", help="time eager launches instead of a CUDA graph")
    p.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline sample budget")
    p.add_argument("--no-reference-gpu", action="store_true",
                   help="skip timing the reference's own GPU path (baseline/_ref, backend='auto')")
    args = p.parse_args(argv)
    if args.steps is None:
        args.steps = {2: 200, 3: 20, 4: 20, 5: 10}[args.config]
    args.warmup = max(3, args.warmup) if args.impl == "b200" else args.warmup
    return args


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


# ----------------------------------------------------------------------------- workloads
def per_rank_batch(cfg, world: int) -> int:
    if cfg["scaling"] == "weak":
        return cfg["batch"]
    if cfg["batch"] % world:
        raise SystemExit(f"global batch {cfg['batch']} does not split over {world} GPUs")
    return cfg["batch"] // world


def _seeded_normal(shape, seed: int, dtype) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


def _token_ids(batch: int, seq: int, vocab: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (batch, seq + 1), generator=g)


class ModuleWorkload:
    """SharedDictionaryAttention forward (or forward+backward) on one rank's batch."""

    def __init__(self, cfg, device, rank: int, world: int) -> None:
        from double_attention_b200 import SharedDictionaryAttention, experiment_config

        self.cfg, self.device = cfg, device
        self.batch = per_rank_batch(cfg, world)
        self.train = cfg["mode"] == "fwdbwd"
        torch.manual_seed(0)
        module = SharedDictionaryAttention(experiment_config(cfg["preset"])).to(device=device, dtype=cfg["dtype"])
        self.module = module.train(self.train)
        shape = (self.batch, cfg["seq"], 512)
        self.x_host = _seeded_normal(shape, 1 + rank, cfg["dtype"]).pin_memory()
        self.x = self.x_host.to(device)
        self.out_host = torch.empty(shape, dtype=cfg["dtype"]).pin_memory()
        if self.train:
            self.dy_host = _seeded_normal(shape, 1000 + rank, cfg["dtype"]).pin_memory()
            self.dy = self.dy_host.to(device)
            self.x.requires_grad_(True)
        self.tokens = self.batch * cfg["seq"]
        self.h2d = self.x_host.numel() * self.x_host.element_size() * (2 if self.train else 1)
        self.d2h = self.out_host.numel() * self.out_host.element_size()
        self.capturable = True

    def step(self) -> None:
        if not self.train:
            with torch.no_grad():
                self.module(self.x)
            return
        for p in self.module.parameters():
            p.grad = None
        self.x.grad = None
        self.module(self.x).backward(self.dy)

    def e2e_region(self, steps: int, flush: torch.Tensor, stream, graphed: bool = True) -> float:
        """Device time (ms) of `steps` end-to-end steps, copies included, timed as one region.

        Every step copies its inputs from pinned host memory and its result (y, or dx when training)
        back to pinned host memory.  The staging is double-buffered, as a prefetching input pipeline
        does it: step k+1's inputs go host -> device on one copy stream while step k computes, and step
        k's result goes device -> host on a second copy stream (PCIe carries both directions at once)
        while step k+1 computes.  The region opens before the first step's input copy and closes
        after the last step's result copy; the L2 flush before every step lies inside it.  With
        `graphed` the module step is the package's GraphedModuleStep (one graph launch per step: the
        staged inputs are copied into its static buffers and its result into one of two result
        buffers, device to device, inside the region); otherwise the eager module call.
        """
        if not hasattr(self, "_staging"):
            from double_attention_b200 import GraphedModuleStep

            shape, dt = self.x_host.shape, self.x_host.dtype
            self._staging = {
                "in": torch.cuda.Stream(self.device), "out": torch.cuda.Stream(self.device),
                "x": [torch.empty(shape, dtype=dt, device=self.device) for _ in range(2)],
                "dy": [torch.empty(shape, dtype=dt, device=self.device) for _ in range(2)] if self.train else None,
                "res": [torch.empty(shape, dtype=dt, device=self.device) for _ in range(2)],
                "graph": GraphedModuleStep(self.module, tuple(shape), dt, backward=self.train) if graphed else None,
            }
        st = self._staging
        copy_in, copy_out = st["in"], st["out"]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        staged = [torch.cuda.Event() for _ in range(steps)]
        consumed = [torch.cuda.Event() for _ in range(steps)]
        sent = [torch.cuda.Event() for _ in range(steps)]

        def stage(k: int) -> None:
            i = k % 2
            copy_in.wait_event(consumed[k - 2] if k >= 2 else start)  # buffer i free again
            with torch.cuda.stream(copy_in):
                st["x"][i].copy_(self.x_host, non_blocking=True)
                if self.train:
                    st["dy"][i].copy_(self.dy_host, non_blocking=True)
            staged[k].record(copy_in)

        start.record(stream)
        stage(0)
        for k in range(steps):
            flush.zero_()
            if k + 1 < steps:
                stage(k + 1)
            stream.wait_event(staged[k])
            i = k % 2
            if st["graph"] is not None:
                res = st["graph"](st["x"][i], st["dy"][i] if self.train else None)
                if k >= 2:
                    stream.wait_event(sent[k - 2])  # result buffer i is on its way to the host no longer
                st["res"][i].copy_(res)
                out = st["res"][i]
            elif self.train:
                for p in self.module.parameters():
                    p.grad = None
                xd = st["x"][i].detach().requires_grad_(True)
                self.module(xd).backward(st["dy"][i])
                out = xd.grad  # the input gradient is the step's result
                out.record_stream(copy_out)
            else:
                with torch.no_grad():
                    out = self.module(st["x"][i])
                out.record_stream(copy_out)
            consumed[k].record(stream)
            copy_out.wait_event(consumed[k])
            with torch.cuda.stream(copy_out):
                self.out_host.copy_(out, non_blocking=True)
            sent[k].record(copy_out)
            del out
        stream.wait_stream(copy_out)
        end.record(stream)
        torch.cuda.synchronize()
        return start.elapsed_time(end)


class LMWorkload:
    """One DoubleAttentionLM training step (forward, backward, gradient average, AdamW)."""

    def __init__(self, cfg, device, rank: int, world: int) -> None:
        from double_attention_b200 import DoubleAttentionLM, experiment_config
        from double_attention_b200.data_parallel import GradientAllReduce

        self.cfg, self.device = cfg, device
        self.batch = per_rank_batch(cfg, world)
        torch.manual_seed(0)
        model = DoubleAttentionLM(cfg["vocab"], cfg["seq"], experiment_config(cfg["preset"]), cfg["layers"],
                                  dictionary_group_size=cfg["layers"], feedforward_dim=cfg["ffn"])
        self.model = model.to(device).train()
        self.opt = torch.optim.AdamW(self.model.parameters(), lr=3e-4, fused=True)
        banks = [p for bank in self.model.stack.banks for p in bank.parameters()]
        self.reducer = GradientAllReduce(self.model.parameters(), last=banks)
        ids = _token_ids(self.batch, cfg["seq"], cfg["vocab"], seed=2 + rank)
        self.ids_host = ids[:, :-1].contiguous().pin_memory()
        self.tgt_host = ids[:, 1:].contiguous().pin_memory()
        self.ids, self.tgt = self.ids_host.to(device), self.tgt_host.to(device)
        self.loss_host = torch.empty((), dtype=torch.float32).pin_memory()
        self.tokens = self.batch * cfg["seq"]
        self.h2d = 2 * self.ids_host.numel() * self.ids_host.element_size()
        self.d2h = 4
        self.capturable = False  # NCCL collectives and the optimiser run eagerly

    def _train(self, ids, tgt):
        self.opt.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=self.cfg["dtype"]):
            _, loss = self.model(ids, tgt)
        loss.backward()
        self.reducer.finish()
        self.opt.step()
        return loss

    def step(self) -> None:
        self._train(self.ids, self.tgt)

    def e2e_step(self) -> None:
        ids = self.ids_host.to(self.device, non_blocking=True)
        tgt = self.tgt_host.to(self.device, non_blocking=True)
        self.loss_host.copy_(self._train(ids, tgt).detach().float(), non_blocking=True)

    def e2e_region(self, steps: int, flush: torch.Tensor, stream, graphed: bool = False) -> float:
        """Device time (ms) of `steps` end-to-end training steps (1 MB of token ids in, the loss out)."""
        return sum(time_steps(self.e2e_step, steps, flush, stream))


def make_workload(cfg, device, rank, world):
    return (LMWorkload if cfg["kind"] == "lm" else ModuleWorkload)(cfg, device, rank, world)


# ----------------------------------------------------------------------------- timing
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


def capture(fn, device, stream):
    """CUDA graph of `fn` (None if it cannot be captured)."""
    try:
        side = torch.cuda.Stream(device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            fn()
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        graph.replay()
        torch.cuda.synchronize()
        return graph
    except Exception as exc:  # graph capture is an optimisation only
        print(f"[bench] CUDA graph capture failed ({exc}); timing eager launches", file=sys.stderr)
        torch.cuda.synchronize()
        return None


def kernel_rooflines(cfg, config: int, device, batch: int):
    """Live per-launch duration and algorithmic FLOPs of the main kernels at the shapes one rank runs."""
    from double_attention_b200 import kernel_bench

    out = {}
    for name in ROOFLINE_KERNELS[cfg["mode"]]:
        run, flops = kernel_bench.make_case(name, config, device, batch=batch)
        ms = kernel_bench.time_kernel(run, 20, device, graph=name in kernel_bench.GRAPH_CASES)
        out[name] = (ms, flops)
        del run
    torch.cuda.empty_cache()
    return out


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


# ----------------------------------------------------------------------------- CPU reference
def cpu_reference(cfg, seconds: float, steps: int | None = None, warmup: int = 0):
    """The reference algorithm (the fp32 CPU oracle restatement) on host cores, on a bounded sample.

    Returns (tokens/s, threads, samples, sample batch, median seconds)."""
    import oracle
    from double_attention_b200 import experiment_config

    threads = torch.get_num_threads()
    seq = cfg["seq"]
    sample_batch = 1 if (cfg["mode"] != "fwd" or seq > 2048) else cfg["batch"]
    if cfg["kind"] == "lm":
        from double_attention_b200 import DoubleAttentionLM

        torch.manual_seed(0)
        model = DoubleAttentionLM(cfg["vocab"], seq, experiment_config(cfg["preset"]), cfg["layers"],
                                  dictionary_group_size=cfg["layers"], feedforward_dim=cfg["ffn"])
        params = {k: v.detach().float().clone().requires_grad_() for k, v in model.named_parameters()}
        state = {k: v.detach().float() for k, v in model.state_dict().items()}
        opt = torch.optim.AdamW(params.values(), lr=3e-4)
        ids = _token_ids(sample_batch, seq, cfg["vocab"], seed=2)

        def one():
            opt.zero_grad(set_to_none=True)
            full = dict(state)
            full.update(params)
            full["lm_head.weight"] = full["token_embedding.weight"]
            _, loss = oracle.lm_forward(full, ids[:, :-1], ids[:, 1:], model.stack.config, cfg["layers"],
                                        cfg["layers"])
            loss.backward()
            opt.step()
    else:
        from double_attention_b200 import SharedDictionaryAttention

        torch.manual_seed(0)
        module = SharedDictionaryAttention(experiment_config(cfg["preset"]))
        train = cfg["mode"] == "fwdbwd"
        params = {k: v.detach().float().clone().requires_grad_(train) for k, v in module.state_dict().items()}
        x = _seeded_normal((sample_batch, seq, 512), 1, torch.float32)
        dy = _seeded_normal((sample_batch, seq, 512), 1000, torch.float32)

        def one():
            if train:
                xr = x.clone().requires_grad_()
                oracle.attention_forward(params, xr, module.config).backward(dy)
            else:
                with torch.no_grad():
                    oracle.attention_forward(params, x, module.config)
    for _ in range(max(1, warmup)):
        one()
    times = []
    t_end = time.perf_counter() + seconds
    while (steps is None and time.perf_counter() < t_end) or (steps is not None and len(times) < steps):
        t0 = time.perf_counter()
        one()
        times.append(time.perf_counter() - t0)
        if steps is None and len(times) >= 1000:
            break
    sec = statistics.median(times)
    return sample_batch * seq / sec, threads, len(times), sample_batch, sec


REF_DIR = REPO / "baseline" / "_ref"


def reference_gpu(cfg, device, steps: int, flush: torch.Tensor, ours_out: torch.Tensor | None):
    """The reference's own GPU path as the speed bar: the UNMODIFIED Ahnd6474/double-attention package
    (installed into baseline/_ref) with backend="auto" -- its Triton kernels and cuBLAS -- on the same
    seeded weights and inputs, timed like this arm (CUDA events, L2 flushed, eager launches as in the
    reference's benchmarks/benchmark_attention.py).  Returns a dict for the JSON line, or None when the
    package is not installed."""
    if not (REF_DIR / "double_attention").is_dir():
        return {"unavailable": "reference not installed in baseline/_ref"}
    sys.path.insert(0, str(REF_DIR))
    try:
        import double_attention as ref
        from double_attention.config import experiment_config as ref_config
        from double_attention.triton_kernels import TRITON_AVAILABLE
    finally:
        sys.path.remove(str(REF_DIR))
    if not ref.__file__.startswith(str(REF_DIR)):
        return {"unavailable": f"imported another double_attention ({ref.__file__})"}
    if not TRITON_AVAILABLE:
        return {"unavailable": "triton does not import on this box"}
    stream = torch.cuda.current_stream(device)
    if cfg["kind"] == "lm":
        torch.manual_seed(0)
        model = ref.DoubleAttentionLM(cfg["vocab"], cfg["seq"], ref_config(cfg["preset"], backend="auto"),
                                      cfg["layers"], dictionary_group_size=cfg["layers"],
                                      feedforward_dim=cfg["ffn"]).to(device).train()
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4, fused=True)
        ids = _token_ids(cfg["batch"], cfg["seq"], cfg["vocab"], seed=2).to(device)

        def step():
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=cfg["dtype"]):
                _, loss = model(ids[:, :-1], ids[:, 1:])
            loss.backward()
            opt.step()
        out = None
    else:
        torch.manual_seed(0)
        module = ref.SharedDictionaryAttention(ref_config(cfg["preset"], backend="auto"))
        module = module.to(device=device, dtype=cfg["dtype"]).train(cfg["mode"] == "fwdbwd")
        shape = (cfg["batch"], cfg["seq"], 512)
        x = _seeded_normal(shape, 1, cfg["dtype"]).to(device)
        train = cfg["mode"] == "fwdbwd"
        if train:
            dy = _seeded_normal(shape, 1000, cfg["dtype"]).to(device)
            x.requires_grad_(True)

        def step():
            if not train:
                with torch.no_grad():
                    module(x)
                return
            for p in module.parameters():
                p.grad = None
            x.grad = None
            module(x).backward(dy)
        with torch.no_grad():
            out = module(x.detach())
    for _ in range(3):  # includes Triton's JIT compilation
        step()
    torch.cuda.synchronize()
    with ClockSampler(device.index or 0) as clocks:
        time.sleep(0.05)
        times = time_steps(step, steps, flush, stream)
    ms = sum(times) / len(times)
    line = {"impl": "Ahnd6474/double-attention 0.1.0, unmodified, backend='auto' (Triton kernels + cuBLAS)",
            "value": cfg["batch"] * cfg["seq"] / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "steps": steps, "clocks": clocks.summary()}
    if out is not None and ours_out is not None:
        line["max_abs_vs_this_output"] = float((out.float() - ours_out.float()).abs().max())
    return line


def _mode_words(cfg) -> str:
    return {"fwd": "forward", "fwdbwd": "forward+backward", "train": "LM training step (fwd, bwd, AdamW)"}[cfg["mode"]]


# ----------------------------------------------------------------------------- arms
def run_reference(args, cfg, world, rank):
    if rank != 0:
        return
    # torchrun sets OMP_NUM_THREADS=1 for every rank; the reference arm runs on rank 0 alone and uses
    # every host core
    torch.set_num_threads(os.cpu_count() or 1)
    tps, threads, n, sb, sec = cpu_reference(cfg, args.cpu_seconds, steps=args.steps, warmup=args.warmup)
    sample = (f"{n} steps of the fp32 CPU oracle {_mode_words(cfg)} on {sb}x{cfg['seq']} tokens "
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
        "scaling": cfg["scaling"],
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic",
        "config": {"workload": cfg["workload"], "preset": cfg["preset"], "seq_len": cfg["seq"],
                   "mode": cfg["mode"], "parallelism": f"dp{args.gpus}", "device": "host cpu"},
        "cpu_baseline": {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args, cfg, world, rank, local):
    from double_attention_b200 import _lib

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    work = make_workload(cfg, device, rank, world)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    # --- device-resident step, captured in a CUDA graph when possible
    for _ in range(args.warmup):
        work.step()
    torch.cuda.synchronize()
    launches0 = _lib.kernel_launches()
    work.step()
    torch.cuda.synchronize()
    launches_per_step = _lib.kernel_launches() - launches0
    graph = None
    if work.capturable and not args.no_graph:
        graph = capture(work.step, device, stream)
    used_graph = graph is not None
    step = graph.replay if used_graph else work.step
    for _ in range(3):
        step()
    barrier(world)
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        time.sleep(0.05)  # let the sampler take its first readings
        times = time_steps(step, args.steps, flush, stream)
    barrier(world)
    torch.cuda.synchronize()
    ms = max_over_ranks(sum(times) / len(times), world)
    value = work.tokens * world / (ms / 1e3)

    # --- end to end through the public API: pinned host in, result back to pinned host
    # the value step's graph is released first: the end-to-end step captures its own
    del step, graph
    torch.cuda.empty_cache()
    e2e_graphed = work.capturable and not args.no_graph
    work.e2e_region(3, flush, stream, graphed=e2e_graphed)
    barrier(world)
    torch.cuda.synchronize()
    e2e_total = work.e2e_region(args.steps, flush, stream, graphed=e2e_graphed)
    barrier(world)
    e2e_ms = max_over_ranks(e2e_total / args.steps, world)
    e2e_value = work.tokens * world / (e2e_ms / 1e3)
    h2d, d2h = work.h2d, work.d2h

    # --- roofline of the dominant kernel (rank 0 only; each kernel timed alone, L2 flushed)
    roofline = cpu_base = ref_gpu = None
    ours_out = None
    if rank == 0 and world == 1 and cfg["kind"] == "module" and not args.no_reference_gpu:
        with torch.no_grad():
            ours_out = work.module(work.x.detach()).float()
    if rank == 0:
        del work
        torch.cuda.empty_cache()
        kernels = kernel_rooflines(cfg, args.config, device, per_rank_batch(cfg, world))
        top = max(kernels, key=lambda k: kernels[k][0])
        peak_tf, _hbm, peak_kind = load_peaks()
        ms_top, flops_top = kernels[top]
        achieved = flops_top / (ms_top / 1e3) / 1e12
        roofline = {
            "kernel": top, "bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
            "frac": achieved / peak_tf, "peak_source": f"{peak_kind} bf16 dense (burst)",
            "flops_per_launch": flops_top, "ms_per_launch": ms_top,
            "traffic": load_traffic(top, f"config{args.config}"),
            "other_kernels": {k: {"ms": v[0], "tflops": v[1] / (v[0] / 1e3) / 1e12,
                                  "traffic": load_traffic(k, f"config{args.config}")}
                              for k, v in kernels.items() if k != top},
        }
        if world == 1 and not args.no_reference_gpu:
            try:
                ref_gpu = reference_gpu(cfg, device, min(args.steps, 10), flush, ours_out)
            except Exception as exc:  # reported, never fatal to this arm
                ref_gpu = {"unavailable": f"{type(exc).__name__}: {exc}"[:300]}
            if ref_gpu.get("value"):
                ref_gpu["ratio_this_over_reference"] = value / ref_gpu["value"]
            del ours_out
            torch.cuda.empty_cache()
        if world == 1:
            torch.set_num_threads(os.cpu_count() or 1)
            tps, threads, n, sb, sec = cpu_reference(cfg, args.cpu_seconds)
            cpu_base = {"value": tps, "unit": "tokens/s", "cores": threads, "kind": "port",
                        "sample": f"{n} fp32 CPU oracle {_mode_words(cfg)} steps on {sb}x{cfg['seq']} tokens in "
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
            "scaling": cfg["scaling"],
            "vs_baseline": None,
            "dtype": "fp16" if cfg["dtype"] == torch.float16 else "bf16",
            "data": "synthetic",
            "config": {
                "workload": cfg["workload"], "preset": cfg["preset"],
                **({"operands": cfg["operands"]} if "operands" in cfg else {}),
                "batch_per_gpu": per_rank_batch(cfg, world), "global_batch": per_rank_batch(cfg, world) * world,
                "seq_len": cfg["seq"], "mode": cfg["mode"], "parallelism": f"dp{world}",
                "l2": "flushed before every timed step (512 MiB write)", "cuda_graph": used_graph,
            },
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms,
                    "timing": ("one region over all steps, L2 flush before every step inside it; inputs staged "
                               "double-buffered on a host-to-device copy stream, results on a device-to-host "
                               "copy stream" if cfg["kind"] == "module" else
                               "per-step events around the copies and the eager training step"),
                    "call": ("double_attention_b200.GraphedModuleStep (one CUDA graph launch per step)"
                             if e2e_graphed else "eager module call")},
            "roofline": roofline,
            "cpu_baseline": cpu_base,
            "reference_gpu": ref_gpu,
            "clocks": clock_summary,
            "gpu_launches": launches_per_step * args.steps,
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
