"""Single-kernel driver: runs one sm_100a kernel on a BASELINE workload shape.

Used for per-kernel timing and for focused profiler captures, e.g.

    python -m double_attention_b200.kernel_bench --kernel route --config 2 --reps 3
    ncu --set full --clock-control none -k regex:route_fwd -c 1 \\
        python -m double_attention_b200.kernel_bench --kernel route --config 2 --reps 3

Inputs are synthetic (seeded N(0,1) activations, normalised random
dictionaries / routed vectors) with the shapes of the named config.  With
``--time`` the kernel is timed with CUDA events (L2 flushed between
launches) and one JSON line with the algorithmic FLOPs and achieved
TFLOP/s is printed.
"""

from __future__ import annotations

import argparse
import json
import statistics

import torch
import torch.nn.functional as F

from . import ops

# (preset, batch, seq, dtype) per BASELINE.json config (per GPU)
SHAPES = {
    2: ("a1", 8, 512, torch.float16),
    3: ("qk4-s4", 16, 2048, torch.bfloat16),
    4: ("a1-r512-d1536", 4, 8192, torch.bfloat16),
    5: ("a1", 32, 1024, torch.bfloat16),
}


KERNELS = ("route", "attention", "route_bwd", "route_bwd_rows", "dict_grads_splitk", "attention_bwd", "projection")


class _Cfg:
    def __init__(self, maps: int) -> None:
        self.outer_maps = maps
        self.causal = True


def make_case(kernel: str, config: int, device: torch.device, batch: int | None = None):
    from .config import experiment_config

    preset, default_batch, seq, dtype = SHAPES[config]
    batch = batch or default_batch
    cfg = experiment_config(preset)
    h, r, m, d = cfg.qk_branches, cfg.routing_dim, cfg.dictionary_size, cfg.model_dim
    g = torch.Generator().manual_seed(config)
    if kernel == "route":
        proj = torch.randn(batch * seq, 2 * h * r, generator=g).to(dtype).to(device)
        dk = F.normalize(torch.randn(r, m, generator=g), dim=0).to(dtype).to(device)
        dv = F.normalize(torch.randn(r, m, generator=g), dim=0).to(dtype).to(device)
        views = ops.dictionary_views_from_normalized(dk, dv, dtype)
        beta = torch.tensor(cfg.beta, device=device)
        rows = 2 * batch * seq * h

        def run():
            ops._route_forward(proj, batch * seq, 2 * h, r, views, beta, cfg.eps, True, True)

        return run, 4.0 * r * m * rows
    if kernel == "attention":
        routed = F.normalize(torch.randn(2, h, batch, seq, r, generator=g), dim=-1).to(dtype).to(device)
        value = torch.randn(batch, seq, d, generator=g).to(torch.bfloat16).to(device)
        scales = torch.full((cfg.outer_maps,), cfg.initial_score_scale, device=device)
        mix = torch.full((cfg.outer_maps,), 1.0 / cfg.outer_maps, device=device) if cfg.outer_maps > 1 else None
        c = _Cfg(cfg.outer_maps)

        def run():
            ops.routed_attention_mixed(routed, value, scales, mix, c)

        return run, float(batch) * seq * seq * (cfg.outer_maps * r + d)
    if kernel in ("route_bwd", "route_bwd_rows"):
        # route_bwd: the whole route backward as autograd runs it (da_route_bwd_fused: the row pass, the
        # atom-parallel dictionary-gradient kernel and the fixed-order reduction of its partial sums);
        # route_bwd_rows: the row pass alone (da_route_bwd without [rows, M] outputs)
        proj = torch.randn(batch * seq, 2 * h * r, generator=g).to(dtype).to(device)
        dk = F.normalize(torch.randn(r, m, generator=g), dim=0).to(dtype).to(device)
        dv = F.normalize(torch.randn(r, m, generator=g), dim=0).to(dtype).to(device)
        views = ops.dictionary_views_from_normalized(dk, dv, dtype)
        beta = torch.tensor(cfg.beta, device=device)
        rows, groups = batch * seq, 2 * h
        z, lse, onorm = ops._route_forward(proj, rows, groups, r, views, beta, cfg.eps, True, True)
        dz = torch.randn(groups, rows, r, generator=g).to(dtype).to(device)
        dq = torch.empty_like(proj)
        ws = ops.workspace(device)
        beta32 = beta.float().reshape(1)
        if kernel == "route_bwd":
            def run():
                ops._route_backward_fused(proj, views.key_t, views.value_t, beta32, z, dz, lse, onorm, dq, rows,
                                          groups, r, cfg.eps, True, True, True, True, True)

            # dP, dq_hat, dDv and dDk over every route row
            return run, 8.0 * r * m * groups * rows
        g_out = torch.empty(groups, rows, r, dtype=torch.bfloat16, device=device)

        def run():
            ops.call("da_route_bwd", proj.data_ptr(), rows, proj.shape[1], proj.stride(0), groups, r, r, m,
                     ops.dtype_code(dtype), views.key_t.data_ptr(), views.value_t.data_ptr(), beta32.data_ptr(),
                     cfg.eps, 1, 1, z.data_ptr(), dz.data_ptr(), lse.data_ptr(), onorm.data_ptr(), dq.data_ptr(),
                     None, None, g_out.data_ptr(), None, None, 0, ws.status.data_ptr(), ops.stream_ptr(device))

        # dP and dq_hat
        return run, 4.0 * r * m * groups * rows
    if kernel == "dict_grads_splitk":  # the unfused path's dDk and dDv split-K GEMMs over stored [rows, M] rows
        rows, groups = batch * seq, 2 * h
        proj = torch.randn(rows, 2 * h * r, generator=g).to(dtype).to(device)
        dl_out = (torch.randn(groups, rows, m, generator=g) * 1e-2).to(dtype).to(device)
        p_out = torch.rand(groups, rows, m, generator=g).to(torch.bfloat16).to(device)
        g_out = torch.randn(groups, rows, r, generator=g).to(torch.bfloat16).to(device)
        d_key = torch.zeros(r, m, device=device)
        d_value = torch.zeros(r, m, device=device)

        def run():
            ops.key_dictionary_grad(proj, r, dl_out, d_key)
            ops.gemm_splitk(g_out.view(-1, r), r, True, p_out.view(-1, m), m, True, r, m, groups * rows, d_value)

        return run, 4.0 * r * m * groups * rows
    if kernel == "attention_bwd":  # the whole attention backward op (delta pass, dQ, dK and dV launches)
        # The op as _MixedAttention.backward runs it (gradients stored once in the input dtype when the
        # maps sit on disjoint branches, else fresh zeroed fp32 ones; the delta pass for one map), called
        # directly rather than through autograd so that it can be captured.
        maps = cfg.outer_maps
        routed = F.normalize(torch.randn(2, h, batch, seq, r, generator=g), dim=-1).to(dtype).to(device)
        value = torch.randn(batch, seq, d, generator=g).to(dtype).to(device)
        scales = torch.full((maps,), cfg.initial_score_scale, device=device)
        mix = torch.full((maps,), 1.0 / maps, device=device) if maps > 1 else None
        dy = torch.randn(batch, seq, d, generator=g).to(dtype).to(device)
        flat = routed.view(-1, r)
        group, branch0 = ops._map_layout(h, maps)
        qmap = ops.RowMap(flat, 0, seq, batch * seq)
        kmap = ops.RowMap(flat, h * batch * seq, seq, batch * seq)
        y, lse = ops._attention_forward(qmap, kmap, value, batch, seq, r, maps, group, branch0, True, scales, mix,
                                        None, 1.0, dtype)

        overwrite = h >= maps  # as the module path: gradients stored once in the input dtype

        def run():
            alloc, gdt = (torch.empty, dtype) if overwrite else (torch.zeros, torch.float32)
            droute = alloc(flat.shape, dtype=gdt, device=device)
            dv = alloc(batch * seq, d, dtype=gdt, device=device)
            dscale = torch.zeros(maps, dtype=torch.float32, device=device)
            dweight = torch.zeros(maps, dtype=torch.float32, device=device) if mix is not None else None
            if maps == 1:
                delta, given = ops._attention_delta(dy, y).view(batch, 1, seq), True
            else:
                delta, given = torch.empty(batch, maps, seq, dtype=torch.float32, device=device), False
            ops._attention_backward(qmap, kmap, value, dy, batch, seq, r, maps, group, branch0, True, scales, mix,
                                    lse, delta, given, droute, droute, dv, dscale, dweight, overwrite=overwrite)

        return run, float(batch) * seq * seq * (2 * cfg.outer_maps * r + 2 * d)
    if kernel == "projection":
        x = torch.randn(batch * seq, d, generator=g).to(dtype).to(device)
        w = (torch.randn(2 * h * r, d, generator=g) * d**-0.5).to(dtype).to(device)
        out = torch.empty(batch * seq, 2 * h * r, dtype=dtype, device=device)

        def run():
            ops.gemm(x, False, w, False, batch * seq, 2 * h * r, d, out)

        return run, 2.0 * batch * seq * d * 2 * h * r
    raise ValueError(f"unknown kernel {kernel!r}")


# cases that enqueue several launches (and memsets): timed as CUDA-graph replays so that host
# enqueue work cannot fall inside the timed region
GRAPH_CASES = ("attention_bwd", "route_bwd")


def time_kernel(run, reps: int, device: torch.device, graph: bool = False) -> float:
    """Mean device time (ms) of `run`, L2 flushed before each launch.

    Each launch is bracketed by CUDA events on the launching stream right behind a 512 MiB flush
    (~0.1 ms of device work, during which the host has long enqueued the events and the launch), so
    the bracket holds the kernel and its launch latency only.  With `graph` the launches are
    replayed from a CUDA graph instead (for multi-launch cases whose host enqueue takes longer).
    """
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(3):
        run()
    launch = run
    if graph:
        g = torch.cuda.CUDAGraph()
        try:
            side = torch.cuda.Stream(device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                run()
            stream.wait_stream(side)
            with torch.cuda.graph(g):
                run()
            launch = g.replay
        except RuntimeError:  # not capturable: time eager launches
            torch.cuda.synchronize()
    events = []
    for _ in range(reps):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        launch()
        e.record(stream)
        events.append((s, e))
    torch.cuda.synchronize()
    return statistics.mean(s.elapsed_time(e) for s, e in events)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--kernel", required=True, help=f"comma-separated list of {', '.join(KERNELS)}")
    p.add_argument("--config", type=int, choices=sorted(SHAPES), default=2)
    p.add_argument("--reps", type=int, default=3)
    p.add_argument("--batch", type=int, default=None, help="override the config's per-GPU batch (small captures)")
    p.add_argument("--time", action="store_true")
    args = p.parse_args(argv)
    device = torch.device("cuda", 0)
    for kernel in args.kernel.split(","):
        if kernel not in KERNELS:
            raise SystemExit(f"unknown kernel {kernel!r}")
        run, flops = make_case(kernel, args.config, device, args.batch)
        if args.time:
            ms = time_kernel(run, args.reps, device, graph=kernel in GRAPH_CASES)
            print(json.dumps({"kernel": kernel, "config": args.config, "ms": ms, "flops": flops,
                              "tflops": flops / (ms / 1e3) / 1e12}))
        else:
            for _ in range(args.reps):
                run()
            torch.cuda.synchronize()
        del run
        ops.device_status(device)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
