"""Host logic of the data-parallel gradient average, on two gloo ranks (CPU).

Each rank runs a small model on its own batch; after backward the bucketed
all-reduce must leave every rank with the mean of the ranks' gradients,
with the `last` parameters (stand-ins for the shared dictionary banks) in
the final bucket and earlier buckets already launched during backward.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from double_attention_b200.data_parallel import GradientAllReduce


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Net(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.bank = nn.Parameter(torch.randn(8, 16))      # read by every layer, like a dictionary bank
        self.layers = nn.ModuleList(nn.Linear(16, 16) for _ in range(3))
        self.head = nn.Linear(16, 4, bias=False)

    def forward(self, x):
        for layer in self.layers:
            x = torch.tanh(layer(x) + x @ self.bank.t() @ self.bank)
        return self.head(x)


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        net = _Net()
        reducer = GradientAllReduce(net.parameters(), last=[net.bank], bucket_bytes=1024)
        assert reducer.buckets[-1] == [net.bank]
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randn(5, 16, generator=g)
        for step in range(2):  # twice: the reducer must re-arm itself
            net.zero_grad(set_to_none=True)
            net(x * (step + 1)).square().mean().backward()
            launched_early = sum(h is not None for h in reducer._handles[:-1])
            local = [p.grad.clone() for p in net.parameters()]
            reducer.finish()
            gathered = []
            for t in local:  # the expected mean, by an independent all_gather
                parts = [torch.empty_like(t) for _ in range(world)]
                dist.all_gather(parts, t)
                gathered.append(torch.stack(parts).mean(0))
            ok = all(torch.allclose(p.grad, e, atol=1e-6) for p, e in zip(net.parameters(), gathered))
            out.put((rank, step, ok, launched_early, len(reducer.buckets)))
        reducer.close()
    finally:
        dist.destroy_process_group()


def test_bucketed_average_on_two_gloo_ranks() -> None:
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = [out.get(timeout=120) for _ in range(2 * world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert len(results) == 2 * world
    for rank, step, ok, launched_early, buckets in results:
        assert ok, f"rank {rank} step {step}: gradients are not the mean over ranks"
        assert buckets >= 3
        assert launched_early == buckets - 1, "early buckets should launch during backward"


def _failing_worker(rank: int, world: int, port: int, out) -> None:
    """Rank 1 raises in its forward pass (it never reaches the all-reduce); rank 0 runs backward and
    finish(), whose wait must end with an error well inside the process group's timeout."""
    import datetime
    import time

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    torch.manual_seed(0)
    net = _Net()
    reducer = GradientAllReduce(net.parameters(), last=[net.bank], bucket_bytes=1024)
    x = torch.randn(5, 16)
    if rank == 1:
        out.put((rank, "raised", 0.0))
        out.close()
        out.join_thread()  # flush the queue before leaving
        os._exit(3)  # the failure: this rank leaves without joining any collective
    t0 = time.monotonic()
    try:
        net(x).square().mean().backward()
        reducer.finish(timeout=datetime.timedelta(seconds=5))
        out.put((rank, "no error", time.monotonic() - t0))
    except RuntimeError as exc:
        out.put((rank, f"error: {exc}", time.monotonic() - t0))
    out.close()
    out.join_thread()
    os._exit(0)  # skip the process-group teardown with a dead peer


def test_a_rank_that_leaves_makes_the_others_finish_fail() -> None:
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, what, seconds = out.get(timeout=90)
        results[rank] = (what, seconds)
    for p in procs:
        p.join(timeout=60)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    what, seconds = results[0]
    assert what.startswith("error: gradient all-reduce of bucket"), what
    assert seconds < 20.0, f"the failure took {seconds:.1f} s to surface"


def test_single_process_is_a_no_op() -> None:
    net = _Net()
    reducer = GradientAllReduce(net.parameters(), last=[net.bank])
    net(torch.randn(3, 16)).sum().backward()
    before = [p.grad.clone() for p in net.parameters()]
    reducer.finish()
    assert all(torch.equal(a, p.grad) for a, p in zip(before, net.parameters()))


if __name__ == "__main__":
    pytest.main([__file__, "-q"])
