"""GraphedModuleStep: a module step replayed from a CUDA graph gives the eager call's results.

The replayed graph launches the same kernels on the same inputs as the eager call, and every kernel
on the path reduces in a fixed order, so the output, the input gradient and every parameter gradient
must equal the eager ones bit for bit.  Two replays with different inputs check that the static
buffers carry each call's inputs and results.
"""

from __future__ import annotations

import pytest
import torch

from double_attention_b200 import GraphedModuleStep, SharedDictionaryAttention, experiment_config, ops

pytestmark = pytest.mark.gpu


def _inputs(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype).cuda()


@pytest.mark.parametrize(("name", "dtype", "batch", "length"),
                         [("a1", torch.float16, 8, 512), ("qk4-s4", torch.bfloat16, 2, 256)])
def test_graphed_forward_equals_eager(name, dtype, batch, length) -> None:
    torch.manual_seed(0)
    module = SharedDictionaryAttention(experiment_config(name)).cuda().to(dtype).eval()
    shape = (batch, length, module.config.model_dim)
    step = GraphedModuleStep(module, shape, dtype)
    for seed in (1, 2):
        x = _inputs(shape, dtype, seed)
        with torch.no_grad():
            want = module(x)
        got = step(x).clone()
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    assert ops.device_status(torch.device("cuda")) == 0


def test_graphed_forward_backward_equals_eager() -> None:
    dtype = torch.bfloat16
    torch.manual_seed(0)
    module = SharedDictionaryAttention(experiment_config("qk4-s4")).cuda().to(dtype).train()
    shape = (2, 256, module.config.model_dim)
    step = GraphedModuleStep(module, shape, dtype, backward=True)
    graph_grads = {n: p.grad for n, p in module.named_parameters()}
    for seed in (3, 4):
        x, dy = _inputs(shape, dtype, seed), _inputs(shape, dtype, seed + 100)
        dx = step(x, dy).clone()
        got = {n: g.clone() for n, g in graph_grads.items()}
        torch.cuda.synchronize()
        # the eager step on the same inputs (it replaces .grad; the graph's buffers keep their contents)
        for p in module.parameters():
            p.grad = None
        xe = x.detach().requires_grad_(True)
        module(xe).backward(dy)
        torch.cuda.synchronize()
        assert torch.equal(dx, xe.grad)
        for n, p in module.named_parameters():
            assert torch.equal(got[n], p.grad), n
        for n, p in module.named_parameters():  # hand the graph its own gradient buffers back
            p.grad = graph_grads[n]
    assert ops.device_status(torch.device("cuda")) == 0


def test_graphed_step_rejects_cpu_module() -> None:
    module = SharedDictionaryAttention(experiment_config("a1"))
    with pytest.raises(RuntimeError, match="CUDA device"):
        GraphedModuleStep(module, (1, 4, 512), torch.float32)


def test_capture_takes_a_prezeroed_workspace() -> None:
    """A stream first seen while a graph is being captured gets one of the zero-filled workspaces made
    beforehand outside any capture, so the graph records no workspace fills (which every replay would
    otherwise repeat)."""
    dev = torch.device("cuda")
    idx = torch.cuda.current_device()
    ops.workspace(dev)  # the current stream's workspace; the device's spares are made with it
    spares = list(ops._spare_workspaces[idx])
    assert spares
    graph = torch.cuda.CUDAGraph()
    capture_stream = torch.cuda.Stream(dev)  # never used before, so it has no workspace yet
    scratch = torch.zeros(4, device=dev)
    with torch.cuda.graph(graph, stream=capture_stream):
        ws = ops.workspace(dev)
        scratch.add_(1.0)
    assert any(ws is s for s in spares)
    graph.replay()
    torch.cuda.synchronize()
    assert int(ws.route_work.abs().sum()) == 0 and int(ws.status.abs().sum()) == 0
    assert torch.equal(scratch, torch.ones(4, device=dev))
