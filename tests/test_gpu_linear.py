"""The Linear layers around the routed attention on the tcgen05 GEMM, against fp32 PyTorch.

* ``da_gemm_ex``: bias, GELU with the pre-activation kept, GELU-derivative multiply, and two K
  segments (the value projection's dX joined to the Q/K projection's);
* ``ops.linear`` (the output projection, modules.py:272) and ``ops.feedforward`` (Linear -> GELU ->
  Linear, modules.py:339-346) forward and backward under bf16 autocast, fp32 parameters.

Operands are rounded to the kernel dtype and the reference runs in fp32 on their upcast.  Bar:
outputs max-abs 2e-2 * max(1, max |ref|) and cosine >= 0.9995; gradients cosine >= 0.999 and
max-abs 3e-2 * max(1, max |ref|).  Weight gradients come from split-K products added in a fixed
order, so two backward passes agree bit for bit.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from double_attention_b200 import ops

pytestmark = pytest.mark.gpu


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    return float(F.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


def _close(name: str, got: torch.Tensor, ref: torch.Tensor, rel: float, min_cos: float) -> None:
    got, ref = got.float().cpu(), ref.float().cpu()
    bound = rel * max(1.0, ref.abs().max().item())
    err, cos = (got - ref).abs().max().item(), _cos(got, ref)
    assert err <= bound and cos >= min_cos, f"{name}: max-abs {err:.3e} (bound {bound:.3e}) cosine {cos:.6f}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("m", "k", "n", "k2"), [(1000, 512, 1536, 0), (300, 1024, 512, 512), (4096, 512, 512, 0)])
def test_gemm_ex_epilogues(m, k, n, k2, dtype) -> None:
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(m + n + k2)
    a = (torch.randn(m, k, generator=g) * 0.5).to(dtype)
    b = (torch.randn(n, k, generator=g) * k**-0.5).to(dtype)
    bias = torch.randn(n, generator=g).to(dtype)
    ref = a.float() @ b.float().t()
    a2 = b2 = None
    if k2:
        a2 = (torch.randn(m, k2, generator=g) * 0.5).to(dtype)
        b2 = (torch.randn(n, k2, generator=g) * k2**-0.5).to(dtype)
        ref = ref + a2.float() @ b2.float().t()
    ad, bd = a.to(dev), b.to(dev)
    a2d = None if a2 is None else a2.to(dev)
    b2d = None if b2 is None else b2.to(dev)
    # plain, K-major B
    out = torch.empty(m, n, dtype=dtype, device=dev)
    ops.gemm_ex(ad, bd, False, out, a2=a2d, b2=b2d)
    _close("plain", out, ref, 2e-2, 0.9995)
    # MN-major B (the transposed weight of a backward product)
    out_t = torch.empty(m, n, dtype=dtype, device=dev)
    b2t = None if b2d is None else b2d.t().contiguous()
    ops.gemm_ex(ad, bd.t().contiguous(), True, out_t, a2=a2d, b2=b2t)
    _close("MN-major B", out_t, ref, 2e-2, 0.9995)
    # bias + GELU, pre-activation kept
    z = torch.empty(m, n, dtype=dtype, device=dev)
    h = torch.empty(m, n, dtype=dtype, device=dev)
    ops.gemm_ex(ad, bd, False, h, a2=a2d, b2=b2d, bias=bias.to(dev), act=1, aux=z)
    pre = ref + bias.float()
    _close("pre-activation", z, pre, 2e-2, 0.9995)
    _close("GELU", h, F.gelu(pre), 2e-2, 0.9995)
    # times GELU'(z): d/dz of GELU applied to an upstream product
    dz = torch.empty(m, n, dtype=dtype, device=dev)
    ops.gemm_ex(ad, bd, False, dz, a2=a2d, b2=b2d, act=2, aux=z)
    zr = z.float().cpu().requires_grad_()
    F.gelu(zr).backward(torch.ones_like(zr))
    _close("GELU backward", dz, ref * zr.grad, 2e-2, 0.9995)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0


def test_output_projection_and_feedforward_match_torch() -> None:
    """The block's Linear layers under bf16 autocast with fp32 parameters (the training configuration)."""
    dev = torch.device("cuda")
    torch.manual_seed(0)
    proj = nn.Linear(512, 512, bias=False).to(dev)
    ff1, ff2 = nn.Linear(512, 1536).to(dev), nn.Linear(1536, 512).to(dev)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 700, 512, generator=g).to(dev)
    dy = torch.randn(2, 700, 512, generator=g).to(dev)
    xd = x.clone().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        assert ops.linear_supported(xd, proj) and ops.feedforward_supported(xd, ff1, ff2)
        y = ops.feedforward(ops.linear(xd, proj), ff1, ff2)
    assert y.dtype == torch.bfloat16
    y.float().backward(dy)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0

    # fp32 reference on the bf16-rounded operands (what autocast feeds the products)
    r = lambda t: t.detach().to(torch.bfloat16).float().cpu()  # noqa: E731
    xr = r(x).requires_grad_()
    wp, w1, b1, w2, b2 = (r(t).requires_grad_() for t in (proj.weight, ff1.weight, ff1.bias, ff2.weight, ff2.bias))
    yr = F.linear(F.gelu(F.linear(F.linear(xr, wp), w1, b1)), w2, b2)
    yr.backward(dy.cpu())
    _close("y", y, yr, 2e-2, 0.9995)
    for name, got, ref in (("x", xd.grad, xr.grad), ("W_out", proj.weight.grad, wp.grad),
                           ("W1", ff1.weight.grad, w1.grad), ("b1", ff1.bias.grad, b1.grad),
                           ("W2", ff2.weight.grad, w2.grad), ("b2", ff2.bias.grad, b2.grad)):
        _close(f"d {name}", got, ref, 3e-2, 0.999)


def test_feedforward_backward_is_bit_reproducible() -> None:
    dev = torch.device("cuda")
    torch.manual_seed(0)
    ff1, ff2 = nn.Linear(512, 1536).to(dev), nn.Linear(1536, 512).to(dev)
    x = torch.randn(3000, 512, device=dev)
    dy = torch.randn(3000, 512, device=dev)
    grads = []
    for _ in range(2):
        for prm in (*ff1.parameters(), *ff2.parameters()):
            prm.grad = None
        xd = x.clone().requires_grad_()
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = ops.feedforward(xd, ff1, ff2)
        y.float().backward(dy)
        grads.append([xd.grad.clone()] + [prm.grad.clone() for prm in (*ff1.parameters(), *ff2.parameters())])
    torch.cuda.synchronize()
    for a, b in zip(*grads):
        assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("rows", "cols", "ld"), [(1, 8, 8), (1000, 512, 512), (3000, 1536, 1536), (777, 264, 520),
                                                  (262144, 512, 512)])
def test_bias_grad_column_sums(rows, cols, ld, dtype) -> None:
    """da_col_sum against an fp64 column sum of the same rounded values; two calls agree bit for bit."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(rows + cols)
    full = torch.randn(rows, ld, generator=g).to(dtype)
    d = full.to(dev)[:, :cols]
    got = ops._bias_grad(d)
    again = ops._bias_grad(d)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    assert got.dtype == torch.float32 and got.shape == (cols,)
    ref = full[:, :cols].double().sum(0)
    bound = 1e-5 * rows ** 0.5 * 4 + 1e-6 * ref.abs().max().item()
    assert (got.double().cpu() - ref).abs().max().item() <= bound
    assert torch.equal(got, again)


def test_block_linear_layers_on_either_gemm_agree(monkeypatch) -> None:
    """The block's output projection and feed-forward branch run on cuBLAS by default
    (ops.BLOCK_LINEAR_ON_TCGEN05 = False) or on the tcgen05 GEMM; the two LM steps agree."""
    from double_attention_b200 import DoubleAttentionLM, experiment_config

    dev = torch.device("cuda")
    ids = torch.randint(0, 512, (2, 257), generator=torch.Generator().manual_seed(4)).to(dev)
    results = []
    for flag in (False, True):
        monkeypatch.setattr(ops, "BLOCK_LINEAR_ON_TCGEN05", flag)
        torch.manual_seed(0)
        model = DoubleAttentionLM(512, 256, experiment_config("a1"), 2, dictionary_group_size=2,
                                  feedforward_dim=1536).to(dev)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits, loss = model(ids[:, :-1], ids[:, 1:])
        loss.backward()
        torch.cuda.synchronize()
        assert ops.device_status(dev) == 0
        results.append((logits.float().cpu(), loss.item(), {n: p.grad.float().cpu() for n, p in model.named_parameters()}))
    (l0, loss0, g0), (l1, loss1, g1) = results
    assert abs(loss0 - loss1) <= 2e-3 * abs(loss0)
    _close("logits", l1, l0, 2e-2, 0.9995)
    for name in g0:
        ref, got = g0[name], g1[name]
        scale = ref.abs().max().item()
        err = (got - ref).abs().max().item()
        assert err <= 3e-2 * max(1.0, scale), f"d {name}: max-abs {err:.3e}"
        if scale >= 1e-2:  # the cosine of a near-zero gradient says nothing
            assert _cos(got, ref) >= 0.999, f"d {name}: cosine {_cos(got, ref):.6f}"
