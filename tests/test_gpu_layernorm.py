"""Residual add + LayerNorm kernels (the glue around the block) against PyTorch fp32 on a B200.

Reference composition (modules.py:294-356): ``x_out = x + branch`` on the fp32 residual stream,
``y = nn.LayerNorm(x_out)`` in fp32, cast to the dtype the next Linear reads.  Forward: x_out is
bit-exact (one fp32 add); y within the rounding of its dtype.  Backward against autograd of the
same composition in fp32: dx, d branch, d gamma and d beta.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from double_attention_b200 import ops

pytestmark = pytest.mark.gpu


def _norm(d: int, seed: int) -> nn.LayerNorm:
    torch.manual_seed(seed)
    n = nn.LayerNorm(d).cuda()
    with torch.no_grad():  # non-trivial affine parameters
        n.weight.copy_(1 + 0.1 * torch.randn(d))
        n.bias.copy_(0.1 * torch.randn(d))
    return n


def _tol(dtype: torch.dtype) -> float:
    return {torch.float32: 2e-5, torch.bfloat16: 1.6e-2, torch.float16: 2e-3}[dtype]


@pytest.mark.parametrize("d", [256, 512, 768, 1024])
@pytest.mark.parametrize("rows", [1, 37, 4096])
@pytest.mark.parametrize(("branch_dtype", "out_dtype"),
                         [(None, torch.bfloat16), (torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                          (torch.float16, torch.float16)])
def test_add_layernorm_matches_torch(d: int, rows: int, branch_dtype, out_dtype) -> None:
    norm = _norm(d, 11 + d + rows)
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + d)
    x = (3 * torch.randn(rows, d, device="cuda", generator=g) + 0.5)
    branch = None if branch_dtype is None else torch.randn(rows, d, device="cuda", generator=g).to(branch_dtype)
    dy = torch.randn(rows, d, device="cuda", generator=g).to(out_dtype)
    d_res = torch.randn(rows, d, device="cuda", generator=g) if branch is not None else None

    # reference: fp32 autograd of the composition
    xr = x.clone().requires_grad_(True)
    br = None if branch is None else branch.float().clone().requires_grad_(True)
    wr = norm.weight.detach().clone().requires_grad_(True)
    bbr = norm.bias.detach().clone().requires_grad_(True)
    xo_ref = xr + br if br is not None else xr
    y_ref = F.layer_norm(xo_ref, (d,), wr, bbr, norm.eps)
    loss = (y_ref * dy.float()).sum() + ((xo_ref * d_res).sum() if d_res is not None else 0)
    loss.backward()

    # fused kernels
    xk = x.clone().requires_grad_(True)
    bk = None if branch is None else branch.clone().requires_grad_(True)
    norm.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=out_dtype, enabled=out_dtype != torch.float32):
        if bk is None:
            y = ops.layernorm(xk, norm)
            xo = None
        else:
            xo, y = ops.add_layernorm(xk, bk, norm)
    assert y.dtype == out_dtype
    total = (y.float() * dy.float()).sum()
    if xo is not None:
        assert xo.dtype == torch.float32
        assert torch.equal(xo.detach(), xo_ref.detach()), "x + branch must be exact in fp32"
        total = total + (xo * d_res).sum()
    total.backward()

    tol = _tol(out_dtype)
    err = (y.float() - y_ref.detach()).abs().max().item()
    assert err <= tol * max(1.0, y_ref.detach().abs().max().item()), f"y max-abs {err}"
    gs = xr.grad.abs().max().item()
    assert (xk.grad - xr.grad).abs().max().item() <= 1e-4 * max(1.0, gs), "dx"
    if bk is not None:
        assert bk.grad.dtype == branch.dtype
        assert (bk.grad.float() - br.grad).abs().max().item() <= _tol(branch.dtype) * max(1.0, gs), "d branch"
    for name, got, want in (("d gamma", norm.weight.grad, wr.grad), ("d beta", norm.bias.grad, bbr.grad)):
        scale = max(1.0, want.abs().max().item())
        assert (got - want).abs().max().item() <= 2e-4 * scale * max(1.0, rows ** 0.5 / 8), name


def test_block_uses_fused_norms_and_matches_unfused() -> None:
    """A DoubleAttentionStack step with the fused norms equals the same stack with nn.LayerNorm calls."""
    from double_attention_b200 import DoubleAttentionStack, experiment_config

    torch.manual_seed(0)
    cfg = experiment_config("a1")
    stack = DoubleAttentionStack(cfg, 2, feedforward_dim=1536).cuda()
    x = torch.randn(2, 256, cfg.model_dim, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = stack(x)
    y.float().square().mean().backward()
    fused = {n: p.grad.clone() for n, p in stack.named_parameters() if p.grad is not None}
    stack.zero_grad(set_to_none=True)

    real = ops.layernorm_supported
    ops.layernorm_supported = lambda *a, **k: False  # the module's plain nn.LayerNorm path
    try:
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y2 = stack(x)
        y2.float().square().mean().backward()
    finally:
        ops.layernorm_supported = real
    plain = {n: p.grad.clone() for n, p in stack.named_parameters() if p.grad is not None}
    cos = F.cosine_similarity(y.float().flatten(), y2.float().flatten(), dim=0).item()
    assert cos >= 0.9999, cos
    assert set(fused) == set(plain)
    for n in fused:
        c = F.cosine_similarity(fused[n].float().flatten(), plain[n].float().flatten(), dim=0).item()
        assert c >= 0.999, (n, c)
