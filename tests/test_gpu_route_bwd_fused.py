"""The route backward with fused, deterministic dictionary gradients (da_route_bwd_fused).

Called through the C ABI on the module layout (several route groups side by side in one projected
matrix, as SharedDictionaryAttention routes its Q and K branches) and checked against the oracle's
autograd in fp32 on the same rounded inputs (the value dictionary as the bf16 operand the kernels
read).  Bar as the other route-backward tests: cosine >= 0.9995 and max-abs <= 2e-2 * max(1, max|g|)
per gradient tensor, dbeta within 2e-2 relative.  The dictionary gradients and dbeta come from
per-chunk partial sums added in a fixed order, so two calls must agree bit for bit.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import oracle
from double_attention_b200 import _lib, ops

pytestmark = pytest.mark.gpu


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    return float(F.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


def _close(name: str, got: torch.Tensor, ref: torch.Tensor, rel: float = 2e-2, min_cos: float = 0.9995) -> None:
    got = got.float().cpu()
    bound = rel * max(1.0, ref.abs().max().item())
    err = (got - ref).abs().max().item()
    cos = _cos(got, ref)
    assert err <= bound and cos >= min_cos, f"{name}: max-abs {err:.3e} (bound {bound:.3e}), cosine {cos:.6f}"


def _case(rows, groups, r, m, col_stride, dtype, seed, ni=True):
    g = torch.Generator().manual_seed(seed)
    cols = (groups - 1) * col_stride + r
    cols += (-cols) % 64
    q = torch.randn(rows, cols, generator=g)
    if not ni:
        q = q / r**0.5
    q = q.to(dtype)
    dk = F.normalize(torch.randn(r, m, generator=g), dim=0).to(dtype)
    dv = F.normalize(torch.randn(r, m, generator=g), dim=0).to(dtype)
    dz = torch.randn(groups, rows, r, generator=g).to(dtype)
    return q, dk, dv, dz


def _run_fused(q, dk, dv, dz, rows, groups, r, m, col_stride, beta, ni, no):
    dev = torch.device("cuda")
    qd = q.to(dev)
    views = ops.dictionary_views_from_normalized(dk.to(dev), dv.to(dev), q.dtype)
    beta_t = torch.tensor([beta], device=dev)
    z, lse, onorm = ops._route_forward(qd, rows, groups, col_stride, views, beta_t, 1e-6, ni, no)
    dq = torch.zeros_like(qd)
    d_key, d_value, dbeta = ops._route_backward_fused(qd, views.key_t, views.value_t, beta_t, z, dz.to(dev), lse,
                                                      onorm, dq, rows, groups, col_stride, 1e-6, ni, no, True, True,
                                                      True)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    return dq, d_key, d_value, dbeta


@pytest.mark.parametrize(
    ("rows", "groups", "r", "m", "col_stride", "dtype", "beta", "ni", "no"),
    [
        (2048, 8, 128, 512, 128, torch.bfloat16, 4.0, True, True),   # qk4-s4 module layout (Q and K x 4 branches)
        (1000, 2, 256, 512, 256, torch.bfloat16, 4.0, True, True),   # a1 layout, ragged last tile
        (700, 2, 256, 512, 320, torch.float16, 4.0, True, True),     # fp16, groups not adjacent
        (300, 3, 128, 256, 192, torch.float16, 6.0, False, True),    # unnormalised input, two atom tiles
        (129, 1, 128, 512, 128, torch.bfloat16, 4.0, True, False),   # one full tile + one row, raw output
        (64, 2, 256, 128, 256, torch.bfloat16, 4.0, True, True),     # one 64-row tile per group, one atom tile
    ],
)
def test_fused_route_backward_matches_oracle(rows, groups, r, m, col_stride, dtype, beta, ni, no) -> None:
    q, dk, dv, dz = _case(rows, groups, r, m, col_stride, dtype, seed=rows + groups + r, ni=ni)
    assert ops.route_bwd_fused_supported(q, rows, col_stride, r, m)
    dq, d_key, d_value, dbeta = _run_fused(q, dk, dv, dz, rows, groups, r, m, col_stride, beta, ni, no)

    dkr = dk.float().requires_grad_()
    dvr = dv.to(torch.bfloat16).float().requires_grad_()  # the kernels' value operand is bf16
    br = torch.tensor(beta, requires_grad=True)
    qr = q.float().requires_grad_()
    total = 0.0
    seen = []
    for grp in range(groups):
        seen.append({})
        zr = oracle.dictionary_route(qr[:, grp * col_stride:grp * col_stride + r], dkr, dvr, br, 1e-6,
                                     normalize_input=ni, normalize_output=no, inspect=seen[-1])
        total = total + (zr * dz[grp].float()).sum()
    total.backward()
    for grp in range(groups):
        sl = slice(grp * col_stride, grp * col_stride + r)
        _close(f"d q (group {grp})", dq[:, sl], qr.grad[:, sl])
    _close("d key dictionary", d_key, dkr.grad)
    _close("d value dictionary", d_value, dvr.grad)
    # d beta = sum over rows and atoms of logit * d loss / d (beta logit): terms of both signs that cancel
    # (they sum to zero over the atoms of a row), so the bf16 rounding of g moves it by more than its own
    # size suggests.  Bar as for the route variants: 2e-2 relative plus 1e-4 of the summed term magnitude.
    terms = sum((d["logits"] * d["scaled"].grad).abs().sum().item() for d in seen)
    tol = 2e-2 * abs(br.grad.item()) + 1e-4 * terms
    assert abs(dbeta.item() - br.grad.item()) <= tol, f"d beta {dbeta.item()} vs {br.grad.item()} (tol {tol})"


@pytest.mark.parametrize(("r", "dtype"), [(128, torch.bfloat16), (256, torch.float16)])
def test_fused_route_backward_is_bit_reproducible(r: int, dtype: torch.dtype) -> None:
    rows, groups, m = 3000, 4, 512
    q, dk, dv, dz = _case(rows, groups, r, m, r, dtype, seed=17)
    first = _run_fused(q, dk, dv, dz, rows, groups, r, m, r, 4.0, True, True)
    second = _run_fused(q, dk, dv, dz, rows, groups, r, m, r, 4.0, True, True)
    for name, a, b in zip(("dq", "d_key", "d_value", "dbeta"), first, second):
        assert torch.equal(a, b), f"{name} differs between two identical calls"


def test_fused_route_backward_agrees_with_the_stored_weights_path() -> None:
    """The fused path's dq comes from the same row kernel as the unfused path's; its dictionary gradients
    agree with the split-K GEMMs over the stored [rows, M] weights within rounding."""
    rows, groups, r, m = 4096, 2, 256, 512
    q, dk, dv, dz = _case(rows, groups, r, m, r, torch.bfloat16, seed=23)
    dq, d_key, d_value, dbeta = _run_fused(q, dk, dv, dz, rows, groups, r, m, r, 4.0, True, True)
    dev = torch.device("cuda")
    qd = q.to(dev)
    views = ops.dictionary_views_from_normalized(dk.to(dev), dv.to(dev), q.dtype)
    beta_t = torch.tensor([4.0], device=dev)
    z, lse, onorm = ops._route_forward(qd, rows, groups, r, views, beta_t, 1e-6, True, True)
    dq2 = torch.zeros_like(qd)
    p_out = torch.empty(groups, rows, m, dtype=torch.bfloat16, device=dev)
    dl_out = torch.empty(groups, rows, m, dtype=q.dtype, device=dev)
    g_out = torch.empty(groups, rows, r, dtype=torch.bfloat16, device=dev)
    dbeta2 = torch.zeros(1, device=dev)
    ops.call("da_route_bwd", qd.data_ptr(), rows, qd.shape[1], qd.stride(0), groups, r, r, m, _lib.DA_BF16,
             views.key_t.data_ptr(), views.value_t.data_ptr(), beta_t.data_ptr(), 1e-6, 1, 1, z.data_ptr(),
             dz.to(dev).data_ptr(), lse.data_ptr(), onorm.data_ptr(), dq2.data_ptr(), p_out.data_ptr(),
             dl_out.data_ptr(), g_out.data_ptr(), dbeta2.data_ptr(), None, 0, ops.workspace(dev).status.data_ptr(),
             ops.stream_ptr(dev))
    d_key2 = torch.zeros(r, m, device=dev)
    ops.key_dictionary_grad(qd, r, dl_out, d_key2)
    d_value2 = torch.zeros(r, m, device=dev)
    ops.gemm_splitk(g_out.view(-1, r), r, True, p_out.view(-1, m), m, True, r, m, groups * rows, d_value2)
    torch.cuda.synchronize()
    assert torch.equal(dq, dq2)
    _close("d key dictionary", d_key, d_key2.cpu(), min_cos=0.99999)
    _close("d value dictionary", d_value, d_value2.cpu(), min_cos=0.99999)
    assert abs(dbeta.item() - dbeta2.item()) <= 1e-3 * max(1.0, abs(dbeta2.item()))


def test_fused_route_backward_checks_its_workspace() -> None:
    handle = _lib.lib()
    need = int(handle.da_route_bwd_workspace_size(4096, 2, 256, 512))
    assert need >= 2 * 4096 * 256 * 2 + 2 * 4096 * 8  # at least g and the row statistics
    assert int(handle.da_route_bwd_workspace_size(4096, 2, 512, 512)) == -1  # R 512: not this entry's
    dev = torch.device("cuda")
    rows, groups, r, m = 4096, 2, 256, 512
    q, dk, dv, dz = _case(rows, groups, r, m, r, torch.bfloat16, seed=3)
    qd, dzd = q.to(dev), dz.to(dev)
    views = ops.dictionary_views_from_normalized(dk.to(dev), dv.to(dev), q.dtype)
    beta_t = torch.tensor([4.0], device=dev)
    z, lse, onorm = ops._route_forward(qd, rows, groups, r, views, beta_t, 1e-6, True, True)
    small = torch.empty(need - 256, dtype=torch.uint8, device=dev)
    out = torch.empty(r, m, device=dev)
    rc = handle.da_route_bwd_fused(qd.data_ptr(), rows, qd.shape[1], qd.stride(0), groups, r, r, m, _lib.DA_BF16,
                                   views.key_t.data_ptr(), views.value_t.data_ptr(), beta_t.data_ptr(), 1e-6, 1, 1,
                                   z.data_ptr(), dzd.data_ptr(), lse.data_ptr(), onorm.data_ptr(),
                                   torch.empty_like(qd).data_ptr(), out.data_ptr(), out.data_ptr(), None,
                                   small.data_ptr(), small.numel(), ops.workspace(dev).status.data_ptr(),
                                   ops.stream_ptr(dev))
    assert rc == _lib.DA_ERR_WORKSPACE
