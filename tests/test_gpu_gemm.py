"""tcgen05 GEMM (fused Q/K projection and its backward) against fp32 matmul."""

from __future__ import annotations

import pytest
import torch

from double_attention_b200 import _lib, ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("a_mn", "b_mn"), [(False, False), (False, True), (True, True)])
@pytest.mark.parametrize(("m", "n", "k"), [(4096, 512, 512), (300, 1024, 512), (512, 512, 4104), (256, 256, 96)])
def test_gemm_layouts(m, n, k, a_mn, b_mn, dtype) -> None:
    if a_mn and m % 128:
        pytest.skip("MN-major A needs M % 128 == 0")
    torch.manual_seed(m + n + k)
    dev = torch.device("cuda")
    a = torch.randn(m, k, device=dev).to(dtype)
    b = torch.randn(n, k, device=dev).to(dtype)
    a_arg = a.t().contiguous() if a_mn else a
    b_arg = b.t().contiguous() if b_mn else b
    out = torch.empty(m, n, device=dev, dtype=torch.float32)
    ops.gemm(a_arg, a_mn, b_arg, b_mn, m, n, k, out)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    expected = a.float() @ b.float().t()
    torch.testing.assert_close(out, expected, atol=2e-3 * k**0.5, rtol=1e-3)
    # dtype output and fp32 accumulation
    out16 = torch.empty(m, n, device=dev, dtype=dtype)
    ops.gemm(a_arg, a_mn, b_arg, b_mn, m, n, k, out16)
    torch.testing.assert_close(out16.float(), expected, atol=2e-3 * k**0.5, rtol=1e-2)
    ops.gemm(a_arg, a_mn, b_arg, b_mn, m, n, k, out, accumulate=True)
    torch.testing.assert_close(out, 2 * expected, atol=4e-3 * k**0.5, rtol=1e-3)


def test_projection_autograd() -> None:
    torch.manual_seed(3)
    dev = torch.device("cuda")
    x = torch.randn(2, 300, 512, device=dev).to(torch.bfloat16).requires_grad_()
    w = (torch.randn(1024, 512, device=dev) * 0.04).to(torch.bfloat16).requires_grad_()
    y = ops.qk_projection(x, w)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr, wr = x.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    yr = xr.reshape(-1, 512) @ wr.t()
    yr.backward(dy.float())
    torch.testing.assert_close(y.float(), yr, atol=2e-2, rtol=1e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, atol=5e-2, rtol=2e-2)
    torch.testing.assert_close(w.grad.float(), wr.grad, atol=1e-1, rtol=2e-2)


@pytest.mark.parametrize(("groups", "rows", "r", "m", "cs"), [(8, 512, 128, 512, 128), (2, 4096, 256, 512, 256),
                                                             (3, 192, 128, 384, 136)])
@pytest.mark.parametrize("deterministic", [True, False])
def test_grouped_splitk_matches_reference(groups, rows, r, m, cs, deterministic) -> None:
    """da_gemm_splitk_grouped: C += sum_g A_g^T B_g with A_g the g-th column block of a row-major matrix,
    the splits' partial sums added in a fixed order through a workspace, or with atomics without one."""
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(groups + rows)
    a = torch.randn(rows, (groups - 1) * cs + r + 8, generator=g).to(torch.bfloat16)
    b = torch.randn(groups, rows, m, generator=g).to(torch.bfloat16)
    ad, bd = a.to(dev), b.to(dev)
    ws = ops.workspace(dev)
    elems = int(_lib.lib().da_gemm_splitk_workspace_elems(r, m, rows * groups, 0))
    part = torch.empty(elems, device=dev) if deterministic else None
    outs = []
    for _ in range(2):
        out = torch.full((r, m), 0.5, dtype=torch.float32, device=dev)  # C += ...: the initial value stays
        ops.call("da_gemm_splitk_grouped", ad.data_ptr(), ad.stride(0), cs, bd.data_ptr(), m, out.data_ptr(), m, r,
                 m, rows, groups, 1, 0, None if part is None else part.data_ptr(), 0 if part is None else elems,
                 ws.status.data_ptr(), ops.stream_ptr(dev))
        outs.append(out)
    torch.cuda.synchronize()
    ref = sum(a[:, k * cs:k * cs + r].double().t() @ b[k].double() for k in range(groups)) + 0.5
    err = (outs[0].double().cpu() - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item(), err
    if deterministic:
        assert torch.equal(outs[0], outs[1])


def test_splitk_rejects_a_short_workspace() -> None:
    dev = torch.device("cuda")
    a = torch.zeros(1024, 256, dtype=torch.bfloat16, device=dev)
    b = torch.zeros(1024, 512, dtype=torch.bfloat16, device=dev)
    out = torch.zeros(256, 512, device=dev)
    elems = int(_lib.lib().da_gemm_splitk_workspace_elems(256, 512, 1024, 0))
    assert elems >= 256 * 512
    part = torch.empty(elems - 4, device=dev)
    rc = _lib.lib().da_gemm_splitk(a.data_ptr(), 256, 1, b.data_ptr(), 512, 1, out.data_ptr(), 512, 256, 512, 1024,
                                   _lib.DA_BF16, 0, part.data_ptr(), part.numel(),
                                   ops.workspace(dev).status.data_ptr(), ops.stream_ptr(dev))
    assert rc == _lib.DA_ERR_WORKSPACE


@pytest.mark.parametrize(("m", "n", "k"), [(1024, 512, 32768), (512, 512, 4096), (256, 256, 64)])
@pytest.mark.parametrize("store", [torch.bfloat16, torch.float32])
def test_splitk_store_equals_accumulate_into_zeros(m, n, k, store) -> None:
    """da_gemm_splitk_store (C = A^T B stored once, in fp32 or the operand dtype) against da_gemm_splitk
    into a zero-filled fp32 C then cast: the same fixed-order split sums, so bit for bit equal -- at the
    weight-gradient shapes of the config-3 projections (B16 and B2 rows) and at a one-split size."""
    torch.manual_seed(m + n + k)
    dev = torch.device("cuda")
    a = torch.randn(k, m, device=dev).to(torch.bfloat16)
    b = torch.randn(k, n, device=dev).to(torch.bfloat16)
    want = torch.zeros(m, n, device=dev)
    ops.gemm_splitk(a, m, True, b, n, True, m, n, k, want)
    got = ops.weight_grad(a, b, m, n, k, store)
    torch.cuda.synchronize()
    assert got.dtype == store
    assert torch.equal(got, want.to(store))
    assert ops.device_status(dev) == 0
    ref = a.float().t() @ b.float()
    assert (want - ref).abs().max().item() <= 1e-3 * ref.abs().max().item()
