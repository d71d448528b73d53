"""Tensor-core building blocks and the dictionary normalisation kernel on a B200.

The MMA self-test computes one 128 x N tile with the same TMA layouts,
shared-memory descriptors and TMEM read-back the routing kernels use, and
compares it element by element with an fp32 matmul of the same bf16 inputs.
"""

from __future__ import annotations

import pytest
import torch

from double_attention_b200 import _lib

pytestmark = pytest.mark.gpu

CASES = [
    (1, 64, False),
    (1, 128, False),
    (1, 256, False),
    (1, 128, True),
    (1, 256, True),
    (2, 64, False),
    (2, 128, False),
    (2, 256, False),
    (2, 128, True),
    (2, 256, True),
]


@pytest.mark.parametrize("k", [64, 256])
@pytest.mark.parametrize(("cta_group", "n", "b_mn"), CASES)
def test_selftest_mma_tile(cta_group: int, n: int, b_mn: bool, k: int) -> None:
    torch.manual_seed(1000 + 7 * n + k + cta_group)
    dev = torch.device("cuda")
    a = torch.randn(128, k, device=dev).to(torch.bfloat16)
    b = torch.randn(n, k, device=dev).to(torch.bfloat16)
    b_arg = b.t().contiguous() if b_mn else b
    d = torch.full((128, n), float("nan"), device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    _lib.call(
        "da_selftest_mma", cta_group, n, int(b_mn), k, a.data_ptr(), b_arg.data_ptr(), d.data_ptr(),
        status.data_ptr(), _lib.stream_ptr(),
    )
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0]
    expected = a.float() @ b.float().t()
    torch.testing.assert_close(d, expected, atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("r", "m"), [(256, 512), (128, 512), (512, 1536), (8, 16)])
def test_dict_norm_forward_backward(dtype: torch.dtype, r: int, m: int) -> None:
    torch.manual_seed(r + m)
    dev = torch.device("cuda")
    raw = (torch.randn(r, m, device=dev) * r**-0.5).requires_grad_()
    raw.data[:, 3] = 0.0  # a column below eps takes the clamped branch
    out = torch.empty(r, m, device=dev, dtype=dtype)
    out_t = torch.empty(m, r, device=dev, dtype=dtype)
    denom = torch.empty(m, device=dev)
    max_norm = torch.empty(1, device=dev)
    eps = 1e-6
    _lib.call(
        "da_dict_norm_fwd", raw.data_ptr(), r, m, eps, _lib.dtype_code(dtype), out.data_ptr(), out_t.data_ptr(),
        denom.data_ptr(), max_norm.data_ptr(), _lib.stream_ptr(),
    )
    expected = torch.nn.functional.normalize(raw, dim=0, eps=eps)
    # the column norm's summation order differs from torch's: allow 1 ulp
    torch.testing.assert_close(out, expected.detach().to(dtype))
    torch.testing.assert_close(out_t.float(), out.float().t(), atol=0, rtol=0)
    torch.testing.assert_close(denom, raw.detach().norm(dim=0).clamp_min(eps), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(max_norm[0], out.float().norm(dim=0).max(), atol=1e-6, rtol=1e-5)

    grad = torch.randn(r, m, device=dev)
    grad_t = torch.randn(m, r, device=dev)
    expected.backward(grad + grad_t.t())
    grad_raw = torch.empty(r, m, device=dev)
    _lib.call(
        "da_dict_norm_bwd", raw.data_ptr(), denom.data_ptr(), grad.data_ptr(), grad_t.data_ptr(), r, m, eps,
        grad_raw.data_ptr(), 0, _lib.stream_ptr(),
    )
    torch.testing.assert_close(grad_raw, raw.grad, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("r", "m"), [(256, 512), (128, 512), (512, 1536), (8, 20)])
def test_dict_norm_pair_matches_single_bank_calls(dtype: torch.dtype, r: int, m: int) -> None:
    """One launch for the key bank (compute dtype) and the value bank (bf16)."""
    torch.manual_seed(r * m)
    dev = torch.device("cuda")
    raw_k = torch.randn(r, m, device=dev) * r**-0.5
    raw_v = torch.randn(r, m, device=dev) * r**-0.5
    raw_k[:, 1] = 0.0
    eps = 1e-6
    key, key_t = torch.empty(r, m, device=dev, dtype=dtype), torch.empty(m, r, device=dev, dtype=dtype)
    val, val_t = (torch.empty(r, m, device=dev, dtype=torch.bfloat16),
                  torch.empty(m, r, device=dev, dtype=torch.bfloat16))
    kden, vden, kmax = torch.empty(m, device=dev), torch.empty(m, device=dev), torch.empty(1, device=dev)
    _lib.call("da_dict_norm_pair_fwd", raw_k.data_ptr(), raw_v.data_ptr(), _lib.DA_F32, r, m, eps, _lib.dtype_code(dtype),
              key.data_ptr(), key_t.data_ptr(), kden.data_ptr(), kmax.data_ptr(), val.data_ptr(), val_t.data_ptr(),
              vden.data_ptr(), _lib.stream_ptr())
    torch.testing.assert_close(key, torch.nn.functional.normalize(raw_k, dim=0, eps=eps).to(dtype))
    torch.testing.assert_close(val, torch.nn.functional.normalize(raw_v, dim=0, eps=eps).to(torch.bfloat16))
    assert torch.equal(key_t, key.t()) and torch.equal(val_t, val.t())
    torch.testing.assert_close(kden, raw_k.norm(dim=0).clamp_min(eps), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(vden, raw_v.norm(dim=0).clamp_min(eps), atol=1e-6, rtol=1e-5)
    torch.testing.assert_close(kmax[0], key.float().norm(dim=0).max(), atol=1e-6, rtol=1e-5)


@pytest.mark.parametrize("raw_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_dict_norm_bwd_typed_equals_convert_call_cast(raw_dtype: torch.dtype) -> None:
    """da_dict_norm_bwd_typed on a bank in its own dtype, gradient stored in that dtype, against the
    fp32 call on the bank converted to fp32 and its result cast: the same arithmetic, so bit for bit
    equal; accumulate into fp32 likewise, and accumulate into a half type is refused."""
    torch.manual_seed(11)
    dev = torch.device("cuda")
    r, m, eps = 128, 320, 1e-6
    raw = torch.randn(r, m, device=dev).to(raw_dtype)
    raw[:, 7] = 0  # a clamped column
    raw32 = raw.float().contiguous()
    denom = raw32.norm(dim=0).clamp_min(eps).contiguous()
    grad = torch.randn(r, m, device=dev)
    grad_t = torch.randn(m, r, device=dev)
    want = torch.empty(r, m, device=dev)
    _lib.call("da_dict_norm_bwd", raw32.data_ptr(), denom.data_ptr(), grad.data_ptr(), grad_t.data_ptr(), r, m, eps,
              want.data_ptr(), 0, 0)
    got = torch.empty(r, m, dtype=raw_dtype, device=dev)
    _lib.call("da_dict_norm_bwd_typed", raw.data_ptr(), _lib.dtype_code(raw_dtype), denom.data_ptr(), grad.data_ptr(),
              grad_t.data_ptr(), r, m, eps, got.data_ptr(), _lib.dtype_code(raw_dtype), 0, 0)
    acc = torch.ones(r, m, device=dev)
    _lib.call("da_dict_norm_bwd_typed", raw.data_ptr(), _lib.dtype_code(raw_dtype), denom.data_ptr(), grad.data_ptr(),
              None, r, m, eps, acc.data_ptr(), _lib.DA_F32, 1, 0)
    want_acc = torch.ones(r, m, device=dev)
    _lib.call("da_dict_norm_bwd", raw32.data_ptr(), denom.data_ptr(), grad.data_ptr(), None, r, m, eps,
              want_acc.data_ptr(), 1, 0)
    torch.cuda.synchronize()
    assert torch.equal(got, want.to(raw_dtype))
    assert torch.equal(acc, want_acc)
    if raw_dtype != torch.float32:
        with pytest.raises(NotImplementedError):
            _lib.call("da_dict_norm_bwd_typed", raw.data_ptr(), _lib.dtype_code(raw_dtype), denom.data_ptr(),
                      grad.data_ptr(), None, r, m, eps, got.data_ptr(), _lib.dtype_code(raw_dtype), 1, 0)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_temperatures_backward_equals_autograd(dtype: torch.dtype) -> None:
    """da_temperatures_bwd against torch autograd of exp(clamp(log, lo, hi)) (modules.py:130-132,
    ops.py:160-161) in the log's dtype, with logs inside, outside and exactly on both bounds: the
    gradient passes where lo <= log <= hi, bit for bit."""
    from double_attention_b200 import ops

    dev = torch.device("cuda")
    lo_b, hi_b = ops.BETA_LOG_RANGE
    lo_s, hi_s = ops.SCALE_LOG_RANGE
    # bounds as the kernel compares them: rounded to fp32 (then to the log's dtype, which may move them)
    log_beta = torch.tensor([0.7], dtype=dtype, device=dev)
    log_scales = torch.tensor([lo_s - 1.0, float(torch.tensor(lo_s, dtype=torch.float32)), 2.5, hi_s + 0.5,
                               float(torch.tensor(hi_s, dtype=torch.float32)), 0.0], dtype=dtype, device=dev)
    for lb_value in (0.7, lo_b - 0.3, hi_b + 0.1):
        log_beta.fill_(lb_value)
        lb = log_beta.clone().requires_grad_()
        ls = log_scales.clone().requires_grad_()
        beta, scales = ops._Temperatures.apply(lb, ls)
        g_beta = torch.tensor([1.75], device=dev)
        g_scales = torch.linspace(-2.0, 3.0, log_scales.numel(), device=dev)
        torch.autograd.backward((beta, scales), (g_beta, g_scales))
        lb_ref = log_beta.clone().requires_grad_()
        ls_ref = log_scales.clone().requires_grad_()
        beta_ref = lb_ref.float().clamp(lo_b, hi_b).exp()
        scales_ref = ls_ref.float().clamp(lo_s, hi_s).exp()
        torch.autograd.backward((beta_ref, scales_ref), (g_beta, g_scales))
        torch.cuda.synchronize()
        assert lb.grad.dtype == dtype and ls.grad.dtype == dtype
        assert torch.equal(beta, beta_ref) and torch.equal(scales, scales_ref)
        assert torch.equal(lb.grad, lb_ref.grad), (lb_value, lb.grad, lb_ref.grad)
        assert torch.equal(ls.grad, ls_ref.grad), (ls.grad, ls_ref.grad)
