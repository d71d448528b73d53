"""The allocation-free route entry point (da_route_fwd_static) on a B200.

This entry point exists for callers that cannot allocate device memory while
they run the route (code under CUDA stream capture, or engines that hand a
plugin only its inputs and outputs): its work area is a __device__ array
inside the library.  Here it is called through the C ABI and checked against
the regular entry point (da_route_fwd, which takes a caller-allocated work
buffer) on the same inputs, twice in a row.

Only the 64-atom-tile route kernel uses the work area (a CTA ticket, a count
of rows to recompute exactly and their list, recomputed by the last CTA); the
wide-tile kernels that R >= 128 with M a multiple of 128 select keep their
repair lists in shared memory.  So the cases that exercise the array use
R = 64, or M not a multiple of 128, and include inputs whose every row takes
the exact repair pass (beta 60, unnormalised inputs of norm ~3 sqrt(R)), plus
a call at the array's limit of 65536 route rows.  The wide-tile cases check
that the entry point also serves the shapes that never touch the array.  The
file is named so pytest collects it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn.functional as F

import oracle
from double_attention_b200 import _lib, ops

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2


def _inputs(rows: int, r: int, m: int, groups: int, dtype: torch.dtype, seed: int, scale: float):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    q = (torch.randn(rows, groups * r, generator=g) * scale).to(dtype).to(dev)
    dk = F.normalize(torch.randn(r, m, generator=g), dim=0).to(dtype).to(dev)
    dv = F.normalize(torch.randn(r, m, generator=g), dim=0).to(dtype).to(dev)
    return q, ops.dictionary_views_from_normalized(dk, dv, dtype)


def _static_call(q, rows, groups, views, beta, normalize_input):
    r, m = views.routing_dim, views.size
    dev = q.device
    z = torch.full((groups, rows, r), float("nan"), dtype=q.dtype, device=dev)
    lse = torch.full((groups, rows), float("nan"), device=dev)
    onorm = torch.full((groups, rows), float("nan"), device=dev)
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    beta32 = torch.tensor([beta], device=dev)
    rc = _lib.lib().da_route_fwd_static(
        q.data_ptr(), rows, q.shape[1], q.stride(0), groups, r, r, m, _lib.dtype_code(q.dtype),
        views.key_t.data_ptr(), views.value.data_ptr(), beta32.data_ptr(), views.key_max.data_ptr(),
        ctypes.c_float(1e-6), int(normalize_input), 1, z.data_ptr(), lse.data_ptr(), onorm.data_ptr(), None,
        status.data_ptr(), _lib.stream_ptr(dev))
    assert rc == _lib.DA_OK, _lib.lib().da_status_string(rc)
    torch.cuda.synchronize()
    assert status.tolist() == [0, 0]
    return z, lse, onorm


@pytest.mark.parametrize(
    ("rows", "r", "m", "groups", "dtype", "beta", "scale", "normalize_input"),
    [
        # 64-atom-tile kernel: global ticket, repair count and row list in the static array
        (4096, 64, 128, 1, torch.bfloat16, 4.0, 1.0, True),
        (1000, 128, 192, 2, torch.float16, 4.0, 1.0, True),      # M not a multiple of 128, two groups
        (2000, 64, 128, 1, torch.bfloat16, 60.0, 3.0, False),    # every row repaired from the array's list
        (700, 128, 192, 1, torch.bfloat16, 60.0, 3.0, False),    # the same with a ragged tail tile
        (32768, 64, 128, 2, torch.bfloat16, 4.0, 1.0, True),     # groups * rows == 65536, the array's limit
        # wide-tile kernels (repair lists in shared memory)
        (4096, 256, 512, 2, torch.float16, 4.0, 1.0, True),      # config-2 route rows (Q and K groups)
        (512, 128, 512, 1, torch.bfloat16, 60.0, 3.0, False),    # every row repaired
    ],
)
def test_static_entry_matches_regular_entry_twice(rows, r, m, groups, dtype, beta, scale, normalize_input) -> None:
    q, views = _inputs(rows, r, m, groups, dtype, seed=rows + r, scale=scale)
    dev = q.device
    z_ref, lse_ref, on_ref = ops._route_forward(q, rows, groups, r, views, torch.tensor(beta, device=dev), 1e-6,
                                                normalize_input, True)
    torch.cuda.synchronize()
    # the regular entry itself against the fp32 oracle (value dictionary as the bf16 operand it reads)
    dk, dv = views.key_t.t().float().cpu(), views.value.float().cpu()
    for grp in range(groups):
        expected = oracle.dictionary_route(q[:, grp * r:(grp + 1) * r].float().cpu(), dk, dv, beta, 1e-6,
                                           normalize_input=normalize_input)
        assert (z_ref[grp].float().cpu() - expected).abs().max().item() <= MAX_ABS
    for _ in range(2):  # the shared work area must come back clean for the next call
        z, lse, onorm = _static_call(q, rows, groups, views, beta, normalize_input)
        assert torch.isfinite(z.float()).all()
        assert (z.float() - z_ref.float()).abs().max().item() <= MAX_ABS
        torch.testing.assert_close(lse, lse_ref, atol=2e-3, rtol=1e-4)
        torch.testing.assert_close(onorm, on_ref, atol=2e-3, rtol=5e-3)


def test_static_entry_rejects_rows_beyond_its_work_area() -> None:
    q, views = _inputs(128, 128, 512, 1, torch.bfloat16, seed=1, scale=1.0)
    dev = q.device
    out = torch.empty(1, dtype=torch.float32, device=dev)
    rc = _lib.lib().da_route_fwd_static(
        q.data_ptr(), 65537, 128, 128, 1, 128, 128, 512, _lib.DA_BF16, views.key_t.data_ptr(),
        views.value.data_ptr(), out.data_ptr(), views.key_max.data_ptr(), ctypes.c_float(1e-6), 1, 1,
        out.data_ptr(), out.data_ptr(), out.data_ptr(), None, out.data_ptr(), _lib.stream_ptr(dev))
    assert rc == _lib.DA_ERR_WORKSPACE
