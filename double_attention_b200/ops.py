"""Op layer: autograd Functions over the sm_100a C ABI.

Public op-level API mirroring the reference's Triton seam
(src/double_attention/triton_kernels.py:1984-2019 and :2290-2305):

* :func:`dictionary_route` -- same arguments, meaning and errors as
  ``dictionary_route_triton``;
* :func:`routed_attention` -- same as ``routed_attention_triton``;

plus the module-path helpers used by ``SharedDictionaryAttention``.
Every numeric step runs in the B200 kernels of ``libda_b200.so``; there is
no CPU or PyTorch fallback -- unsupported inputs raise.
"""

from __future__ import annotations

import ctypes
import math
import threading
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _lib
from ._lib import call, dtype_code, ptr, stream_ptr

REPAIR_CAP = 4096
_HALF = (torch.float16, torch.bfloat16)


# ----------------------------------------------------------------------------- dispatch
def compute_dtype(x: Tensor) -> torch.dtype:
    """The fp16/bf16 dtype the kernels compute in for input ``x``."""
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return x.dtype


_capability: dict[int, tuple[int, int]] = {}


def resolve_backend(backend: str, x: Tensor, dtype: torch.dtype | None = None) -> str:
    """Counterpart of ops.py:142-157.  Only the B200 kernels exist here:
    ``"auto"``/``"triton"``/``"b200"`` select them and fail loudly when they
    cannot run; ``"torch"`` is rejected (no CPU implementation ships)."""
    if backend == "torch":
        raise NotImplementedError(
            "backend='torch' is not provided by double_attention_b200; it ships only the B200 kernels"
        )
    dtype = dtype or x.dtype
    if not x.is_cuda or dtype not in _HALF:
        raise RuntimeError("B200 backend requested but unavailable: CUDA fp16/bf16 tensors are required")
    idx = x.device.index if x.device.index is not None else torch.cuda.current_device()
    cap = _capability.get(idx)
    if cap is None:
        cap = _capability[idx] = torch.cuda.get_device_capability(idx)
    major, minor = cap
    if (major, minor) != (10, 0):
        raise RuntimeError(f"B200 backend requested but unavailable: sm_100 GPU required, found sm_{major}{minor}")
    return "b200"


def score_scale_from_log(log_scale: Tensor) -> Tensor:
    """ops.py:160-161."""
    return log_scale.clamp(math.log(0.25), math.log(1024.0)).exp()


def assemble_score_maps(query: Tensor, key: Tensor, outer_maps: int) -> tuple[Tensor, Tensor]:
    """Index mapping of ops.py:96-139 (used for the aux outputs; the
    attention kernel applies the same mapping through its addressing)."""
    if query.ndim != 4 or query.shape != key.shape:
        raise ValueError("query and key must have matching [B, H, T, R] shapes")
    branches = query.shape[1]
    if branches == outer_maps:
        return query, key
    if branches > outer_maps:
        if branches % outer_maps:
            raise ValueError("qk_branches must be divisible by outer_maps")
        group = branches // outer_maps
        s = group ** -0.25
        b, _, t, r = query.shape

        def fold(z: Tensor) -> Tensor:
            return z.reshape(b, outer_maps, group, t, r).permute(0, 1, 3, 2, 4).reshape(b, outer_maps, t, group * r) * s

        return fold(query), fold(key)
    if outer_maps % branches:
        raise ValueError("outer_maps must be divisible by qk_branches")
    rep = outer_maps // branches
    return query.repeat_interleave(rep, dim=1), key.repeat_interleave(rep, dim=1)


# ----------------------------------------------------------------------------- workspaces
class _Workspace:
    """Per-(device, stream) scratch the kernels keep between calls: the route
    kernel's CTA ticket / repair list (zero-initialised once, reset by the
    kernel itself) and a device status word."""

    def __init__(self, device: torch.device) -> None:
        self.route_work = torch.zeros(2 + REPAIR_CAP, dtype=torch.int32, device=device)
        self.status = torch.zeros(2, dtype=torch.int32, device=device)


_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], _Workspace] = {}
# Zero-filled workspaces made outside any graph capture, for streams first seen while one is captured:
# a workspace made during the capture would put its zero fills into the graph, replayed every step.
_spare_workspaces: dict[int, list[_Workspace]] = {}
_SPARES = 4


def workspace(device: torch.device) -> _Workspace:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, stream_ptr(device))
    ws = _workspaces.get(key)
    if ws is None:
        with _ws_lock:
            ws = _workspaces.get(key)
            if ws is None:
                spares = _spare_workspaces.setdefault(idx, [])
                capturing = torch.cuda.is_current_stream_capturing()
                if capturing and spares:
                    ws = spares.pop()
                else:
                    ws = _Workspace(device)
                    while not capturing and len(spares) < _SPARES:
                        spares.append(_Workspace(device))
                _workspaces[key] = ws
    return ws


def device_status(device: torch.device | None = None, reset: bool = True) -> int:
    """OR of all status bits kernels on this device/stream reported (syncs).

    Raises when a kernel reported a device-side wait that gave up, naming
    the wait site (a logic error in a kernel, never expected)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    ws = workspace(device)
    flags, site = (int(v) for v in ws.status.tolist())
    if reset:
        ws.status.zero_()
    if flags & 1:
        raise _lib.DAError("device status", _lib.DA_ERR_DEVICE_TIMEOUT, f"bounded wait gave up at site {site}")
    return flags


def _grad_wanted(*tensors: Tensor | None) -> bool:
    """True when autograd must record this op (grad mode on and an input requires grad); otherwise
    the wrappers below call the kernels directly, without the autograd Function machinery."""
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _check_half_cuda(name: str, *tensors: Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise ValueError(f"{name} requires CUDA tensors")
    dt = tensors[0].dtype
    if dt not in _HALF or any(t.dtype != dt for t in tensors):
        raise ValueError(f"{name} requires fp16 or bf16 inputs of one matching dtype")


# ----------------------------------------------------------------------------- dictionaries
@dataclass
class DictionaryViews:
    """Kernel operands of one normalised dictionary bank in one dtype.

    key   [R, M], key_t [M, R] in the compute dtype (q . Dk operands)
    value [R, M], value_t [M, R] in bf16 (probability . Dv operands)
    key_max: max column norm of ``key`` as rounded (softmax offset bound).
    key_anchor / value_anchor: [R, M] tensors through which the route
    backward returns the dictionary gradients in fp32 (their contents are
    never read), so gradients from every block sharing a bank accumulate in
    fp32 before one normalisation backward.
    """

    key: Tensor
    key_t: Tensor
    value: Tensor
    value_t: Tensor
    key_max: Tensor
    key_anchor: Tensor
    value_anchor: Tensor

    @property
    def routing_dim(self) -> int:
        return self.key.shape[0]

    @property
    def size(self) -> int:
        return self.key.shape[1]


class _DictNorm(torch.autograd.Function):
    """Column normalisation + cast of a bank (modules.py:45-48, :229-231)."""

    @staticmethod
    def forward(ctx, raw: Tensor, eps: float, dtype: torch.dtype):  # type: ignore[override]
        raw = raw.detach().contiguous().float()
        r, m = raw.shape
        out = torch.empty(r, m, dtype=dtype, device=raw.device)
        out_t = torch.empty(m, r, dtype=dtype, device=raw.device)
        denom = torch.empty(m, dtype=torch.float32, device=raw.device)
        mx = torch.empty(1, dtype=torch.float32, device=raw.device)
        call("da_dict_norm_fwd", raw.data_ptr(), r, m, eps, dtype_code(dtype), out.data_ptr(), out_t.data_ptr(),
             denom.data_ptr(), mx.data_ptr(), stream_ptr(raw.device))
        ctx.save_for_backward(raw, denom)
        ctx.eps = eps
        ctx.mark_non_differentiable(mx)
        ctx.set_materialize_grads(False)  # views nothing differentiates stay None (no zero fills)
        anchor = torch.empty(r, m, dtype=torch.float32, device=raw.device)  # fp32 gradient entry, never read
        return out, out_t, mx, anchor

    @staticmethod
    def backward(ctx, g_out: Tensor | None, g_out_t: Tensor | None, _g_mx, g_anchor: Tensor | None):  # type: ignore[override]
        raw, denom = ctx.saved_tensors
        if g_anchor is not None:
            g_out = g_anchor if g_out is None else g_anchor + g_out.float()
        if g_out is None and g_out_t is None:
            return None, None, None
        r, m = raw.shape
        ga = None if g_out is None else g_out.float().contiguous()
        gb = None if g_out_t is None else g_out_t.float().contiguous()
        grad = torch.empty_like(raw)
        call("da_dict_norm_bwd", raw.data_ptr(), denom.data_ptr(), ptr(ga), ptr(gb), r, m, ctx.eps,
             grad.data_ptr(), 0, stream_ptr(raw.device))
        return grad, None, None


class _DictNormPair(torch.autograd.Function):
    """Key bank (compute dtype) and value bank (bf16) normalised in one launch.

    ``raw_value`` None means a tied dictionary whose value views are a bf16
    normalisation of ``raw_key`` (the compute dtype is not bf16)."""

    @staticmethod
    def forward(ctx, raw_key: Tensor, raw_value: Tensor | None, eps: float, dtype: torch.dtype):  # type: ignore[override]
        rk = raw_key.detach().contiguous()  # fp32, or the half type of a cast module (read as is)
        rv = rk if raw_value is None else raw_value.detach().to(rk.dtype).contiguous()
        r, m = rk.shape
        dev = rk.device
        key = torch.empty(r, m, dtype=dtype, device=dev)
        key_t = torch.empty(m, r, dtype=dtype, device=dev)
        value = torch.empty(r, m, dtype=torch.bfloat16, device=dev)
        value_t = torch.empty(m, r, dtype=torch.bfloat16, device=dev)
        kden = torch.empty(m, dtype=torch.float32, device=dev)
        vden = torch.empty(m, dtype=torch.float32, device=dev)
        kmax = torch.empty(1, dtype=torch.float32, device=dev)
        call("da_dict_norm_pair_fwd", rk.data_ptr(), rv.data_ptr(), dtype_code(rk.dtype), r, m, eps, dtype_code(dtype),
             key.data_ptr(),
             key_t.data_ptr(), kden.data_ptr(), kmax.data_ptr(), value.data_ptr(), value_t.data_ptr(),
             vden.data_ptr(), stream_ptr(dev))
        ctx.save_for_backward(rk, rv, kden, vden)
        ctx.raw_dtype = raw_key.dtype
        ctx.eps = eps
        ctx.tied = raw_value is None
        ctx.mark_non_differentiable(kmax)
        # the route's backward gives the fp32 anchors their gradients and the bf16 views none: those stay
        # None instead of zero-filled tensors that the backward would convert and add
        ctx.set_materialize_grads(False)
        key_anchor = torch.empty(r, m, dtype=torch.float32, device=dev)  # fp32 gradient entries, never read
        value_anchor = torch.empty(r, m, dtype=torch.float32, device=dev)
        return key, key_t, kmax, key_anchor, value, value_t, value_anchor

    @staticmethod
    def backward(ctx, g_key, g_key_t, _g_kmax, g_key_anchor, g_value, g_value_t, g_value_anchor):  # type: ignore[override]
        rk, rv, kden, vden = ctx.saved_tensors  # the banks in their own dtype, read exactly by the kernel
        r, m = rk.shape
        dev = rk.device
        rdt = dtype_code(rk.dtype)

        def merged(g, anchor):
            if anchor is None:
                return None if g is None else g.float().contiguous()
            return anchor.contiguous() if g is None else (anchor + g.float()).contiguous()

        gk, gv = merged(g_key, g_key_anchor), merged(g_value, g_value_anchor)
        gkt = None if g_key_t is None else g_key_t.float().contiguous()
        gvt = None if g_value_t is None else g_value_t.float().contiguous()
        want_key = gk is not None or gkt is not None
        want_value = gv is not None or gvt is not None

        def norm_bwd(raw, den, g, gt, out, accumulate):
            call("da_dict_norm_bwd_typed", raw.data_ptr(), rdt, den.data_ptr(), ptr(g), ptr(gt), r, m, ctx.eps,
                 out.data_ptr(), dtype_code(out.dtype), accumulate, stream_ptr(dev))

        grad_key = grad_value = None
        if ctx.tied and want_value:  # the value bank is the key bank: both gradients added in fp32 on raw_key
            grad_key = (torch.empty if want_key else torch.zeros)(r, m, dtype=torch.float32, device=dev)
            if want_key:
                norm_bwd(rk, kden, gk, gkt, grad_key, 0)
            norm_bwd(rk, vden, gv, gvt, grad_key, 1)
            grad_key = grad_key.to(ctx.raw_dtype)
        else:  # each gradient stored once in its bank's dtype
            if want_key:
                grad_key = torch.empty(r, m, dtype=ctx.raw_dtype, device=dev)
                norm_bwd(rk, kden, gk, gkt, grad_key, 0)
            if want_value:
                grad_value = torch.empty(r, m, dtype=ctx.raw_dtype, device=dev)
                norm_bwd(rv, vden, gv, gvt, grad_value, 0)
        return grad_key, grad_value, None, None


# ----------------------------------------------------------------------------- temperatures
BETA_LOG_RANGE = (math.log(0.05), math.log(64.0))     # modules.py:130-132
SCALE_LOG_RANGE = (math.log(0.25), math.log(1024.0))  # ops.py:160-161


def _temperatures_forward(log_beta: Tensor, log_scales: Tensor) -> tuple[Tensor, Tensor]:
    dev = log_scales.device
    out = torch.empty(1 + log_scales.numel(), dtype=torch.float32, device=dev)
    beta, scales = out[:1], out[1:]
    lb, ls = log_beta.detach().contiguous(), log_scales.detach().contiguous()
    call("da_temperatures", lb.data_ptr(), dtype_code(lb.dtype), BETA_LOG_RANGE[0], BETA_LOG_RANGE[1],
         ls.data_ptr(), dtype_code(ls.dtype), ls.numel(), SCALE_LOG_RANGE[0], SCALE_LOG_RANGE[1],
         beta.data_ptr(), scales.data_ptr(), stream_ptr(dev))
    return beta, scales


class _Temperatures(torch.autograd.Function):
    """beta and the per-map score scales in fp32 from their logs, one launch."""

    @staticmethod
    def forward(ctx, log_beta: Tensor, log_scales: Tensor):  # type: ignore[override]
        beta, scales = _temperatures_forward(log_beta, log_scales)
        ctx.save_for_backward(log_beta, log_scales, beta, scales)
        return beta, scales

    @staticmethod
    def backward(ctx, g_beta, g_scales):  # type: ignore[override]
        # d log = g * value inside the clamp range (inclusive), else 0; both in one launch, each rounded
        # once to its log's dtype
        log_beta, log_scales, beta, scales = ctx.saved_tensors
        if g_beta is None and g_scales is None:
            return None, None
        lb, ls = log_beta.detach().contiguous(), log_scales.detach().contiguous()
        gb = None if g_beta is None else g_beta.float().contiguous()
        gs = None if g_scales is None else g_scales.float().contiguous()
        grad_lb = None if gb is None else torch.empty_like(lb)
        grad_ls = None if gs is None else torch.empty_like(ls)
        call("da_temperatures_bwd", lb.data_ptr(), dtype_code(lb.dtype), BETA_LOG_RANGE[0], BETA_LOG_RANGE[1],
             beta.data_ptr(), ptr(gb), ptr(grad_lb), ls.data_ptr(), dtype_code(ls.dtype), ls.numel(),
             SCALE_LOG_RANGE[0], SCALE_LOG_RANGE[1], scales.data_ptr(), ptr(gs), ptr(grad_ls), stream_ptr(lb.device))
        return grad_lb, grad_ls


def temperatures(log_beta: Tensor, log_scales: Tensor) -> tuple[Tensor, Tensor]:
    """``(beta [1], scales [S])`` in fp32: exp of the clamped logs (modules.py:130-132, ops.py:160-161)."""
    if not _grad_wanted(log_beta, log_scales):
        return _temperatures_forward(log_beta, log_scales)
    return _Temperatures.apply(log_beta, log_scales)


def _dictionary_views_nograd(raw_key: Tensor, raw_value: Tensor | None, eps: float,
                             dtype: torch.dtype) -> DictionaryViews:
    """The views of dictionary_views without autograd (one launch)."""
    rk = raw_key.detach().contiguous()
    rv = rk if raw_value is None else raw_value.detach().to(rk.dtype).contiguous()
    r, m = rk.shape
    dev = rk.device
    key, key_t = torch.empty(r, m, dtype=dtype, device=dev), torch.empty(m, r, dtype=dtype, device=dev)
    value = torch.empty(r, m, dtype=torch.bfloat16, device=dev)
    value_t = torch.empty(m, r, dtype=torch.bfloat16, device=dev)
    stats = torch.empty(2 * m + 4, dtype=torch.float32, device=dev)  # key / value denominators, max
    kden, vden, kmax = stats[:m], stats[m:2 * m], stats[2 * m:2 * m + 1]
    call("da_dict_norm_pair_fwd", rk.data_ptr(), rv.data_ptr(), dtype_code(rk.dtype), r, m, eps, dtype_code(dtype),
         key.data_ptr(), key_t.data_ptr(), kden.data_ptr(), kmax.data_ptr(), value.data_ptr(), value_t.data_ptr(),
         vden.data_ptr(), stream_ptr(rk.device))
    return DictionaryViews(key, key_t, value, value_t, kmax, key, value)


def dictionary_views(raw_key: Tensor, raw_value: Tensor | None, eps: float, dtype: torch.dtype) -> DictionaryViews:
    """Normalise a bank's raw parameters into kernel operands (autograd-aware)."""
    if not raw_key.is_cuda:
        raise RuntimeError("B200 backend requested but unavailable: CUDA fp16/bf16 tensors are required")
    if not _grad_wanted(raw_key, raw_value):
        return _dictionary_views_nograd(raw_key, raw_value, eps, dtype)
    if raw_value is None and dtype == torch.bfloat16:  # tied dictionary: one set of bf16 views serves both
        key, key_t, key_max, key_anchor = _DictNorm.apply(raw_key, eps, dtype)
        return DictionaryViews(key, key_t, key, key_t, key_max, key_anchor, key_anchor)
    key, key_t, key_max, key_anchor, value, value_t, value_anchor = _DictNormPair.apply(raw_key, raw_value, eps,
                                                                                      dtype)
    return DictionaryViews(key, key_t, value, value_t, key_max, key_anchor, value_anchor)


def _col_norm_max(d: Tensor) -> Tensor:
    out = torch.empty(1, dtype=torch.float32, device=d.device)
    call("da_col_norm_max", d.data_ptr(), d.shape[0], d.shape[1], dtype_code(d.dtype), out.data_ptr(),
         stream_ptr(d.device))
    return out


def dictionary_views_from_normalized(key: Tensor, value: Tensor, dtype: torch.dtype) -> DictionaryViews:
    """Kernel operands from caller-normalised dictionaries (cast + transpose).

    The caller's tensors themselves are the gradient anchors: the route
    backward returns the dictionary gradients to them."""
    k = key.detach().to(dtype).contiguous()
    v = value.detach().to(torch.bfloat16).contiguous()
    return DictionaryViews(k, k.t().contiguous(), v, v.t().contiguous(), _col_norm_max(k), key, value)


# ----------------------------------------------------------------------------- route
def _route_supported(r: int, m: int) -> None:
    if r not in (64, 128, 256, 512):
        raise NotImplementedError(f"dictionary route kernels support routing widths 64/128/256/512, got {r}")
    if m % 64:
        raise NotImplementedError(f"dictionary route kernels need a dictionary size divisible by 64, got {m}")


def _route_forward(q: Tensor, rows: int, groups: int, col_stride: int, views: DictionaryViews, beta: Tensor,
                   eps: float, normalize_input: bool, normalize_output: bool,
                   argmax: Tensor | None = None) -> tuple[Tensor, Tensor, Tensor]:
    r, m = views.routing_dim, views.size
    _route_supported(r, m)
    dev = q.device
    z = torch.empty(groups, rows, r, dtype=q.dtype, device=dev)
    lse = torch.empty(groups, rows, dtype=torch.float32, device=dev)
    onorm = torch.empty(groups, rows, dtype=torch.float32, device=dev)
    ws = workspace(dev)
    beta32 = beta.detach().float().reshape(1).contiguous()
    call("da_route_fwd", q.data_ptr(), rows, q.shape[1], q.stride(0), groups, col_stride, r, m, dtype_code(q.dtype),
         views.key_t.data_ptr(), views.value.data_ptr(), beta32.data_ptr(), views.key_max.data_ptr(), eps,
         int(normalize_input), int(normalize_output), z.data_ptr(), lse.data_ptr(), onorm.data_ptr(), ptr(argmax),
         ws.route_work.data_ptr(), REPAIR_CAP, ws.status.data_ptr(), stream_ptr(dev))
    return z, lse, onorm


class _Route(torch.autograd.Function):
    """Dictionary route over ``groups`` column blocks of a [rows, cols] matrix."""

    @staticmethod
    def forward(ctx, q: Tensor, key: Tensor, key_t: Tensor, value: Tensor, value_t: Tensor, key_max: Tensor,  # type: ignore[override]
                key_anchor: Tensor, value_anchor: Tensor, beta: Tensor, rows: int, groups: int, col_stride: int,
                eps: float, normalize_input: bool, normalize_output: bool):
        views = DictionaryViews(key, key_t, value, value_t, key_max, key_anchor, value_anchor)
        z, lse, onorm = _route_forward(q, rows, groups, col_stride, views, beta, eps, normalize_input,
                                       normalize_output)
        ctx.save_for_backward(q, key_t, value_t, beta, z, lse, onorm)
        ctx.meta = (rows, groups, col_stride, eps, normalize_input, normalize_output,
                    key_anchor.dtype, value_anchor.dtype)
        return z

    @staticmethod
    def backward(ctx, dz: Tensor):  # type: ignore[override]
        return _route_backward(ctx, dz)


def gemm_splitk(a: Tensor, lda: int, a_mn: bool, b: Tensor, ldb: int, b_mn: bool, m: int, n: int, k: int,
                out: Tensor, splits: int = 0) -> Tensor:
    """out[m, n] += sum_k A(m, k) B(n, k) in fp32, K split over CTAs whose partial sums are added in a fixed
    order (see da_gemm_splitk), so the result is bit-reproducible."""
    ws = workspace(out.device)
    elems = int(_lib.lib().da_gemm_splitk_workspace_elems(m, n, k, splits))
    part = torch.empty(max(elems, 4), dtype=torch.float32, device=out.device)
    call("da_gemm_splitk", a.data_ptr(), lda, int(a_mn), b.data_ptr(), ldb, int(b_mn), out.data_ptr(), out.stride(0),
         m, n, k, dtype_code(a.dtype), splits, part.data_ptr(), part.numel(), ws.status.data_ptr(),
         stream_ptr(out.device))
    return out


def weight_grad(a: Tensor, b: Tensor, m: int, n: int, k: int, dtype: torch.dtype) -> Tensor:
    """A new [m, n] tensor = sum over the k rows of a [k, m]^T . b [k, n] (a weight gradient dY^T . X),
    the rows split over CTAs and the partial sums added in a fixed order, stored once in ``dtype`` (fp32,
    or the operands' dtype; another dtype goes through fp32 and a cast)."""
    store = dtype if dtype in (torch.float32, a.dtype) else torch.float32
    out = torch.empty(m, n, dtype=store, device=a.device)
    elems = int(_lib.lib().da_gemm_splitk_workspace_elems(m, n, k, 0))
    part = torch.empty(max(elems, 4), dtype=torch.float32, device=a.device)
    call("da_gemm_splitk_store", a.data_ptr(), a.stride(0), 1, b.data_ptr(), b.stride(0), 1, out.data_ptr(),
         out.stride(0), dtype_code(store), m, n, k, dtype_code(a.dtype), 0, part.data_ptr(), part.numel(),
         workspace(a.device).status.data_ptr(), stream_ptr(a.device))
    return out if store == dtype else out.to(dtype)


def key_dictionary_grad(q: Tensor, col_stride: int, dl: Tensor, out: Tensor) -> Tensor:
    """out [R, M] fp32 += sum_g q_g^T dl[g]: q_g the g-th column block (width R, stride col_stride) of
    the routed matrix q [rows, cols], dl [groups, rows, M] -- one split-K launch over every group
    when the rows divide into 64-row stages, else one per group."""
    groups, rows, m = dl.shape
    r = out.shape[0]
    if groups > 1 and rows % 64 == 0 and col_stride % 8 == 0:
        elems = int(_lib.lib().da_gemm_splitk_workspace_elems(r, m, rows * groups, 0))
        part = torch.empty(max(elems, 4), dtype=torch.float32, device=q.device)
        call("da_gemm_splitk_grouped", q.data_ptr(), q.stride(0), col_stride, dl.data_ptr(), m, out.data_ptr(),
             out.stride(0), r, m, rows, groups, dtype_code(q.dtype), 0, part.data_ptr(), part.numel(),
             workspace(q.device).status.data_ptr(), stream_ptr(q.device))
    else:
        for g in range(groups):
            gemm_splitk(q[:, g * col_stride:], q.stride(0), True, dl[g], m, True, r, m, rows, out)
    return out


def route_bwd_fused_supported(q: Tensor, rows: int, col_stride: int, r: int, m: int) -> bool:
    """Shapes the deterministic fused route backward (da_route_bwd_fused) takes; others use da_route_bwd
    plus split-K GEMMs over stored [rows, M] weights."""
    return (r in (128, 256) and m % 128 == 0 and q.shape[1] % 64 == 0 and col_stride % 64 == 0
            and q.stride(0) % 8 == 0 and rows >= (128 if r == 128 else 64))


def _route_backward_fused(q: Tensor, key_t: Tensor, value_t: Tensor, beta: Tensor, z: Tensor, dz: Tensor,
                          lse: Tensor, onorm: Tensor, dq: Tensor, rows: int, groups: int, col_stride: int, eps: float,
                          ni: bool, no: bool, need_key: bool, need_value: bool, need_beta: bool):
    """dq (into ``dq``) and fp32 dDk, dDv [R, M], dbeta [1] from one da_route_bwd_fused call."""
    m, r = key_t.shape
    dev = q.device
    handle = _lib.lib()
    ws_bytes = int(handle.da_route_bwd_workspace_size(rows, groups, r, m))
    scratch = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    d_key = torch.empty(r, m, dtype=torch.float32, device=dev) if need_key else None
    d_value = torch.empty(r, m, dtype=torch.float32, device=dev) if need_value else None
    dbeta = torch.empty(1, dtype=torch.float32, device=dev) if need_beta else None
    beta32 = beta.detach().float().reshape(1).contiguous()
    call("da_route_bwd_fused", q.data_ptr(), rows, q.shape[1], q.stride(0), groups, col_stride, r, m,
         dtype_code(q.dtype), key_t.data_ptr(), value_t.data_ptr(), beta32.data_ptr(), eps, int(ni), int(no),
         z.data_ptr(), dz.data_ptr(), lse.data_ptr(), onorm.data_ptr(), dq.data_ptr(), ptr(d_key), ptr(d_value),
         ptr(dbeta), scratch.data_ptr(), ws_bytes, workspace(dev).status.data_ptr(), stream_ptr(dev))
    return d_key, d_value, dbeta


def _route_backward(ctx, dz: Tensor):
    """dq, fp32 dDk / dDv (into the anchors) and dbeta of one route call."""
    q, key_t, value_t, beta, z, lse, onorm = ctx.saved_tensors
    rows, groups, col_stride, eps, ni, no, key_dtype, value_dtype = ctx.meta
    need = ctx.needs_input_grad
    m, r = key_t.shape
    dev = q.device
    dz = dz.to(z.dtype).contiguous()
    full = groups * col_stride == q.shape[1] and col_stride == r and q.stride(0) == q.shape[1]
    dq = torch.empty_like(q) if full else torch.zeros_like(q)
    if route_bwd_fused_supported(q, rows, col_stride, r, m):
        d_key, d_value, dbeta = _route_backward_fused(q, key_t, value_t, beta, z, dz, lse, onorm, dq, rows, groups,
                                                      col_stride, eps, ni, no, need[6], need[7], need[8])
        return (dq if need[0] else None, None, None, None, None, None,
                None if d_key is None else d_key.to(key_dtype),
                None if d_value is None else d_value.to(value_dtype),
                None if dbeta is None else dbeta.view(beta.shape).to(beta.dtype),
                None, None, None, None, None, None)
    p_out = torch.empty(groups, rows, m, dtype=torch.bfloat16, device=dev)
    dl_out = torch.empty(groups, rows, m, dtype=q.dtype, device=dev)
    g_out = torch.empty(groups, rows, r, dtype=torch.bfloat16, device=dev)
    dbeta = torch.zeros(1, dtype=torch.float32, device=dev) if need[8] else None
    # per-(CTA, warp) dbeta partials, added in a fixed order by the library
    dbeta_work = torch.empty(8 * groups * ((rows + 127) // 128), dtype=torch.float32, device=dev) if need[8] else None
    ws = workspace(dev)
    beta32 = beta.detach().float().reshape(1).contiguous()
    call("da_route_bwd", q.data_ptr(), rows, q.shape[1], q.stride(0), groups, col_stride, r, m, dtype_code(q.dtype),
         key_t.data_ptr(), value_t.data_ptr(), beta32.data_ptr(), eps, int(ni), int(no), z.data_ptr(), dz.data_ptr(),
         lse.data_ptr(), onorm.data_ptr(), dq.data_ptr(), p_out.data_ptr(), dl_out.data_ptr(), g_out.data_ptr(),
         ptr(dbeta), ptr(dbeta_work), 0 if dbeta_work is None else dbeta_work.numel(), ws.status.data_ptr(),
         stream_ptr(dev))
    d_key = d_value = None
    if need[6]:  # dDk = sum_groups q_g^T dL'_g  (dL' already carries 1 / ||q||)
        d_key = torch.zeros(r, m, dtype=torch.float32, device=dev)
        key_dictionary_grad(q, col_stride, dl_out, d_key)
    if need[7]:  # dDv = G^T P over every routed row
        d_value = torch.zeros(r, m, dtype=torch.float32, device=dev)
        gemm_splitk(g_out.view(-1, r), r, True, p_out.view(-1, m), m, True, r, m, groups * rows, d_value)
    return (dq if need[0] else None, None, None, None, None, None,
            None if d_key is None else d_key.to(key_dtype),
            None if d_value is None else d_value.to(value_dtype),
            None if dbeta is None else dbeta.view(beta.shape).to(beta.dtype),
            None, None, None, None, None, None)


# ----------------------------------------------------------------------------- route variants
# Flag bits of the variant row stages (include/da_b200.h DA_ROUTE_*).
ROUTE_SILU_LOGITS, ROUTE_STANDARDIZE, ROUTE_DIRECT_SILU, ROUTE_NORM_INPUT = 1, 2, 4, 8


@dataclass(frozen=True)
class RouteVariant:
    """The switches of dictionary_route_reference (ops.py:16-62) other than
    identity logits with softmax assignment: ``flags`` (ROUTE_* bits), the
    direct-SiLU gain and the standardised-logit scale."""

    flags: int
    silu_gain: float = 1.0
    std_scale: float = 1.0


def route_variant(activation: str, assignment: str, silu_gain: float, standardize: bool,
                  standardized_logit_scale: float | None, routing_dim: int) -> RouteVariant | None:
    """The variant of a route configuration, or None for identity logits with softmax (the fused kernel)."""
    if activation not in ("identity", "silu"):
        raise ValueError(f"unsupported dictionary activation: {activation}")
    if assignment not in ("softmax", "silu"):
        raise ValueError(f"unsupported dictionary assignment: {assignment}")
    flags = (ROUTE_SILU_LOGITS if activation == "silu" else 0) | (ROUTE_STANDARDIZE if standardize else 0) \
        | (ROUTE_DIRECT_SILU if assignment == "silu" else 0)
    if not flags:
        return None
    scale = routing_dim ** -0.5 if standardized_logit_scale is None else float(standardized_logit_scale)
    return RouteVariant(flags, float(silu_gain), scale)


def _variant_supported(r: int, m: int) -> None:
    if r % 128:
        raise NotImplementedError(f"route variants need a routing width divisible by 128, got {r}")
    if m % 128 or m > 2048:
        raise NotImplementedError(f"route variants need a dictionary size divisible by 128 and <= 2048, got {m}")


class _RouteVariantFn(torch.autograd.Function):
    """A route variant over ``groups`` column blocks of a [rows, cols] matrix.

    Per group: S = q.Dk on the tcgen05 GEMM, the variant's row stage
    (da_route_var_weights), r = W.Dv^T on the GEMM, the output normalisation;
    backward the same products in reverse (da_route_var_* row stages around
    da_gemm / da_gemm_splitk)."""

    @staticmethod
    def forward(ctx, q: Tensor, key: Tensor, key_t: Tensor, value: Tensor, value_t: Tensor,  # type: ignore[override]
                key_anchor: Tensor, value_anchor: Tensor, beta: Tensor, rows: int, groups: int, col_stride: int,
                eps: float, normalize_input: bool, normalize_output: bool, variant: RouteVariant):
        m, r = key_t.shape
        _variant_supported(r, m)
        dev, dt = q.device, dtype_code(q.dtype)
        flags = variant.flags | (ROUTE_NORM_INPUT if normalize_input else 0)
        z = torch.empty(groups, rows, r, dtype=q.dtype, device=dev)
        onorm = torch.empty(groups, rows, dtype=torch.float32, device=dev)
        stats = torch.empty(groups, rows, 4, dtype=torch.float32, device=dev)
        s_buf = torch.empty(rows, m, dtype=torch.float32, device=dev)
        w_buf = torch.empty(rows, m, dtype=torch.bfloat16, device=dev)
        r_buf = torch.empty(rows, r, dtype=torch.float32, device=dev)
        beta32 = beta.detach().float().reshape(1).contiguous()
        st = stream_ptr(dev)
        for g in range(groups):
            qg = q[:, g * col_stride:]
            gemm(qg, False, key_t, False, rows, m, r, s_buf)  # S = q . Dk
            call("da_route_var_weights", s_buf.data_ptr(), rows, m, qg.data_ptr(), q.stride(0), r, dt, flags,
                 variant.silu_gain, variant.std_scale, beta32.data_ptr(), eps, w_buf.data_ptr(), stats[g].data_ptr(),
                 st)
            gemm(w_buf, False, value, False, rows, r, m, r_buf)  # r = W . Dv^T
            call("da_route_var_output", r_buf.data_ptr(), rows, r, dt, int(normalize_output), eps, z[g].data_ptr(),
                 onorm[g].data_ptr(), st)
        ctx.save_for_backward(q, key, key_t, value_t, beta32, z, onorm, stats)
        ctx.meta = (rows, groups, col_stride, eps, normalize_input, normalize_output, flags, variant,
                    key_anchor.dtype, value_anchor.dtype, beta.shape, beta.dtype)
        return z

    @staticmethod
    def backward(ctx, dz: Tensor):  # type: ignore[override]
        q, key, key_t, value_t, beta32, z, onorm, stats = ctx.saved_tensors
        (rows, groups, col_stride, eps, ni, no, flags, variant, key_dtype, value_dtype, beta_shape,
         beta_dtype) = ctx.meta
        need = ctx.needs_input_grad
        m, r = key_t.shape
        dev, dt = q.device, dtype_code(q.dtype)
        st = stream_ptr(dev)
        dz = dz.to(z.dtype).contiguous()
        full = groups * col_stride == q.shape[1] and col_stride == r and q.stride(0) == q.shape[1]
        dq = torch.empty_like(q) if full else torch.zeros_like(q)
        softmax = not flags & ROUTE_DIRECT_SILU
        dbeta = torch.zeros(1, dtype=torch.float32, device=dev) if need[7] and softmax else None
        d_key = torch.zeros(r, m, dtype=torch.float32, device=dev) if need[5] else None
        d_value = torch.zeros(r, m, dtype=torch.float32, device=dev) if need[6] else None
        g_buf = torch.empty(rows, r, dtype=torch.bfloat16, device=dev)
        delta = torch.empty(rows, dtype=torch.float32, device=dev)
        s_buf = torch.empty(rows, m, dtype=torch.float32, device=dev)
        dw_buf = torch.empty(rows, m, dtype=torch.float32, device=dev)
        ds_buf = torch.empty(rows, m, dtype=q.dtype, device=dev)
        w_buf = torch.empty(rows, m, dtype=torch.bfloat16, device=dev)
        u_buf = torch.empty(rows, r, dtype=torch.float32, device=dev)
        dbeta_work = torch.empty((rows + 7) // 8, dtype=torch.float32, device=dev)  # per-8-row dbeta partials
        for g in range(groups):
            qg = q[:, g * col_stride:]
            call("da_route_var_output_bwd", z[g].data_ptr(), dz[g].data_ptr(), onorm[g].data_ptr(), rows, r, dt,
                 int(no), eps, g_buf.data_ptr(), delta.data_ptr(), st)
            gemm(qg, False, key_t, False, rows, m, r, s_buf)  # S = q . Dk again
            gemm(g_buf, False, value_t, False, rows, m, r, dw_buf)  # dW = g . Dv
            call("da_route_var_weights_bwd", s_buf.data_ptr(), dw_buf.data_ptr(), rows, m, stats[g].data_ptr(),
                 delta.data_ptr(), flags, variant.silu_gain, variant.std_scale, beta32.data_ptr(), dt, ds_buf.data_ptr(),
                 w_buf.data_ptr(), ptr(dbeta), dbeta_work.data_ptr(), dbeta_work.numel(), st)
            if need[0]:
                gemm(ds_buf, False, key, False, rows, r, m, u_buf)  # u = dS . Dk^T
                call("da_route_var_input_bwd", u_buf.data_ptr(), qg.data_ptr(), q.stride(0), stats[g].data_ptr(),
                     rows, r, dt, int(ni), eps, dq[:, g * col_stride:].data_ptr(), dq.stride(0), st)
            if d_key is not None:  # dDk += q_g^T dS_g
                gemm_splitk(qg, q.stride(0), True, ds_buf, m, True, r, m, rows, d_key)
            if d_value is not None:  # dDv += g_g^T W_g
                gemm_splitk(g_buf, r, True, w_buf, m, True, r, m, rows, d_value)
        return (dq if need[0] else None, None, None, None, None,
                None if d_key is None else d_key.to(key_dtype),
                None if d_value is None else d_value.to(value_dtype),
                None if dbeta is None else dbeta.view(beta_shape).to(beta_dtype),
                None, None, None, None, None, None, None)


def _route_rows(q: Tensor, views: DictionaryViews, beta: Tensor, rows: int, groups: int, col_stride: int, eps: float,
                normalize_input: bool, normalize_output: bool, variant: RouteVariant | None) -> Tensor:
    if variant is None and not _grad_wanted(q, views.key_anchor, views.value_anchor, beta):
        return _route_forward(q, rows, groups, col_stride, views, beta, eps, normalize_input, normalize_output)[0]
    if variant is None:
        return _Route.apply(q, views.key, views.key_t, views.value, views.value_t, views.key_max, views.key_anchor,
                            views.value_anchor, beta, rows, groups, col_stride, eps, normalize_input,
                            normalize_output)
    return _RouteVariantFn.apply(q, views.key, views.key_t, views.value, views.value_t, views.key_anchor,
                                 views.value_anchor, beta, rows, groups, col_stride, eps, normalize_input,
                                 normalize_output, variant)


def route_projected(projected: Tensor, views: DictionaryViews, beta: Tensor, cfg, batch: int, length: int) -> Tensor:
    """Route the Q and K branches of a fused projection ``[B*T, 2*H*R]``.

    Returns ``[2, H, B, T, R]`` (index 0: routed queries, 1: routed keys);
    the concatenation of modules.py:239 is only an index mapping here.
    """
    h, r = cfg.qk_branches, cfg.routing_dim
    variant = route_variant(cfg.dictionary_activation, cfg.dictionary_assignment, cfg.dictionary_silu_gain,
                            cfg.standardize_dictionary_logits, cfg.standardized_logit_scale, r)
    z = _route_rows(projected, views, beta, batch * length, 2 * h, r, cfg.eps, cfg.normalize_routing_input,
                    cfg.normalize_routing_output, variant)
    return z.view(2, h, batch, length, r)


def dictionary_route(
    input: Tensor,
    dictionary_key: Tensor,
    dictionary_value: Tensor,
    beta: Tensor,
    eps: float = 1e-6,
    silu_logits: bool = False,
    direct_silu: bool = False,
    silu_gain: float = 1.0,
    standardize_logits: bool = False,
    standardized_logit_scale: float | None = None,
    normalize_input: bool = True,
    normalize_output: bool = True,
) -> Tensor:
    """B200 counterpart of ``dictionary_route_triton`` (triton_kernels.py:1984-2019).

    ``input`` [..., R]; ``dictionary_key``/``dictionary_value`` [R, M]
    (already column-normalised, same fp16/bf16 dtype as ``input``).
    """
    _check_half_cuda("dictionary route", input, dictionary_key, dictionary_value)
    r = input.shape[-1]
    variant = route_variant("silu" if silu_logits else "identity", "silu" if direct_silu else "softmax", silu_gain,
                            standardize_logits, standardized_logit_scale, r)
    if dictionary_key.shape[0] != r or dictionary_value.shape != dictionary_key.shape:
        raise ValueError("dictionaries must be [routing_dim, M] matching the input")
    shape = input.shape
    flat = input.contiguous().view(-1, r)
    views = dictionary_views_from_normalized(dictionary_key, dictionary_value, input.dtype)
    if not torch.is_tensor(beta):
        beta = torch.tensor(float(beta), device=input.device)
    z = _route_rows(flat, views, beta, flat.shape[0], 1, r, eps, normalize_input, normalize_output, variant)
    return z.view(shape)


# ----------------------------------------------------------------------------- outer attention
MAX_MAPS = 4


@dataclass
class RowMap:
    """Rows of a [rows, R] matrix: row(b, branch, t) = base + b*sb + branch*sbr + t."""

    tensor: Tensor
    base: int
    sb: int
    sbr: int

    @property
    def rows(self) -> int:
        return self.tensor.shape[0]


def _attention_supported(r: int, d: int, maps: int, group: int) -> None:
    if r % 64:
        raise NotImplementedError(f"outer attention kernels need a routing width divisible by 64, got {r}")
    if d not in (128, 256, 512):
        raise NotImplementedError(f"outer attention kernels support value widths 128/256/512, got {d}")
    if maps > MAX_MAPS or maps * group * r > 512:
        raise NotImplementedError(
            f"outer attention kernels support up to {MAX_MAPS} maps and maps*group*R <= 512 "
            f"(got maps={maps}, group={group}, R={r})"
        )


def _attention_forward(q: RowMap, k: RowMap, v: Tensor, batch: int, length: int, r: int, maps: int, group: int,
                       branch0: list[int], causal: bool, scales: Tensor, weights: Tensor | None,
                       key_norm_max: Tensor | None, key_norm_bound: float, out_dtype: torch.dtype):
    d = v.shape[-1]
    _attention_supported(r, d, maps, group)
    dev = v.device
    v16 = v.contiguous() if v.dtype == torch.bfloat16 else v.to(torch.bfloat16).contiguous()
    y = torch.empty(batch, length, d, dtype=out_dtype, device=dev)
    lse = torch.empty(batch, maps, length, dtype=torch.float32, device=dev)
    ws = workspace(dev)
    sc = scales.detach().float().contiguous()
    wt = None if weights is None else weights.detach().float().contiguous()
    kn = None if key_norm_max is None else key_norm_max.detach().float().contiguous()
    b0 = (ctypes_int_array(MAX_MAPS))(*(branch0 + [0] * (MAX_MAPS - len(branch0))))
    b0_addr = ctypes_addressof(b0)
    # several maps over few query tiles: the library splits every tile's key range over two CTA pairs and
    # asks for a workspace for the partial row sums and outputs
    ws_bytes = int(_lib.lib().da_attn_fwd_workspace_size(batch, length, maps, d)) if maps > 1 else 0
    if ws_bytes > 0:
        work = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        call("da_attn_fwd_ws", q.tensor.data_ptr(), q.rows, q.base, q.sb, q.sbr, k.tensor.data_ptr(), k.rows, k.base,
             k.sb, k.sbr, v16.data_ptr(), batch, length, r, d, maps, group, b0_addr, int(causal),
             dtype_code(q.tensor.dtype), sc.data_ptr(), ptr(wt), ptr(kn), float(key_norm_bound), y.data_ptr(),
             lse.data_ptr(), work.data_ptr(), ws_bytes, ws.status.data_ptr(), stream_ptr(dev))
        return y, lse
    call("da_attn_fwd", q.tensor.data_ptr(), q.rows, q.base, q.sb, q.sbr, k.tensor.data_ptr(), k.rows, k.base, k.sb,
         k.sbr, v16.data_ptr(), batch, length, r, d, maps, group, b0_addr, int(causal), dtype_code(q.tensor.dtype),
         sc.data_ptr(), ptr(wt), ptr(kn), float(key_norm_bound), y.data_ptr(), lse.data_ptr(), ws.status.data_ptr(),
         stream_ptr(dev))
    return y, lse


def _attention_bwd_supported(r: int, d: int, group: int) -> None:
    if d not in (256, 512) or group * r not in (128, 256, 512):
        raise NotImplementedError(
            "outer attention backward kernels support value widths 256/512 and group*R in 128/256/512 "
            f"(got D={d}, group={group}, R={r})"
        )


def _attention_delta(dy: Tensor, y: Tensor) -> Tensor:
    """delta[b*T + t] = <dY, Y> per row (fp32), Y the output of one map alone."""
    rows, d = dy.numel() // dy.shape[-1], dy.shape[-1]
    delta = torch.empty(rows, dtype=torch.float32, device=dy.device)
    call("da_attn_bwd_delta", dy.data_ptr(), y.data_ptr(), rows, d, dtype_code(dy.dtype), delta.data_ptr(),
         stream_ptr(dy.device))
    return delta


def _attention_backward(q: RowMap, k: RowMap, v: Tensor, dy: Tensor, batch: int, length: int, r: int, maps: int,
                        group: int, branch0: list[int], causal: bool, scales: Tensor, weights: Tensor | None,
                        lse: Tensor, delta: Tensor, delta_given: bool, dq: Tensor | None, dk: Tensor | None,
                        dv: Tensor | None, dscale: Tensor | None, dweight: Tensor | None,
                        overwrite: bool = False, split: bool = True) -> None:
    """All maps of one attention (da_attn_bwd_mixed): fp32 gradients accumulated in place, or with
    `overwrite` (maps on disjoint branches, da_attn_bwd_mixed_ow) every produced row of dq, dk and dv
    stored once in the input dtype.  `split=False` keeps the library's unsplit form at sizes where it
    would split every pair's long row over two CTA pairs."""
    d = v.shape[-1]
    _attention_bwd_supported(r, d, group)
    if maps * group * r > 512:
        raise NotImplementedError(f"outer attention backward supports maps*group*R <= 512, got {maps * group * r}")
    dev = v.device
    ws = workspace(dev)
    b0 = (ctypes_int_array(MAX_MAPS))(*(branch0 + [0] * (MAX_MAPS - len(branch0))))
    # per-(CTA, warp) partial sums of d gamma / d alpha, added in a fixed order by the library; at small
    # batches with several maps also the split form's partial rows (every pair's long row over two CTA
    # pairs, the shares added in order by the library)
    part_bytes = int(_lib.lib().da_attn_bwd_workspace_size(batch, length, maps))
    if split:
        part_bytes = max(part_bytes, int(_lib.lib().da_attn_bwd_split_workspace_size(batch, length, r, d, maps, group)))
    part = torch.empty(part_bytes, dtype=torch.uint8, device=dev)

    entry = "da_attn_bwd_mixed_ow" if overwrite else "da_attn_bwd_mixed"

    def launch(dq_, dk_, dv_, dscale_, dweight_, given, stream) -> None:
        call(entry, q.tensor.data_ptr(), q.rows, q.base, q.sb, q.sbr, k.tensor.data_ptr(), k.rows,
             k.base, k.sb, k.sbr, v.data_ptr(), dy.data_ptr(), batch, length, r, d, maps, group, ctypes_addressof(b0),
             int(causal), dtype_code(q.tensor.dtype), scales.data_ptr(), ptr(weights), lse.data_ptr(),
             delta.data_ptr(), int(given), ptr(dq_), ptr(dk_), ptr(dv_), ptr(dscale_), ptr(dweight_),
             part.data_ptr(), part_bytes, ws.status.data_ptr(), stream)

    # Small batches (one kernel's CTAs, two per pair, fit on the SMs at once) leave most SMs idle in
    # each of the three kernels, so independent launches run side by side on two more streams (fork
    # and join on stream events, which graph capture keeps): dV, which reads neither delta nor anything
    # the others write, beside everything; without a given delta, the delta sweep runs alone first
    # (with d alpha), then the dK kernel on a side stream beside a single-sweep dQ launch that takes
    # the stored delta.  The library's status word stays this stream's.
    pairs = batch * ((length + 127) // 128)
    if dv is not None and (dq is not None or dk is not None) and 2 * pairs <= _sm_count(dev):
        main = torch.cuda.current_stream(dev)
        side_v, side_k = _side_streams_of(dev)
        side_v.wait_stream(main)
        launch(None, None, dv, None, None, True, side_v.cuda_stream)
        if not delta_given:
            launch(None, None, None, None, dweight, False, main.cuda_stream)  # delta (and d alpha) only
            dweight, delta_given = None, True
        if dk is not None and (dq is not None or dscale is not None):
            side_k.wait_stream(main)
            launch(None, dk, None, None, None, True, side_k.cuda_stream)
            launch(dq, None, None, dscale, dweight, delta_given, main.cuda_stream)
            main.wait_stream(side_k)
        else:
            launch(dq, dk, None, dscale, dweight, delta_given, main.cuda_stream)
        main.wait_stream(side_v)
        return
    launch(dq, dk, dv, dscale, dweight, delta_given, stream_ptr(dev))


_side_streams: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream]] = {}
_sm_counts: dict[int, int] = {}


def _side_streams_of(dev: torch.device) -> tuple[torch.cuda.Stream, torch.cuda.Stream]:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    st = _side_streams.get(idx)
    if st is None:
        d = torch.device("cuda", idx)
        st = _side_streams.setdefault(idx, (torch.cuda.Stream(d), torch.cuda.Stream(d)))
    return st


def _sm_count(dev: torch.device) -> int:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    n = _sm_counts.get(idx)
    if n is None:
        n = _sm_counts.setdefault(idx, torch.cuda.get_device_properties(idx).multi_processor_count)
    return n


def ctypes_int_array(n: int):
    import ctypes

    return ctypes.c_int * n


def ctypes_addressof(obj) -> int:
    import ctypes

    return ctypes.addressof(obj)


def _map_layout(h: int, s: int) -> tuple[int, list[int]]:
    """Branches per map and first branch of each map (ops.py:96-139)."""
    if h >= s:
        group = h // s
        return group, [i * group for i in range(s)]
    rep = s // h
    return 1, [i // rep for i in range(s)]


class _MixedAttention(torch.autograd.Function):
    """Y = sum_s alpha_s softmax_causal(gamma_s Q_s K_s^T) V for routed [2,H,B,T,R]."""

    @staticmethod
    def forward(ctx, routed: Tensor, value: Tensor, scales: Tensor, weights: Tensor | None, maps: int,  # type: ignore[override]
                causal: bool, key_norm_bound: float):
        _two, h, batch, length, r = routed.shape
        flat = routed.view(-1, r)
        group, branch0 = _map_layout(h, maps)
        qmap = RowMap(flat, 0, length, batch * length)
        kmap = RowMap(flat, h * batch * length, length, batch * length)
        y, lse = _attention_forward(qmap, kmap, value, batch, length, r, maps, group, branch0, causal, scales,
                                    weights if maps > 1 else None, None, key_norm_bound, routed.dtype)
        ctx.save_for_backward(routed, value, scales, weights if weights is not None else scales, y, lse)
        ctx.meta = (maps, causal, key_norm_bound, weights is not None)
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        routed, value, scales, weights, y, lse = ctx.saved_tensors
        maps, causal, key_norm_bound, has_weights = ctx.meta
        _two, h, batch, length, r = routed.shape
        dtype, d = routed.dtype, value.shape[-1]
        flat = routed.view(-1, r)
        group, branch0 = _map_layout(h, maps)
        qmap = RowMap(flat, 0, length, batch * length)
        kmap = RowMap(flat, h * batch * length, length, batch * length)
        v16 = value.detach().to(dtype).contiguous()
        dy16 = dy.to(dtype).contiguous()
        need = ctx.needs_input_grad
        # maps on disjoint branches (H >= S): every routed and value row has one writer, which stores its
        # gradient in the input dtype -- no zero-filled fp32 buffers, no casts afterwards
        overwrite = h >= maps
        gdt = dtype if overwrite else torch.float32
        alloc = torch.empty if overwrite else torch.zeros
        droute = alloc(flat.shape, dtype=gdt, device=flat.device) if need[0] else None
        dv = alloc(batch * length, d, dtype=gdt, device=flat.device) if need[1] else None
        # (with overwrite the library also stores d gamma and d alpha once instead of adding to them)
        dscale = alloc(maps, dtype=torch.float32, device=flat.device)
        sc = scales.detach().float().contiguous()
        wt = weights.detach().float().contiguous() if has_weights and maps > 1 else None
        dweight = alloc(maps, dtype=torch.float32, device=flat.device) if wt is not None else None
        if maps == 1:  # delta from the saved output
            delta, given = _attention_delta(dy16, y).view(batch, 1, length), True
        else:  # computed exactly by the kernel's first sweep (the per-map outputs are never stored)
            delta, given = torch.empty(batch, maps, length, dtype=torch.float32, device=flat.device), False
        _attention_backward(qmap, kmap, v16, dy16, batch, length, r, maps, group, branch0, causal, sc, wt,
                            lse.contiguous(), delta, given, droute, droute, dv, dscale if need[2] else None, dweight,
                            overwrite=overwrite)
        g_routed = droute.view(routed.shape).to(dtype) if droute is not None else None
        g_value = dv.view(value.shape).to(value.dtype) if dv is not None else None
        g_scales = dscale.to(scales.dtype) if need[2] else None
        g_weights = dweight.to(weights.dtype) if (dweight is not None and need[3]) else None
        return g_routed, g_value, g_scales, g_weights, None, None, None


def routed_attention_mixed(routed: Tensor, value: Tensor, scales: Tensor, map_weights: Tensor | None, cfg) -> Tensor:
    """Module path: mixed outer attention over the routed [2, H, B, T, R] tensor."""
    maps = cfg.outer_maps
    # Routed vectors have norm <= 1 (normalised outputs, or convex combinations
    # of unit dictionary atoms), which bounds every score by gamma_s.
    if not _grad_wanted(routed, value, scales, map_weights):
        _two, h, batch, length, r = routed.shape
        flat = routed.view(-1, r)
        group, branch0 = _map_layout(h, maps)
        y, _lse = _attention_forward(RowMap(flat, 0, length, batch * length),
                                     RowMap(flat, h * batch * length, length, batch * length), value, batch, length,
                                     r, maps, group, branch0, cfg.causal, scales,
                                     map_weights if maps > 1 else None, None, 1.0, routed.dtype)
        return y
    return _MixedAttention.apply(routed, value, scales, map_weights, maps, cfg.causal, 1.0)


def routed_attention_maps(routed: Tensor, value: Tensor, scales: Tensor, cfg) -> Tensor:
    """Per-map outputs [B, S, T, D] (map_combine='concat'): one launch per map."""
    outs = []
    for s in range(cfg.outer_maps):
        outs.append(_SingleMapAttention.apply(routed, value, scales, s, cfg.outer_maps, cfg.causal))
    return torch.stack(outs, dim=1)


class _SingleMapAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, routed: Tensor, value: Tensor, scales: Tensor, s: int, maps: int, causal: bool):  # type: ignore[override]
        _two, h, batch, length, r = routed.shape
        flat = routed.view(-1, r)
        group, branch0 = _map_layout(h, maps)
        qmap = RowMap(flat, 0, length, batch * length)
        kmap = RowMap(flat, h * batch * length, length, batch * length)
        y, lse = _attention_forward(qmap, kmap, value, batch, length, r, 1, group, [branch0[s]], causal,
                                    scales[s:s + 1], None, None, 1.0, routed.dtype)
        ctx.save_for_backward(routed, value, scales, y, lse)
        ctx.meta = (s, maps, causal)
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        routed, value, scales, y, lse = ctx.saved_tensors
        s, maps, causal = ctx.meta
        _two, h, batch, length, r = routed.shape
        dtype, d = routed.dtype, value.shape[-1]
        flat = routed.view(-1, r)
        group, branch0 = _map_layout(h, maps)
        qmap = RowMap(flat, 0, length, batch * length)
        kmap = RowMap(flat, h * batch * length, length, batch * length)
        v16 = value.detach().to(dtype).contiguous()
        dy16 = dy.to(dtype).contiguous()
        need = ctx.needs_input_grad
        droute = torch.zeros(flat.shape, dtype=torch.float32, device=flat.device) if need[0] else None
        dv = torch.zeros(batch * length, d, dtype=torch.float32, device=flat.device) if need[1] else None
        dscale = torch.zeros(scales.shape[0], dtype=torch.float32, device=flat.device)
        delta = _attention_delta(dy16, y).view(batch, 1, length)
        _attention_backward(qmap, kmap, v16, dy16, batch, length, r, 1, group, [branch0[s]], causal,
                            scales.detach().float()[s:s + 1].contiguous(), None, lse.contiguous(), delta, True,
                            droute, droute, dv, dscale[s:s + 1] if need[2] else None, None)
        return (droute.view(routed.shape).to(dtype) if droute is not None else None,
                dv.view(value.shape).to(value.dtype) if dv is not None else None,
                dscale.to(scales.dtype) if need[2] else None, None, None, None)


class _PerMapAttention(torch.autograd.Function):
    """Op-level routed attention: [B, S, T, R] query/key -> [B, S, T, D]."""

    @staticmethod
    def forward(ctx, query: Tensor, key: Tensor, value: Tensor, scales: Tensor, causal: bool):  # type: ignore[override]
        batch, maps, length, r = query.shape
        qf = query.contiguous().view(-1, r)
        kf = key.contiguous().view(-1, r)
        kmax = key.detach().float().norm(dim=-1).amax(dim=-1).contiguous()  # [B, S] score bound
        outs, lses = [], []
        qmap = RowMap(qf, 0, maps * length, length)
        kmap = RowMap(kf, 0, maps * length, length)
        for s in range(maps):
            y, lse = _attention_forward(qmap, kmap, value, batch, length, r, 1, 1, [s], causal, scales[s:s + 1],
                                        None, kmax[:, s].contiguous(), 1.0, query.dtype)
            outs.append(y)
            lses.append(lse[:, 0])
        out = torch.stack(outs, dim=1)
        ctx.save_for_backward(qf, kf, value, scales, out, torch.stack(lses, dim=0))
        ctx.meta = (batch, maps, length, r, causal)
        return out

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        qf, kf, value, scales, out, lses = ctx.saved_tensors
        batch, maps, length, r, causal = ctx.meta
        dtype, d = qf.dtype, value.shape[-1]
        qmap = RowMap(qf, 0, maps * length, length)
        kmap = RowMap(kf, 0, maps * length, length)
        v16 = value.detach().to(dtype).contiguous()
        need = ctx.needs_input_grad
        dq = torch.zeros(qf.shape, dtype=torch.float32, device=qf.device) if need[0] else None
        dk = torch.zeros(kf.shape, dtype=torch.float32, device=qf.device) if need[1] else None
        dv = torch.zeros(batch * length, d, dtype=torch.float32, device=qf.device) if need[2] else None
        dscale = torch.zeros(maps, dtype=torch.float32, device=qf.device)
        sc = scales.detach().float().contiguous()
        for s in range(maps):
            dy_s = dy[:, s].to(dtype).contiguous()
            delta = _attention_delta(dy_s, out[:, s].contiguous()).view(batch, 1, length)
            _attention_backward(qmap, kmap, v16, dy_s, batch, length, r, 1, 1, [s], causal, sc[s:s + 1], None,
                                lses[s].contiguous().view(batch, 1, length), delta, True, dq, dk, dv,
                                dscale[s:s + 1] if need[3] else None, None)
        shape = (batch, maps, length, r)
        return (dq.view(shape).to(dtype) if dq is not None else None,
                dk.view(shape).to(dtype) if dk is not None else None,
                dv.view(value.shape).to(value.dtype) if dv is not None else None,
                dscale.to(scales.dtype) if need[3] else None, None)


def routed_attention(query: Tensor, key: Tensor, value: Tensor, scales: Tensor, causal: bool = True) -> Tensor:
    """B200 counterpart of ``routed_attention_triton`` (triton_kernels.py:2290-2305).

    ``query``/``key`` [B, S, T, R], ``value`` [B, T, D] (one fp16/bf16 dtype),
    ``scales`` [S]; returns [B, S, T, D].
    """
    if query.ndim != 4 or key.shape != query.shape:
        raise ValueError("query and key must have matching [B, S, T, R] shapes")
    if value.ndim != 3 or value.shape[:2] != (query.shape[0], query.shape[2]):
        raise ValueError("value must have shape [B, T, D] matching query")
    if scales.shape != (query.shape[1],):
        raise ValueError(f"scales must have shape [{query.shape[1]}]")
    _check_half_cuda("routed attention", query, key, value)
    return _PerMapAttention.apply(query, key, value, scales, causal)


# ----------------------------------------------------------------------------- projection GEMM
def gemm(a: Tensor, a_mn: bool, b: Tensor, b_mn: bool, m: int, n: int, k: int, out: Tensor,
         accumulate: bool = False) -> Tensor:
    """out[m, n] (+)= sum_k A(m, k) B(n, k) on the tcgen05 GEMM (see da_gemm)."""
    if a.dtype != b.dtype or a.dtype not in _HALF:
        raise ValueError("gemm operands must share one fp16/bf16 dtype")
    if a.stride(-1) != 1 or b.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("gemm operands must be row-major")
    ws = workspace(a.device)
    call("da_gemm", a.data_ptr(), a.stride(0), int(a_mn), b.data_ptr(), b.stride(0), int(b_mn), out.data_ptr(),
         out.stride(0), m, n, k, dtype_code(a.dtype), int(out.dtype == torch.float32), int(accumulate),
         ws.status.data_ptr(), stream_ptr(a.device))
    return out


def gemm_ex(a: Tensor, b: Tensor, b_mn: bool, out: Tensor, a2: Tensor | None = None, b2: Tensor | None = None,
            bias: Tensor | None = None, act: int = 0, aux: Tensor | None = None) -> Tensor:
    """out [M, N] = act(A . B^T [+ A2 . B2^T] + bias) in the operand dtype (see da_gemm_ex): A [M, K] row-major;
    B [N, K], or [K, N] with ``b_mn``; act 0 none, 1 GELU (pre-activation into ``aux`` when given), 2 times
    GELU'(aux)."""
    m, k = a.shape
    n = out.shape[1]
    k2 = 0 if a2 is None else a2.shape[1]
    for t in (a, b, out, a2, b2, bias, aux):
        if t is not None and (t.dtype != a.dtype or t.stride(-1) != 1):
            raise ValueError("gemm_ex tensors must be row-major and share the operand dtype")
    call("da_gemm_ex", a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), int(b_mn), k, ptr(a2),
         0 if a2 is None else a2.stride(0), ptr(b2), 0 if b2 is None else b2.stride(0), k2, out.data_ptr(),
         out.stride(0), m, n, dtype_code(a.dtype), ptr(bias), act, ptr(aux), 0 if aux is None else aux.stride(0),
         workspace(a.device).status.data_ptr(), stream_ptr(a.device))
    return out


def _bias_grad(d: Tensor) -> Tensor:
    """Column sums of a [rows, N] bf16/fp16 gradient in fp32 (the bias gradient of a Linear), one
    HBM pass whose partial sums are added in a fixed order (da_col_sum)."""
    d = d.reshape(-1, d.shape[-1])
    if d.stride(-1) != 1:
        d = d.contiguous()
    rows, cols = d.shape
    elems = int(_lib.lib().da_col_sum_workspace_elems(rows, cols))
    work = torch.empty(max(elems, 4), dtype=torch.float32, device=d.device)
    out = torch.empty(cols, dtype=torch.float32, device=d.device)
    call("da_col_sum", d.data_ptr(), rows, cols, d.stride(0), dtype_code(d.dtype), out.data_ptr(), work.data_ptr(),
         work.numel(), stream_ptr(d.device))
    return out


class _Linear(torch.autograd.Function):
    """y [M, N] = x [M, K] . W[N, K]^T (+ b) on the tcgen05 GEMM, in the compute dtype: the output projection
    of SharedDictionaryAttention (modules.py:272) and any Linear of the block."""

    @staticmethod
    def forward(ctx, x2d: Tensor, weight: Tensor, bias: Tensor | None, dtype: torch.dtype):  # type: ignore[override]
        w = weight.to(dtype)
        b = None if bias is None else bias.to(dtype)
        out = torch.empty(x2d.shape[0], w.shape[0], dtype=dtype, device=x2d.device)
        gemm_ex(x2d, w, False, out, bias=b)
        ctx.save_for_backward(x2d, w)
        ctx.param_dtypes = (weight.dtype, None if bias is None else bias.dtype)
        return out

    @staticmethod
    def backward(ctx, dout: Tensor):  # type: ignore[override]
        x2d, w = ctx.saved_tensors
        need = ctx.needs_input_grad
        dout = dout.to(w.dtype).contiguous()
        m, k = x2d.shape
        n = w.shape[0]
        dx = dw = db = None
        if need[0]:
            dx = torch.empty(m, k, dtype=w.dtype, device=x2d.device)
            gemm_ex(dout, w, True, dx)  # dX = dY . W
        if need[1]:
            dw = weight_grad(dout, x2d, n, k, m, ctx.param_dtypes[0])  # dW = dY^T . X
        if need[2]:
            db = _bias_grad(dout).to(ctx.param_dtypes[1])
        return dx, dw, db, None


def _linear_dtype(x: Tensor) -> torch.dtype:
    return torch.get_autocast_dtype("cuda") if torch.is_autocast_enabled("cuda") else x.dtype


# The block's plain Linear layers (SharedDictionaryAttention's output projection, modules.py:272, and the
# feed-forward branch of the block, modules.py:339-346) lie outside the routed-attention path.  PyTorch's
# cuBLAS runs them faster on B200 than this library's persistent GEMM does, even with GELU fused into the
# latter's epilogues (LM training step, a1, 6 layers, B256 T1024: 89.7 ms against 96.2 ms per step), so
# the modules call F.linear / nn.GELU for them by default, as the reference does; True routes them
# through ops.linear / ops.feedforward on the tcgen05 GEMM.
BLOCK_LINEAR_ON_TCGEN05 = False


def linear_supported(x: Tensor, layer: torch.nn.Linear) -> bool:
    """Whether the tcgen05 GEMM covers ``layer(x)``: CUDA, half-precision compute (autocast, or x and the
    weight in one half dtype, as F.linear requires), widths multiples of 128 (out) and 8 (in)."""
    dtype = _linear_dtype(x)
    return (x.is_cuda and x.numel() > 0 and dtype in _HALF and layer.out_features % 128 == 0
            and layer.in_features % 8 == 0
            and (torch.is_autocast_enabled("cuda") or layer.weight.dtype == dtype))


def linear(x: Tensor, layer: torch.nn.Linear) -> Tensor:
    """``layer(x)`` on the tcgen05 GEMM, with F.linear's autocast behaviour (operands and output in the
    autocast dtype under autocast, else in x's dtype)."""
    dtype = _linear_dtype(x)
    x2d = x.reshape(-1, x.shape[-1]).to(dtype)
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    out = _Linear.apply(x2d, layer.weight, layer.bias, dtype)
    return out.view(*x.shape[:-1], out.shape[-1])


class _FeedForward(torch.autograd.Function):
    """Linear -> GELU -> Linear (modules.py:339-346, the block's feed-forward branch) on the tcgen05 GEMM:
    the first product's epilogue adds its bias, applies GELU and keeps the pre-activation; the backward's
    first product (dOut . W2) multiplies by GELU'(pre-activation) in its epilogue, so no separate GELU
    pass runs in either direction."""

    @staticmethod
    def forward(ctx, x2d: Tensor, w1: Tensor, b1: Tensor | None, w2: Tensor, b2: Tensor | None,  # type: ignore[override]
                dtype: torch.dtype):
        m = x2d.shape[0]
        w1c, w2c = w1.to(dtype), w2.to(dtype)
        b1c = None if b1 is None else b1.to(dtype)
        b2c = None if b2 is None else b2.to(dtype)
        hidden = w1c.shape[0]
        z = torch.empty(m, hidden, dtype=dtype, device=x2d.device)
        h = torch.empty(m, hidden, dtype=dtype, device=x2d.device)
        gemm_ex(x2d, w1c, False, h, bias=b1c, act=1, aux=z)  # h = GELU(x W1^T + b1), z kept
        out = torch.empty(m, w2c.shape[0], dtype=dtype, device=x2d.device)
        gemm_ex(h, w2c, False, out, bias=b2c)
        ctx.save_for_backward(x2d, w1c, w2c, z, h)
        ctx.param_dtypes = (w1.dtype, None if b1 is None else b1.dtype, w2.dtype, None if b2 is None else b2.dtype)
        return out

    @staticmethod
    def backward(ctx, dout: Tensor):  # type: ignore[override]
        x2d, w1c, w2c, z, h = ctx.saved_tensors
        need = ctx.needs_input_grad
        dt = w1c.dtype
        dout = dout.to(dt).contiguous()
        m, k = x2d.shape
        hidden, n = w1c.shape[0], w2c.shape[0]
        pd = ctx.param_dtypes
        dx = dw1 = db1 = dw2 = db2 = None
        if need[3]:
            dw2 = weight_grad(dout, h, n, hidden, m, pd[2])  # dW2 = dOut^T . h
        if need[4]:
            db2 = _bias_grad(dout).to(pd[3])
        dz = torch.empty(m, hidden, dtype=dt, device=x2d.device)
        gemm_ex(dout, w2c, True, dz, act=2, aux=z)  # dZ = (dOut . W2) * GELU'(z)
        if need[1]:
            dw1 = weight_grad(dz, x2d, hidden, k, m, pd[0])  # dW1 = dZ^T . x
        if need[2]:
            db1 = _bias_grad(dz).to(pd[1])
        if need[0]:
            dx = torch.empty(m, k, dtype=dt, device=x2d.device)
            gemm_ex(dz, w1c, True, dx)  # dX = dZ . W1
        return dx, dw1, db1, dw2, db2, None


def feedforward_supported(x: Tensor, first: torch.nn.Linear, second: torch.nn.Linear) -> bool:
    return linear_supported(x, first) and linear_supported(x, second) and first.out_features == second.in_features


def feedforward(x: Tensor, first: torch.nn.Linear, second: torch.nn.Linear) -> Tensor:
    """``second(GELU(first(x)))`` (F.linear autocast behaviour) on the tcgen05 GEMM with fused GELU."""
    dtype = _linear_dtype(x)
    x2d = x.reshape(-1, x.shape[-1]).to(dtype)
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    out = _FeedForward.apply(x2d, first.weight, first.bias, second.weight, second.bias, dtype)
    return out.view(*x.shape[:-1], out.shape[-1])


class _Projection(torch.autograd.Function):
    """[B*T, N] = x [B*T, K] . W[N, K]^T  (the fused Q/K projection)."""

    @staticmethod
    def forward(ctx, x2d: Tensor, weight: Tensor):  # type: ignore[override]
        m, k = x2d.shape
        n = weight.shape[0]
        out = torch.empty(m, n, dtype=x2d.dtype, device=x2d.device)
        gemm(x2d, False, weight, False, m, n, k, out)
        ctx.save_for_backward(x2d, weight)
        return out

    @staticmethod
    def backward(ctx, dout: Tensor):  # type: ignore[override]
        x2d, weight = ctx.saved_tensors
        dout = dout.contiguous()
        m, k = x2d.shape
        n = weight.shape[0]
        dx = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(m, k, dtype=x2d.dtype, device=x2d.device)
            gemm(dout, False, weight, True, m, k, n, dx)          # dX = dC . W
        if ctx.needs_input_grad[1]:
            dw = weight_grad(dout, x2d, n, k, m, weight.dtype)  # dW = dC^T . X, rows split
        return dx, dw


_PTR3 = ctypes.c_void_p * 3
_I64X3 = ctypes.c_int64 * 3
_I32X3 = ctypes.c_int * 3


def _qkv_forward(x2d: Tensor, wq: Tensor, wk: Tensor, wv: Tensor, bv: Tensor | None) -> tuple[Tensor, Tensor]:
    m, k = x2d.shape
    hr, d = wq.shape[0], wv.shape[0]
    dev = x2d.device
    proj = torch.empty(m, 2 * hr, dtype=x2d.dtype, device=dev)
    value = torch.empty(m, d, dtype=torch.bfloat16, device=dev)
    dt = dtype_code(x2d.dtype)
    call("da_gemm_segments", x2d.data_ptr(), x2d.stride(0), m, k, dt, 3,
         _PTR3(wq.data_ptr(), wk.data_ptr(), wv.data_ptr()), _I64X3(wq.stride(0), wk.stride(0), wv.stride(0)),
         _I64X3(hr, hr, d), _PTR3(proj.data_ptr(), proj.data_ptr() + hr * proj.element_size(), value.data_ptr()),
         _I64X3(2 * hr, 2 * hr, d), _I32X3(dt, dt, _lib.DA_BF16),
         _PTR3(None, None, None if bv is None else bv.data_ptr()), workspace(dev).status.data_ptr(),
         stream_ptr(dev))
    return proj, value


class _QKVProjection(torch.autograd.Function):
    """Q/K projection [B*T, 2*H*R] (compute dtype) and value projection [B*T, D] (bf16, + bias) of one
    input in one launch (modules.py:143-157 and the value Linear)."""

    @staticmethod
    def forward(ctx, x2d: Tensor, wq: Tensor, wk: Tensor, wv: Tensor, bv: Tensor | None):  # type: ignore[override]
        proj, value = _qkv_forward(x2d, wq, wk, wv, bv)
        ctx.save_for_backward(x2d, wq, wk, wv)
        ctx.has_bias = bv is not None
        return proj, value

    @staticmethod
    def backward(ctx, dproj: Tensor | None, dvalue: Tensor | None):  # type: ignore[override]
        x2d, wq, wk, wv = ctx.saved_tensors
        need = ctx.needs_input_grad
        m, k = x2d.shape
        hr = wq.shape[0]
        dt = x2d.dtype
        dx = dwq = dwk = dwv = dbv = None
        dv = None if dvalue is None else dvalue.to(dt).contiguous()
        if dproj is not None:
            dproj = dproj.to(dt).contiguous()
        if need[0]:  # dX = dC . [Wq; Wk] + dV . Wv in one launch (two K segments)
            dx = torch.empty(m, k, dtype=dt, device=x2d.device)
            if dproj is not None and dv is not None:
                gemm_ex(dproj, torch.cat((wq, wk), 0), True, dx, a2=dv, b2=wv)
            elif dproj is not None:
                gemm_ex(dproj, torch.cat((wq, wk), 0), True, dx)
            elif dv is not None:
                gemm_ex(dv, wv, True, dx)
            else:
                dx = None
        if dproj is not None and (need[1] or need[2]):
            # dW = dC^T . X (fp32): a [2HR, K] output of a few tiles over all B*T rows, so the row
            # dimension is split over CTAs (partial sums added in a fixed order)
            if wq.dtype == wk.dtype:  # one [2HR, K] gradient, its two row blocks handed out as views
                dw = weight_grad(dproj, x2d, 2 * hr, k, m, wq.dtype)
                dwq, dwk = dw[:hr], dw[hr:]
            else:
                dw = weight_grad(dproj, x2d, 2 * hr, k, m, torch.float32)
                dwq, dwk = dw[:hr].to(wq.dtype), dw[hr:].to(wk.dtype)
        if dv is not None:
            if need[3]:  # dWv = dV^T . X, rows split over CTAs as above
                dwv = weight_grad(dv, x2d, wv.shape[0], k, m, wv.dtype)
            if ctx.has_bias and need[4]:
                dbv = _bias_grad(dv).to(wv.dtype)
        return dx, dwq, dwk, dwv, dbv


def qkv_projection(x: Tensor, wq: Tensor, wk: Tensor, wv: Tensor, bv: Tensor | None) -> tuple[Tensor, Tensor]:
    """``x [B, T, K]`` -> projected ``[B*T, 2*H*R]`` (x's dtype) and value ``[B*T, D]`` (bf16)."""
    x2d = x.reshape(-1, x.shape[-1])
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    args = (x2d, wq.contiguous(), wk.contiguous(), wv.contiguous(), None if bv is None else bv.contiguous())
    if not _grad_wanted(*args):
        return _qkv_forward(*args)
    return _QKVProjection.apply(*args)


def qk_projection(x: Tensor, fused_weight: Tensor) -> Tensor:
    """Fused Q/K projection ``x [B, T, D] -> [B*T, 2*H*R]`` (modules.py:143-157)."""
    x2d = x.reshape(-1, x.shape[-1])
    if not x2d.is_contiguous():
        x2d = x2d.contiguous()
    return _Projection.apply(x2d, fused_weight.contiguous())


# ----------------------------------------------------------------------------- residual add + LayerNorm
# The glue around the block (modules.py:294-356, :415-460): ``x + branch`` on the fp32 residual
# stream followed by ``nn.LayerNorm``.  One kernel adds, normalises and writes the normalised rows
# directly in the dtype the next Linear reads (the autocast dtype under autocast, else x's dtype),
# so the reference's separate add, fp32 LayerNorm output and autocast cast become one pass; the
# backward adds the residual gradient and writes the branch gradient in the same pass.
LAYERNORM_WIDTHS = (256, 512, 768, 1024)


def layernorm_supported(x: Tensor, *norms) -> bool:
    """Whether the fused kernels cover ``norm(x)`` for every given ``nn.LayerNorm``."""
    if not (x.is_cuda and x.dtype == torch.float32 and x.numel() > 0 and x.shape[-1] in LAYERNORM_WIDTHS):
        return False  # (an empty batch keeps nn.LayerNorm's behaviour)
    for n in norms:
        if (n.weight is None or n.bias is None or n.weight.dtype != torch.float32
                or tuple(n.normalized_shape) != (x.shape[-1],)):
            return False
    return True


def _layernorm_out_dtype(x: Tensor) -> torch.dtype:
    if torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return x.dtype


def _ln_forward(x: Tensor, branch: Tensor | None, weight: Tensor, bias: Tensor, eps: float,
                out_dtype: torch.dtype) -> tuple[Tensor | None, Tensor, Tensor, Tensor]:
    d = x.shape[-1]
    rows = x.numel() // d
    x_out = torch.empty_like(x) if branch is not None else None
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    mean = torch.empty(rows, dtype=torch.float32, device=x.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    call("da_add_layernorm_fwd", x.data_ptr(), ptr(branch), dtype_code(branch.dtype) if branch is not None else 0,
         weight.data_ptr(), bias.data_ptr(), rows, d, float(eps), ptr(x_out), y.data_ptr(), dtype_code(out_dtype),
         mean.data_ptr(), rstd.data_ptr(), stream_ptr(x.device))
    return x_out, y, mean, rstd


def _ln_backward(ctx, d_res: Tensor | None, dy: Tensor | None):
    x_norm, mean, rstd, weight = ctx.saved_tensors
    need = ctx.needs_input_grad
    d = x_norm.shape[-1]
    rows = x_norm.numel() // d
    if dy is None:  # y unused downstream: the residual gradient passes through
        dx = d_res if d_res is not None else torch.zeros_like(x_norm)
        db = dx.to(ctx.branch_dtype) if ctx.has_branch and need[1] else None
        return dx, db, None, None
    dy = dy.contiguous()
    d_res = None if d_res is None else d_res.contiguous()
    dx = torch.empty_like(x_norm)
    db = torch.empty(x_norm.shape, dtype=ctx.branch_dtype, device=x_norm.device) if ctx.has_branch and need[1] else None
    blocks = int(_lib.lib().da_layernorm_bwd_blocks(rows))
    partial = torch.empty((blocks, 2, d), dtype=torch.float32, device=x_norm.device)
    wi = 2 if ctx.has_branch else 1
    dgamma = torch.empty(d, dtype=torch.float32, device=x_norm.device) if need[wi] else None
    dbeta = torch.empty(d, dtype=torch.float32, device=x_norm.device) if need[wi + 1] else None
    call("da_add_layernorm_bwd", dy.data_ptr(), dtype_code(dy.dtype), ptr(d_res), x_norm.data_ptr(), mean.data_ptr(),
         rstd.data_ptr(), weight.data_ptr(), rows, d, dx.data_ptr(), ptr(db),
         dtype_code(ctx.branch_dtype) if ctx.has_branch else 0, partial.data_ptr(), blocks, ptr(dgamma), ptr(dbeta),
         stream_ptr(x_norm.device))
    return dx, db, dgamma, dbeta


class _LayerNormCast(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps, out_dtype):
        _, y, mean, rstd = _ln_forward(x, None, weight, bias, eps, out_dtype)
        ctx.save_for_backward(x, mean, rstd, weight)
        ctx.has_branch, ctx.branch_dtype = False, None
        return y

    @staticmethod
    def backward(ctx, dy):
        dx, _, dgamma, dbeta = _ln_backward(ctx, None, dy)
        return dx, dgamma, dbeta, None, None


class _AddLayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, branch, weight, bias, eps, out_dtype):
        x_out, y, mean, rstd = _ln_forward(x, branch, weight, bias, eps, out_dtype)
        ctx.save_for_backward(x_out, mean, rstd, weight)
        ctx.has_branch, ctx.branch_dtype = True, branch.dtype
        return x_out, y

    @staticmethod
    def backward(ctx, d_xout, dy):
        dx, db, dgamma, dbeta = _ln_backward(ctx, d_xout, dy)
        return dx, db, dgamma, dbeta, None, None


def layernorm(x: Tensor, norm) -> Tensor:
    """``norm(x)`` for an ``nn.LayerNorm`` over the last dimension of fp32 ``x``, written in the dtype the
    next Linear reads (the autocast dtype under autocast)."""
    xc = x if x.is_contiguous() else x.contiguous()
    return _LayerNormCast.apply(xc, norm.weight, norm.bias, norm.eps, _layernorm_out_dtype(x))


def add_layernorm(x: Tensor, branch: Tensor, norm) -> tuple[Tensor, Tensor]:
    """``(x + branch, norm(x + branch))``: the residual update (fp32) and its normalised rows (in the
    dtype the next Linear reads)."""
    if branch.shape != x.shape:
        raise ValueError(f"branch shape {tuple(branch.shape)} does not match the residual {tuple(x.shape)}")
    xc = x if x.is_contiguous() else x.contiguous()
    bc = branch if branch.is_contiguous() else branch.contiguous()
    return _AddLayerNorm.apply(xc, bc, norm.weight, norm.bias, norm.eps, _layernorm_out_dtype(x))
