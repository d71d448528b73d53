"""Outer routed attention backward (per map, mixed maps, op level) against the oracle.

The oracle is the fp32 restatement of the reference's attention; its
gradients come from torch autograd on the dtype-rounded inputs.  Bar for every
gradient: cosine >= 0.9995 and max |g - g_ref| <= 2e-2 * max(1, max |g_ref|);
scalar gradients (scales, mix weights) within 2e-2 relative.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import oracle
from double_attention_b200 import ops

pytestmark = pytest.mark.gpu

MIN_COS = 0.9995
REL = 2e-2


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    return float(F.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


def _close(name: str, got: torch.Tensor, ref: torch.Tensor) -> None:
    got = got.float().cpu()
    bound = REL * max(1.0, ref.abs().max().item())
    err = (got - ref).abs().max().item()
    cos = _cos(got, ref)
    assert err <= bound and cos >= MIN_COS, f"{name}: max-abs {err:.3e} (bound {bound:.3e}), cosine {cos:.6f}"


def _scalar_close(name: str, got: torch.Tensor, ref: torch.Tensor) -> None:
    got = got.float().cpu()
    tol = REL * max(ref.abs().max().item(), 1e-3)
    assert (got - ref).abs().max().item() <= tol, f"{name}: {got.tolist()} vs {ref.tolist()}"


class _Cfg:
    def __init__(self, maps: int, causal: bool = True) -> None:
        self.outer_maps = maps
        self.causal = causal


def _inputs(h, maps, batch, length, r, d, scale0, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    routed = F.normalize(torch.randn(2, h, batch, length, r, generator=g), dim=-1).to(dtype)
    value = torch.randn(batch, length, d, generator=g).to(dtype)
    dy = torch.randn(batch, length, d, generator=g).to(dtype)
    log_scales = math.log(scale0) + torch.linspace(-0.05, 0.05, maps) if maps > 1 else torch.tensor([math.log(scale0)])
    scales = log_scales.exp()
    mix = torch.softmax(torch.randn(maps, generator=g), 0) if maps > 1 else None
    return routed, value, dy, scales, mix


def _oracle_grads(routed, value, dy, scales, mix, maps, causal):
    rq = routed.float().requires_grad_()
    val = value.float().requires_grad_()
    sc = scales.clone().requires_grad_()
    mx = None if mix is None else mix.clone().requires_grad_()
    zq, zk = rq[0].permute(1, 0, 2, 3), rq[1].permute(1, 0, 2, 3)
    sq, sk = oracle.assemble_score_maps(zq, zk, maps)
    per_map = oracle.routed_attention(sq, sk, val, sc, causal)
    out = per_map[:, 0] if mx is None else torch.einsum("s,bstd->btd", mx, per_map)
    out.backward(dy.float())
    return rq.grad, val.grad, sc.grad, None if mx is None else mx.grad


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(
    ("h", "maps", "batch", "length", "r", "d", "scale0", "causal"),
    [
        (1, 1, 2, 512, 256, 512, 16.0, True),     # a1 (one map, routing width 256)
        (4, 4, 2, 256, 128, 512, 16.0, True),     # qk4-s4 (four mixed maps, width 128)
        (2, 1, 2, 130, 128, 512, 16.0, True),     # two branches concatenated per map, ragged tail
        (1, 2, 2, 65, 256, 256, 16.0, True),      # one branch repeated over two maps, D=256
        (4, 4, 1, 257, 128, 256, 12.0, False),    # non-causal, ragged tail
        (1, 1, 1, 384, 512, 256, 512.0**0.5, True),  # routing width 512
    ],
)
def test_mixed_attention_backward(h, maps, batch, length, r, d, scale0, causal, dtype) -> None:
    dev = torch.device("cuda")
    routed, value, dy, scales, mix = _inputs(h, maps, batch, length, r, d, scale0, dtype, seed=length + maps + r)
    rd = routed.to(dev).requires_grad_()
    vd = value.to(dev).requires_grad_()
    sd = scales.to(dev).requires_grad_()
    md = None if mix is None else mix.to(dev).requires_grad_()
    y = ops.routed_attention_mixed(rd, vd, sd, md, _Cfg(maps, causal))
    y.backward(dy.to(dev))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0

    g_routed, g_value, g_scales, g_mix = _oracle_grads(routed, value, dy, scales, mix, maps, causal)
    _close("d routed", rd.grad, g_routed)
    _close("d value", vd.grad, g_value)
    _scalar_close("d scales", sd.grad, g_scales)
    if mix is not None:
        _scalar_close("d mix weights", md.grad, g_mix)


def test_concat_maps_backward() -> None:
    """map_combine='concat': one launch per map, gradients summed over maps."""
    dev = torch.device("cuda")
    dtype = torch.bfloat16
    h, maps, batch, length, r, d = 2, 2, 2, 200, 128, 256
    routed, value, dy, scales, _ = _inputs(h, maps, batch, length, r, d, 16.0, dtype, seed=11)
    g = torch.Generator().manual_seed(12)
    dyp = torch.randn(batch, maps, length, d, generator=g).to(dtype)
    rd = routed.to(dev).requires_grad_()
    vd = value.to(dev).requires_grad_()
    sd = scales.to(dev).requires_grad_()
    out = ops.routed_attention_maps(rd, vd, sd, _Cfg(maps))
    out.backward(dyp.to(dev))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0

    rq = routed.float().requires_grad_()
    val = value.float().requires_grad_()
    sc = scales.clone().requires_grad_()
    zq, zk = rq[0].permute(1, 0, 2, 3), rq[1].permute(1, 0, 2, 3)
    sq, sk = oracle.assemble_score_maps(zq, zk, maps)
    oracle.routed_attention(sq, sk, val, sc, True).backward(dyp.float())
    _close("d routed", rd.grad, rq.grad)
    _close("d value", vd.grad, val.grad)
    _scalar_close("d scales", sd.grad, sc.grad)


@pytest.mark.parametrize("causal", [True, False])
def test_op_level_routed_attention_backward(causal: bool) -> None:
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(5)
    batch, maps, length, r, d = 2, 3, 193, 128, 256
    q = F.normalize(torch.randn(batch, maps, length, r, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(batch, maps, length, r, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(batch, length, d, generator=g).to(torch.bfloat16)
    dy = torch.randn(batch, maps, length, d, generator=g).to(torch.bfloat16)
    scales = torch.tensor([8.0, 11.0, 16.0])
    qd, kd, vd = (t.to(dev).requires_grad_() for t in (q, k, v))
    sd = scales.to(dev).requires_grad_()
    ops.routed_attention(qd, kd, vd, sd, causal).backward(dy.to(dev))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0

    qr, kr, vr = (t.float().requires_grad_() for t in (q, k, v))
    sr = scales.clone().requires_grad_()
    oracle.routed_attention(qr, kr, vr, sr, causal).backward(dy.float())
    _close("d query", qd.grad, qr.grad)
    _close("d key", kd.grad, kr.grad)
    _close("d value", vd.grad, vr.grad)
    _scalar_close("d scales", sd.grad, sr.grad)


def test_backward_is_repeatable() -> None:
    """Two backward passes on the same inputs give bit-identical gradients, the score scales' and the
    map weights' (sums over every query row, added in a fixed order) included."""
    dev = torch.device("cuda")
    routed, value, dy, scales, mix = _inputs(4, 4, 3, 700, 128, 512, 16.0, torch.bfloat16, seed=3)
    grads = []
    for _ in range(2):
        rd = routed.to(dev).requires_grad_()
        vd = value.to(dev).requires_grad_()
        sd = scales.to(dev).requires_grad_()
        md = mix.to(dev).requires_grad_()
        ops.routed_attention_mixed(rd, vd, sd, md, _Cfg(4)).backward(dy.to(dev))
        grads.append((rd.grad.clone(), vd.grad.clone(), sd.grad.clone(), md.grad.clone()))
    torch.cuda.synchronize()
    for name, a, b in zip(("routed", "value", "scales", "map weights"), grads[0], grads[1]):
        assert torch.equal(a, b), f"d {name} differs between two identical backward passes"


@pytest.mark.parametrize("batch", [2, 32])
def test_overwrite_gradients_equal_the_accumulated_ones(batch: int) -> None:
    """da_attn_bwd_mixed_ow (maps on disjoint branches: each gradient row stored once in the input dtype)
    against da_attn_bwd_mixed into zeroed fp32 buffers then cast: the same fp32 values rounded once, so
    bit for bit equal -- at B2 T512 (the three-stream small-batch schedule) and B32 T512 (one stream)."""
    dev, dtype = torch.device("cuda"), torch.bfloat16
    h = maps = 4
    length, r, d = 512, 128, 512
    routed, value, dy, scales, mix = _inputs(h, maps, batch, length, r, d, 16.0, dtype, seed=5)
    routed, value, dy = routed.to(dev), value.to(dev).to(dtype), dy.to(dev).to(dtype)
    scales, mix = scales.to(dev).float(), mix.to(dev).float()
    flat = routed.view(-1, r)
    group, branch0 = ops._map_layout(h, maps)
    qmap = ops.RowMap(flat, 0, length, batch * length)
    kmap = ops.RowMap(flat, h * batch * length, length, batch * length)
    _y, lse = ops._attention_forward(qmap, kmap, value, batch, length, r, maps, group, branch0, True, scales, mix,
                                     None, 1.0, dtype)
    out = {}
    for overwrite in (False, True):
        gdt, alloc = (dtype, torch.empty) if overwrite else (torch.float32, torch.zeros)
        droute = alloc(flat.shape, dtype=gdt, device=dev)
        dv = alloc(batch * length, d, dtype=gdt, device=dev)
        # the overwrite entry stores d gamma and d alpha (=): NaN-filled outputs must come back finite
        fill = float("nan") if overwrite else 0.0
        dscale = torch.full((maps,), fill, dtype=torch.float32, device=dev)
        dweight = torch.full((maps,), fill, dtype=torch.float32, device=dev)
        delta = torch.empty(batch, maps, length, dtype=torch.float32, device=dev)
        ops._attention_backward(qmap, kmap, value, dy, batch, length, r, maps, group, branch0, True, scales, mix,
                                lse, delta, False, droute, droute, dv, dscale, dweight, overwrite=overwrite)
        out[overwrite] = (droute.to(dtype), dv.to(dtype), dscale, dweight)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    for name, a, b in zip(("routed", "value", "scales", "map weights"), out[False], out[True]):
        assert torch.equal(a, b), f"d {name}: overwrite and accumulate paths differ"


@pytest.mark.parametrize(("batch", "length", "causal"), [(2, 2048, True), (1, 640, True), (1, 640, False)])
def test_split_form_matches_the_unsplit_one(batch: int, length: int, causal: bool) -> None:
    """With several maps on disjoint branches and few query tiles the library splits every pair's long row
    over two CTA pairs (da_attn_bwd_split_workspace_size > 0) and adds the shares' fp32 partial rows in
    share order.  Against the unsplit form on the same inputs the gradients differ by fp32 reassociation
    only (a bf16 rounding step at most per element), the split form repeats bit for bit, and its delta
    is the unsplit sweep's.  B2 T2048 is the config-3 shape at eight GPUs; T640 has a ragged last tile
    and, causal, first query tiles whose second key share is empty."""
    dev, dtype = torch.device("cuda"), torch.bfloat16
    h = maps = 4
    r, d = 128, 512
    routed, value, dy, scales, mix = _inputs(h, maps, batch, length, r, d, 16.0, dtype, seed=9)
    routed, value, dy = routed.to(dev), value.to(dev).to(dtype), dy.to(dev).to(dtype)
    scales, mix = scales.to(dev).float(), mix.to(dev).float()
    flat = routed.view(-1, r)
    group, branch0 = ops._map_layout(h, maps)
    lib = ops._lib.lib()
    assert lib.da_attn_bwd_split_workspace_size(batch, length, r, d, maps, group) > 0
    assert lib.da_attn_bwd_split_workspace_size(batch, length, r, d, 1, group) == 0  # one map never splits
    qmap = ops.RowMap(flat, 0, length, batch * length)
    kmap = ops.RowMap(flat, h * batch * length, length, batch * length)
    _y, lse = ops._attention_forward(qmap, kmap, value, batch, length, r, maps, group, branch0, causal, scales, mix,
                                     None, 1.0, dtype)

    def run(split: bool):
        droute = torch.empty(flat.shape, dtype=dtype, device=dev)
        dv = torch.empty(batch * length, d, dtype=dtype, device=dev)
        dscale = torch.zeros(maps, dtype=torch.float32, device=dev)
        dweight = torch.zeros(maps, dtype=torch.float32, device=dev)
        delta = torch.empty(batch, maps, length, dtype=torch.float32, device=dev)
        ops._attention_backward(qmap, kmap, value, dy, batch, length, r, maps, group, branch0, causal, scales, mix,
                                lse, delta, False, droute, droute, dv, dscale, dweight, overwrite=True, split=split)
        return droute, dv, dscale, dweight, delta

    whole, first, again = run(False), run(True), run(True)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    names = ("routed", "value", "scales", "map weights", "delta")
    for name, a, b in zip(names, first, again):
        assert torch.equal(a, b), f"d {name}: two split passes differ"
    for name, a, b in zip(names, first, whole):
        a, b = a.float(), b.float()
        scale = max(b.abs().max().item(), 1e-30)
        tol = 1e-5 if name in ("scales", "map weights", "delta") else 2 ** -7
        err = (a - b).abs().max().item() / scale
        assert err <= tol, f"d {name}: split vs unsplit max error {err:.2e} of max |g| (bound {tol:.1e})"
        assert _cos(a, b) >= 0.99999, name
