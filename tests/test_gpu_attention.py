"""Outer routed attention forward (with the fused alpha mix) against the oracle.

Bar: max |y - y_ref| <= 2e-2 and cosine >= 0.9995; the per-map log-sum-exp
within 2e-3.  Inputs are rounded to the kernel dtype and the oracle runs in
fp32 on their upcast; the value operand of the probability product is bf16.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import oracle
from double_attention_b200 import ops

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    return float(F.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


def _routed(h: int, batch: int, length: int, r: int, dtype: torch.dtype, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return F.normalize(torch.randn(2, h, batch, length, r, generator=g), dim=-1).to(dtype)


class _Cfg:
    def __init__(self, maps: int, causal: bool = True) -> None:
        self.outer_maps = maps
        self.causal = causal


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(
    ("h", "maps", "batch", "length", "r", "d", "scale0"),
    [
        (1, 1, 8, 512, 256, 512, 16.0),            # a1, config-2 attention
        (4, 4, 2, 256, 128, 512, 16.0),            # qk4-s4 (mixed maps)
        (1, 1, 1, 1024, 512, 512, 512.0**0.5),     # a1-r512-d1536 width
        (2, 1, 2, 130, 256, 512, 16.0),            # qk2-s1: two branches concatenated per map
        (1, 2, 2, 65, 256, 256, 16.0),             # qk1-s2: one branch repeated over two maps
        (4, 4, 1, 257, 128, 128, 12.0),            # ragged tail, narrow value
    ],
)
def test_mixed_attention_forward(h, maps, batch, length, r, d, scale0, dtype) -> None:
    dev = torch.device("cuda")
    routed = _routed(h, batch, length, r, dtype, seed=length + r + maps)
    g = torch.Generator().manual_seed(7)
    value = torch.randn(batch, length, d, generator=g).to(dtype)
    log_scales = math.log(scale0) + torch.linspace(-0.05, 0.05, maps) if maps > 1 else torch.tensor([math.log(scale0)])
    scales = log_scales.exp()
    mix = torch.softmax(torch.randn(maps, generator=g), 0) if maps > 1 else None
    y = ops.routed_attention_mixed(routed.to(dev), value.to(dev), scales.to(dev),
                                   None if mix is None else mix.to(dev), _Cfg(maps))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0

    zq, zk = routed[0].float().permute(1, 0, 2, 3), routed[1].float().permute(1, 0, 2, 3)
    sq, sk = oracle.assemble_score_maps(zq, zk, maps)
    per_map = oracle.routed_attention(sq, sk, value.to(torch.bfloat16).float(), scales, True)
    expected = per_map[:, 0] if mix is None else torch.einsum("s,bstd->btd", mix, per_map)
    got = y.float().cpu()
    assert (got - expected).abs().max().item() <= MAX_ABS
    assert _cos(got, expected) >= MIN_COS


@pytest.mark.parametrize("causal", [True, False])
def test_op_level_routed_attention(causal: bool) -> None:
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(2)
    q = F.normalize(torch.randn(2, 2, 65, 64, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(2, 2, 65, 64, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(2, 65, 128, generator=g).to(torch.bfloat16)
    scales = torch.tensor([12.0, 17.0])
    y = ops.routed_attention(q.to(dev), k.to(dev), v.to(dev), scales.to(dev), causal)
    assert y.shape == (2, 2, 65, 128) and y.dtype == torch.bfloat16
    expected = oracle.routed_attention(q.float(), k.float(), v.float(), scales, causal)
    got = y.float().cpu()
    assert (got - expected).abs().max().item() <= MAX_ABS
    assert _cos(got, expected) >= MIN_COS


def test_attention_lse_matches() -> None:
    dev = torch.device("cuda")
    routed = _routed(4, 1, 200, 128, torch.bfloat16, seed=3)
    value = torch.randn(1, 200, 512).to(torch.bfloat16)
    scales = torch.full((4,), 16.0)
    mix = torch.full((4,), 0.25)
    flat = routed.to(dev).view(-1, 128)
    qmap = ops.RowMap(flat, 0, 200, 200)
    kmap = ops.RowMap(flat, 4 * 200, 200, 200)
    _, lse = ops._attention_forward(qmap, kmap, value.to(dev), 1, 200, 128, 4, 1, [0, 1, 2, 3], True,
                                    scales.to(dev), mix.to(dev), None, 1.0, torch.bfloat16)
    zq, zk = routed[0].float().permute(1, 0, 2, 3), routed[1].float().permute(1, 0, 2, 3)
    s = torch.einsum("bstr,bsur->bstu", zq, zk) * 16.0
    s = s.masked_fill(torch.ones(200, 200, dtype=torch.bool).triu(1), float("-inf"))
    torch.testing.assert_close(lse.cpu(), torch.logsumexp(s, -1), atol=2e-3, rtol=1e-4)


def test_key_split_forward_matches_one_launch() -> None:
    """Several maps over few query tiles (qk4-s4 at B2 T2048): the key range of each tile is split over two
    CTA pairs (partial row sums, then partial outputs added in share order).  The result matches the
    single-launch kernel (da_attn_fwd, no workspace) to fp32 reassociation and repeats bit for bit."""
    from double_attention_b200 import _lib

    dev, dtype = torch.device("cuda"), torch.bfloat16
    h = maps = 4
    batch, length, r, d = 2, 2048, 128, 512
    assert int(_lib.lib().da_attn_fwd_workspace_size(batch, length, maps, d)) > 0  # the split runs here
    routed = _routed(h, batch, length, r, dtype, seed=11).to(dev)
    g = torch.Generator().manual_seed(12)
    value = torch.randn(batch, length, d, generator=g).to(dtype).to(dev)
    scales = torch.full((maps,), 16.0, device=dev)
    mix = torch.softmax(torch.randn(maps, generator=g), 0).to(dev)
    flat = routed.view(-1, r)
    group, branch0 = ops._map_layout(h, maps)
    qmap = ops.RowMap(flat, 0, length, batch * length)
    kmap = ops.RowMap(flat, h * batch * length, length, batch * length)
    runs = [ops._attention_forward(qmap, kmap, value, batch, length, r, maps, group, branch0, True, scales, mix,
                                   None, 1.0, dtype) for _ in range(2)]
    # the same op in one launch
    y1 = torch.empty(batch, length, d, dtype=dtype, device=dev)
    lse1 = torch.empty(batch, maps, length, dtype=torch.float32, device=dev)
    b0 = (ops.ctypes_int_array(ops.MAX_MAPS))(*(branch0 + [0] * (ops.MAX_MAPS - len(branch0))))
    status = torch.zeros(2, dtype=torch.int32, device=dev)
    ops.call("da_attn_fwd", flat.data_ptr(), qmap.rows, qmap.base, qmap.sb, qmap.sbr, flat.data_ptr(), kmap.rows,
             kmap.base, kmap.sb, kmap.sbr, value.data_ptr(), batch, length, r, d, maps, group, ops.ctypes_addressof(b0),
             1, ops.dtype_code(dtype), scales.float().contiguous().data_ptr(), mix.float().contiguous().data_ptr(), 0,
             1.0, y1.data_ptr(), lse1.data_ptr(), status.data_ptr(), ops.stream_ptr(dev))
    torch.cuda.synchronize()
    assert int(status[0]) == 0 and ops.device_status(dev) == 0
    (ya, la), (yb, lb) = runs
    assert torch.equal(ya, yb) and torch.equal(la, lb)
    assert (ya.float() - y1.float()).abs().max().item() <= 1e-2
    assert _cos(ya.float(), y1.float()) >= 0.99999
    assert (la - lse1).abs().max().item() <= 1e-4
