"""Parity at the full benchmark shapes, where the kernels pick their throughput layouts.

The kernels choose their layout from the amount of work against the SM count:
the route forward and backward switch to two CTAs per SM (compact) or one CTA
pair per SM with two producer warps per stream (coarse) once the 128-row pairs
outnumber the SMs; the attention forward switches to its coarse layout once
its query tiles do.  The smaller parity cases never reach those layouts, so
these tests run the GPU on the full per-GPU shapes of the benchmark
configurations and check the results against the CPU oracle on a subset:

* route rows are independent, so a seeded sample of rows is routed by the oracle;
* attention sequences are independent (and each query row depends only on the
  keys before it), so the oracle attends a few sequences, or a seeded sample of
  query rows of a sequence;
* parameter gradients are sums over sequences, so the upstream gradient is
  zero on every sequence but a few and the oracle runs those few.

Bars as in the other parity tests: outputs max-abs 2e-2 and cosine >= 0.9995;
route argmax identical on >= 99.9% of rows once fp32 near-ties (top-2 gap
<= 4e-3) are set aside, with strict agreement printed; module parameter
gradients cosine >= 0.999 and max-abs 3e-2 * max(1, max |g_ref|) (the cosine only where
max |g_ref| >= 1e-2); scalars and per-map vectors within 5e-2 relative + 5e-2 absolute.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

import oracle
from double_attention_b200 import DoubleAttentionLM, SharedDictionaryAttention, experiment_config, ops

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MIN_COS = 0.9995
NEAR_TIE = 4e-3


def _cos(a: torch.Tensor, b: torch.Tensor) -> float:
    return float(F.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


def _check(name: str, got: torch.Tensor, ref: torch.Tensor, max_abs: float = MAX_ABS, min_cos: float = MIN_COS):
    got = got.float().cpu()
    err, cos = (got - ref).abs().max().item(), _cos(got, ref)
    assert err <= max_abs and cos >= min_cos, f"{name}: max-abs {err:.3e} (bound {max_abs:.1e}) cosine {cos:.6f}"


def _check_grads(pairs) -> None:
    failures = []
    for key, got, ref in pairs:
        assert got is not None and ref is not None, key
        got = got.float().cpu()
        if ref.numel() <= 4:
            tol = 5e-2 * ref.abs().max().item() + 5e-2
            if (got - ref).abs().max().item() > tol:
                failures.append(f"{key}: {got.tolist()} vs {ref.tolist()}")
            continue
        bound = 3e-2 * max(1.0, ref.abs().max().item())
        err, cos = (got - ref).abs().max().item(), _cos(got, ref)
        # A gradient whose entries are all below 1e-2 is a sum that cancels (the LM's final-norm bias:
        # 2048 bf16-rounded token gradients summing to ~1e-3); its direction is set by bf16 rounding under
        # autocast, so only the absolute bound applies to it.
        if err > bound or (cos < 0.999 and ref.abs().max().item() >= 1e-2):
            failures.append(f"{key}: max-abs {err:.3e} (bound {bound:.3e}) cosine {cos:.6f}")
    assert not failures, "; ".join(failures)


def _attend_rows(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, t_idx: torch.Tensor) -> torch.Tensor:
    """Causal softmax(scale q_t k^T) v of ops.py:65-93 for the query positions t_idx of one sequence and map."""
    s = (q[t_idx] @ k.t()) * scale
    future = torch.arange(k.shape[0])[None, :] > t_idx[:, None]
    return torch.softmax(s.masked_fill(future, float("-inf")), dim=-1) @ v


def _sample_rows(n: int, count: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    edges = torch.cat([torch.arange(0, 128), torch.arange(n - 128, n)])
    return torch.unique(torch.cat([edges, torch.randperm(n, generator=g)[:count]]))


# ----------------------------------------------------------------------------- route forward, config 4
def test_route_forward_config4_rows() -> None:
    """a1-r512-d1536 route at one GPU's config-4 batch (B4 T8192: 32768 Q and 32768 K rows, R 512,
    M 1536): 512 pairs, the one-CTA-pair-per-SM wide kernel with 256-atom tiles."""
    rows, r, m, beta = 4 * 8192, 512, 1536, 4.0 * 2**0.5
    g = torch.Generator().manual_seed(41)
    dev = torch.device("cuda")
    proj = torch.randn(rows, 2 * r, generator=g).to(torch.bfloat16)
    dk = F.normalize(torch.randn(r, m, generator=g), dim=0).to(torch.bfloat16)
    dv = F.normalize(torch.randn(r, m, generator=g), dim=0).to(torch.bfloat16)
    views = ops.dictionary_views_from_normalized(dk.to(dev), dv.to(dev), torch.bfloat16)
    argmax = torch.empty(2, rows, dtype=torch.int32, device=dev)
    z, lse, _ = ops._route_forward(proj.to(dev), rows, 2, r, views, torch.tensor(beta, device=dev), 1e-6, True,
                                   True, argmax=argmax)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0

    idx = _sample_rows(rows, 3000, seed=5)
    strict_all, clear_agree, clear_total = [], 0, 0
    for grp in range(2):
        x = proj[idx, grp * r:(grp + 1) * r].float()
        expected = oracle.dictionary_route(x, dk.float(), dv.float(), beta)
        _check(f"z group {grp}", z[grp, idx.to(dev)], expected)
        logits = F.normalize(x, dim=-1) @ dk.float()
        torch.testing.assert_close(lse[grp, idx.to(dev)].cpu(), torch.logsumexp(beta * logits, -1), atol=2e-3,
                                   rtol=1e-4)
        top2 = logits.topk(2, dim=-1)
        agree = argmax[grp, idx.to(dev)].cpu().long() == top2.indices[:, 0]
        clear = (top2.values[:, 0] - top2.values[:, 1]) > NEAR_TIE
        strict_all.append(agree.float().mean().item())
        clear_agree += int(agree[clear].sum())
        clear_total += int(clear.sum())
    strict = sum(strict_all) / len(strict_all)
    non_tie = clear_agree / max(1, clear_total)
    print(f"config-4 route argmax: strict {strict:.5f}, excluding near-ties {non_tie:.5f} "
          f"({clear_total} of {2 * len(idx)} rows clear)")
    assert non_tie >= 0.999, f"argmax agreement {non_tie:.5f} excluding near-ties (strict {strict:.5f})"


# ----------------------------------------------------------------------------- attention forward
class _Cfg:
    def __init__(self, maps: int) -> None:
        self.outer_maps = maps
        self.causal = True


def test_attention_forward_config4_single_map() -> None:
    """One map, R 512, D 512, B4 T8192: 256 query tiles, the coarse single-map kernel."""
    batch, length, r, d, scale = 4, 8192, 512, 512, 512.0**0.5
    g = torch.Generator().manual_seed(43)
    dev = torch.device("cuda")
    routed = F.normalize(torch.randn(2, 1, batch, length, r, generator=g), dim=-1).to(torch.bfloat16)
    value = torch.randn(batch, length, d, generator=g).to(torch.bfloat16)
    y = ops.routed_attention_mixed(routed.to(dev), value.to(dev), torch.tensor([scale], device=dev), None, _Cfg(1))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    t_idx = _sample_rows(length, 384, seed=6)
    for b in (0, batch - 1):
        expected = _attend_rows(routed[0, 0, b].float(), routed[1, 0, b].float(), value[b].float(), scale, t_idx)
        _check(f"y[{b}]", y[b, t_idx.to(dev)], expected)


def test_attention_forward_config3_mixed_maps() -> None:
    """Four maps mixed by alpha, R 128, D 512, B16 T2048: 256 query tiles, the coarse mixed kernel."""
    batch, length, r, d, maps = 16, 2048, 128, 512, 4
    g = torch.Generator().manual_seed(44)
    dev = torch.device("cuda")
    routed = F.normalize(torch.randn(2, maps, batch, length, r, generator=g), dim=-1).to(torch.bfloat16)
    value = torch.randn(batch, length, d, generator=g).to(torch.bfloat16)
    scales = (math.log(16.0) + torch.linspace(-0.05, 0.05, maps)).exp()
    mix = torch.softmax(torch.randn(maps, generator=g), 0)
    y = ops.routed_attention_mixed(routed.to(dev), value.to(dev), scales.to(dev), mix.to(dev), _Cfg(maps))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    for b in (0, 9, batch - 1):
        zq, zk = routed[0, :, b : b + 1].float().permute(1, 0, 2, 3), routed[1, :, b : b + 1].float().permute(1, 0, 2, 3)
        per_map = oracle.routed_attention(zq, zk, value[b : b + 1].float(), scales, True)
        expected = torch.einsum("s,bstd->btd", mix, per_map)[0]
        _check(f"y[{b}]", y[b], expected)


# ----------------------------------------------------------------------------- modules at full shape
def _params_for_oracle(module: torch.nn.Module):
    params = {k: v.detach().float().cpu().requires_grad_() for k, v in module.named_parameters()}
    state = {k: v.detach().float().cpu() for k, v in module.state_dict().items()}
    state.update(params)
    return params, state


def test_module_config3_forward_backward() -> None:
    """qk4-s4 SharedDictionaryAttention forward+backward at B16 T2048 (the config-3 step: 262144 route rows,
    compact route forward and backward, coarse mixed attention, all three attention backward kernels).
    fp32 parameters under bf16 autocast; dY is non-zero on sequences 0, 7 and 15 only, so every parameter
    gradient is the sum of those three sequences' contributions, which the oracle computes."""
    dev = torch.device("cuda")
    batch, length, live = 16, 2048, (0, 7, 15)
    torch.manual_seed(0)
    module = SharedDictionaryAttention(experiment_config("qk4-s4")).to(dev)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(batch, length, 512, generator=g)
    dy = torch.zeros(batch, length, 512)
    dy[list(live)] = torch.randn(len(live), length, 512, generator=g)
    xd = x.to(dev).requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = module(xd)
    y.float().backward(dy.to(dev))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0

    params, state = _params_for_oracle(module)
    xr = x[list(live)].clone().requires_grad_()
    yr = oracle.attention_forward(state, xr, module.config)
    yr.backward(dy[list(live)])
    _check("y (live sequences)", y[list(live)].detach(), yr.detach())
    _check_grads([("x", xd.grad[list(live)], xr.grad)] +
                 [(k, p.grad, params[k].grad) for k, p in module.named_parameters()])
    assert xd.grad[1:7].abs().max().item() == 0.0  # sequences without an upstream gradient get none


def _module_rows_oracle(state, x: torch.Tensor, cfg, t_idx: torch.Tensor) -> torch.Tensor:
    """SharedDictionaryAttention.forward (modules.py:190-291) of one sequence x [T, 512] for one map
    (H = S = 1), at the query positions t_idx only (keys and values over the whole sequence)."""
    q = x @ state["query.weight"].t()
    k = x @ state["key.weight"].t()
    v = x @ state["value.weight"].t()
    if state.get("value.bias") is not None:
        v = v + state["value.bias"]
    dk, dv = oracle.normalize_bank(state["bank.raw_key"], state.get("bank.raw_value"), cfg.eps)
    beta = oracle.beta_from_log(state["log_beta"])
    zq = oracle.dictionary_route(q[t_idx], dk, dv, beta, cfg.eps)
    zk = oracle.dictionary_route(k, dk, dv, beta, cfg.eps)
    scale = float(oracle.score_scale_from_log(state["log_score_scales"])[0])
    s = (zq @ zk.t()) * scale
    future = torch.arange(x.shape[0])[None, :] > t_idx[:, None]
    out = torch.softmax(s.masked_fill(future, float("-inf")), dim=-1) @ v
    w = state.get("output.weight")
    return out if w is None else out @ w.t()


def test_module_config4_forward() -> None:
    """a1-r512-d1536 forward at one GPU's config-4 batch (B4 T8192, bf16 module): the coarse R 512 route
    over 65536 rows and the coarse single-map attention, checked on sampled query rows of two sequences."""
    dev = torch.device("cuda")
    batch, length = 4, 8192
    torch.manual_seed(0)
    module = SharedDictionaryAttention(experiment_config("a1-r512-d1536")).to(dev, torch.bfloat16)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(batch, length, 512, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        y = module(x.to(dev))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    state = {k: v.detach().float().cpu() for k, v in module.state_dict().items()}
    t_idx = _sample_rows(length, 256, seed=7)
    for b in (0, batch - 1):
        expected = _module_rows_oracle(state, x[b].float(), module.config, t_idx)
        _check(f"y[{b}]", y[b, t_idx.to(dev)], expected)


def test_lm_config5_per_gpu_batch() -> None:
    """The config-5 LM (a1, 6 layers, one bank, FFN 1536, vocab 2048, T 1024) at its one-GPU batch of 256
    sequences under bf16 autocast: 524288 route rows per layer (compact route forward, R 256 route backward),
    coarse attention.  The training loss (cross-entropy, mean over tokens) is taken over sequences 0 and 255
    only, so the parameter gradients are those two sequences' contributions while every kernel runs on the
    whole batch."""
    dev = torch.device("cuda")
    vocab, seq, batch, layers, live = 2048, 1024, 256, 6, [0, 255]
    torch.manual_seed(0)
    model = DoubleAttentionLM(vocab, seq, experiment_config("a1"), layers, dictionary_group_size=layers,
                              feedforward_dim=1536).to(dev)
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, vocab, (batch, seq + 1), generator=g)
    x, y = ids[:, :-1], ids[:, 1:]
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits, _ = model(x.to(dev))
        loss = F.cross_entropy(logits[live].flatten(0, 1), y[live].flatten().to(dev))
    loss.backward()
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    got_logits = logits[live].detach().float().cpu()
    del logits

    params, state = _params_for_oracle(model)
    state["lm_head.weight"] = state["token_embedding.weight"]
    ref_logits, ref_loss = oracle.lm_forward(state, x[live], y[live], model.stack.config, layers, layers)
    ref_loss.backward()
    # the untrained tied-embedding LM's logits reach ~30: the bar scales with their range
    _check("logits (live sequences)", got_logits, ref_logits.detach(),
           max_abs=2e-2 * max(1.0, ref_logits.abs().max().item()))
    assert abs(loss.item() - ref_loss.item()) <= 2e-3 * max(1.0, abs(ref_loss.item())), (loss.item(), ref_loss.item())
    _check_grads([(k, p.grad, params[k].grad) for k, p in model.named_parameters()])


# ----------------------------------------------------------------------------- tied dictionary
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tied_dictionary_module_forward_backward(dtype: torch.dtype) -> None:
    """untied_dictionary=False (reference modules.py:33-43): the value dictionary is the key dictionary.
    bf16 autocast takes the one-normalisation path (both views share one bf16 normalisation), fp16 autocast
    the pair path (key views in fp16, value views a bf16 normalisation of the same bank); both gradients
    land on the one raw bank."""
    dev = torch.device("cuda")
    torch.manual_seed(0)
    module = SharedDictionaryAttention(experiment_config("a1", untied_dictionary=False)).to(dev)
    assert module.bank.raw_value is None
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 256, 512, generator=g)
    dy = torch.randn(2, 256, 512, generator=g)
    xd = x.to(dev).requires_grad_()
    with torch.autocast("cuda", dtype=dtype):
        y = module(xd)
    y.float().backward(dy.to(dev))
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    params, state = _params_for_oracle(module)
    xr = x.clone().requires_grad_()
    yr = oracle.attention_forward(state, xr, module.config)
    yr.backward(dy)
    _check("y", y.detach(), yr.detach())
    _check_grads([("x", xd.grad, xr.grad)] + [(k, p.grad, params[k].grad) for k, p in module.named_parameters()])
