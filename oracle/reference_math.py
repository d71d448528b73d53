"""Plain-PyTorch CPU restatement of the reference hot path (test oracle).

Every function cites the reference source it restates (paths inside the
Ahnd6474/double-attention package).  All arithmetic follows the reference
order of operations: normalisations, softmax and accumulation in the input
dtype (callers pass fp32 or fp64 tensors), with autograd providing the
gradients the backward parity tests compare against.
"""

from __future__ import annotations

import math
from typing import Any, Mapping

import torch
import torch.nn.functional as F
from torch import Tensor


def _normalize(x: Tensor, dim: int, eps: float) -> Tensor:
    # F.normalize: x / max(||x||_2, eps)  (used at ops.py:45, :62, modules.py:46-47)
    return x / x.norm(p=2, dim=dim, keepdim=True).clamp_min(eps)


def normalize_bank(raw_key: Tensor, raw_value: Tensor | None, eps: float = 1e-6) -> tuple[Tensor, Tensor]:
    """SharedDictionaryBank.normalized (modules.py:45-48): column-normalise."""
    key = _normalize(raw_key, 0, eps)
    value = key if raw_value is None else _normalize(raw_value, 0, eps)
    return key, value


def score_scale_from_log(log_scale: Tensor) -> Tensor:
    """ops.py:160-161: exp(clamp(log gamma, ln 1/4, ln 1024))."""
    return log_scale.clamp(math.log(0.25), math.log(1024.0)).exp()


def beta_from_log(log_beta: Tensor) -> Tensor:
    """modules.py:130-132: exp(clamp(log beta, ln 0.05, ln 64))."""
    return log_beta.clamp(math.log(0.05), math.log(64.0)).exp()


def dictionary_route(
    x: Tensor,
    dictionary_key: Tensor,
    dictionary_value: Tensor,
    beta: Tensor | float,
    eps: float = 1e-6,
    activation: str = "identity",
    assignment: str = "softmax",
    silu_gain: float = 1.0,
    standardize_logits: bool = False,
    standardized_logit_scale: float | None = None,
    normalize_input: bool = True,
    normalize_output: bool = True,
    inspect: dict | None = None,
) -> Tensor:
    """ops.py:16-62: z = norm(Dv softmax(beta * Dk^T norm(x)))  (+ variants).

    ``inspect`` (test use): receives the final logits and the softmax input
    (``logits``, ``scaled``; the latter retains its gradient), from which a
    test bounds the conditioning of the beta gradient, the sum over every
    route row and atom of logits * d loss / d scaled."""
    q = _normalize(x, -1, eps) if normalize_input else x
    logits = torch.matmul(q, dictionary_key)
    if activation == "silu":
        logits = 2.0 * F.silu(logits)  # ops.py:39-41
    elif activation != "identity":
        raise ValueError(f"unsupported dictionary activation: {activation}")
    if standardize_logits:  # ops.py:44-53
        centered = logits - logits.mean(dim=-1, keepdim=True)
        inv_std = torch.rsqrt(centered.square().mean(dim=-1, keepdim=True) + eps)
        scale = x.shape[-1] ** -0.5 if standardized_logit_scale is None else standardized_logit_scale
        logits = centered * inv_std * scale
    if assignment == "softmax":  # ops.py:54-59
        scaled = logits * beta
        if inspect is not None:
            scaled.retain_grad()
            inspect.update(logits=logits, scaled=scaled)
        weights = torch.softmax(scaled, dim=-1)
    elif assignment == "silu":
        weights = (2.0 / silu_gain) * F.silu(silu_gain * logits)
    else:
        raise ValueError(f"unsupported dictionary assignment: {assignment}")
    reconstructed = torch.matmul(weights, dictionary_value.transpose(0, 1))
    return _normalize(reconstructed, -1, eps) if normalize_output else reconstructed


def routed_attention(query: Tensor, key: Tensor, value: Tensor, scales: Tensor, causal: bool = True) -> Tensor:
    """ops.py:65-93: per-map causal softmax(scale_s Q_s K_s^T) applied to a shared V.

    query/key [B, S, T, R], value [B, T, D] -> [B, S, T, D].
    """
    if query.ndim != 4 or key.shape != query.shape:
        raise ValueError("query and key must have matching [B, S, T, R] shapes")
    if value.ndim != 3 or value.shape[:2] != (query.shape[0], query.shape[2]):
        raise ValueError("value must have shape [B, T, D] matching query")
    if scales.shape != (query.shape[1],):
        raise ValueError(f"scales must have shape [{query.shape[1]}]")
    scores = torch.matmul(query, key.transpose(-2, -1)) * scales.view(1, -1, 1, 1)
    if causal:
        t = query.shape[-2]
        future = torch.ones(t, t, dtype=torch.bool).triu(1)
        scores = scores.masked_fill(future, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    return torch.matmul(probs, value[:, None])


def assemble_score_maps(query: Tensor, key: Tensor, outer_maps: int) -> tuple[Tensor, Tensor]:
    """ops.py:96-139: map H Q/K branches onto S outer maps."""
    if query.ndim != 4 or query.shape != key.shape:
        raise ValueError("query and key must have matching [B, H, T, R] shapes")
    branches = query.shape[1]
    if branches == outer_maps:
        return query, key
    if branches > outer_maps:  # group-concatenate, scale group^-1/4 (ops.py:113-131)
        if branches % outer_maps:
            raise ValueError("qk_branches must be divisible by outer_maps")
        group = branches // outer_maps
        s = group ** -0.25
        b, _, t, r = query.shape

        def fold(z: Tensor) -> Tensor:
            return (z.view(b, outer_maps, group, t, r).permute(0, 1, 3, 2, 4).reshape(b, outer_maps, t, group * r)) * s

        return fold(query), fold(key)
    if outer_maps % branches:  # repeat (ops.py:133-139)
        raise ValueError("outer_maps must be divisible by qk_branches")
    rep = outer_maps // branches
    return query.repeat_interleave(rep, dim=1), key.repeat_interleave(rep, dim=1)


def _cfg(cfg: Any, name: str) -> Any:
    return cfg[name] if isinstance(cfg, Mapping) else getattr(cfg, name)


def attention_forward(
    params: Mapping[str, Tensor],
    x: Tensor,
    cfg: Any,
    normalized_dictionary: tuple[Tensor, Tensor] | None = None,
    prefix: str = "",
    return_parts: bool = False,
):
    """SharedDictionaryAttention.forward (modules.py:190-291), functional form.

    ``params`` uses the module's state_dict keys (``query.weight``,
    ``key.weight``, ``value.weight``/``value.bias``, ``bank.raw_key``,
    ``bank.raw_value``, ``log_score_scales``, ``log_beta``,
    ``map_mix_logits``, ``output.weight``), optionally under ``prefix``.
    """
    p = lambda k: params.get(prefix + k)  # noqa: E731
    H, S, R = _cfg(cfg, "qk_branches"), _cfg(cfg, "outer_maps"), _cfg(cfg, "routing_dim")
    eps = _cfg(cfg, "eps")
    b, t, _ = x.shape
    q = torch.matmul(x, p("query.weight").t()).view(b, t, H, R).permute(0, 2, 1, 3)  # modules.py:143-157
    k = torch.matmul(x, p("key.weight").t()).view(b, t, H, R).permute(0, 2, 1, 3)
    v = torch.matmul(x, p("value.weight").t())
    if p("value.bias") is not None:
        v = v + p("value.bias")
    if normalized_dictionary is None:
        dk, dv = normalize_bank(p("bank.raw_key"), p("bank.raw_value"), eps)
    else:
        dk, dv = normalized_dictionary
    beta = beta_from_log(p("log_beta"))
    route = lambda z: dictionary_route(  # noqa: E731  modules.py:159-188
        z, dk, dv, beta, eps,
        _cfg(cfg, "dictionary_activation"), _cfg(cfg, "dictionary_assignment"),
        _cfg(cfg, "dictionary_silu_gain"), _cfg(cfg, "standardize_dictionary_logits"),
        _cfg(cfg, "standardized_logit_scale"), _cfg(cfg, "normalize_routing_input"),
        _cfg(cfg, "normalize_routing_output"),
    )
    zq, zk = route(q), route(k)
    sq, sk = assemble_score_maps(zq, zk, S)
    scales = score_scale_from_log(p("log_score_scales"))
    maps = routed_attention(sq, sk, v, scales, _cfg(cfg, "causal"))
    if _cfg(cfg, "map_combine") == "weighted_sum":  # modules.py:265-272
        mix = p("map_mix_logits")
        combined = maps[:, 0] if mix is None else torch.einsum("s,bstd->btd", torch.softmax(mix, 0), maps)
    else:  # concat, modules.py:273-279
        combined = maps.permute(0, 2, 1, 3).flatten(2)
    w_out = p("output.weight")
    out = combined if w_out is None else torch.matmul(combined, w_out.t())
    if return_parts:
        return out, {"zq": zq, "zk": zk, "value": v, "maps": maps, "combined": combined}
    return out


def _layer_norm(x: Tensor, params: Mapping[str, Tensor], prefix: str) -> Tensor:
    return F.layer_norm(x, x.shape[-1:], params[prefix + "weight"], params[prefix + "bias"], 1e-5)


def lm_forward(
    params: Mapping[str, Tensor],
    token_ids: Tensor,
    targets: Tensor | None,
    cfg: Any,
    num_layers: int,
    dictionary_group_size: int | None = None,
) -> tuple[Tensor, Tensor | None]:
    """DoubleAttentionLM.forward (modules.py:444-460) with its stack
    (modules.py:398-412) and blocks (modules.py:332-356), standard FFN only."""
    group = dictionary_group_size or num_layers
    n_banks = math.ceil(num_layers / group)
    eps = _cfg(cfg, "eps")
    t = token_ids.shape[1]
    h = params["token_embedding.weight"][token_ids] + params["position_embedding.weight"][:t][None]
    banks = [
        normalize_bank(params[f"stack.banks.{i}.raw_key"], params.get(f"stack.banks.{i}.raw_value"), eps)
        for i in range(n_banks)
    ]
    for layer in range(num_layers):
        pre = f"stack.blocks.{layer}."
        bank = banks[min(layer // group, n_banks - 1)]
        a = attention_forward(params, _layer_norm(h, params, pre + "attention_norm."), cfg, bank, prefix=pre + "attention.")
        h = h + a
        f = _layer_norm(h, params, pre + "feedforward_norm.")
        f = F.linear(f, params[pre + "feedforward.0.weight"], params[pre + "feedforward.0.bias"])
        f = F.gelu(f)
        f = F.linear(f, params[pre + "feedforward.2.weight"], params[pre + "feedforward.2.bias"])
        h = h + f
    h = _layer_norm(h, params, "final_norm.")
    logits = torch.matmul(h, params["token_embedding.weight"].t())  # tied head, modules.py:441
    loss = None
    if targets is not None:
        loss = F.cross_entropy(logits.flatten(0, 1), targets.flatten())
    return logits, loss
