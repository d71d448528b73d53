"""Drop-in modules: same constructors, parameters and state_dict as the reference.

``SharedDictionaryBank``, ``SharedDictionaryAttention``,
``DoubleAttentionBlock``, ``DoubleAttentionStack`` and ``DoubleAttentionLM``
mirror src/double_attention/modules.py:25-460: identical constructor
signatures, parameter creation order (so ``torch.manual_seed`` builds the
same weights), state_dict keys and forward contracts.  The hot path inside
``SharedDictionaryAttention.forward`` runs on the B200 kernels of this
package (``ops``); the layers around it (value/output projections,
LayerNorm, FFN, embeddings, loss) are ordinary PyTorch modules.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor

from . import ops
from .config import DoubleAttentionConfig

# The reference exposes this switch to compare fused and separate Q/K
# projections (modules.py:22).  The B200 path always runs one fused
# projection GEMM over the concatenated weights; the flag is kept for
# compatibility and selects the same computation either way.
FUSED_QUERY_KEY_PROJECTION = True


class NormalizedDictionary(tuple):
    """``(key, value)`` column-normalised fp32 dictionaries (as the reference
    returns them) that also carries the bank they came from, so attention
    layers can fetch the kernel operands built once per forward."""

    def __new__(cls, key: Tensor, value: Tensor, bank: "SharedDictionaryBank", eps: float):
        obj = super().__new__(cls, (key, value))
        obj.bank = bank
        obj.eps = eps
        obj._views: dict[torch.dtype, ops.DictionaryViews] = {}
        return obj

    def views(self, dtype: torch.dtype) -> "ops.DictionaryViews":
        if dtype not in self._views:
            self._views[dtype] = ops.dictionary_views(self.bank.raw_key, self.bank.raw_value, self.eps, dtype)
        return self._views[dtype]


class SharedDictionaryBank(nn.Module):
    """Globally or stage-wise shared routing dictionary (modules.py:25-54)."""

    def __init__(self, routing_dim: int, dictionary_size: int, *, untied: bool = True) -> None:
        super().__init__()
        self.routing_dim = routing_dim
        self.dictionary_size = dictionary_size
        self.untied = untied
        std = routing_dim**-0.5
        self.raw_key = nn.Parameter(torch.randn(routing_dim, dictionary_size) * std)
        if untied:
            self.raw_value = nn.Parameter(torch.randn(routing_dim, dictionary_size) * std)
        else:
            self.register_parameter("raw_value", None)

    def normalized(self, eps: float = 1e-6) -> NormalizedDictionary:
        key = F.normalize(self.raw_key, dim=0, eps=eps)
        value = key if self.raw_value is None else F.normalize(self.raw_value, dim=0, eps=eps)
        return NormalizedDictionary(key, value, self, eps)

    def extra_repr(self) -> str:
        return f"routing_dim={self.routing_dim}, dictionary_size={self.dictionary_size}, untied={self.untied}"


@dataclass
class DoubleAttentionAux:
    routing_query: Tensor
    routing_key: Tensor
    score_query: Tensor
    score_key: Tensor
    score_scales: Tensor
    map_weights: Tensor
    backend: str


class SharedDictionaryAttention(nn.Module):
    """Content/routing-decoupled attention (modules.py:68-291) on B200 kernels."""

    def __init__(
        self,
        config: DoubleAttentionConfig,
        *,
        bank: SharedDictionaryBank | None = None,
        create_bank: bool = True,
    ) -> None:
        super().__init__()
        self.config = config
        width = config.qk_branches * config.routing_dim
        self.query = nn.Linear(config.model_dim, width, bias=False)
        self.key = nn.Linear(config.model_dim, width, bias=False)
        self.value = nn.Linear(config.model_dim, config.model_dim, bias=config.value_bias)
        if bank is not None:
            self.bank = bank
        elif create_bank:
            self.bank = SharedDictionaryBank(config.routing_dim, config.dictionary_size,
                                             untied=config.untied_dictionary)
        else:
            self.bank = None

        initial_log_scale = math.log(config.initial_score_scale)
        if config.outer_maps == 1:
            initial_scales = torch.tensor([initial_log_scale])
        else:
            # A small deterministic spread keeps repeated maps (QK1-S2) from
            # staying exactly symmetric (modules.py:98-106).
            initial_scales = initial_log_scale + torch.linspace(-0.05, 0.05, config.outer_maps)
        self.log_score_scales = nn.Parameter(initial_scales)
        if config.learnable_beta:
            self.log_beta = nn.Parameter(torch.tensor(math.log(config.beta)))
        else:
            self.register_buffer("log_beta", torch.tensor(math.log(config.beta)), persistent=True)

        if config.map_combine == "weighted_sum":
            if config.outer_maps > 1:
                self.map_mix_logits = nn.Parameter(torch.zeros(config.outer_maps))
            else:
                self.register_parameter("map_mix_logits", None)
            self.output = (
                nn.Linear(config.model_dim, config.model_dim, bias=False)
                if config.output_projection
                else nn.Identity()
            )
        else:
            self.register_parameter("map_mix_logits", None)
            self.output = nn.Linear(config.outer_maps * config.model_dim, config.model_dim, bias=False)

    @property
    def beta(self) -> Tensor:
        return self.log_beta.clamp(math.log(0.05), math.log(64.0)).exp()

    def forward(
        self,
        x: Tensor,
        *,
        bank: SharedDictionaryBank | None = None,
        normalized_dictionary: tuple[Tensor, Tensor] | None = None,
        return_aux: bool = False,
    ) -> Tensor | tuple[Tensor, DoubleAttentionAux]:
        cfg = self.config
        if x.ndim != 3 or x.shape[-1] != cfg.model_dim:
            raise ValueError(f"expected x with shape [B, T, {cfg.model_dim}], got {tuple(x.shape)}")
        active_bank = bank if bank is not None else self.bank
        if active_bank is None:
            raise ValueError("no dictionary bank supplied")
        if active_bank.routing_dim != cfg.routing_dim or active_bank.dictionary_size != cfg.dictionary_size:
            raise ValueError("dictionary bank dimensions do not match the attention config")
        if normalized_dictionary is not None:
            expected = (cfg.routing_dim, cfg.dictionary_size)
            if normalized_dictionary[0].shape != expected or normalized_dictionary[1].shape != expected:
                raise ValueError("normalized dictionary dimensions do not match attention config")

        compute_dtype = ops.compute_dtype(x)
        backend = ops.resolve_backend(cfg.backend, x, compute_dtype)

        if isinstance(normalized_dictionary, NormalizedDictionary):
            views = normalized_dictionary.views(compute_dtype)
        elif normalized_dictionary is not None:
            views = ops.dictionary_views_from_normalized(normalized_dictionary[0], normalized_dictionary[1],
                                                        compute_dtype)
        else:
            views = ops.dictionary_views(active_bank.raw_key, active_bank.raw_value, cfg.eps, compute_dtype)

        xc = x.to(compute_dtype)
        # Q, K and V projections of x in one launch; V comes out in the bf16 the attention reads
        projected, dense_value = ops.qkv_projection(
            xc, self.query.weight.to(compute_dtype), self.key.weight.to(compute_dtype),
            self.value.weight.to(compute_dtype),
            None if self.value.bias is None else self.value.bias.to(compute_dtype))  # [B*T, 2*H*R], [B*T, D]
        dense_value = dense_value.view(x.shape[0], x.shape[1], -1)
        beta, score_scales = ops.temperatures(self.log_beta, self.log_score_scales)  # fp32, one launch

        routed = ops.route_projected(projected, views, beta, cfg, x.shape[0], x.shape[1])  # [2,H,B,T,R]
        if cfg.map_combine == "weighted_sum" and self.map_mix_logits is not None:
            map_weights = torch.softmax(self.map_mix_logits, dim=0)
        else:
            map_weights = None

        if cfg.map_combine == "weighted_sum":
            combined = ops.routed_attention_mixed(routed, dense_value, score_scales, map_weights, cfg)
            if (ops.BLOCK_LINEAR_ON_TCGEN05 and isinstance(self.output, nn.Linear)
                    and ops.linear_supported(combined, self.output)):
                output = ops.linear(combined, self.output)  # the output projection on the tcgen05 GEMM
            else:
                output = self.output(combined.to(self._output_dtype(combined)))
        else:
            per_map = ops.routed_attention_maps(routed, dense_value, score_scales, cfg)  # [B,S,T,D]
            output = self.output(per_map.permute(0, 2, 1, 3).flatten(2))

        if not return_aux:
            return output
        if cfg.map_combine == "weighted_sum":
            map_weights_out = x.new_ones(1) if map_weights is None else map_weights.to(combined.dtype)
        else:
            map_weights_out = x.new_full((cfg.outer_maps,), 1.0 / cfg.outer_maps)
        routed_query, routed_key = routed[0].permute(1, 0, 2, 3), routed[1].permute(1, 0, 2, 3)
        score_query, score_key = ops.assemble_score_maps(routed_query, routed_key, cfg.outer_maps)
        return output, DoubleAttentionAux(
            routing_query=routed_query,
            routing_key=routed_key,
            score_query=score_query,
            score_key=score_key,
            score_scales=score_scales,
            map_weights=map_weights_out,
            backend=backend,
        )

    def _output_dtype(self, t: Tensor) -> torch.dtype:
        w = getattr(self.output, "weight", None)
        if w is None or torch.is_autocast_enabled():
            return t.dtype
        return w.dtype


class DoubleAttentionBlock(nn.Module):
    """Pre-norm block (modules.py:294-356)."""

    def __init__(self, config: DoubleAttentionConfig, *, feedforward_dim: int | None = None,
                 dropout: float = 0.0) -> None:
        super().__init__()
        feedforward_dim = feedforward_dim or 3 * config.model_dim
        if config.q_dictionary_feedforward:
            if config.qk_branches != 1:
                raise ValueError("Q-dictionary FFN requires exactly one Q branch")
            if feedforward_dim != config.dictionary_size:
                raise ValueError("Q-dictionary FFN requires feedforward_dim == dictionary_size")
        self.attention_norm = nn.LayerNorm(config.model_dim)
        self.attention = SharedDictionaryAttention(config, create_bank=False)
        self.feedforward_norm = nn.LayerNorm(config.model_dim)
        if config.q_dictionary_feedforward:
            # feedforward[0] is replaced by the shared D^T Q expansion; the
            # module indices stay those of the standard FFN (modules.py:313-322).
            self.feedforward = nn.Sequential(nn.Identity(), nn.GELU(), nn.Linear(feedforward_dim, config.model_dim),
                                             nn.Dropout(dropout))
        else:
            self.feedforward = nn.Sequential(nn.Linear(config.model_dim, feedforward_dim), nn.GELU(),
                                             nn.Linear(feedforward_dim, config.model_dim), nn.Dropout(dropout))

    def forward(self, x: Tensor, bank: SharedDictionaryBank, *,
                normalized_dictionary: tuple[Tensor, Tensor] | None = None) -> Tensor:
        if ops.layernorm_supported(x, self.attention_norm, self.feedforward_norm):
            x, branch = self._forward_fused(x, None, bank, normalized_dictionary)
            return x + branch
        x = x + self.attention(self.attention_norm(x), bank=bank, normalized_dictionary=normalized_dictionary)
        return x + self._feedforward_branch(self.feedforward_norm(x), bank, normalized_dictionary)

    def _forward_fused(self, x: Tensor, pending: Tensor | None, bank: SharedDictionaryBank,
                       normalized_dictionary: tuple[Tensor, Tensor] | None) -> tuple[Tensor, Tensor]:
        """The block on the fp32 residual stream with fused norms: ``x + pending`` (the previous block's
        feed-forward branch, not yet added) is normalised by the same kernel that adds it; returns the
        residual after the attention branch and this block's feed-forward branch, still to be added."""
        if pending is None:
            normalized_x = ops.layernorm(x, self.attention_norm)
        else:
            x, normalized_x = ops.add_layernorm(x, pending, self.attention_norm)
        branch = self.attention(normalized_x, bank=bank, normalized_dictionary=normalized_dictionary)
        x, normalized_x = ops.add_layernorm(x, branch, self.feedforward_norm)
        return x, self._feedforward_branch(normalized_x, bank, normalized_dictionary)

    def _feedforward_branch(self, normalized_x: Tensor, bank: SharedDictionaryBank,
                            normalized_dictionary: tuple[Tensor, Tensor] | None) -> Tensor:
        if not self.attention.config.q_dictionary_feedforward:
            first, act, second, drop = self.feedforward
            if (ops.BLOCK_LINEAR_ON_TCGEN05 and act.approximate == "none"
                    and ops.feedforward_supported(normalized_x, first, second)):
                return drop(ops.feedforward(normalized_x, first, second))  # GELU fused into the GEMMs
            return self.feedforward(normalized_x)
        if normalized_dictionary is None:
            dictionary_key, _ = bank.normalized(self.attention.config.eps)
        else:
            dictionary_key = normalized_dictionary[0]
        query = self.attention.query(normalized_x)
        if dictionary_key.dtype != query.dtype:
            dictionary_key = dictionary_key.to(query.dtype)
        hidden = F.linear(query, dictionary_key.transpose(0, 1).contiguous())
        return self.feedforward(hidden)


class DoubleAttentionStack(nn.Module):
    """Blocks with global or stage-wise dictionaries (modules.py:359-412)."""

    def __init__(self, config: DoubleAttentionConfig, num_layers: int, *, dictionary_group_size: int | None = None,
                 feedforward_dim: int | None = None, dropout: float = 0.0) -> None:
        super().__init__()
        if num_layers <= 0:
            raise ValueError("num_layers must be positive")
        group_size = dictionary_group_size or num_layers
        if group_size <= 0:
            raise ValueError("dictionary_group_size must be positive")
        self.config = config
        self.num_layers = num_layers
        self.dictionary_group_size = group_size
        bank_count = math.ceil(num_layers / group_size)
        self.banks = nn.ModuleList(
            SharedDictionaryBank(config.routing_dim, config.dictionary_size, untied=config.untied_dictionary)
            for _ in range(bank_count)
        )
        self.blocks = nn.ModuleList(
            DoubleAttentionBlock(config, feedforward_dim=feedforward_dim, dropout=dropout) for _ in range(num_layers)
        )

    def forward(self, x: Tensor) -> Tensor:
        # One normalisation per bank per forward; every block of the group
        # reuses it, so gradients accumulate before one normalisation
        # backward (modules.py:398-412).
        x, pending = self._forward_pending(x)
        return x if pending is None else x + pending

    def _forward_pending(self, x: Tensor) -> tuple[Tensor, Tensor | None]:
        """Runs the blocks; with the fused norms the last block's feed-forward branch is returned
        unadded (``pending``), so that a following norm can add it in its own kernel."""
        normalized = tuple(bank.normalized(self.config.eps) for bank in self.banks)
        fused = all(ops.layernorm_supported(x, b.attention_norm, b.feedforward_norm) for b in self.blocks)
        pending = None
        for index, block in enumerate(self.blocks):
            bank_index = min(index // self.dictionary_group_size, len(self.banks) - 1)
            if fused:
                x, pending = block._forward_fused(x, pending, self.banks[bank_index], normalized[bank_index])
            else:
                x = block(x, self.banks[bank_index], normalized_dictionary=normalized[bank_index])
        return x, pending


class DoubleAttentionLM(nn.Module):
    """Small causal LM wrapper (modules.py:415-460)."""

    def __init__(self, vocab_size: int, max_sequence_length: int, config: DoubleAttentionConfig, num_layers: int, *,
                 dictionary_group_size: int | None = None, feedforward_dim: int | None = None,
                 dropout: float = 0.0) -> None:
        super().__init__()
        self.max_sequence_length = max_sequence_length
        self.token_embedding = nn.Embedding(vocab_size, config.model_dim)
        self.position_embedding = nn.Embedding(max_sequence_length, config.model_dim)
        self.stack = DoubleAttentionStack(config, num_layers, dictionary_group_size=dictionary_group_size,
                                          feedforward_dim=feedforward_dim, dropout=dropout)
        self.final_norm = nn.LayerNorm(config.model_dim)
        self.lm_head = nn.Linear(config.model_dim, vocab_size, bias=False)
        self.lm_head.weight = self.token_embedding.weight

    def forward(self, token_ids: Tensor, targets: Tensor | None = None) -> tuple[Tensor, Tensor | None]:
        if token_ids.ndim != 2:
            raise ValueError("token_ids must have shape [B, T]")
        length = token_ids.shape[1]
        if length > self.max_sequence_length:
            raise ValueError(f"sequence length {length} exceeds configured maximum {self.max_sequence_length}")
        positions = torch.arange(length, device=token_ids.device)
        hidden, pending = self.stack._forward_pending(
            self.token_embedding(token_ids) + self.position_embedding(positions)[None])
        if pending is not None and ops.layernorm_supported(hidden, self.final_norm):
            logits = self.lm_head(ops.add_layernorm(hidden, pending, self.final_norm)[1])
        else:
            if pending is not None:
                hidden = hidden + pending
            if ops.layernorm_supported(hidden, self.final_norm):
                logits = self.lm_head(ops.layernorm(hidden, self.final_norm))
            else:
                logits = self.lm_head(self.final_norm(hidden))
        loss = None
        if targets is not None:
            if targets.shape != token_ids.shape:
                raise ValueError("targets must match token_ids shape")
            loss = F.cross_entropy(logits.flatten(0, 1), targets.flatten())
        return logits, loss
