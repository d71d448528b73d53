"""Host-side behaviour that needs no GPU: configuration semantics, module
construction / state_dict layout, and the loud failure on CPU tensors.

Mirrors the CPU tests of the reference (tests/test_modules.py) for the
parts this package implements."""

from __future__ import annotations

import math

import pytest
import torch

from double_attention_b200 import (
    DoubleAttentionBlock,
    DoubleAttentionConfig,
    DoubleAttentionLM,
    DoubleAttentionStack,
    SharedDictionaryAttention,
    SharedDictionaryBank,
    experiment_config,
    experiment_names,
)
from double_attention_b200 import ops


def small(name: str, **kw) -> DoubleAttentionConfig:
    values = {"model_dim": 32, "routing_dim": 8, "dictionary_size": 16}
    values.update(kw)
    return experiment_config(name, **values)


def test_preset_table_matches_reference_names() -> None:
    assert experiment_names()[:3] == ("a1", "a1-silu", "a1-silu-logitnorm")
    assert len(experiment_names()) == 21
    assert experiment_config("A1").routing_dim == 256
    with pytest.raises(ValueError, match="unknown experiment"):
        experiment_config("nope")


@pytest.mark.parametrize("name,size", [("a1-r512-d512", 512), ("a1-r512-d1024", 1024), ("a1-r512-d1536", 1536),
                                       ("a1-r512-d2855-qffn", 2855), ("a1-r512-d1764-qffn-l8", 1764)])
def test_r512_presets_calibrate_temperature(name: str, size: int) -> None:
    cfg = experiment_config(name)
    assert cfg.routing_dim == 512 and cfg.dictionary_size == size
    assert cfg.beta == pytest.approx(4.0 * 2**0.5)
    assert cfg.initial_score_scale == pytest.approx(512**0.5)


@pytest.mark.parametrize("name,nin,nout", [("a1", True, True), ("a1-no-qnorm", False, True),
                                           ("a1-no-dpnorm", True, False), ("a1-no-norm", False, False)])
def test_normalisation_presets(name: str, nin: bool, nout: bool) -> None:
    cfg = experiment_config(name)
    assert cfg.normalize_routing_input is nin and cfg.normalize_routing_output is nout


def test_qk4_s4_and_direct_silu_presets() -> None:
    cfg = experiment_config("qk4-s4")
    assert (cfg.qk_branches, cfg.outer_maps, cfg.routing_dim, cfg.total_qk_width) == (4, 4, 128, 512)
    assert experiment_config("a1-no-softmax-g4").dictionary_silu_gain == 4.0
    assert experiment_config("a1-silu-logitnorm-t1").standardized_logit_scale == 0.25


def test_config_validation_messages() -> None:
    with pytest.raises(ValueError, match="divide one another"):
        DoubleAttentionConfig(qk_branches=3, outer_maps=2)
    with pytest.raises(ValueError, match="must be positive"):
        DoubleAttentionConfig(beta=0.0)
    with pytest.raises(ValueError, match="concat map combination"):
        DoubleAttentionConfig(map_combine="concat", output_projection=False)
    with pytest.raises(ValueError, match="unsupported backend"):
        DoubleAttentionConfig(backend="tpu")


def test_module_parameters_and_state_dict_keys() -> None:
    m = SharedDictionaryAttention(small("qk2-s2"))
    assert set(m.state_dict()) == {"query.weight", "key.weight", "value.weight", "value.bias", "bank.raw_key",
                                   "bank.raw_value", "log_score_scales", "log_beta", "map_mix_logits",
                                   "output.weight"}
    assert not any("fused" in k for k in m.state_dict())
    assert m.log_score_scales.shape == (2,) and m.log_score_scales[0] != m.log_score_scales[1]
    assert float(m.beta) == pytest.approx(4.0)
    tied = SharedDictionaryAttention(small("a1", untied_dictionary=False))
    assert tied.bank.raw_value is None
    k, v = tied.bank.normalized()
    assert k.data_ptr() == v.data_ptr()


def test_stack_banks_and_lm_tying() -> None:
    stack = DoubleAttentionStack(small("a1"), num_layers=8, dictionary_group_size=4, feedforward_dim=48)
    assert len(stack.banks) == 2
    assert len(DoubleAttentionStack(small("a1"), num_layers=3, feedforward_dim=48).banks) == 1
    lm = DoubleAttentionLM(41, 12, small("a1"), 2, feedforward_dim=48)
    assert lm.lm_head.weight is lm.token_embedding.weight
    with pytest.raises(ValueError, match="exceeds configured maximum"):
        lm(torch.zeros(1, 13, dtype=torch.long))


def test_qffn_block_validation() -> None:
    cfg = experiment_config("a1-d1536-qffn", model_dim=32, routing_dim=8, dictionary_size=48)
    with pytest.raises(ValueError, match="feedforward_dim == dictionary_size"):
        DoubleAttentionBlock(cfg, feedforward_dim=64)
    block = DoubleAttentionBlock(cfg, feedforward_dim=48)
    assert isinstance(block.feedforward[0], torch.nn.Identity)


def test_forward_fails_loudly_without_gpu_kernels() -> None:
    m = SharedDictionaryAttention(small("a1"))
    with pytest.raises(RuntimeError, match="B200 backend requested but unavailable"):
        m(torch.randn(1, 4, 32))
    with pytest.raises(ValueError, match="expected x with shape"):
        m(torch.randn(1, 4, 31))
    with pytest.raises(NotImplementedError, match="backend='torch'"):
        SharedDictionaryAttention(small("a1", backend="torch"))(torch.randn(1, 4, 32))


def test_score_scale_and_assembly_helpers() -> None:
    ls = torch.tensor([math.log(0.1), math.log(16.0), math.log(5000.0)])
    torch.testing.assert_close(ops.score_scale_from_log(ls), torch.tensor([0.25, 16.0, 1024.0]))
    q = torch.randn(2, 4, 5, 8)
    k = torch.randn(2, 4, 5, 8)
    sq, sk = ops.assemble_score_maps(q, k, 2)
    assert sq.shape == (2, 2, 5, 16)
    torch.testing.assert_close(sq[:, 0, :, :8], q[:, 0] * 2 ** -0.25)
    rq, _ = ops.assemble_score_maps(q[:, :1], k[:, :1], 2)
    torch.testing.assert_close(rq[:, 0], rq[:, 1])
    assert ops._map_layout(4, 2) == (2, [0, 2])
    assert ops._map_layout(1, 2) == (1, [0, 0])
    assert ops._map_layout(4, 4) == (1, [0, 1, 2, 3])
