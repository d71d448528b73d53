"""The CPU oracle is pinned to golden vectors made by the reference itself.

``tests/golden/reference_golden.pt`` was produced by running the reference
package (tests/golden/make_golden.py) on the seeded inputs of
``tests/golden/cases.py``; here the oracle reproduces every stored output and
gradient, and this package's module constructors reproduce the reference's
parameters bit for bit under the same seeds.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

import oracle

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN_DIR))
import cases  # noqa: E402

GOLD = torch.load(GOLDEN_DIR / "reference_golden.pt", weights_only=False)
SAME_TORCH = GOLD["torch_version"] == str(torch.__version__)


def _check(actual: torch.Tensor, stored, atol: float = 2e-5, rtol: float = 1e-4) -> None:
    if isinstance(stored, torch.Tensor):
        torch.testing.assert_close(actual.detach(), stored, atol=atol, rtol=rtol)
    else:  # checksum: sum, |sum|, sum of squares, first values
        got = cases.checksum(actual)
        scale = max(1.0, abs(stored[1]))
        assert abs(got[0] - stored[0]) <= 1e-4 * scale, (got[0], stored[0])
        assert abs(got[1] - stored[1]) <= 1e-4 * scale
        assert abs(got[2] - stored[2]) <= 1e-4 * max(1.0, stored[2])
        torch.testing.assert_close(torch.tensor(got[3:]), torch.tensor(stored[3:]), atol=atol, rtol=rtol)


@pytest.mark.parametrize("index", range(len(cases.ROUTE_CASES)))
def test_oracle_route_matches_reference(index: int) -> None:
    case = cases.ROUTE_CASES[index]
    gold = GOLD["routes"][index]
    x, dk, dv, beta, dy = cases.route_inputs(case)
    act, std, scale, nin, nout, assign, gain = case["flags"]
    xs = [t.clone().requires_grad_() for t in (x, dk, dv, beta)]
    y = oracle.dictionary_route(xs[0], xs[1], xs[2], xs[3], activation=act, assignment=assign, silu_gain=gain,
                                standardize_logits=std, standardized_logit_scale=scale, normalize_input=nin,
                                normalize_output=nout)
    y.backward(dy)
    _check(y, gold["y"])
    for t, g in zip(xs, gold["grads"]):
        if g is None:
            assert t.grad is None or not t.grad.abs().any()
        else:
            _check(t.grad, g, atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("index", range(len(cases.ATTENTION_CASES)))
def test_oracle_attention_matches_reference(index: int) -> None:
    case = cases.ATTENTION_CASES[index]
    gold = GOLD["attention"][index]
    q, k, v, sc, dy = cases.attention_inputs(case)
    xs = [z.clone().requires_grad_() for z in (q, k, v, sc)]
    y = oracle.routed_attention(*xs, causal=case["causal"])
    y.backward(dy)
    _check(y, gold["y"])
    for t, g in zip(xs, gold["grads"]):
        _check(t.grad, g, atol=1e-4, rtol=1e-3)


def test_oracle_assemble_matches_reference() -> None:
    a = GOLD["assemble"]
    for c in a["cases"]:
        q, k = (a["q"], a["k"]) if c["branches"] == 4 else (a["q"][:, :1], a["k"][:, :1])
        got = oracle.assemble_score_maps(q, k, c["maps"])
        for x, y in zip(got, c["out"]):
            torch.testing.assert_close(x, y)


@pytest.mark.skipif(not SAME_TORCH, reason="seeded parameter streams are only reproducible on the same torch")
@pytest.mark.parametrize("index", range(len(cases.MODULE_CASES)))
def test_module_weights_and_oracle_forward_match_reference(index: int) -> None:
    from double_attention_b200 import SharedDictionaryAttention, experiment_config

    case = cases.MODULE_CASES[index]
    gold = GOLD["modules"][index]
    torch.manual_seed(case["seed"])
    module = SharedDictionaryAttention(experiment_config(case["name"], **case["overrides"]))
    # identical parameter creation order, state_dict keys and values
    assert [k for k, _ in module.named_parameters()] == gold["param_order"]
    state = module.state_dict()
    assert list(state) == list(gold["state_checksums"])
    for key, stored in gold["state_checksums"].items():
        _check(state[key], stored, atol=0, rtol=0)
    # the oracle forward/backward on those weights reproduces the reference
    params = {k: v.detach().clone().requires_grad_(v.is_floating_point()) for k, v in state.items()}
    x, dy = cases.module_inputs(case)
    xg = x.clone().requires_grad_()
    y = oracle.attention_forward(params, xg, module.config)
    y.backward(dy)
    assert abs(float(y.double().sum()) - gold["y_sum"]) <= 1e-3 * max(1.0, abs(gold["y_sum"]))
    torch.testing.assert_close(y[0, 0, :16].detach(), gold["y_head"], atol=2e-5, rtol=1e-4)
    _check(y, gold["y"])
    _check(xg.grad, gold["x_grad"], atol=1e-4, rtol=1e-3)
    for key, stored in gold["grad_checksums"].items():
        _check(params[key].grad, stored, atol=1e-4, rtol=1e-3)


@pytest.mark.skipif(not SAME_TORCH, reason="seeded parameter streams are only reproducible on the same torch")
def test_lm_weights_and_oracle_forward_match_reference() -> None:
    from double_attention_b200 import DoubleAttentionLM, experiment_config

    c = cases.LM_CASE
    gold = GOLD["lm"]
    torch.manual_seed(c["seed"])
    lm = DoubleAttentionLM(c["vocab"], c["max_len"], experiment_config("a1", **c["overrides"]), c["layers"],
                           dictionary_group_size=c["group"], feedforward_dim=c["ffn"])
    assert [k for k, _ in lm.named_parameters()] == gold["param_order"]
    state = lm.state_dict()
    for key, stored in gold["state_checksums"].items():
        _check(state[key], stored, atol=0, rtol=0)
    params = {k: v.detach().clone().requires_grad_(v.is_floating_point()) for k, v in state.items()}
    params["lm_head.weight"] = params["token_embedding.weight"]  # tied
    ids, targets = cases.lm_inputs(c)
    logits, loss = oracle.lm_forward(params, ids, targets, lm.stack.config, c["layers"], c["group"])
    loss.backward()
    torch.testing.assert_close(logits.detach(), gold["logits"], atol=2e-5, rtol=1e-4)
    assert abs(float(loss) - gold["loss"]) <= 1e-5
    for key, stored in gold["grad_checksums"].items():
        if key == "lm_head.weight":
            continue
        _check(params[key].grad, stored, atol=1e-4, rtol=1e-3)


def test_reference_anchor_value() -> None:
    """The documented anchor of the a1 preset (seed 0, x = randn(2, 64, 512))."""
    gold = GOLD["modules"][0]
    assert cases.MODULE_CASES[0]["name"] == "a1"
    assert abs(gold["y_sum"]) > 0
