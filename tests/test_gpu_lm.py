"""DoubleAttentionLM on the B200 kernels against the oracle LM (training configuration).

fp32 parameters under bf16 autocast, one dictionary bank shared by every
block (normalised once per forward, so the bank gradient collects every
block's contribution before one normalisation backward).  Bar: loss within
2e-3 relative; every parameter gradient with cosine >= 0.999 and max-abs within
3e-2 * max(1, max |g_ref|) (scalars and per-map vectors: 5e-2 relative
+ 5e-2 absolute).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import oracle
from double_attention_b200 import DoubleAttentionLM, experiment_config, ops

pytestmark = pytest.mark.gpu


def _cos(a, b) -> float:
    return float(F.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


@pytest.mark.parametrize(("preset", "layers", "group"), [("a1", 2, 2), ("qk4-s4", 2, 1)])
def test_lm_training_gradients_match_oracle(preset: str, layers: int, group: int) -> None:
    dev = torch.device("cuda")
    vocab, seq, batch = 256, 192, 2
    torch.manual_seed(0)
    model = DoubleAttentionLM(vocab, seq, experiment_config(preset), layers, dictionary_group_size=group,
                              feedforward_dim=1024).to(dev)
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, vocab, (batch, seq + 1), generator=g)
    x, y = ids[:, :-1], ids[:, 1:]
    with torch.autocast("cuda", dtype=torch.bfloat16):
        _, loss = model(x.to(dev), y.to(dev))
    loss.backward()
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0

    params = {k: v.detach().float().cpu().requires_grad_() for k, v in model.named_parameters()}
    state = {k: v.detach().float().cpu() for k, v in model.state_dict().items()}
    state.update(params)
    state["lm_head.weight"] = state["token_embedding.weight"]
    _, ref_loss = oracle.lm_forward(state, x, y, model.stack.config, layers, group)
    ref_loss.backward()
    # an untrained tied-embedding LM has large logits, so the loss is large too
    assert abs(loss.item() - ref_loss.item()) <= 2e-3 * max(1.0, abs(ref_loss.item())), (loss.item(), ref_loss.item())
    failures = []
    for key, p in model.named_parameters():
        ref = params[key].grad
        assert p.grad is not None and ref is not None, key
        got = p.grad.float().cpu()
        if ref.numel() <= 4:
            tol = 5e-2 * ref.abs().max().item() + 5e-2
            if (got - ref).abs().max().item() > tol:
                failures.append(f"{key}: {got.tolist()} vs {ref.tolist()}")
            continue
        bound = 3e-2 * max(1.0, ref.abs().max().item())
        err, cos = (got - ref).abs().max().item(), _cos(got, ref)
        if err > bound or cos < 0.999:
            failures.append(f"{key}: max-abs {err:.3e} (bound {bound:.3e}) cosine {cos:.6f}")
    assert not failures, "; ".join(failures)
