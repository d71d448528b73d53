"""Generate the golden vectors that pin the CPU oracle to the reference.

Runs the reference package (Ahnd6474/double-attention, its pure-PyTorch
``backend="torch"`` path) on the seeded CPU inputs of ``cases.py`` and
stores outputs and gradients in ``reference_golden.pt``.  It needs the
reference source tree and is run by hand in the build container:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py

Nothing at test time imports the reference.  Inputs are rebuilt from the
recipes in ``cases.py``; tensors larger than 16 Ki elements are stored as
checksums (sum, |sum|, sum of squares, first values).  Module cases store
the seed that builds their weights plus per-tensor checksums of the
reference's state_dict, so a re-implementation with the same parameter
creation order can show it builds identical weights.
"""

from __future__ import annotations

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))

import cases  # noqa: E402

SMALL = 16384


def keep(t: torch.Tensor):
    t = t.detach()
    return t.clone() if t.numel() <= SMALL else cases.checksum(t)


def main() -> None:
    try:
        from double_attention import DoubleAttentionLM, SharedDictionaryAttention, experiment_config
        from double_attention.ops import assemble_score_maps, dictionary_route_reference, routed_attention_reference
    except ImportError as exc:
        raise SystemExit(f"reference package not importable ({exc}); set PYTHONPATH=<reference>/src") from exc
    torch.set_num_threads(4)
    out: dict[str, object] = {"torch_version": str(torch.__version__)}

    routes = []
    for case in cases.ROUTE_CASES:
        x, dk, dv, beta, dy = cases.route_inputs(case)
        act, std, scale, nin, nout, assign, gain = case["flags"]
        xs = [t.clone().requires_grad_() for t in (x, dk, dv, beta)]
        y = dictionary_route_reference(
            xs[0], xs[1], xs[2], xs[3], activation=act, assignment=assign, silu_gain=gain,
            standardize_logits=std, standardized_logit_scale=scale, normalize_input=nin, normalize_output=nout,
        )
        y.backward(dy)
        routes.append({"y": keep(y), "grads": [keep(t.grad) if t.grad is not None else None for t in xs]})
    out["routes"] = routes

    attns = []
    for case in cases.ATTENTION_CASES:
        q, k, v, sc, dy = cases.attention_inputs(case)
        xs = [z.clone().requires_grad_() for z in (q, k, v, sc)]
        y = routed_attention_reference(*xs, causal=case["causal"])
        y.backward(dy)
        attns.append({"y": keep(y), "grads": [keep(z.grad) for z in xs]})
    out["attention"] = attns

    g = torch.Generator().manual_seed(300)
    q = torch.randn(2, 4, 5, 8, generator=g)
    k = torch.randn(2, 4, 5, 8, generator=g)
    assemble = [{"maps": m, "branches": 4, "out": tuple(z.clone() for z in assemble_score_maps(q, k, m))} for m in (1, 2, 4)]
    assemble.append({"maps": 2, "branches": 1, "out": tuple(z.clone() for z in assemble_score_maps(q[:, :1], k[:, :1], 2))})
    out["assemble"] = {"q": q, "k": k, "cases": assemble}

    modules = []
    for case in cases.MODULE_CASES:
        torch.manual_seed(case["seed"])
        module = SharedDictionaryAttention(experiment_config(case["name"], backend="torch", **case["overrides"]))
        x, dy = cases.module_inputs(case)
        xg = x.clone().requires_grad_()
        y = module(xg)
        y.backward(dy)
        modules.append({
            "y_sum": float(y.detach().double().sum()),
            "y_head": y[0, 0, :16].detach().clone(),
            "y": keep(y),
            "x_grad": keep(xg.grad),
            "state_checksums": {k: cases.checksum(v) for k, v in module.state_dict().items()},
            "param_order": [k for k, _ in module.named_parameters()],
            "grad_checksums": {k: cases.checksum(p.grad) for k, p in module.named_parameters() if p.grad is not None},
        })
    out["modules"] = modules

    c = cases.LM_CASE
    torch.manual_seed(c["seed"])
    cfg = experiment_config("a1", backend="torch", **c["overrides"])
    lm = DoubleAttentionLM(c["vocab"], c["max_len"], cfg, c["layers"], dictionary_group_size=c["group"],
                           feedforward_dim=c["ffn"])
    ids, targets = cases.lm_inputs(c)
    logits, loss = lm(ids, targets)
    loss.backward()
    out["lm"] = {
        "logits": logits.detach().clone(), "loss": float(loss.detach()),
        "state_checksums": {k: cases.checksum(v) for k, v in lm.state_dict().items()},
        "param_order": [k for k, _ in lm.named_parameters()],
        "grad_checksums": {k: cases.checksum(p.grad) for k, p in lm.named_parameters() if p.grad is not None},
    }

    path = HERE / "reference_golden.pt"
    torch.save(out, path)
    print(f"wrote {path} ({path.stat().st_size / 1024:.0f} KiB)")


if __name__ == "__main__":
    main()
