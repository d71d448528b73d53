"""Seeded input recipes shared by the golden generator and the tests.

The golden file stores outputs (and small inputs); larger inputs are
rebuilt from these recipes so the fixture stays small.  The recipes use
``torch.Generator`` streams on the CPU, which are deterministic for a given
torch version (the fixture records the version it was made with).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

# (activation, standardize, scale, normalize_input, normalize_output,
#  assignment, silu_gain): the route variants of the reference parity suite
# (tests/test_triton_parity.py:113-127, :200-233) plus the wide preset.
ROUTE_CASES = [
    dict(seed=100, x=(2, 3, 17, 64), m=128, beta=4.0, flags=("identity", False, None, True, True, "softmax", 1.0)),
    dict(seed=101, x=(2, 3, 17, 64), m=128, beta=4.0, flags=("silu", False, None, True, True, "softmax", 1.0)),
    dict(seed=102, x=(2, 3, 17, 64), m=128, beta=4.0, flags=("silu", True, None, False, True, "softmax", 1.0)),
    dict(seed=103, x=(2, 3, 17, 64), m=128, beta=4.0, flags=("silu", True, 0.25, False, True, "softmax", 1.0)),
    dict(seed=104, x=(2, 3, 17, 64), m=128, beta=4.0, flags=("identity", False, None, False, True, "softmax", 1.0)),
    dict(seed=105, x=(2, 3, 17, 64), m=128, beta=4.0, flags=("identity", False, None, True, False, "softmax", 1.0)),
    dict(seed=106, x=(2, 3, 17, 64), m=128, beta=4.0, flags=("identity", False, None, False, False, "softmax", 1.0)),
    dict(seed=142, x=(1, 2, 11, 256), m=512, beta=4.0, flags=("identity", False, None, True, True, "silu", 1.0)),
    dict(seed=145, x=(1, 2, 11, 256), m=512, beta=4.0, flags=("identity", False, None, True, True, "silu", 4.0)),
    dict(seed=131, x=(1, 2, 7, 512), m=1536, beta=4.0 * 2.0**0.5,
         flags=("identity", False, None, True, True, "softmax", 1.0)),
]

# (batch, maps, T, R, D, causal, scales): tests/test_triton_parity.py:424-518
ATTENTION_CASES = [
    dict(seed=200, shape=(2, 2, 65, 64), d=96, causal=True, scales=[12.0, 17.0]),
    dict(seed=201, shape=(2, 2, 65, 64), d=96, causal=False, scales=[12.0, 17.0]),
    dict(seed=202, shape=(1, 4, 64, 128), d=512, causal=True, scales=[12.0] * 4),
    dict(seed=203, shape=(1, 2, 257, 64), d=80, causal=True, scales=[11.0, 15.0]),
]


def route_inputs(case: dict, dtype: torch.dtype = torch.float32):
    g = torch.Generator().manual_seed(case["seed"])
    x = torch.randn(*case["x"], generator=g)
    r = case["x"][-1]
    dk = F.normalize(torch.randn(r, case["m"], generator=g), dim=0)
    dv = F.normalize(torch.randn(r, case["m"], generator=g), dim=0)
    dy = torch.randn(*case["x"], generator=g)
    beta = torch.tensor(case["beta"])
    return [t.to(dtype) for t in (x, dk, dv, beta, dy)]


def attention_inputs(case: dict, dtype: torch.dtype = torch.float32):
    g = torch.Generator().manual_seed(case["seed"])
    b, s, t, r = case["shape"]
    q = F.normalize(torch.randn(b, s, t, r, generator=g), dim=-1)
    k = F.normalize(torch.randn(b, s, t, r, generator=g), dim=-1)
    v = torch.randn(b, t, case["d"], generator=g)
    dy = torch.randn(b, s, t, case["d"], generator=g)
    scales = torch.tensor(case["scales"])
    return [z.to(dtype) for z in (q, k, v, scales, dy)]


# Module cases: (preset, torch.manual_seed for the weights, x shape, overrides)
MODULE_CASES = [
    dict(name="a1", seed=0, shape=(2, 64, 512), overrides={}),
    dict(name="qk4-s4", seed=1, shape=(2, 32, 512), overrides={}),
    dict(name="a1-r512-d1536", seed=2, shape=(1, 16, 512), overrides={}),
    dict(name="qk2-s1", seed=3, shape=(1, 9, 32), overrides={"model_dim": 32, "routing_dim": 8, "dictionary_size": 16}),
    dict(name="qk1-s2", seed=4, shape=(1, 9, 32), overrides={"model_dim": 32, "routing_dim": 8, "dictionary_size": 16}),
]


def module_inputs(case: dict):
    g = torch.Generator().manual_seed(case["seed"] + 1000)
    x = torch.randn(*case["shape"], generator=g)
    dy = torch.randn(*case["shape"], generator=g)
    return x, dy


LM_CASE = dict(seed=5, vocab=41, max_len=12, layers=2, group=2, ffn=48, ids_seed=6, ids_shape=(2, 9),
               overrides={"model_dim": 32, "routing_dim": 8, "dictionary_size": 16})


def lm_inputs(case: dict = LM_CASE):
    g = torch.Generator().manual_seed(case["ids_seed"])
    ids = torch.randint(0, case["vocab"], case["ids_shape"], generator=g)
    return ids, ids.roll(-1, dims=1)


def checksum(t: torch.Tensor) -> list[float]:
    """Order-insensitive summary of a tensor plus its first values."""
    t = t.detach().double().flatten()
    return [float(t.sum()), float(t.abs().sum()), float(t.square().sum()), *map(float, t[:4])]
