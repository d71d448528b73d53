"""SharedDictionaryAttention forward on the B200 against the oracle module.

Weights come from ``torch.manual_seed`` exactly as in the reference (same
parameter creation order), are cast to the kernel dtype with the module,
and the oracle runs in fp32 on their upcast with the same input.
Bar: max-abs 2e-2 and cosine >= 0.9995 on the module output.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import oracle
from double_attention_b200 import SharedDictionaryAttention, experiment_config, ops

pytestmark = pytest.mark.gpu


def _cos(a, b) -> float:
    return float(F.cosine_similarity(a.double().flatten(), b.double().flatten(), dim=0))


@pytest.mark.parametrize(
    ("name", "dtype", "batch", "length"),
    [
        ("a1", torch.float16, 8, 512),          # config 2
        ("a1", torch.bfloat16, 2, 200),
        ("qk4-s4", torch.bfloat16, 2, 256),     # config 3 width
        ("a1-r512-d1536", torch.bfloat16, 1, 1024),
        ("qk2-s1", torch.bfloat16, 2, 130),
        ("qk1-s2", torch.bfloat16, 2, 65),
        ("qk2-s2", torch.bfloat16, 1, 128),
    ],
)
def test_module_forward_matches_oracle(name, dtype, batch, length) -> None:
    dev = torch.device("cuda")
    torch.manual_seed(0)
    module = SharedDictionaryAttention(experiment_config(name)).to(dev, dtype)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(batch, length, module.config.model_dim, generator=g).to(dtype)
    with torch.no_grad():
        y, aux = module(x.to(dev), return_aux=True)
    torch.cuda.synchronize()
    assert ops.device_status(dev) == 0
    assert aux.backend == "b200" and y.dtype == dtype
    params = {k: v.detach().float().cpu() for k, v in module.state_dict().items()}
    expected, parts = oracle.attention_forward(params, x.float(), module.config, return_parts=True)
    got = y.float().cpu()
    assert (got - expected).abs().max().item() <= 2e-2
    assert _cos(got, expected) >= 0.9995
    zq = aux.routing_query.float().cpu()
    assert (zq - parts["zq"]).abs().max().item() <= 2e-2


def test_module_rejects_cpu_and_torch_backend() -> None:
    module = SharedDictionaryAttention(experiment_config("a1"))
    with pytest.raises(RuntimeError, match="B200 backend requested"):
        module(torch.randn(1, 4, 512))
    module = SharedDictionaryAttention(experiment_config("a1", backend="torch")).cuda().half()
    with pytest.raises(NotImplementedError):
        module(torch.randn(1, 4, 512, device="cuda", dtype=torch.float16))
