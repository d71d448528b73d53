"""CPU oracle for the routed-attention hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in plain PyTorch on the CPU (fp32 by default, fp64 on
request), the reference algorithm of Ahnd6474/double-attention for the hot
path the B200 kernels implement:

* ``dictionary_route``     -- src/double_attention/ops.py:16-62
* ``routed_attention``     -- src/double_attention/ops.py:65-93
* ``assemble_score_maps``  -- src/double_attention/ops.py:96-139
* ``score_scale_from_log`` -- src/double_attention/ops.py:160-161
* ``beta_from_log``        -- src/double_attention/modules.py:130-132
* ``normalize_bank``       -- src/double_attention/modules.py:45-48
* ``attention_forward``    -- SharedDictionaryAttention.forward, modules.py:190-291
* ``lm_forward``           -- DoubleAttentionLM / Stack / Block, modules.py:294-460

It is the checker, never the thing measured or shipped: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path
(``double_attention_b200``) never imports this package and has no CPU
fallback.

The oracle is pinned against golden vectors produced by running the
reference package itself (``tests/golden/make_golden.py``); see
``tests/test_oracle_golden.py``.
"""

from .reference_math import (
    assemble_score_maps,
    attention_forward,
    beta_from_log,
    dictionary_route,
    lm_forward,
    normalize_bank,
    routed_attention,
    score_scale_from_log,
)

__all__ = [
    "assemble_score_maps",
    "attention_forward",
    "beta_from_log",
    "dictionary_route",
    "lm_forward",
    "normalize_bank",
    "routed_attention",
    "score_scale_from_log",
]
