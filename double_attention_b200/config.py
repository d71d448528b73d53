"""Experiment configuration, kept semantically identical to the reference.

Mirrors ``DoubleAttentionConfig`` / ``experiment_config`` /
``experiment_names`` of src/double_attention/config.py:14-211: the same
fields, defaults, validation messages, preset table and per-preset
overrides, so configurations built for the reference build the same modules
here.  ``backend`` additionally accepts ``"b200"``; ``"auto"`` and
``"triton"`` select the B200 kernels as well (there is no other GPU
backend), while ``"torch"`` is rejected when a module runs, because this
package ships no CPU implementation.
"""

from __future__ import annotations

from dataclasses import dataclass, fields, replace
from typing import Literal

Backend = Literal["auto", "torch", "triton", "b200"]
MapCombine = Literal["weighted_sum", "concat"]
DictionaryActivation = Literal["identity", "silu"]
DictionaryAssignment = Literal["softmax", "silu"]

_BACKENDS = ("auto", "torch", "triton", "b200")


@dataclass(frozen=True)
class DoubleAttentionConfig:
    """One shared-dictionary attention experiment (config.py:14-89).

    ``routing_dim`` is the width of each Q/K branch; the total Q/K
    projection width is ``routing_dim * qk_branches``.
    """

    model_dim: int = 512
    routing_dim: int = 256
    dictionary_size: int = 512
    qk_branches: int = 1
    outer_maps: int = 1
    beta: float = 4.0
    initial_score_scale: float = 16.0
    learnable_beta: bool = False
    dictionary_activation: DictionaryActivation = "identity"
    dictionary_assignment: DictionaryAssignment = "softmax"
    dictionary_silu_gain: float = 1.0
    standardize_dictionary_logits: bool = False
    standardized_logit_scale: float | None = None
    normalize_routing_input: bool = True
    normalize_routing_output: bool = True
    q_dictionary_feedforward: bool = False
    untied_dictionary: bool = True
    output_projection: bool = True
    value_bias: bool = True
    map_combine: MapCombine = "weighted_sum"
    causal: bool = True
    backend: Backend = "auto"
    eps: float = 1e-6

    def __post_init__(self) -> None:
        for name in ("model_dim", "routing_dim", "dictionary_size", "qk_branches", "outer_maps", "beta",
                     "initial_score_scale", "dictionary_silu_gain", "eps"):
            value = getattr(self, name)
            if value <= 0:
                raise ValueError(f"{name} must be positive, got {value!r}")
        if self.standardized_logit_scale is not None and self.standardized_logit_scale <= 0:
            raise ValueError("standardized_logit_scale must be positive when provided")
        big, small = max(self.qk_branches, self.outer_maps), min(self.qk_branches, self.outer_maps)
        if big % small:
            raise ValueError(
                "qk_branches and outer_maps must divide one another so score "
                "maps can be grouped or repeated without an ambiguous mapping"
            )
        if self.backend not in _BACKENDS:
            raise ValueError(f"unsupported backend: {self.backend}")
        if self.map_combine not in ("weighted_sum", "concat"):
            raise ValueError(f"unsupported map_combine: {self.map_combine}")
        if self.dictionary_activation not in ("identity", "silu"):
            raise ValueError(f"unsupported dictionary activation: {self.dictionary_activation}")
        if self.dictionary_assignment not in ("softmax", "silu"):
            raise ValueError(f"unsupported dictionary assignment: {self.dictionary_assignment}")
        if self.map_combine == "concat" and not self.output_projection:
            raise ValueError("concat map combination requires output_projection=True")

    @property
    def total_qk_width(self) -> int:
        return self.routing_dim * self.qk_branches

    def with_updates(self, **updates: object) -> "DoubleAttentionConfig":
        return replace(self, **updates)


# Preset table (config.py:92-119): name -> (Q/K branches, outer maps, routing
# width, activation, standardize logits, explicit pre-beta scale, input norm,
# output norm).  The table is data the presets are defined by; it must match
# the reference entry for entry.
_PRESETS: dict[str, tuple[int, int, int, str, bool, float | None, bool, bool]] = {
    "a1": (1, 1, 256, "identity", False, None, True, True),
    "a1-silu": (1, 1, 256, "silu", False, None, True, True),
    "a1-silu-logitnorm": (1, 1, 256, "silu", True, None, False, True),
    "a1-silu-logitnorm-t1": (1, 1, 256, "silu", True, 0.25, False, True),
    "a1-r512-d512": (1, 1, 512, "identity", False, None, True, True),
    "a1-r512-d1024": (1, 1, 512, "identity", False, None, True, True),
    "a1-r512-d1536": (1, 1, 512, "identity", False, None, True, True),
    "a1-r512-d1536-qffn": (1, 1, 512, "identity", False, None, True, True),
    "a1-r512-d2855-qffn": (1, 1, 512, "identity", False, None, True, True),
    "a1-r512-d1764-qffn-l8": (1, 1, 512, "identity", False, None, True, True),
    "a1-d1536": (1, 1, 256, "identity", False, None, True, True),
    "a1-d1536-qffn": (1, 1, 256, "identity", False, None, True, True),
    "a1-no-softmax": (1, 1, 256, "identity", False, None, True, True),
    "a1-no-softmax-g4": (1, 1, 256, "identity", False, None, True, True),
    "a1-no-qnorm": (1, 1, 256, "identity", False, None, False, True),
    "a1-no-dpnorm": (1, 1, 256, "identity", False, None, True, False),
    "a1-no-norm": (1, 1, 256, "identity", False, None, False, False),
    "qk2-s1": (2, 1, 256, "identity", False, None, True, True),
    "qk1-s2": (1, 2, 256, "identity", False, None, True, True),
    "qk2-s2": (2, 2, 256, "identity", False, None, True, True),
    "qk4-s4": (4, 4, 128, "identity", False, None, True, True),
}

_R512 = {"beta": 4.0 * (2.0**0.5), "initial_score_scale": 512.0**0.5}

# Per-preset overrides (config.py:121-170): the r512 presets keep the
# dictionary-logit and outer-score variances of the 256-wide baseline.
_PRESET_OVERRIDES: dict[str, dict[str, object]] = {
    "a1-r512-d512": {"dictionary_size": 512, **_R512},
    "a1-r512-d1024": {"dictionary_size": 1024, **_R512},
    "a1-r512-d1536": {"dictionary_size": 1536, **_R512},
    "a1-r512-d1536-qffn": {"dictionary_size": 1536, **_R512, "q_dictionary_feedforward": True},
    "a1-r512-d2855-qffn": {"dictionary_size": 2855, **_R512, "q_dictionary_feedforward": True},
    "a1-r512-d1764-qffn-l8": {"dictionary_size": 1764, **_R512, "q_dictionary_feedforward": True},
    "a1-d1536": {"dictionary_size": 1536},
    "a1-d1536-qffn": {"dictionary_size": 1536, "q_dictionary_feedforward": True},
    "a1-no-softmax": {"dictionary_assignment": "silu", "dictionary_silu_gain": 1.0},
    "a1-no-softmax-g4": {"dictionary_assignment": "silu", "dictionary_silu_gain": 4.0},
}

_PRESET_FIELDS = (
    "qk_branches",
    "outer_maps",
    "routing_dim",
    "dictionary_activation",
    "standardize_dictionary_logits",
    "standardized_logit_scale",
    "normalize_routing_input",
    "normalize_routing_output",
)


def experiment_config(name: str, **overrides: object) -> DoubleAttentionConfig:
    """Build a named experiment variant (config.py:173-207)."""
    key = name.lower().replace("_", "-")
    if key not in _PRESETS:
        choices = ", ".join(sorted(_PRESETS))
        raise ValueError(f"unknown experiment {name!r}; choose one of: {choices}")
    values: dict[str, object] = dict(zip(_PRESET_FIELDS, _PRESETS[key]))
    values.update(_PRESET_OVERRIDES.get(key, {}))
    values.update(overrides)
    return DoubleAttentionConfig(**values)


def experiment_names() -> tuple[str, ...]:
    """All preset names, in table order (config.py:210-211)."""
    return tuple(_PRESETS)


def config_field_names() -> tuple[str, ...]:
    return tuple(f.name for f in fields(DoubleAttentionConfig))
