"""B200-native (sm_100a) routed-attention hot path of Double Attention.

Drop-in for the reference package's module/config API
(src/double_attention/__init__.py): the same constructors, parameters and
state_dict keys, with the dictionary normalisation, fused Q/K projection,
dictionary route and outer routed attention running in hand-written
tcgen05 kernels (``libda_b200.so``, C ABI in ``include/da_b200.h``).
"""

from .config import DoubleAttentionConfig, experiment_config, experiment_names
from .graphs import GraphedModuleStep
from .modules import (
    DoubleAttentionAux,
    DoubleAttentionBlock,
    DoubleAttentionLM,
    DoubleAttentionStack,
    SharedDictionaryAttention,
    SharedDictionaryBank,
)
from .ops import assemble_score_maps, dictionary_route, routed_attention

__all__ = [
    "DoubleAttentionAux",
    "DoubleAttentionBlock",
    "DoubleAttentionConfig",
    "DoubleAttentionLM",
    "DoubleAttentionStack",
    "GraphedModuleStep",
    "SharedDictionaryAttention",
    "SharedDictionaryBank",
    "assemble_score_maps",
    "dictionary_route",
    "experiment_config",
    "experiment_names",
    "routed_attention",
]
