"""The C-ABI library loads on a CPU-only host and exports every entry point
declared in include/*.h; no compute is called here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from double_attention_b200 import _lib

REPO = Path(__file__).resolve().parent.parent


def declared_symbols() -> list[str]:
    names = []
    for header in sorted((REPO / "include").glob("*.h")):
        names += re.findall(r"^DA_API\s+[\w\s\*]+?\b(da_\w+)\s*\(", header.read_text(), flags=re.M)
    return names


def test_header_declares_entry_points() -> None:
    names = declared_symbols()
    for required in ("da_dict_norm_fwd", "da_route_fwd", "da_attn_fwd", "da_gemm", "da_status_string"):
        assert required in names


def test_library_loads_and_exports_every_declared_symbol() -> None:
    handle = _lib.lib()
    for name in declared_symbols():
        assert hasattr(handle, name), name
    assert b"sm_100a" in handle.da_version()
    assert handle.da_status_string(_lib.DA_ERR_SHAPE) == b"unsupported or inconsistent shape"
    assert _lib.kernel_launches() >= 0


def test_bound_signatures_cover_compute_entry_points() -> None:
    for name in declared_symbols():
        if name in ("da_version", "da_status_string", "da_last_cuda_error", "da_kernel_launches"):
            continue
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_argument_validation_happens_before_any_device_work() -> None:
    handle = _lib.lib()
    # null pointers are rejected on the host (no CUDA call is made)
    assert handle.da_route_fwd(*([None] * 1), *([0] * 8), *([None] * 4), ctypes.c_float(1e-6), 1, 1,
                               *([None] * 5), 0, None, None) == _lib.DA_ERR_NULL
    with pytest.raises(ValueError):
        _lib.check("da_gemm", _lib.DA_ERR_SHAPE)
    with pytest.raises(NotImplementedError):
        _lib.check("da_attn_fwd", _lib.DA_ERR_UNSUPPORTED)


def test_layernorm_entry_points_validate_on_the_host() -> None:
    handle = _lib.lib()
    f32 = ctypes.c_float(1e-5)
    # a null input, then an unsupported width: both refused before any CUDA call
    assert handle.da_add_layernorm_fwd(None, None, 0, None, None, 8, 512, f32, None, None, 1, None, None,
                                       None) == _lib.DA_ERR_NULL
    buf = (ctypes.c_float * 4096)()
    p = ctypes.addressof(buf)
    assert handle.da_add_layernorm_fwd(p, None, 0, p, p, 8, 500, f32, None, p, 1, p, p, None) == _lib.DA_ERR_SHAPE
    assert handle.da_add_layernorm_fwd(p, None, 0, p, p, 8, 512, f32, None, p, 7, p, p, None) == _lib.DA_ERR_DTYPE
    # the backward's partial-sum buffer must have the queried number of blocks
    blocks = handle.da_layernorm_bwd_blocks(1)
    assert blocks == 1
    assert handle.da_add_layernorm_bwd(p, 1, None, p, p, p, p, 1, 512, p, None, 0, p, blocks + 1, None, None,
                                       None) == _lib.DA_ERR_WORKSPACE


def test_fused_norms_only_for_cuda_fp32_rows() -> None:
    import torch
    import torch.nn as nn

    from double_attention_b200 import ops

    norm = nn.LayerNorm(512)
    assert not ops.layernorm_supported(torch.zeros(2, 512), norm)            # CPU tensor: plain nn.LayerNorm
    assert not ops.layernorm_supported(torch.zeros(2, 500), nn.LayerNorm(500))
