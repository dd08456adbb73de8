"""CPU checks of the C-ABI boundary: the library loads and exports every entry
point declared in include/h3_b200.h (no compute calls: there is no GPU here)."""
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    text = open(os.path.join(ROOT, "include", "h3_b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char \*)\s*(h3_\w+)\s*\(", text, re.M)))


def test_header_declares_entry_points():
    names = _declared()
    for required in ("h3_rms_norm", "h3_swiglu", "h3_rms_modulate", "h3_rope", "h3_gated_residual",
                     "h3_gated_residual_rms_modulate", "h3_qk_norm_rope", "h3_rope_cache", "h3_mha",
                     "h3_linear", "h3_linear_swiglu", "h3_linear_gated_residual"):
        assert required in names


def test_library_exports_every_declared_symbol():
    import h3b200
    lib = h3b200.load()
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert lib.h3_abi_version() == 1
    assert lib.h3_status_string(2) == b"bad shape"


def test_python_signatures_cover_header():
    import h3b200._lib as L
    assert set(_declared()) <= set(L.SIGNATURES)


def test_ops_refuse_cpu_tensors():
    import torch
    import h3b200
    x = torch.zeros(2, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        h3b200.h3_gated_residual(x, x, x)
