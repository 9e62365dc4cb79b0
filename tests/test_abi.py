"""The C-ABI library: loads, exports every declared symbol, validates
parameters on the host.  No kernel is launched (runs without a GPU)."""
import ctypes
import os
import re

import pytest

from conftest import PKG_DIR, REPO

HEADER = os.path.join(REPO, "include", "fa_sm100.h")
LIB = os.path.join(PKG_DIR, "flash_attention", "libfa_sm100.so")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"FA_API\s+[\w\s\*]*?\b(fa_sm100_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "fa_sm100_fwd" in names and "fa_sm100_check_params" in names
    assert len(names) >= 7


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} not exported"


def test_params_layout_matches_binding():
    from flash_attention import _C

    assert _C.lib.fa_sm100_params_size() == ctypes.sizeof(_C.FaParams)


def _params(**kw):
    from flash_attention import _C

    p = _C.FaParams()
    p.batch, p.seqlen_q, p.seqlen_k, p.heads, p.heads_k, p.head_dim = 1, 128, 128, 2, 2, 64
    p.q = p.k = p.v = p.o = 1 << 20
    p.q_batch_stride = p.k_batch_stride = p.v_batch_stride = p.o_batch_stride = 128 * 2 * 64
    p.q_row_stride = p.k_row_stride = p.v_row_stride = p.o_row_stride = 2 * 64
    p.q_head_stride = p.k_head_stride = p.v_head_stride = p.o_head_stride = 64
    p.softmax_scale = 0.125
    for k, v in kw.items():
        setattr(p, k, v)
    return p


@pytest.mark.parametrize(
    "kw,expected",
    [
        ({}, 0),
        ({"head_dim": 96}, -2),
        ({"heads_k": 1}, 0),
        ({"heads": 4, "heads_k": 3}, -1),
        ({"batch": -1}, -1),
        ({"q": (1 << 20) + 2}, -3),
        ({"q_row_stride": 2 * 64 + 4}, -3),
        ({"softmax_scale": float("nan")}, -1),
        ({"o": None}, -1),
        ({"batch": 0, "q": None}, 0),
    ],
)
def test_check_params(kw, expected):
    from flash_attention import _C

    assert _C.lib.fa_sm100_check_params(ctypes.byref(_params(**kw))) == expected


def test_status_strings():
    from flash_attention import _C

    for rc in (0, -1, -2, -3, -4, -5, -6):
        assert _C.status_string(rc)
    assert _C.status_string(-6) == "device-side wait timed out"
