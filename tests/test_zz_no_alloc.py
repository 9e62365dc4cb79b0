"""The allocation-free split entry point, fa_sm100_fwd_split_noalloc, against
the regular entry point fa_sm100_fwd, both called through the C ABI.

The split entry point is for callers that cannot allocate device memory where
they run attention (an engine whose memory pool owns the GPU, a loop where an
allocation and the synchronisation it can trigger are not allowed, a C or FFI
caller that only holds pointers to its own tensors).  Its per-split partial
results live in one scratch array inside the library, kept from call to call,
so the test makes two different calls in a row: the second must not be
disturbed by what the first left in the scratch.  This file is collected last
on purpose; it passes alone and after the other tests.
"""
import ctypes

import pytest
import torch

from oracle.attention_oracle import make_inputs

pytestmark = pytest.mark.gpu

O_TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
LSE_TOL = 1e-3
FA_ERR_SCRATCH_LIMIT = -7


def _abi():
    from flash_attention import _C

    lib = _C.lib
    lib.fa_sm100_fwd_split_noalloc.argtypes = [ctypes.POINTER(_C.FaParams), ctypes.c_int32, ctypes.c_void_p]
    lib.fa_sm100_fwd_split_noalloc.restype = ctypes.c_int
    lib.fa_sm100_split_scratch_bytes.argtypes = []
    lib.fa_sm100_split_scratch_bytes.restype = ctypes.c_size_t
    return _C, lib


def _call(q, k, v, causal, splits=None):
    """Run one entry point on fresh NaN-filled outputs; return (status, o, lse)."""
    _C, lib = _abi()
    b, sq, h, _ = q.shape
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, sq), float("nan"), dtype=torch.float32, device=q.device)
    p = _C.fill_params(q, k, v, o, lse, causal)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if splits is None:
        rc = lib.fa_sm100_fwd(ctypes.byref(p), stream)
    else:
        rc = lib.fa_sm100_fwd_split_noalloc(ctypes.byref(p), splits, stream)
    torch.cuda.synchronize()
    return rc, o, lse


# (batch, seqlen_q, seqlen_k, heads, heads_k, head_dim, dtype, causal, splits)
CASES = [
    (2, 700, 1500, 4, 2, 128, torch.bfloat16, True, 3),
    (1, 300, 2000, 8, 8, 64, torch.float16, False, 4),
]


def test_two_calls_in_a_row_match_the_regular_entry_point():
    for i, (b, sq, sk, h, hk, d, dtype, causal, splits) in enumerate(CASES):
        q, k, v = (t.cuda() for t in make_inputs(b, sq, h, d, dtype, seed=50 + i, seqlen_k=sk, heads_k=hk))
        rc_ref, o_ref, lse_ref = _call(q, k, v, causal)
        rc, o, lse = _call(q, k, v, causal, splits=splits)
        assert rc_ref == 0 and rc == 0, (rc_ref, rc)
        assert not torch.isnan(o).any() and not torch.isnan(lse).any()
        assert (o.float() - o_ref.float()).abs().max().item() <= O_TOL[dtype]
        assert (lse - lse_ref).abs().max().item() <= LSE_TOL


def test_problem_larger_than_the_scratch_is_rejected_before_launch():
    _, lib = _abi()
    limit = lib.fa_sm100_split_scratch_bytes()
    b, sq, h, d, splits = 1, 4096, 64, 128, 4
    assert splits * b * sq * h * 4 * (d + 1) > limit
    q = torch.zeros(b, sq, h, d, dtype=torch.bfloat16, device="cuda")
    rc, o, _ = _call(q, q, q, False, splits=splits)
    assert rc == FA_ERR_SCRATCH_LIMIT
    assert torch.isnan(o).all()  # nothing was launched
