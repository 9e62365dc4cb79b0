"""Host-side behaviour of flash_attn_func that needs no GPU: the input checks
raise RuntimeError with the reference's messages (csrc/flash_api.cpp:14-29)
before anything is launched."""
import pytest
import torch

from flash_attention import flash_attn_func


def _qkv(dtype=torch.float16, d=64):
    return [torch.zeros(1, 8, 2, d, dtype=dtype) for _ in range(3)]


def test_cpu_tensor_rejected():
    with pytest.raises(RuntimeError, match="q must be on CUDA"):
        flash_attn_func(*_qkv())


def test_signature_matches_reference():
    import inspect

    params = list(inspect.signature(flash_attn_func).parameters.values())
    assert [p.name for p in params[:4]] == ["q", "k", "v", "causal"]
    assert params[3].default is False
    assert params[4].kind is inspect.Parameter.KEYWORD_ONLY


def test_module_layout_matches_reference():
    import flash_attention
    from flash_attention import _C
    from flash_attention.interface import flash_attn_func as f2

    # the reference's one export first; the host-streaming call is an addition
    assert flash_attention.__all__[0] == "flash_attn_func"
    assert set(flash_attention.__all__) == {"flash_attn_func", "flash_attn_func_host"}
    assert callable(_C.forward) and f2 is flash_attn_func


def test_host_streaming_rejects_unpinned_tensors():
    from flash_attention import flash_attn_func_host

    x = torch.zeros(1, 8, 2, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="pinned host memory"):
        flash_attn_func_host(x, x, x)
    with pytest.raises(RuntimeError, match="contiguous"):
        y = torch.zeros(1, 8, 2, 128, dtype=torch.float16)[..., ::2]
        flash_attn_func_host(y, y, y)


def test_backward_binding_matches_library_struct():
    import ctypes

    from flash_attention import _C
    from flash_attention.backward import FaBwdParams

    assert _C.lib.fa_sm100_bwd_params_size() == ctypes.sizeof(FaBwdParams)


def test_pybind_module_exports_and_shares_the_library():
    """forward() runs in the pybind11 module, which links the same
    libfa_sm100.so that ctypes loaded (one copy of its state in the process)."""
    import inspect

    from flash_attention import _C, _fa_torch

    assert "forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool)" in _fa_torch.forward.__doc__
    assert callable(_fa_torch.forward_with_lse)
    assert _fa_torch.params_size() == _C.lib.fa_sm100_params_size()
    assert list(inspect.signature(_C.forward).parameters) == ["q", "k", "v", "causal"]
    with open("/proc/self/maps") as f:
        paths = {line.split()[-1] for line in f if line.rstrip().endswith("libfa_sm100.so")}
    assert len(paths) == 1, paths


def test_pybind_module_error_messages_on_cpu():
    from flash_attention._fa_torch import forward

    x = torch.zeros(1, 4, 2, 64)
    with pytest.raises(RuntimeError, match="q must be on CUDA"):
        forward(x, x, x, False)
