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
