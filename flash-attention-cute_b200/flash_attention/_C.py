"""Binding of libfa_sm100.so -- the stand-in for the reference's compiled
``flash_attention._C`` module (pybind11, csrc/flash_api.cpp:70-72).

``forward(q, k, v, causal)`` keeps the reference signature and error
behaviour: the same input checks with the same messages raised as
``RuntimeError`` (csrc/flash_api.cpp:14-29), output allocated with
``torch.empty_like(q)`` (flash_api.cpp:31), softmax scale ``1/sqrt(d)``
(flash_api.cpp:59-60), launched on the current stream of q's device
(flash_api.cpp:64; a device guard is added).  The native call goes through
the C ABI declared in ``include/fa_sm100.h`` via ctypes; there is no CPU
path: if the library is missing, importing this module fails.
"""
from __future__ import annotations

import ctypes
import math
import os
import struct

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libfa_sm100.so")

FA_OK = 0


class FaParams(ctypes.Structure):
    """Mirror of ``struct FaParams`` in include/fa_sm100.h."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("batch", ctypes.c_int32),
        ("seqlen_q", ctypes.c_int32),
        ("seqlen_k", ctypes.c_int32),
        ("heads", ctypes.c_int32),
        ("heads_k", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("q_batch_stride", ctypes.c_int64),
        ("q_row_stride", ctypes.c_int64),
        ("q_head_stride", ctypes.c_int64),
        ("k_batch_stride", ctypes.c_int64),
        ("k_row_stride", ctypes.c_int64),
        ("k_head_stride", ctypes.c_int64),
        ("v_batch_stride", ctypes.c_int64),
        ("v_row_stride", ctypes.c_int64),
        ("v_head_stride", ctypes.c_int64),
        ("o_batch_stride", ctypes.c_int64),
        ("o_row_stride", ctypes.c_int64),
        ("o_head_stride", ctypes.c_int64),
        ("lse_batch_stride", ctypes.c_int64),
        ("lse_head_stride", ctypes.c_int64),
        ("softmax_scale", ctypes.c_float),
        ("is_causal", ctypes.c_int32),
        ("is_bf16", ctypes.c_int32),
        ("q_pos_offset", ctypes.c_int64),
        ("k_pos_offset", ctypes.c_int64),
        ("error_flag", ctypes.c_void_p),
        ("out_f32", ctypes.c_int32),
    ]


def _load() -> ctypes.CDLL:
    if not os.path.exists(_LIB_PATH):
        raise ImportError(
            f"{_LIB_PATH} is missing: build it with `python flash-attention-cute_b200/build_ext.py` "
            "(there is no fallback implementation)"
        )
    lib = ctypes.CDLL(_LIB_PATH)
    lib.fa_sm100_check_params.argtypes = [ctypes.POINTER(FaParams)]
    lib.fa_sm100_check_params.restype = ctypes.c_int
    lib.fa_sm100_fwd.argtypes = [ctypes.POINTER(FaParams), ctypes.c_void_p]
    lib.fa_sm100_fwd.restype = ctypes.c_int
    lib.fa_sm100_lse_merge.argtypes = [
        ctypes.POINTER(ctypes.c_void_p),
        ctypes.POINTER(ctypes.c_void_p),
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.c_int32,
        ctypes.c_void_p,
        ctypes.c_int64,
        ctypes.c_int64,
        ctypes.c_int32,
        ctypes.c_void_p,
        ctypes.c_void_p,
    ]
    lib.fa_sm100_lse_merge.restype = ctypes.c_int
    lib.fa_sm100_take_device_error.argtypes = [ctypes.c_int]
    lib.fa_sm100_take_device_error.restype = ctypes.c_int
    lib.fa_sm100_status_string.argtypes = [ctypes.c_int]
    lib.fa_sm100_status_string.restype = ctypes.c_char_p
    lib.fa_sm100_num_sms.argtypes = [ctypes.c_int]
    lib.fa_sm100_num_sms.restype = ctypes.c_int
    lib.fa_sm100_params_size.argtypes = []
    lib.fa_sm100_params_size.restype = ctypes.c_int
    lib.fa_sm100_set_timeout_ns.argtypes = [ctypes.c_uint64]
    lib.fa_sm100_set_timeout_ns.restype = ctypes.c_uint64
    if lib.fa_sm100_params_size() != ctypes.sizeof(FaParams):
        raise ImportError(
            f"FaParams layout mismatch: library {lib.fa_sm100_params_size()} bytes, "
            f"binding {ctypes.sizeof(FaParams)} bytes"
        )
    return lib


lib = _load()

# Fast launch path: FaParams packed with one struct.pack call (layout checked
# against the ctypes mirror below) and passed as a byte buffer.  For small
# problems the per-call host cost is comparable to the kernel itself.
_PACKED = struct.Struct("=5Q6i14qf2i4x2qQi4x")
_fwd_packed = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_char_p, ctypes.c_void_p)(("fa_sm100_fwd", lib))
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _check_packed_layout() -> None:
    vals = (1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, *range(12, 26), 0.5, 1, 1, 26, 27, 28, 1)
    mirror = FaParams(*vals)
    if _PACKED.size != ctypes.sizeof(FaParams) or _PACKED.pack(*vals) != bytes(mirror):
        raise ImportError("packed FaParams layout does not match the ctypes mirror")


_check_packed_layout()


def status_string(rc: int) -> str:
    return lib.fa_sm100_status_string(rc).decode()


def _check(rc: int, what: str) -> None:
    if rc != FA_OK:
        raise RuntimeError(f"{what} failed: {status_string(rc)} (status {rc})")


def _validate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    # Same checks and messages as csrc/flash_api.cpp:14-29 ...
    if not q.is_cuda:
        raise RuntimeError("q must be on CUDA")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError("q must be fp16 or bf16")
    if q.stride(-1) != 1:
        raise RuntimeError("q must be contiguous in last dim")
    if k.stride(-1) != 1:
        raise RuntimeError("k must be contiguous in last dim")
    if v.stride(-1) != 1:
        raise RuntimeError("v must be contiguous in last dim")
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise RuntimeError("q, k, v must be 4-D (batch, seqlen, heads, head_dim)")
    head_dim = q.size(3)
    if head_dim not in (64, 128):
        raise RuntimeError("head_dim must be 64 or 128")
    if q.size(2) % k.size(2) != 0:
        raise RuntimeError("heads must be divisible by heads_k (for GQA)")
    # ... plus the ones the reference leaves out (its kernel would read K/V
    # of the wrong type, device or head otherwise).
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise RuntimeError("q, k and v must have the same dtype")
    if k.device != q.device or v.device != q.device:
        raise RuntimeError("q, k and v must be on the same device")
    if k.shape != v.shape or k.size(0) != q.size(0) or k.size(3) != head_dim:
        raise RuntimeError("k and v must be (batch, seqlen_k, heads_k, head_dim) matching q")


def fill_params(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    o: torch.Tensor,
    lse: torch.Tensor | None,
    causal: bool,
    softmax_scale: float | None = None,
    q_pos_offset: int = 0,
    k_pos_offset: int = 0,
) -> FaParams:
    # One positional constructor call (field order of struct FaParams): the
    # per-call host cost matters for small problems.
    b, sq, h, d = q.shape
    qs, ks, vs, os_ = q.stride(), k.stride(), v.stride(), o.stride()
    ls = lse.stride() if lse is not None else (0, 0, 0)
    return FaParams(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr() if lse is not None else None,
        b, sq, k.shape[1], h, k.shape[2], d,
        qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1], vs[2], os_[0], os_[1], os_[2],
        ls[0], ls[1],
        (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale),
        1 if causal else 0,
        1 if q.dtype == torch.bfloat16 else 0,
        int(q_pos_offset),
        int(k_pos_offset),
        None,
        1 if o.dtype == torch.float32 else 0,
    )


def launch(p: FaParams, device: torch.device) -> None:
    """Enqueue the kernel for filled params on the current stream of `device`."""
    if device.index is None or device.index == torch.cuda.current_device():
        stream = torch.cuda.current_stream().cuda_stream
        _check(lib.fa_sm100_fwd(ctypes.byref(p), stream), "fa_sm100_fwd")
        return
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        _check(lib.fa_sm100_fwd(ctypes.byref(p), stream), "fa_sm100_fwd")


def forward_with_lse(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    *,
    softmax_scale: float | None = None,
    q_pos_offset: int = 0,
    k_pos_offset: int = 0,
    want_lse: bool = True,
    out: torch.Tensor | None = None,
    lse_out: torch.Tensor | None = None,
):
    _validate(q, k, v)
    if out is not None and (out.shape != q.shape or out.dtype not in (q.dtype, torch.float32)
                            or out.device != q.device or out.stride(-1) != 1):
        raise RuntimeError("out must match q's shape and device, with q's dtype or fp32, contiguous in last dim")
    b, sq, h, d = q.shape
    o = torch.empty_like(q) if out is None else out
    lse = None
    if want_lse:
        lse = q.new_empty((b, h, sq), dtype=torch.float32) if lse_out is None else lse_out
    qs, ks, vs, os_ = q.stride(), k.stride(), v.stride(), o.stride()
    ls = lse.stride() if lse is not None else (0, 0, 0)
    packed = _PACKED.pack(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr() if lse is not None else 0,
        b, sq, k.shape[1], h, k.shape[2], d,
        qs[0], qs[1], qs[2], ks[0], ks[1], ks[2], vs[0], vs[1], vs[2], os_[0], os_[1], os_[2], ls[0], ls[1],
        (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale),
        1 if causal else 0,
        1 if q.dtype == torch.bfloat16 else 0,
        int(q_pos_offset), int(k_pos_offset), 0,
        1 if o.dtype == torch.float32 else 0,
    )
    idx = q.device.index
    if idx == torch.cuda.current_device():
        stream = _raw_stream(idx) if _raw_stream is not None else torch.cuda.current_stream().cuda_stream
        _check(_fwd_packed(packed, stream), "fa_sm100_fwd")
    else:
        with torch.cuda.device(q.device):
            _check(_fwd_packed(packed, torch.cuda.current_stream(q.device).cuda_stream), "fa_sm100_fwd")
    return o, lse


def forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool) -> torch.Tensor:
    """``flash_attention._C.forward(q, k, v, causal) -> o`` (csrc/flash_api.cpp:9-68)."""
    o, _ = forward_with_lse(q, k, v, causal, want_lse=False)
    return o


def lse_merge(o_parts, lse_parts, o_out: torch.Tensor, lse_out: torch.Tensor | None = None) -> None:
    """Merge fp32 partials (rows, heads, d) / (heads, rows) into o_out (rows, heads, d)."""
    n = len(o_parts)
    rows, heads, d = o_parts[0].shape
    for t in list(o_parts) + list(lse_parts):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.device != o_out.device:
            raise RuntimeError("partials must be contiguous fp32 tensors on the output's device")
    arr_o = (ctypes.c_void_p * n)(*[t.data_ptr() for t in o_parts])
    arr_l = (ctypes.c_void_p * n)(*[t.data_ptr() for t in lse_parts])
    with torch.cuda.device(o_out.device):
        stream = torch.cuda.current_stream(o_out.device).cuda_stream
        rc = lib.fa_sm100_lse_merge(
            arr_o,
            arr_l,
            n,
            rows,
            heads,
            d,
            o_out.data_ptr(),
            o_out.stride(0),
            o_out.stride(1),
            1 if o_out.dtype == torch.bfloat16 else 0,
            lse_out.data_ptr() if lse_out is not None else None,
            ctypes.c_void_p(stream),
        )
    _check(rc, "fa_sm100_lse_merge")


def take_device_error(device_index: int) -> int:
    """Read and clear the device's sticky kernel status (FA_OK or FA_ERR_TIMEOUT)."""
    return lib.fa_sm100_take_device_error(int(device_index))


def set_timeout_ns(ns: int) -> int:
    """Bound every device-side wait of later launches to `ns` nanoseconds
    (0 restores the default); returns the previous bound."""
    return int(lib.fa_sm100_set_timeout_ns(int(ns)))
