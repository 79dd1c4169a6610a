"""torch-facing wrappers of the single-kernel C-ABI entry points.

All tensors must live on the current CUDA device; the calls are ordered on
torch's current stream.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import abi
from ._lib import check, lib


def _stream() -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: torch.Tensor | None) -> C.c_void_p:
    if t is None:
        return C.c_void_p(0)
    if not t.is_cuda:
        raise ValueError("rec_b200 kernels need CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("rec_b200 kernels need contiguous tensors")
    return C.c_void_p(t.data_ptr())


def scale_dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return abi.REC_SCALE_FP16
    if dtype == torch.bfloat16:
        return abi.REC_SCALE_BF16
    raise ValueError(f"unsupported scale dtype {dtype}")


def qmat(w: torch.Tensor, s: torch.Tensor, b: torch.Tensor) -> abi.RecQMat:
    return abi.RecQMat(_ptr(w).value, _ptr(s).value, _ptr(b).value)


def gemv_int4(w: torch.Tensor, s: torch.Tensor, b: torch.Tensor, x: torch.Tensor,
              norm_weight: torch.Tensor | None = None, eps: float = 1e-6) -> torch.Tensor:
    """y = W x for an int4 g64 matrix in MLX layout (w uint32/int32 [N, K/8])."""
    n, k8 = w.shape
    k = k8 * 8
    if x.dtype != torch.bfloat16 or x.numel() != k:
        raise ValueError("x must be bf16 with K elements")
    y = torch.empty(n, dtype=torch.bfloat16, device=w.device)
    m = qmat(w, s, b)
    check(lib().rec_gemv_int4(C.byref(m), scale_dtype_code(s.dtype), n, k, _ptr(x), _ptr(norm_weight),
                              float(eps), _ptr(y), _stream()), "rec_gemv_int4")
    return y


def quantize_affine(w: torch.Tensor, bits: int = 4, scale_dtype: torch.dtype = torch.float16):
    """MLX affine quantization (group 64) of a float32 CUDA tensor [..., K]."""
    if w.dtype != torch.float32:
        raise ValueError("quantize_affine takes float32 input")
    w = w.contiguous()
    *lead, k = w.shape
    if k % 64:
        raise ValueError("last dimension must be a multiple of 64")
    groups = w.numel() // 64
    codes = torch.empty(*lead, k * bits // 32, dtype=torch.int32, device=w.device)
    scales = torch.empty(*lead, k // 64, dtype=scale_dtype, device=w.device)
    biases = torch.empty_like(scales)
    check(lib().rec_quantize_affine(_ptr(w), groups, bits, scale_dtype_code(scale_dtype), _ptr(codes),
                                    _ptr(scales), _ptr(biases), _stream()), "rec_quantize_affine")
    return codes, scales, biases
