"""Stand-alone INT8 GEMM kernels on torch tensors (device memory plumbing).

``gemm_i8_i32``            C = A @ B (int32), the MATMUL instruction at any size
``gemm_i8_requant_pc``     int8 = clip(rint(f32(A @ B) * f32(scale[n]))), MATMUL + REQUANT_PC
                           (``golden_model/systolic.py:31-71``, ``golden_model/simulator.py:661-688``)
``gemm_i8_requant_shift``  int8 = clip((acc * mult[n] + 2^(shift[n]-1)) >> shift[n]) (int64),
                           an integer-multiplier epilogue with no reference counterpart
"""
from __future__ import annotations

from . import _lib as L


def _ptr(t):
    return t.data_ptr()


def _check(A, B):
    import torch
    if A.dtype != torch.int8 or B.dtype != torch.int8 or not A.is_cuda or not B.is_cuda:
        raise TypeError("A and B must be int8 CUDA tensors")
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[0]:
        raise ValueError(f"shape mismatch {tuple(A.shape)} @ {tuple(B.shape)}")
    if not (A.is_contiguous() and B.is_contiguous()):
        raise ValueError("A and B must be contiguous (row-major)")
    return A.shape[0], B.shape[1], A.shape[1]


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def gemm_i8_i32(A, B, out=None):
    import torch
    M, N, K = _check(A, B)
    out = torch.empty((M, N), dtype=torch.int32, device=A.device) if out is None else out
    L.check(L.lib.tac_gemm_i8_i32(_ptr(A), _ptr(B), _ptr(out), M, N, K, _stream()), "tac_gemm_i8_i32")
    return out


def gemm_i8_requant_pc(A, B, scale_f16, out=None):
    import torch
    M, N, K = _check(A, B)
    if scale_f16.dtype != torch.float16 or scale_f16.numel() != N:
        raise ValueError("scale_f16 must be float16 with N elements")
    out = torch.empty((M, N), dtype=torch.int8, device=A.device) if out is None else out
    L.check(L.lib.tac_gemm_i8_requant_pc(_ptr(A), _ptr(B), _ptr(scale_f16.contiguous()), _ptr(out), M, N, K,
                                         _stream()), "tac_gemm_i8_requant_pc")
    return out


def gemm_i8_requant_shift(A, B, mult, shift, out=None):
    import torch
    M, N, K = _check(A, B)
    if mult.dtype != torch.int32 or shift.dtype != torch.int32 or mult.numel() != N or shift.numel() != N:
        raise ValueError("mult and shift must be int32 with N elements")
    out = torch.empty((M, N), dtype=torch.int8, device=A.device) if out is None else out
    L.check(L.lib.tac_gemm_i8_requant_shift(_ptr(A), _ptr(B), _ptr(mult.contiguous()), _ptr(shift.contiguous()),
                                            _ptr(out), M, N, K, _stream()), "tac_gemm_i8_requant_shift")
    return out
