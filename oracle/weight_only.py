"""Oracle for the weight-only INT8 GEMM: TEST INFRASTRUCTURE ONLY.

Restates the reference's W8A32 weight-only path
(software/taccel/runtime/fp32_reference.py:330-345,
_weight_only_qdq_per_channel, and its use by
build_weight_only_int8_reference, :389): each output channel (row of the
[out, in] float32 weight) is quantised symmetrically to INT8 with the float32
scale max(max|w_row|, 1e-10) / 127 (round half to even, clipped to
[-128, 127]) and dequantised back to float32 as q * scale; the layer is then
the float32 product x @ W_deq^T (+ bias).  Only tests and the CPU baseline
may import this module.
"""
from __future__ import annotations

from typing import Optional

import numpy as np


def quantize_per_channel(w_out_in: np.ndarray):
    """(q int8 [out, in], scale float32 [out]) of fp32_reference.py:330-345."""
    arr = np.asarray(w_out_in, dtype=np.float32)
    max_abs = np.maximum(np.max(np.abs(arr), axis=1, keepdims=True), np.float32(1e-10))
    scale = (max_abs / np.float32(127.0)).astype(np.float32)
    q = np.clip(np.round(arr / scale), -128, 127).astype(np.int8)
    return q, scale[:, 0]


def dequantize(q: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """q * scale in float32, one scale per row of q [out, in]."""
    return (q.astype(np.float32) * scale.astype(np.float32)[:, None]).astype(np.float32)


def weight_only_linear(x_f16: np.ndarray, q_out_in: np.ndarray, scale: np.ndarray,
                       bias: Optional[np.ndarray] = None) -> np.ndarray:
    """float32 x @ dequant(q)^T (+ bias), the reference's W8A32 layer."""
    y = np.asarray(x_f16, dtype=np.float32) @ dequantize(q_out_in, scale).T
    if bias is not None:
        y = (y + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    return y.astype(np.float32)


def error_bound(x_f16: np.ndarray, q_out_in: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """Bound on the difference between two float32 evaluations of the layer
    that differ only in summation order and in where the scale is applied:
    2 * (K + 2) * 2^-24 * sum_k |x[m,k]| * |dequant(q)[n,k]|, plus a tiny
    absolute floor."""
    k = x_f16.shape[1]
    mag = np.abs(np.asarray(x_f16, dtype=np.float64)) @ np.abs(dequantize(q_out_in, scale).astype(np.float64)).T
    return 2.0 * (k + 2) * 2.0 ** -24 * mag + 1e-30
