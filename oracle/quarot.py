"""Oracle for the QuaRot W8A16 layer: TEST INFRASTRUCTURE ONLY.

The reference applies QuaRot offline (a rotation folded into the weights) and
has no runtime Hadamard, so this path has no reference run to pin against
end to end.  The oracle fixes the layer as:

  1. rotate each row of X (FP16 [M, K]) by the normalised block
     Walsh-Hadamard H = I_(K/b) (x) H_b / sqrt(b), H_b the Sylvester matrix
     of software/taccel/quantizer/rotation.py:108-114, evaluated as an
     in-place fast transform in float32 (stages of half-width 1, 2, 4, ...;
     pair (a, c) -> (a + c, a - c) with a the lower index), then scaled by
     float32(1 / sqrt(b)) and rounded once to FP16;
  2. the W8A16 dynamic matmul of
     software/taccel/runtime/w8a16_simulator_reference.py:96-135 on the
     rotated rows: per-tensor max|x| with a 2^-9 floor, FP16 inverse and
     forward scales computed in float64, INT8 round-half-even quantisation,
     int32 GEMM, (f32(acc) * f32(pc[n])) * f32(fwd) (+ f32(bias[n])), FP16.

Step 2 is pinned to the reference function itself (tests import it when the
reference checkout is present and compare bit for bit; tests/golden holds the
committed vectors).  Step 1 is checked against the dense Sylvester matrix
product; its float32 evaluation order is this oracle's own definition, which
the CUDA kernel follows exactly.
"""
from __future__ import annotations

import math
from typing import Optional

import numpy as np


def sylvester_hadamard(n: int) -> np.ndarray:
    """Dense Sylvester Hadamard matrix of size n (a power of two), float64."""
    if n < 1 or n & (n - 1):
        raise ValueError(f"size must be a power of two, got {n}")
    h = np.ones((1, 1))
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    return h


def fwht_blocks(x_f16: np.ndarray, block: int) -> np.ndarray:
    """Rows of x rotated by I (x) H_block / sqrt(block); returns FP16."""
    x = np.asarray(x_f16, dtype=np.float16)
    m, k = x.shape
    if block < 2 or block & (block - 1) or k % block:
        raise ValueError(f"block {block} must be a power of two dividing {k}")
    v = x.astype(np.float32).reshape(m, k // block, block).copy()
    h = 1
    while h < block:
        w = v.reshape(m, k // block, block // (2 * h), 2, h)
        a = w[:, :, :, 0, :].copy()
        c = w[:, :, :, 1, :].copy()
        w[:, :, :, 0, :] = a + c
        w[:, :, :, 1, :] = a - c
        h *= 2
    v = v * np.float32(1.0 / math.sqrt(block))
    return v.reshape(m, k).astype(np.float16)


def act_scales(x_f16: np.ndarray):
    """(max|x|, inverse FP16 scale, forward FP16 scale) of the dynamic quantiser."""
    xf = np.asarray(x_f16, dtype=np.float16).astype(np.float32)
    max_abs = float(np.max(np.abs(xf))) if xf.size else 0.0
    m = max(max_abs, 2.0 ** -9)
    return max_abs, np.float16(127.0 / m), np.float16(m / 127.0)


def quantize_act(x_f16: np.ndarray, inv_f16) -> np.ndarray:
    xf = np.asarray(x_f16, dtype=np.float16).astype(np.float32)
    return np.clip(np.round(xf * np.float32(inv_f16)), -128, 127).astype(np.int8)


def w8a16_dynamic_matmul(x_f16: np.ndarray, w_int8: np.ndarray, w_scale_f16: np.ndarray,
                         bias_f16: Optional[np.ndarray] = None) -> np.ndarray:
    """FP16 [M, N] output of the W8A16 dynamic matmul on FP16 activations."""
    _, inv, fwd = act_scales(x_f16)
    xq = quantize_act(x_f16, inv)
    acc = xq.astype(np.int64) @ np.asarray(w_int8).astype(np.int64)   # exact; fits int32
    acc = acc.astype(np.int32)
    y = acc.astype(np.float32) * np.asarray(w_scale_f16, np.float16).astype(np.float32).reshape(1, -1)
    y = y * np.float32(fwd)
    if bias_f16 is not None:
        y = y + np.asarray(bias_f16, np.float16).astype(np.float32).reshape(1, -1)
    return y.astype(np.float16)


def quarot_w8a16_layer(x_f16, w_int8, w_scale_f16, bias_f16=None, block: int = 256) -> np.ndarray:
    return w8a16_dynamic_matmul(fwht_blocks(x_f16, block), w_int8, w_scale_f16, bias_f16)


def layer_inputs(m: int = 1024, k: int = 768, n: int = 3072, seed: int = 0, outlier_frac: float = 0.01,
                 outlier_gain: float = 50.0):
    """Seeded inputs with the shapes and value distributions of the QuaRot W8A16
    layer workload: X ~ N(0, 1) FP16 with 1% of channels scaled x50; INT8
    weights per-output-channel quantised from N(0, 0.02) (scale = max|w| / 127,
    stored FP16, as software/taccel/runtime/w8a16_simulator_reference.py:78-93)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    ch = rng.choice(k, max(1, int(round(outlier_frac * k))), replace=False)
    x[:, ch] *= np.float32(outlier_gain)
    x = x.astype(np.float16)
    w = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    scale = (np.maximum(np.max(np.abs(w), axis=0), 1e-8) / 127.0).astype(np.float16)
    w_int8 = np.clip(np.round(w / scale.astype(np.float32).reshape(1, -1)), -128, 127).astype(np.int8)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float16)
    return x, w_int8, scale, bias
