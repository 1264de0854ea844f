"""Weight-only INT8 GEMM (tac_gemm_wo_f16_i8): FP16 activations x INT8 weights
dequantised with per-output-channel float32 scales, float32 out.

* CPU: the oracle's quantiser equals the reference's own
  _weight_only_qdq_per_channel (software/taccel/runtime/fp32_reference.py:330-345)
  when the reference package is importable.
* GPU: the kernel against the oracle's float32 layer, within the bound of two
  float32 evaluations that differ only in summation order
  (oracle.weight_only.error_bound: 2 (K + 2) 2^-24 sum |x| |w|), at the W8A16
  layer workload (1024 x 768 activations, 768 x 3072 weights), ragged shapes
  and a decode row.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from helpers import import_reference
from oracle import weight_only as WO


def _inputs(M, K, N, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float16)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    w[:, rng.choice(K, max(1, K // 100), replace=False)] *= 8.0
    q, s = WO.quantize_per_channel(w)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    return x, q, s, b


@pytest.mark.reference
def test_oracle_quantiser_equals_reference():
    assert import_reference()
    from taccel.runtime.fp32_reference import _weight_only_qdq_per_channel
    for seed, shape in ((0, (64, 48)), (1, (3072, 768)), (2, (5, 7))):
        w = (np.random.default_rng(seed).standard_normal(shape) * 0.05).astype(np.float32)
        w[0] = 0.0   # an all-zero channel takes the 1e-10 floor
        q, s = WO.quantize_per_channel(w)
        np.testing.assert_array_equal(WO.dequantize(q, s), _weight_only_qdq_per_channel(w))


def test_oracle_layer_is_the_float32_product():
    x, q, s, b = _inputs(8, 64, 48, 3)
    y = WO.weight_only_linear(x, q, s, b)
    exact = x.astype(np.float64) @ WO.dequantize(q, s).astype(np.float64).T + b.astype(np.float64)
    assert np.all(np.abs(y - exact) <= WO.error_bound(x, q, s))


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N,with_bias", [(1024, 768, 3072, True), (1024, 768, 3072, False),
                                             (100, 200, 48, True), (300, 1000, 272, True), (1, 768, 3072, True),
                                             (257, 64, 16, False)])
def test_weight_only_gemm_within_float32_bound(M, K, N, with_bias):
    import torch
    from llm_accelerator_b200 import _lib as L
    from llm_accelerator_b200.gemm import gemm_wo_f16_i8
    x, q, s, b = _inputs(M, K, N, M + K + N)
    bias = b if with_bias else None
    want = WO.weight_only_linear(x, q, s, bias)
    bound = WO.error_bound(x, q, s)
    dX = torch.from_numpy(x).cuda()
    dQ = torch.from_numpy(np.ascontiguousarray(q.T)).cuda()        # [K, N], the ISA's weight layout
    dS = torch.from_numpy(s).cuda()
    dB = torch.from_numpy(b).cuda() if with_bias else None
    for _ in range(2):
        y = gemm_wo_f16_i8(dX, dQ, dS, dB).cpu().numpy()
        err = np.abs(y.astype(np.float64) - want.astype(np.float64))
        worst = float(np.max(err / bound))
        print(f"{M}x{K}x{N}: max |y - ref| {float(err.max()):.3g}, {worst:.3f} of the bound")
        assert np.all(err <= bound)
    assert L.lib.tac_gemm_status(None) == L.OK


@pytest.mark.gpu
def test_weight_only_gemm_rejects_unsupported_shapes():
    from llm_accelerator_b200 import _lib as L
    p = C.c_void_p(256)
    assert L.lib.tac_gemm_wo_f16_i8(p, p, p, None, p, 4, 64, 20, None) == L.E_ARGUMENT    # K not a multiple of 8
    assert L.lib.tac_gemm_wo_f16_i8(p, p, p, None, p, 4, 40, 64, None) == L.E_ARGUMENT    # N not a multiple of 16
    assert L.lib.tac_gemm_wo_f16_i8(C.c_void_p(258), p, p, None, p, 4, 64, 64, None) == L.E_ARGUMENT   # unaligned X
