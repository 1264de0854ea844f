"""The QuaRot W8A16 oracle against the reference (CPU)."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import quarot as Q

GOLDEN = Path(__file__).parent / "golden" / "quarot_case.npz"


def _case():
    z = np.load(GOLDEN)
    M, K, N, seed, block = (int(v) for v in z["shape"])
    x, w, s, b = Q.layer_inputs(M, K, N, seed=seed)
    h = hashlib.sha256()
    for a in (x, w, s, b):
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.hexdigest() == str(z["inputs_sha"]), "input generator changed"
    return x, w, s, b, block, z


def test_w8a16_restatement_is_bit_exact_against_reference_vectors():
    x, w, s, b, block, z = _case()
    y = Q.w8a16_dynamic_matmul(z["xr_dense"], w, s, b)
    np.testing.assert_array_equal(y.view(np.uint16), z["y_ref"].view(np.uint16))


def test_fwht_matches_dense_sylvester_rotation_within_one_ulp():
    x, w, s, b, block, z = _case()
    xr = Q.fwht_blocks(x, block)
    a = xr.view(np.int16).astype(np.int32)
    d = z["xr_dense"].view(np.int16).astype(np.int32)
    # same-sign FP16 bit patterns: ulp distance
    ulp = np.abs(np.where(a < 0, -(a & 0x7FFF), a) - np.where(d < 0, -(d & 0x7FFF), d))
    assert ulp.max() <= 1 and np.mean(ulp == 0) > 0.999


@pytest.mark.parametrize("block", [32, 64, 256, 1024])
def test_fwht_is_the_dense_block_hadamard(block):
    rng = np.random.default_rng(block)
    x = rng.standard_normal((8, 2048)).astype(np.float16)
    H = np.kron(np.eye(2048 // block), Q.sylvester_hadamard(block) / np.sqrt(block))
    dense = x.astype(np.float64) @ H.T
    got = Q.fwht_blocks(x, block).astype(np.float64)
    assert np.max(np.abs(got - dense) / np.maximum(np.abs(dense), 2.0 ** -6)) < 2e-3
    # orthogonal: rotating twice gives the input back (up to FP16 rounding)
    back = Q.fwht_blocks(Q.fwht_blocks(x, block), block).astype(np.float64)
    assert np.max(np.abs(back - x.astype(np.float64))) < 2e-2


@pytest.mark.reference
def test_w8a16_restatement_matches_reference_function_directly():
    from helpers import import_reference
    assert import_reference()
    from taccel.runtime.w8a16_simulator_reference import _w8a16_dynamic_matmul
    for seed in range(3):
        x, w, s, b = Q.layer_inputs(32, 512, 128, seed=seed)
        xr = Q.fwht_blocks(x, 256)
        ref = _w8a16_dynamic_matmul(xr.astype(np.float32), w, s, b.astype(np.float32)).astype(np.float16)
        np.testing.assert_array_equal(Q.w8a16_dynamic_matmul(xr, w, s, b).view(np.uint16), ref.view(np.uint16))
