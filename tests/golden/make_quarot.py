"""Writes tests/golden/quarot_case.npz from the reference itself.

Inputs are regenerated from a seed by oracle.quarot.layer_inputs (their
SHA-256 digests are stored to catch a change of generator).  Outputs:
  xr_dense  FP16 rows rotated with the reference's dense Sylvester matrix
            (software/taccel/quantizer/rotation.py:108 _sylvester_hadamard),
            I_3 (x) H_256 / 16, as a float64 product;
  y_ref     the reference's W8A16 dynamic matmul
            (software/taccel/runtime/w8a16_simulator_reference.py:96
            _w8a16_dynamic_matmul) of xr_dense, FP16.
Run from the repository root with the reference checkout at /root/reference.
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(Path(os.environ.get("TACCEL_REFERENCE", "/root/reference")) / "software"))

from oracle.quarot import layer_inputs  # noqa: E402
from taccel.quantizer.rotation import _sylvester_hadamard  # noqa: E402
from taccel.runtime.w8a16_simulator_reference import _w8a16_dynamic_matmul  # noqa: E402

M, K, N, SEED, BLOCK = 64, 768, 256, 7, 256


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def main():
    x, w, s, b = layer_inputs(M, K, N, seed=SEED)
    hb = _sylvester_hadamard(BLOCK) / np.sqrt(float(BLOCK))
    H = np.kron(np.eye(K // BLOCK), hb)
    xr = (x.astype(np.float64) @ H.T).astype(np.float16)
    y = _w8a16_dynamic_matmul(xr.astype(np.float32), w, s, b.astype(np.float32)).astype(np.float16)
    np.savez_compressed(ROOT / "tests" / "golden" / "quarot_case.npz", shape=np.array([M, K, N, SEED, BLOCK]),
                        inputs_sha=np.array(digest(x, w, s, b)), xr_dense=xr, y_ref=y)
    print("wrote quarot_case.npz", xr.shape, y.shape)


if __name__ == "__main__":
    main()
