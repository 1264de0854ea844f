"""Writes tests/golden/ptq_cases.npz from the reference itself.

Each case is a seeded float32 weight (oracle.ptq.weight_case; its SHA-256 is
stored to catch a change of generator) passed through the reference's
_quantize_linear_weight (software/taccel/runtime/tiny_fixture.py:149), which
calls quantize_tensor (software/taccel/quantizer/quantize.py:6).  Stored:
q_kn and the FP16 scales.  A rotation case: a seeded two-layer, two-head
state dict (oracle.ptq.rotation_case) rotated by the reference's
rotate_residual_stream_state_dict (software/taccel/quantizer/rotation.py:158)
with build_random_orthogonal(64) (rotation.py:51).  Run from the repository root with the reference
checkout at /root/reference.
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

from oracle.ptq import rotation_case, weight_case  # noqa: E402
from taccel.quantizer.rotation import build_random_orthogonal, rotate_residual_stream_state_dict  # noqa: E402
from taccel.runtime.tiny_fixture import _quantize_linear_weight  # noqa: E402

# (out_ch, in_features, seed, per_channel, zero_rows, outlier)
CASES = [
    (64, 64, 1, True, (), 0.0),
    (50, 70, 2, True, (3,), 0.0),
    (33, 16, 3, False, (), 0.0),
    (96, 200, 4, True, (0, 95), 40.0),
    (17, 48, 5, False, (2,), 25.0),
    (1, 768, 6, True, (), 0.0),
    (128, 768, 7, True, (), 8.0),
]


def main():
    out = {}
    for i, (o, k, seed, pc, zr, outl) in enumerate(CASES):
        w = weight_case(o, k, seed, zero_rows=zr, outlier=outl)
        q, s = _quantize_linear_weight(w, per_channel=pc)
        out[f"c{i}_meta"] = np.array([o, k, seed, int(pc), int(outl)], dtype=np.int64)
        out[f"c{i}_zero_rows"] = np.array(zr, dtype=np.int64)
        out[f"c{i}_sha"] = np.frombuffer(hashlib.sha256(w.tobytes()).digest(), dtype=np.uint8)
        out[f"c{i}_q"] = q
        out[f"c{i}_s"] = s.view(np.uint16)
    sd, args = rotation_case()
    R = build_random_orthogonal(args["n_embd"], seed=0xCAFE)
    keys = rotate_residual_stream_state_dict(sd, args, R)
    out["rot_R"] = R.astype(np.float32)
    out["rot_keys"] = np.array(keys)
    for i, k in enumerate(keys):
        out[f"rot_{i}"] = np.asarray(sd[k], dtype=np.float32)
    np.savez_compressed(ROOT / "tests" / "golden" / "ptq_cases.npz", **out)
    print("wrote", len(CASES), "cases")


if __name__ == "__main__":
    main()
