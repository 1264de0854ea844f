"""The offline weight-quantisation oracle against the reference (CPU)."""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import REFERENCE
from oracle import ptq as P

GOLDEN = Path(__file__).parent / "golden" / "ptq_cases.npz"


def golden_cases():
    z = np.load(GOLDEN)
    out = []
    i = 0
    while f"c{i}_meta" in z.files:
        o, k, seed, pc, outl = (int(v) for v in z[f"c{i}_meta"])
        w = P.weight_case(o, k, seed, zero_rows=tuple(int(r) for r in z[f"c{i}_zero_rows"]), outlier=float(outl))
        assert hashlib.sha256(w.tobytes()).digest() == z[f"c{i}_sha"].tobytes(), "weight generator changed"
        out.append((w, bool(pc), z[f"c{i}_q"], z[f"c{i}_s"]))
        i += 1
    return out


def test_quantize_linear_weight_bit_exact_against_reference_vectors():
    cases = golden_cases()
    assert len(cases) >= 7
    for w, pc, q_ref, s_ref in cases:
        q, s = P.quantize_linear_weight(w, per_channel=pc)
        np.testing.assert_array_equal(q, q_ref)
        np.testing.assert_array_equal(s.view(np.uint16), s_ref)


def test_quantize_tensor_layout_and_padding():
    w = P.weight_case(20, 30, 9, zero_rows=(19,))
    q, s = P.quantize_tensor(w)
    qk, sk = P.quantize_linear_weight(w)
    assert qk.shape == (32, 32) and sk.shape == (32,)
    np.testing.assert_array_equal(qk[:30, :20], q.T)
    assert not qk[30:].any() and not qk[:, 20:].any()
    assert (sk[20:] == s[-1]).all()
    assert s[19] == 0 and not q[19].any()   # all-zero channel: scale 1e-8 / 127 rounds to FP16 zero


@pytest.mark.reference
@pytest.mark.parametrize("o,k,seed,pc", [(40, 100, 21, True), (40, 100, 22, False), (300, 64, 23, True),
                                         (7, 513, 24, True)])
def test_oracle_matches_reference_function(o, k, seed, pc):
    sys.path.insert(0, str(REFERENCE / "software"))
    from taccel.quantizer.quantize import quantize_tensor
    from taccel.runtime.tiny_fixture import _quantize_linear_weight
    w = P.weight_case(o, k, seed, outlier=30.0 if seed % 2 else 0.0)
    q_r, s_r = quantize_tensor(w, per_channel=pc)
    q, s = P.quantize_tensor(w, per_channel=pc)
    np.testing.assert_array_equal(q, q_r)
    np.testing.assert_array_equal(s.view(np.uint16), s_r.view(np.uint16))
    qk_r, sk_r = _quantize_linear_weight(w, per_channel=pc)
    qk, sk = P.quantize_linear_weight(w, per_channel=pc)
    np.testing.assert_array_equal(qk, qk_r)
    np.testing.assert_array_equal(sk.view(np.uint16), sk_r.view(np.uint16))


def test_rotation_fixture_keys_cover_the_state_dict():
    z = np.load(GOLDEN)
    sd, args = P.rotation_case()
    keys = [str(k) for k in z["rot_keys"]]
    assert set(keys) == set(sd)   # every key of the synthetic dict is rotated
    R = z["rot_R"].astype(np.float64)
    np.testing.assert_allclose(R @ R.T, np.eye(args["n_embd"]), atol=1e-5)
    np.testing.assert_allclose(R @ np.ones(args["n_embd"]), np.ones(args["n_embd"]), atol=1e-5)
