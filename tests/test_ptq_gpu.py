"""GPU parity of the offline weight quantiser (bit-exact against the
reference's vectors and the oracle) and of the residual-stream rotation
(float32 products: within 1e-6 of the reference's NumPy float32 result, whose
entries are below 0.2 in magnitude)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import ptq as P
from test_ptq_oracle import GOLDEN, golden_cases

pytestmark = pytest.mark.gpu


def _run(w, pc):
    import torch
    from llm_accelerator_b200 import ptq
    q, s = ptq.quantize_linear_weight(torch.from_numpy(w).cuda(), per_channel=pc)
    return q.cpu().numpy(), s.cpu().numpy()


def test_quantizer_bit_exact_against_reference_vectors():
    for w, pc, q_ref, s_ref in golden_cases():
        q, s = _run(w, pc)
        np.testing.assert_array_equal(q, q_ref)
        np.testing.assert_array_equal(s.view(np.uint16), s_ref)


@pytest.mark.parametrize("o,k,pc", [(3072, 768, True), (768, 3072, True), (1024, 4096, False), (50257, 768, True),
                                    (1, 1, True), (31, 17, False), (4096, 1024, True)])
def test_quantizer_bit_exact_against_oracle(o, k, pc):
    w = P.weight_case(o, k, seed=o + k, zero_rows=(0,) if o > 1 else (), outlier=50.0 if o % 2 else 0.0)
    q, s = _run(w, pc)
    q_ref, s_ref = P.quantize_linear_weight(w, per_channel=pc)
    np.testing.assert_array_equal(q, q_ref)
    np.testing.assert_array_equal(s.view(np.uint16), s_ref.view(np.uint16))


def test_quantize_tensor_layout():
    import torch
    from llm_accelerator_b200 import ptq
    w = P.weight_case(100, 33, 5)
    q, s = ptq.quantize_tensor(torch.from_numpy(w).cuda())
    q_ref, s_ref = P.quantize_tensor(w)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), s_ref.view(np.uint16))


def test_rotation_matches_reference_result():
    import torch
    from llm_accelerator_b200 import ptq
    z = np.load(GOLDEN)
    sd, args = P.rotation_case()
    sd_t = {k: torch.from_numpy(v) for k, v in sd.items()}
    keys = ptq.rotate_residual_stream_state_dict(sd_t, args, z["rot_R"])
    assert keys == [str(k) for k in z["rot_keys"]]
    for i, k in enumerate(keys):
        got = sd_t[k].numpy()
        assert got.dtype == np.float32 and got.shape == z[f"rot_{i}"].shape
        np.testing.assert_allclose(got, z[f"rot_{i}"], rtol=0, atol=1e-6)
