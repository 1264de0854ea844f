"""Activation calibration (llm_accelerator_b200/calibration.py) against the
reference's build_calibration_scales (software/taccel/runtime/calibration.py:104)
on a seeded 2-layer GPT-2 payload: the calibration windows exactly, every
node's scale to float32 rounding (the forward's GEMMs and reductions sum in
another order than NumPy's), on the CPU through torch and on the GPU."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from llm_accelerator_b200 import calibration as CAL

GOLDEN = Path(__file__).resolve().parent / "golden" / "calibration_tiny.npz"
SETTINGS = {"p999": dict(percentile=99.9), "p100": dict(percentile=100.0),
            "override": dict(percentile=99.9, activation_percentile_overrides={"block0_fc1": 99.0, "ln_f": 100.0})}
RTOL = 2e-5   # float32 rounding of the node statistics, relative


def _payload():
    z = np.load(GOLDEN)
    sd = {k[4:]: z[k] for k in z.files if k.startswith("sd::")}
    return z, {"state_dict": sd, "model_args": json.loads(bytes(z["model_args"]).decode()),
               "text": bytes(z["text"]).decode(), "stoi": json.loads(bytes(z["stoi"]).decode())}


def _expected(z, tag):
    names = json.loads(bytes(z[f"{tag}::names"]).decode())
    return dict(zip(names, z[f"{tag}::scales"].tolist()))


def test_calibration_windows_match_reference():
    z, payload = _payload()
    assert CAL.build_calibration_seqs(payload) == z["windows"].tolist()
    toks = [payload["stoi"][c] for c in payload["text"]]
    assert CAL.build_calibration_seqs_from_token_ids(toks) == z["windows"].tolist()
    assert CAL.build_calibration_seqs({"text": "", "stoi": {}}, seq_len=5) == [[0] * 5]


def _check(device, tag):
    z, payload = _payload()
    got = CAL.build_calibration_scales(payload, device=device, **SETTINGS[tag])
    want = _expected(z, tag)
    assert sorted(got) == sorted(want)
    g = np.asarray([got[k] for k in sorted(want)])
    w = np.asarray([want[k] for k in sorted(want)])
    err = np.abs(g - w) / np.abs(w)
    assert err.max() <= RTOL, (sorted(want)[int(err.argmax())], err.max())


@pytest.mark.parametrize("tag", sorted(SETTINGS))
def test_calibration_scales_match_reference_on_cpu(tag):
    _check("cpu", tag)


def test_unknown_override_is_rejected():
    _, payload = _payload()
    with pytest.raises(ValueError, match="unknown activation percentile override"):
        CAL.build_calibration_scales(payload, device="cpu", activation_percentile_overrides={"no_such_node": 99.0})


@pytest.mark.gpu
@pytest.mark.parametrize("tag", sorted(SETTINGS))
def test_calibration_scales_match_reference_on_gpu(tag):
    _check("cuda", tag)
