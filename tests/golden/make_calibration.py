"""Writes tests/golden/calibration_tiny.npz: a seeded random-init 2-layer GPT-2
payload (d_model 64, 4 heads, a 65-character vocabulary, synthetic seeded
text) and the per-node scales the reference's build_calibration_scales
(software/taccel/runtime/calibration.py:104) returns for it, at three
settings: percentile 99.9, percentile 100 (maxima), and 99.9 with a per-node
override.

    python tests/golden/make_calibration.py

Reads the reference checkout at $TACCEL_REFERENCE (default /root/reference).
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

REF = Path(os.environ.get("TACCEL_REFERENCE", "/root/reference"))
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(REF / "software"))
sys.path.insert(0, str(REF / "software" / "tools"))
sys.dont_write_bytecode = True

SETTINGS = {"p999": dict(percentile=99.9), "p100": dict(percentile=100.0),
            "override": dict(percentile=99.9, activation_percentile_overrides={"block0_fc1": 99.0, "ln_f": 100.0})}


def main() -> None:
    import torch
    from transformers import GPT2Config, GPT2LMHeadModel
    from convert_hf_gpt2_to_nanogpt import convert_hf_state_dict_to_nanogpt
    from taccel.runtime.calibration import build_calibration_scales, build_calibration_seqs
    torch.manual_seed(0)
    hf = GPT2Config(n_layer=2, n_embd=64, n_head=4, n_positions=64, vocab_size=65)
    payload = convert_hf_state_dict_to_nanogpt(GPT2LMHeadModel(hf).state_dict(), hf)
    alphabet = [chr(c) for c in range(33, 33 + 65)]
    rng = np.random.default_rng(0)
    payload["text"] = "".join(rng.choice(alphabet, 600))
    payload["stoi"] = {ch: i for i, ch in enumerate(alphabet)}
    sd = {k: np.asarray(v.detach().cpu().numpy() if hasattr(v, "detach") else v, np.float32)
          for k, v in payload["state_dict"].items()}
    out = {f"sd::{k}": v for k, v in sd.items()}
    out["model_args"] = np.frombuffer(json.dumps(payload["model_args"]).encode(), np.uint8)
    out["text"] = np.frombuffer(payload["text"].encode(), np.uint8)
    out["stoi"] = np.frombuffer(json.dumps(payload["stoi"]).encode(), np.uint8)
    out["windows"] = np.asarray(build_calibration_seqs(payload), np.int64)
    for tag, kw in SETTINGS.items():
        scales = build_calibration_scales(payload, **kw)
        names = sorted(scales)
        out[f"{tag}::names"] = np.frombuffer(json.dumps(names).encode(), np.uint8)
        out[f"{tag}::scales"] = np.asarray([scales[n] for n in names], np.float64)
    np.savez_compressed(HERE / "calibration_tiny.npz", **out)
    print("wrote", HERE / "calibration_tiny.npz")


if __name__ == "__main__":
    main()
