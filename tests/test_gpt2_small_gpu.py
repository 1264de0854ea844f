"""GPT-2 small (12 layers, d_model 768, vocab 50257) decoder bundle on the GPU
against the oracle run on the same host: prefill + decode steps, greedy
tokens and logits.  Uses the bundle under bundles/ (compiled by the reference
toolchain with tests/golden/make_bundles.py)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from helpers import fp16_ulp_diff
from oracle import golden as G

pytestmark = pytest.mark.gpu
BUNDLE = Path(__file__).resolve().parent.parent / "bundles" / "gpt2_small_l12_s47.npz"


@pytest.mark.skipif(not BUNDLE.exists(), reason="GPT-2 small bundle not generated")
def test_gpt2_small_decode_matches_oracle():
    from llm_accelerator_b200.bundle import ProgramBundle
    from llm_accelerator_b200.runner import HostRunner
    from llm_accelerator_b200.simulator import B200Simulator
    from test_oracle_pin import _Runner
    vocab, steps = 50257, 4
    prompt = np.random.default_rng(0).integers(0, vocab, 16)
    bg = ProgramBundle.load(BUNDLE)
    bo = ProgramBundle.load(BUNDLE)
    r = HostRunner(bg, simulator=B200Simulator(), logits_dtype=np.float16)
    ro = _Runner(bo, G.OracleSimulator())
    lg = [r.run_prefill([int(prompt[0])])]
    lo = [ro.step("prefill", int(prompt[0]), 0)]
    for pos in range(1, steps):
        lg.append(r.run_decode_step(int(prompt[pos]), pos))
        lo.append(ro.step("decode", int(prompt[pos]), pos))
    lg, lo = np.stack(lg), np.stack(lo)
    ulp = fp16_ulp_diff(lg.view(np.uint8).ravel().copy(), lo.view(np.uint8).ravel().copy())
    print(f"GPT-2 small logits: bit-exact fraction {np.mean(ulp == 0):.5f}, max ulp {ulp.max()}, "
          f"max abs {np.max(np.abs(lg.astype(np.float32) - lo.astype(np.float32))):.3g}")
    assert [int(np.argmax(x[:vocab])) for x in lg] == [int(np.argmax(x[:vocab])) for x in lo]
    assert np.mean(ulp == 0) >= 0.95
