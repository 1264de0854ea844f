"""GPT-2 small (12 layers, d_model 768, 12 heads, vocab 50257), the compiled
W8A16 program of the reference's compiler (regenerated from the committed
recipe): prefill + 47 decode steps through HostRunner on the GPU, 16
teacher-forced prompt tokens then 32 greedy tokens, against the reference
golden simulator's own run of the same program (tests/golden/run_gpt2_small.npz,
written by tests/golden/make_bundles.py).

Tokens must match one for one.  The FP16 logits of every step are compared by
their SHA-256 digest; a step may differ only through the transcendental ops
(GELU's tanh, softmax's exp), which the engine evaluates in float64 and rounds
once while NumPy's float32 SIMD routines are not correctly rounded: a one-ulp
FP16 difference there can move an INT8 quantisation step further down the
network.  Most steps are bit-exact; steps kept in full are compared value by
value."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from helpers import fp16_ulp_diff

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"
# largest logit perturbation accepted on a step that is not bit-exact, as a
# fraction of the step's largest |logit|
LOGIT_TOL = 0.05


def test_gpt2_small_48_steps_token_for_token():
    from llm_accelerator_b200.recipe import load_recipe
    from llm_accelerator_b200.runner import HostRunner
    gold = np.load(GOLDEN / "run_gpt2_small.npz")
    vocab, prompt = int(gold["vocab"][0]), [int(t) for t in gold["prompt"]]
    n_steps = int(gold["n_steps"][0])
    r = HostRunner(load_recipe(GOLDEN / "recipe_gpt2_small.npz"), logits_dtype=np.float16)
    logits = [r.run_prefill([prompt[0]])]
    toks = list(prompt)
    for pos in range(1, n_steps):
        tok = prompt[pos] if pos < len(prompt) else int(np.argmax(logits[-1][:vocab]))
        if pos >= len(prompt):
            toks.append(tok)
        logits.append(r.run_decode_step(tok, pos))
    assert toks == [int(t) for t in gold["tokens"]]
    digests = np.stack([np.frombuffer(hashlib.sha256(x.tobytes()).digest(), np.uint8) for x in logits])
    exact = np.all(digests == gold["logits_digest"], axis=1)
    print(f"logits bit-exact (SHA-256) on {int(exact.sum())} of {len(exact)} steps")
    for i, step in enumerate(gold["kept_steps"]):
        got, want = logits[int(step)][:vocab], gold["kept_logits"][i][:vocab]
        ulp = fp16_ulp_diff(got.view(np.uint8).copy(), want.view(np.uint8).copy())
        diff = np.abs(got.astype(np.float32) - want.astype(np.float32))
        print(f"step {int(step)}: max ulp {int(ulp.max())}, bit-exact fraction {np.mean(ulp == 0):.5f}, "
              f"max abs {float(diff.max()):.4g} (logit range {float(np.abs(want.astype(np.float32)).max()):.3g})")
        # argmax agrees and the perturbation is small against the logits' scale
        assert int(np.argmax(got)) == int(np.argmax(want))
        assert float(diff.max()) <= LOGIT_TOL * float(np.abs(want.astype(np.float32)).max())
    assert exact.mean() >= 0.9
