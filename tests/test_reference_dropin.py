"""The reference's own runtime drives B200Simulator unchanged.

``taccel.runtime.host_runner.HostRunner(bundle, simulator=B200Simulator())``
(``software/taccel/runtime/host_runner.py:15-20,84,94``) with the reference's
own ``ProgramBundle`` object (``software/taccel/assembler/assembler.py:163``):
the runner patches that object's runtime streams, calls ``load_bundle`` /
``run_program`` and reads logits back through ``state.dram[a:b]``.

* CPU (needs the reference package): the simulator's host side runs for real
  (bundle upload, stream writes, site handling, planning by the C++ compiler,
  read-back) with the plan executed by ``tests/plan_engine.py`` instead of the
  CUDA engine.  Logits, tokens and the cycle count equal the reference
  simulator's own run bit for bit, and the uploaded image equals the
  reference's ``materialize()``.
* GPU (needs the reference package and a B200): the same with the CUDA engine.

The reference package is found under ``baseline/_ref`` when it is installed
there, else in the checkout named by TACCEL_REFERENCE; the tests are skipped
when neither exists.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import fp16_ulp_diff, import_reference, load_bundle, load_run, to_reference_bundle

pytestmark = pytest.mark.reference
TINY = ["tiny_l1_d64", "tiny_l2_d128"]


@pytest.fixture
def plan_engine(monkeypatch):
    import llm_accelerator_b200.simulator as S
    from plan_engine import PlanEngine
    monkeypatch.setattr(S, "Engine", PlanEngine)
    return PlanEngine


def _drive(rb, sim, prompt, n_steps, vocab):
    """The reference HostRunner's prefill + decode loop (teacher-forced over
    the prompt, greedy after it)."""
    from taccel.runtime.host_runner import HostRunner
    r = HostRunner(rb, simulator=sim, logits_dtype=np.float16)
    logits = [r.run_prefill([int(prompt[0])])]
    toks = [int(t) for t in prompt]
    for pos in range(1, n_steps):
        tok = int(prompt[pos]) if pos < len(prompt) else int(np.argmax(logits[-1][:vocab]))
        if pos >= len(prompt):
            toks.append(tok)
        logits.append(r.run_decode_step(tok, pos))
    return toks, np.stack(logits)


def test_reference_bundle_passes_every_host_side_call(plan_engine):
    """load_bundle with the reference's ProgramBundle: the device image equals
    the reference's materialize(), the shared data is handed over as the
    bundle's own buffer (no materialised copy), and every runtime site of
    both streams is planned."""
    assert import_reference()
    from llm_accelerator_b200.simulator import B200Simulator
    b = load_bundle("tiny_l2_d128")
    rb = to_reference_bundle(b)
    sim = B200Simulator()
    sim.load_bundle(rb)
    eng = sim._eng()
    want = rb.materialize(reset_runtime=True)
    assert eng.read_dram(0, 0, len(want)) == want
    shared = [u for u in eng.uploads if u[1] == rb.data_base]
    assert shared == [(-1, rb.data_base, len(rb.shared_data), "bytes")]
    assert all(u[2] < len(rb.shared_data) for u in eng.uploads if u[1] != rb.data_base)
    for name in ("prefill", "decode"):
        sites = sim._bundle_sites(rb)
        region = sim._masked_region(sites)
        sim._reset_volatile(rb.prefill_pc if name == "prefill" else rb.decode_pc)
        prog = sim._plan(region, sites, 10_000_000, True)
        assert not prog.info.faulted and prog.info.halted
        assert prog.n_var_words == sum(2 if s.kind == 0 else 1 for s in sites)


@pytest.mark.parametrize("name", TINY)
def test_reference_host_runner_on_b200_simulator_cpu_plan(name, plan_engine):
    assert import_reference()
    from llm_accelerator_b200.simulator import B200Simulator
    b, gold = load_bundle(name), load_run(name)
    sim = B200Simulator()
    toks, logits = _drive(to_reference_bundle(b), sim, gold["prompt"], len(gold["logits"]), int(gold["vocab"][0]))
    assert toks == gold["tokens"].tolist()
    np.testing.assert_array_equal(logits.view(np.uint16), gold["logits"].view(np.uint16))
    assert sim.state.cycle_count == int(gold["cycles"][0])
    assert sim._eng().runs == len(gold["logits"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", TINY)
def test_reference_host_runner_on_b200_simulator_gpu(name):
    assert import_reference()
    from llm_accelerator_b200.simulator import B200Simulator
    b, gold = load_bundle(name), load_run(name)
    sim = B200Simulator()
    toks, logits = _drive(to_reference_bundle(b), sim, gold["prompt"], len(gold["logits"]), int(gold["vocab"][0]))
    assert toks == gold["tokens"].tolist()
    ulp = fp16_ulp_diff(logits.view(np.uint8).ravel().copy(), gold["logits"].view(np.uint8).ravel().copy())
    assert float(np.mean(ulp == 0)) >= 0.99
    assert np.max(np.abs(logits.astype(np.float32) - gold["logits"].astype(np.float32))) < 5e-2
    assert sim.state.cycle_count == int(gold["cycles"][0])
