"""GPU parity of the CUDA engine (B200).

Integer / byte work (MATMUL, REQUANT*, QUANT, MAX_ABS, DMA, transposes,
DEQUANT*, VADD*, LayerNorm) must be bit-exact against the reference goldens.
GELU and softmax use exp / tanh / x**3 that NumPy's float32 SIMD code does not
round correctly; the engine evaluates them in float64 and rounds once.  Their
FP16 outputs are held to FP16_TOL: at most 2 FP16 ulp where |ref| >= 2^-6 and
at most 2^-14 absolute below that (GELU's 1 + tanh(x) cancels for large
negative x, which magnifies a one-ulp float32 tanh difference there); legacy
INT8-I/O outputs to one int8 step.
"""
from __future__ import annotations

import numpy as np
import pytest

import op_cases as oc
from helpers import (ProgramStub, expected_post, fp16_ulp_diff, load_bundle, load_op_golden, load_run,
                     run_bundle_sequence, vadd_chain_program)
from oracle import isa as OI

pytestmark = pytest.mark.gpu

CASES = oc.case_list()
GOLD = load_op_golden()
FP16_OUT = {0x1B, 0x1C, 0x1D}
FP16_TOL_ULP, FP16_TOL_SMALL, FP16_TOL_ABS = 2, 2.0 ** -6, 2.0 ** -14


def assert_fp16_close(got: np.ndarray, want: np.ndarray, what: str = ""):
    """FP16_TOL check on two byte arrays holding FP16 values."""
    g = got.view(np.float16).astype(np.float32)
    w = want.view(np.float16).astype(np.float32)
    ulp = fp16_ulp_diff(got, want)
    small = np.abs(w) < FP16_TOL_SMALL
    bad = np.where(small, np.abs(g - w) > FP16_TOL_ABS, ulp > FP16_TOL_ULP)
    assert not bad.any(), f"{what}: {int(bad.sum())} values out of tolerance, max ulp {int(ulp.max())}, " \
                          f"max abs {float(np.max(np.abs(g - w))):.3g}"
    return float(np.mean(ulp == 0))


I8_OUT_TRANSC = {0x0E, 0x10, 0x15, 0x12, 0x16}


def _sim():
    from llm_accelerator_b200.simulator import B200Simulator
    return B200Simulator()


def _run_case_gpu(case):
    sim = _sim()
    abuf, wbuf, accum, sregs, dram = oc.pre_state(case)
    if case["kind"] == "program":
        sim.load_program(ProgramStub(case["words"]))
        sim.state.dram[:len(dram)] = dram.tobytes()
    st = sim.state
    st.abuf[:] = abuf.tobytes()
    st.wbuf[:] = wbuf.tobytes()
    st.accum.view(np.uint8)[:] = accum.tobytes()
    st.scale_regs[:] = sregs.view(np.float16)
    if case["tile"] is not None:
        st.tile_config = tuple(case["tile"])
    v, q, k, m = case["attn"]
    if v:
        st.attn_context = {"is_valid": True, "query_row_base": q, "valid_kv_len": k, "mode": m}
    err = ""
    try:
        if case["kind"] == "program":
            sim.run()
        else:
            sim._execute(OI.decode_word(int(case["words"][0])))
    except Exception as e:
        err = type(e).__name__
    post = dict(abuf=np.frombuffer(bytes(st.abuf), np.uint8), wbuf=np.frombuffer(bytes(st.wbuf), np.uint8),
                accum=np.frombuffer(bytes(st.accum.view(np.uint8)), np.uint8),
                sregs=np.asarray(st.scale_regs).view(np.uint8))
    if dram is not None:
        post["dram"] = np.frombuffer(bytes(st.dram[:len(dram)]), np.uint8)
    return err, post, st.cycle_count


@pytest.mark.parametrize("i", range(len(CASES)))
def test_engine_op_case(i):
    case, rec = CASES[i], GOLD[i]
    err, post, cycles = _run_case_gpu(case)
    assert err == rec["err"]
    assert cycles == rec["cycles"]
    exp = expected_post(case, rec)
    op = case["op"]
    for nm, got in post.items():
        want = exp[nm]
        if op in FP16_OUT and nm == "abuf":
            assert_fp16_close(got.copy(), want.copy(), nm)
        elif op in I8_OUT_TRANSC and nm == "abuf":
            d = np.abs(got.view(np.int8).astype(np.int16) - want.view(np.int8).astype(np.int16))
            assert d.max() <= 1, f"{nm}: max int8 step {d.max()}"
        else:
            np.testing.assert_array_equal(got, want, err_msg=nm)


@pytest.mark.parametrize("commute", [False, True], ids=["sum-first", "sum-second"])
@pytest.mark.parametrize("produced", [False, True], ids=["loaded", "produced"])
@pytest.mark.parametrize("shape,parts", [((16, 32), 8), ((16, 256), 8), ((16, 512), 8), ((16, 256), 11)],
                         ids=["16x32", "16x256", "16x512", "16x256-11-parts"])
def test_engine_running_fp16_sum(shape, parts, produced, commute):
    """A running FP16 sum over VADD_FP32s (K_VADD_CHAIN ops on the device,
    operands staged by bulk copies, tasks of 4096 elements) is bit-exact
    against the oracle, including the intermediate sum a STORE writes to
    DRAM."""
    from types import SimpleNamespace
    from oracle import golden as G
    words, img, _ = vadd_chain_program(*shape, parts=parts, commute=commute, produced=produced)
    sim = _sim()
    sim.load_program(ProgramStub(words))
    sim.state.dram[:len(img)] = img.tobytes()
    sim.run()
    orc = G.OracleSimulator()
    stub = ProgramStub(words)
    orc.load_program(SimpleNamespace(instructions=stub.instructions, data_base=0, data=img.tobytes(), entry_point=0,
                                     insn_count=stub.insn_count))
    orc.run()
    for nm in ("abuf", "wbuf"):
        assert bytes(getattr(sim.state, nm)) == bytes(getattr(orc.state, nm)), nm
    assert bytes(sim.state.dram[:len(img)]) == bytes(orc.state.dram[:len(img)])
    assert sim.state.cycle_count == orc.state.cycle_count


@pytest.mark.parametrize("scale", [0x3C00, 0x2000, 0x50B0, 0x7BFF, 0x0001, 0xC200, 0x7C00, 0x7E00],
                         ids=["1", "2^-7", "37.5", "65504", "2^-24", "-3", "inf", "nan"])
def test_engine_quant_every_fp16_value(scale):
    """QUANT_FP32_INT8 of all 65536 FP16 bit patterns (NaNs, infinities,
    subnormals, halfway cases) with one scale register is bit-exact against
    the oracle: rint(x * s) ties to even, NaN -> 0, clipped to int8."""
    from types import SimpleNamespace
    from llm_accelerator_b200 import isa
    from oracle import golden as G
    X = 8192 // 16
    prog = [dict(opcode=0x05, addr_reg=0, imm28=0), dict(opcode=0x06, addr_reg=0, imm28=0),
            dict(opcode=0x03, M=64 // 16 - 1, N=1024 // 16 - 1, K=0),
            dict(opcode=0x07, buf_id=0, sram_off=0, xfer_len=8192, addr_reg=0, dram_off=X),
            dict(opcode=0x04, sreg=1, src_mode=0, imm16=scale),
            dict(opcode=0x18, src1_buf=0, src1_off=0, src2_buf=0, src2_off=0, dst_buf=1, dst_off=0, sreg=1),
            dict(opcode=0x01)]
    words = [isa.word_of(isa.encode(SimpleNamespace(**d))) for d in prog]
    img = np.zeros(X * 16 + 131072 + 4096, np.uint8)
    img[X * 16:X * 16 + 131072] = np.arange(65536, dtype=np.uint16).view(np.uint8)
    sim = _sim()
    sim.load_program(ProgramStub(words))
    sim.state.dram[:len(img)] = img.tobytes()
    sim.run()
    orc = G.OracleSimulator()
    stub = ProgramStub(words)
    orc.load_program(SimpleNamespace(instructions=stub.instructions, data_base=0, data=img.tobytes(), entry_point=0,
                                     insn_count=stub.insn_count))
    orc.run()
    got = np.frombuffer(bytes(sim.state.wbuf), np.int8)[:65536]
    want = np.frombuffer(bytes(orc.state.wbuf), np.int8)[:65536]
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"{bad.size} values differ, first FP16 bits {bad[:4]}: got {got[bad[:4]]} want {want[bad[:4]]}"


@pytest.mark.parametrize("name", ["tiny_l1_d64", "tiny_l2_d128"])
def test_engine_bundle_run_matches_reference(name):
    from llm_accelerator_b200.runner import HostRunner
    b, gold = load_bundle(name), load_run(name)
    toks, logits, sim = run_bundle_sequence(_sim, b, gold["prompt"], len(gold["logits"]), int(gold["vocab"][0]),
                                            HostRunner)
    assert toks == gold["tokens"].tolist()
    ulp = fp16_ulp_diff(logits.view(np.uint8).ravel().copy(), gold["logits"].view(np.uint8).ravel().copy())
    exact = float(np.mean(ulp == 0))
    print(f"{name}: logits bit-exact fraction {exact:.5f}, max ulp {ulp.max()}")
    assert exact >= 0.99
    assert np.max(np.abs(logits.astype(np.float32) - gold["logits"].astype(np.float32))) < 5e-2
    assert sim.state.cycle_count == int(gold["cycles"][0])


@pytest.mark.parametrize("path", ["words", "formulas"])
def test_batched_runner_matches_single_sequence_runs(path):
    """BatchedRunner.step (runtime words) and step_async (parameters from
    tokens and positions through the site formulas) both reproduce
    single-sequence runs bit for bit."""
    from llm_accelerator_b200.runner import BatchedRunner, HostRunner
    b = load_bundle("tiny_l2_d128")
    B, steps, vocab = 4, 6, 512
    rng = np.random.default_rng(11)
    prompts = rng.integers(0, vocab, (B, steps))
    br = BatchedRunner(b, B)
    batched = []
    for pos in range(steps):
        name = "prefill" if pos == 0 else "decode"
        if path == "words":
            br.step(name, prompts[:, pos], np.full(B, pos))
        else:
            br.step_async(name, prompts[:, pos], np.full(B, pos))
            br.engine.check_device()
        batched.append(np.stack([br.logits(name, s) for s in range(B)]))
    batched = np.stack(batched, axis=1)   # [B, steps, vocab_pad]
    for s in range(B):
        b2 = load_bundle("tiny_l2_d128")
        _, single, _ = run_bundle_sequence(_sim, b2, prompts[s], steps, vocab, HostRunner)
        np.testing.assert_array_equal(batched[s].view(np.uint16), single.view(np.uint16))


@pytest.mark.parametrize("B", [80, 150])
def test_batched_runner_head_groups_match_single_sequence_runs(B):
    """At batches whose attention pairs run in head groups (2 pairs a task at
    80 sequences, 4 at 150), sampled sequences of the batch reproduce their
    single-sequence runs bit for bit, one of them at a ragged position."""
    from llm_accelerator_b200.runner import BatchedRunner, HostRunner
    b = load_bundle("tiny_l2_d128")
    steps, vocab = 4, 512
    rng = np.random.default_rng(B)
    prompts = rng.integers(0, vocab, (B, steps))
    br = BatchedRunner(b, B)
    ops, _, tasks, lv = br.plans["decode"].dump()
    assert (ops[tasks[:int(lv[-1])]["op"]]["flags2"] & 2048).any(), "no head-group tasks in the plan"
    br.step("prefill", prompts[:, 0], np.zeros(B, int))
    for pos in range(1, steps):
        br.step("decode", prompts[:, pos], np.full(B, pos))
    # the last token once more: at its own position for every sequence but
    # sequence 1, which takes it at the position before
    br.step("decode", prompts[:, steps - 1], np.where(np.arange(B) == 1, steps - 2, steps - 1))
    for s in (0, 1, B // 2, B - 1):
        r = HostRunner(load_bundle("tiny_l2_d128"), simulator=_sim(), logits_dtype=np.float16)
        r.run_prefill([int(prompts[s, 0])])
        last = steps - 2 if s == 1 else steps - 1
        for pos in range(1, last + 1 if s != 1 else last):
            r.run_decode_step(int(prompts[s, pos]), pos)
        want = r.run_decode_step(int(prompts[s, steps - 1]), last)
        np.testing.assert_array_equal(br.logits("decode", s).view(np.uint16), want.view(np.uint16))


def test_batched_runner_ragged_positions():
    """Sequences at different positions in one step (per-sequence runtime words):
    sequence 1 re-runs position 1 while sequences 0 and 2 move to position 2."""
    from llm_accelerator_b200.runner import BatchedRunner, HostRunner
    b = load_bundle("tiny_l1_d64")
    B = 3
    br = BatchedRunner(b, B)
    br.step("prefill", np.array([5, 6, 7]), np.zeros(B, int))
    br.step("decode", np.array([9, 10, 11]), np.array([1, 1, 1]))
    br.step("decode", np.array([12, 13, 14]), np.array([2, 1, 2]))
    for seq, (t0, t1, t2, p2) in enumerate([(5, 9, 12, 2), (6, 10, 13, 1), (7, 11, 14, 2)]):
        r = HostRunner(load_bundle("tiny_l1_d64"), simulator=_sim(), logits_dtype=np.float16)
        r.run_prefill([t0])
        r.run_decode_step(t1, 1)
        want = r.run_decode_step(t2, p2)
        np.testing.assert_array_equal(br.logits("decode", seq).view(np.uint16), want.view(np.uint16))


# ---- the reference's gen2 known-answer vectors on the engine (tests/golden/gen2_kats.npz) ----
from test_oracle_pin import gen2_cases, gen2_setup  # noqa: E402


@pytest.mark.parametrize("case", [c[0] for c in gen2_cases()])
def test_engine_replays_reference_gen2_kats(case):
    """Each gen2 vector through B200Simulator._execute: bit-exact, except the
    transcendental GELU and masked softmax outputs (FP16_TOL)."""
    name, meta, files = next(c for c in gen2_cases() if c[0] == case)
    insn, s1buf, s2buf, attn = gen2_setup(meta, files)
    sim = _sim()
    st = sim.state
    st.tile_config = (meta["M"] // 16 - 1, meta["N"] // 16 - 1, 0)
    st.scale_regs[:] = np.frombuffer(files["scale_regs_pre.raw"], dtype=np.float16)

    def put(buf, off, data):
        view = st.accum.view(np.uint8) if buf == OI.ACCUM else (st.abuf if buf == OI.ABUF else st.wbuf)
        view[off * 16:off * 16 + len(data)] = data

    put(s1buf, meta["src1_off"], files["input_src1.raw"])
    if "input_src2.raw" in files:
        put(s2buf, meta["src2_off"], files["input_src2.raw"])
    if attn:
        st.attn_context = attn
    sim._execute(insn)
    exp = files["expected_out.raw"]
    sregs = np.asarray(st.scale_regs).tobytes()
    if insn.opcode == OI.MAX_ABS_REDUCE_FP32:
        assert sregs == exp, name
    elif exp:
        got = bytes(st.abuf[meta["dst_off"] * 16:meta["dst_off"] * 16 + len(exp)])
        if insn.opcode in (OI.GELU_FP32, OI.MASKED_SOFTMAX_FP32):
            assert_fp16_close(np.frombuffer(got, np.uint8).copy(), np.frombuffer(exp, np.uint8).copy(), name)
        else:
            assert got == exp, name
    assert sregs == files["scale_regs_post.raw"], name
