"""CPU tests of the C++ stream compiler (no GPU needed).

The compiler must (a) fault exactly where and how the reference faults,
(b) count retired instructions and analytic cycles like the reference, and
(c) produce a plan whose execution, in level order, reproduces the oracle's
machine state bit-for-bit.  (c) runs the plan through tests/plan_exec.py with
the oracle's NumPy arithmetic, so it checks the dataflow transformation
(renaming, aliasing, gathers, levels, final materialisation) in isolation.
"""
from __future__ import annotations

import numpy as np
import pytest

import op_cases as oc
import plan_exec as PE
from helpers import GOLDEN, load_bundle, load_op_golden, load_run, vadd_chain_program
from llm_accelerator_b200 import _lib as L
from llm_accelerator_b200.engine import Site, compile_program
from oracle import golden as G

CASES = oc.case_list()
GOLD = load_op_golden()
DRAM = 16 * 1024 * 1024
ERR_OF_STATUS = {L.E_SIMULATOR: "SimulatorError", L.E_ILLEGAL_OPCODE: "IllegalOpcodeError",
                 L.E_ILLEGAL_BUFFER: "IllegalBufferError", L.E_CONFIG: "ConfigError",
                 L.E_SRAM_ACCESS: "SRAMAccessError", L.E_DRAM_ACCESS: "DRAMAccessError", L.E_VALUE: "ValueError"}


def _regs(case):
    r = L.Regs()
    if case["tile"] is not None:
        r.tile_valid = 1
        r.tile[0], r.tile[1], r.tile[2] = case["tile"]
    v, q, k, m = case["attn"]
    if v:
        r.attn_valid, r.attn_qrb, r.attn_vkl, r.attn_mode = 1, q, k, m
    return r


def _compile_case(case):
    region = b"".join(int(w).to_bytes(8, "big") for w in case["words"])
    return compile_program(1, DRAM, 0, region, 0, 10_000_000 if case["kind"] == "program" else 1, _regs(case),
                           False, ())


@pytest.mark.parametrize("i", range(len(CASES)))
def test_compiler_faults_and_cycles_match_reference(i):
    case, rec = CASES[i], GOLD[i]
    p = _compile_case(case)
    err = ERR_OF_STATUS.get(int(p.fault.status), "") if p.info.faulted else ""
    assert err == rec["err"], p.fault.message
    assert int(p.info.cycles) == rec["cycles"]


@pytest.mark.parametrize("i", [i for i, c in enumerate(CASES) if c["op"] not in
                               (0x0F, 0x0E, 0x10, 0x15, 0x12, 0x16)])
def test_plan_reproduces_reference_op_case(i):
    """Executes the compiled plan with NumPy and compares with the golden record."""
    case, rec = CASES[i], GOLD[i]
    if rec["err"]:
        pytest.skip("faulting case (covered by the fault test)")
    p = _compile_case(case)
    abuf, wbuf, accum, sregs, dram = oc.pre_state(case)
    img = np.zeros(DRAM, np.uint8)
    if dram is not None:
        img[:len(dram)] = dram
    img[:len(case["words"]) * 8] = np.frombuffer(b"".join(int(w).to_bytes(8, "big") for w in case["words"]), np.uint8) \
        if case["kind"] == "program" and dram is None else img[:len(case["words"]) * 8]
    m = PE.PlanMachine(img.tobytes(), 0, int(p.info.arena_bytes), int(p.info.n_slots))
    m.block[:131072] = abuf
    m.block[131072:393216] = wbuf
    m.block[393216:458752] = accum
    m.sregs[:16] = sregs
    ops, segs, tasks, lv = p.dump()
    PE.run_plan(m, ops, segs, lv)
    f = PE.final_state(m)
    from helpers import expected_post
    exp = expected_post(case, rec)
    assert f["abuf"] == exp["abuf"].tobytes()
    assert f["wbuf"] == exp["wbuf"].tobytes()
    assert f["accum"] == exp["accum"].tobytes()
    assert f["sregs"] == exp["sregs"].tobytes()
    if "dram" in exp:
        assert f["dram"][:len(exp["dram"])] == exp["dram"].tobytes()


def _sites(b, name):
    sites = []
    for s in b.runtime_patch_sites:
        if s.stream == name:
            lo, hi = b.symbol_extent(s.base_symbol)
            sites.append(Site(0, s.addr_reg, s.absolute_lo_pc, s.absolute_hi_pc, lo, hi))
    for s in b.runtime_config_attn_sites:
        if s.stream == name:
            sites.append(Site(1, 0, s.absolute_pc))
    return sites


def _params(region, sites):
    out = []
    for s in sites:
        if s.kind == 0:
            lo = int.from_bytes(region[s.lo_pc * 8:s.lo_pc * 8 + 8], "big")
            hi = int.from_bytes(region[s.hi_pc * 8:s.hi_pc * 8 + 8], "big")
            out.append((((hi >> 29) & 0xFFFFFFF) << 28) | ((lo >> 29) & 0xFFFFFFF))
        else:
            w = int.from_bytes(region[s.lo_pc * 8:s.lo_pc * 8 + 8], "big")
            out.append(((w >> 47) & 0xFFF) | (((w >> 35) & 0xFFF) << 16) | (((w >> 33) & 3) << 32))
    return out


def _narrow_kv(b, nm, sites, plan):
    """KV sites narrowed to base + key_cols * kv_step_bytes, as BatchedRunner does."""
    keys = plan.attn_key_cols()
    meta = [s for s in b.runtime_patch_sites if s.stream == nm]
    out = []
    for i, site in enumerate(sites):
        if site.kind == 0 and i < len(meta) and meta[i].kind == "kv_base" and keys:
            site = Site(0, site.addr_reg, site.lo_pc, site.hi_pc, site.range_lo,
                        min(site.range_hi, site.range_lo + keys * b.kv_step_bytes))
        out.append(site)
    return out


def _check_plans_against_oracle(b, tokens, reverse: bool, narrow: bool, pack: bool = True):
    """Compiles b's prefill and decode streams once (runtime sites as plan
    parameters), runs prefill + decode steps of `tokens` through the plans
    with each step's parameters, and compares the whole machine state with the
    oracle's after every step.  pack=False: plans without arena reuse, whose
    uncomputed rows (ops narrowed to the rows read) are overwritten with NaN
    bytes after each op, so any read of them shows."""
    orc = G.OracleSimulator()
    orc.load_bundle(b)
    dram_bytes, shared = len(orc.state.dram), b.temp_base // 16 * 16
    plans = {}
    for nm in ("prefill", "decode"):
        sites = _sites(b, nm)
        region = bytearray(b.instruction_region())
        for s in sites:
            for pc in ((s.lo_pc, s.hi_pc) if s.kind == 0 else (s.lo_pc,)):
                w = int.from_bytes(region[pc * 8:pc * 8 + 8], "big") & (0x7F << 57)
                region[pc * 8:pc * 8 + 8] = w.to_bytes(8, "big")
        entry = b.prefill_pc if nm == "prefill" else b.decode_pc
        plan = compile_program(1, dram_bytes, shared, bytes(region), entry, 10_000_000, L.Regs(), True, sites,
                               pack=pack)
        if narrow:
            sites = _narrow_kv(b, nm, sites, plan)
            plan = compile_program(1, dram_bytes, shared, bytes(region), entry, 10_000_000, L.Regs(), True, sites,
                                   pack=pack)
        plans[nm] = (plan, sites)
    arena = max(int(p.info.arena_bytes) for p, _ in plans.values())
    slots = max(int(p.info.n_slots) for p, _ in plans.values())
    m = PE.PlanMachine(bytes(orc.state.dram), shared, arena, slots)
    for pos, tok in enumerate(tokens):
        nm = "prefill" if pos == 0 else "decode"
        row = b.embedding_row_bytes
        for s in b.runtime_patch_sites:
            if s.stream == nm:
                b.patch_runtime_site(s, {"token_embed": tok * row, "pos_embed": pos * row,
                                         "kv_base": pos * b.kv_step_bytes}[s.kind])
        for s in b.runtime_config_attn_sites:
            if s.stream == nm:
                b.patch_config_attn_site(s, query_row_base=pos, valid_kv_len=pos + 1)
        region = bytes(b.instruction_region())
        m.shared[:len(region)] = np.frombuffer(region, np.uint8)
        p, sites = plans[nm]
        ops, segs, tasks, lv = p.dump()
        PE.run_plan(m, ops, segs, lv, _params(region, sites), reverse=reverse, poison=not pack)
        n = orc.run_program(b, nm)
        assert n == int(p.info.executed)
        f = PE.final_state(m)
        st = orc.state
        assert f["abuf"] == bytes(st.abuf) and f["wbuf"] == bytes(st.wbuf)
        assert f["accum"] == st.accum.tobytes() and f["sregs"] == st.scale_regs.tobytes()
        assert f["dram"] == bytes(st.dram[:len(f["dram"])])


@pytest.mark.parametrize("pack", [True, False], ids=["packed", "unpacked-poisoned"])
@pytest.mark.parametrize("narrow", [False, True], ids=["symbol-ranges", "kv-window-ranges"])
@pytest.mark.parametrize("reverse", [False, True], ids=["level-order", "level-reversed"])
@pytest.mark.parametrize("name", ["tiny_l1_d64", "tiny_l2_d128"])
def test_plan_reproduces_oracle_bundle_run(name, reverse, narrow, pack):
    """Prefill + decode steps: one plan per stream compiled with runtime sites,
    executed with each step's parameters, equals the oracle bit-for-bit, also
    with every level's ops run in reverse order (no hidden intra-level
    dependency, e.g. between the KV-cache appends of one step), and without
    arena reuse with the rows narrowed ops skip overwritten."""
    b = load_bundle(name)
    gold = load_run(name)
    prompt = gold["prompt"]
    tokens = [int(prompt[pos]) if pos < len(prompt) else int(gold["tokens"][pos]) for pos in range(6)]
    _check_plans_against_oracle(b, tokens, reverse, narrow, pack)


@pytest.mark.parametrize("pack", [True, False], ids=["packed", "unpacked-poisoned"])
def test_plan_reproduces_oracle_gpt2_small(pack):
    """GPT-2 small (12 layers, d_model 768): the decode plan carries every
    fusion of the full-size streams (tcgen05 projections with their dequant
    epilogues, the K-split partial sums as VADD chains, MAX_ABS + QUANT,
    attention with the softmax in the QK^T task, row-wise ops narrowed to the
    rows read); prefill and two decode steps equal the oracle bit-for-bit."""
    from llm_accelerator_b200.recipe import load_recipe
    b = load_recipe(GOLDEN / "recipe_gpt2_small.npz")
    _check_plans_against_oracle(b, [464, 2068, 7586], reverse=True, narrow=True, pack=pack)


def test_runtime_site_out_of_range_requests_recompile():
    """A patched word outside its compiled range is reported, not executed."""
    b = load_bundle("tiny_l1_d64")
    sites = _sites(b, "decode")
    assert sites and sites[0].kind == 0
    region = bytes(b.instruction_region())
    p = compile_program(1, 16 << 20, b.temp_base // 16 * 16, region, b.decode_pc, 10_000_000, L.Regs(), True, sites)
    assert int(p.info.n_var_words) == sum(2 if s.kind == 0 else 1 for s in sites)
    assert int(p.info.n_levels) > 0 and not p.info.faulted


def _check_prefetch_hints(p, dram_bytes, shared_bytes):
    """Every task's L2 prefetch range lies inside the memory its op reads:
    the per-sequence block [SRAM | writable DRAM | arena] or the shared image."""
    ops, segs, tasks, lv = p.dump()
    block_units = PE.SRAM_UNITS + (dram_bytes - shared_bytes + 15) // 16 + int(p.info.arena_bytes) // 16
    hinted = tasks[tasks["pf_units"] > 0]
    assert len(hinted) > 0
    phys = hinted["pf_phys"].astype(np.uint64)
    units = hinted["pf_units"].astype(np.uint64)
    shared = (phys >> np.uint64(63)) == 1
    off = phys & np.uint64((1 << 63) - 1)
    end = off + units
    assert np.all(end[shared] <= np.uint64(shared_bytes // 16))
    assert np.all(end[~shared] <= np.uint64(block_units))
    tc = (ops[hinted["op"]]["flags"] & 8) != 0   # tcgen05 tasks hint their whole weight matrix, up to 256 KB
    assert np.all(units[~tc] <= 4096) and np.all(units[tc] <= 16384)
    # a per-sequence MATMUL operand B: the hint covers at most B's bytes (FP16 under F_QB)
    for t in hinted:
        op = ops[int(t["op"])]
        if int(op["kind"]) == PE.K["MATMUL"] and not int(op["b"]) >> 63 and not int(op["flags"]) & 8:
            b_units = int(op["K"]) * int(op["N"]) * (2 if int(op["flags"]) & 512 else 1) // 16
            assert int(t["pf_phys"]) == int(op["b"]) and int(t["pf_units"]) == min(b_units, 4096)


@pytest.mark.parametrize("name", ["tiny_l1_d64", "tiny_l2_d128"])
@pytest.mark.parametrize("batch", [1, 4])
def test_prefetch_hints_stay_inside_operands(name, batch):
    b = load_bundle(name)
    shared = b.temp_base // 16 * 16
    for nm in ("prefill", "decode"):
        entry = b.prefill_pc if nm == "prefill" else b.decode_pc
        p = compile_program(batch, 16 << 20, shared, bytes(b.instruction_region()), entry, 10_000_000, L.Regs(),
                            True, _sites(b, nm))
        _check_prefetch_hints(p, 16 << 20, shared)


def _var_words(region, sites):
    words = []
    for s in sites:
        pcs = (s.lo_pc, s.hi_pc) if s.kind == 0 else (s.lo_pc,)
        words += [int.from_bytes(region[pc * 8:pc * 8 + 8], "big") for pc in pcs]
    return np.array(words, np.uint64)


def test_sites_over_one_symbol_must_carry_one_value():
    """The KV-cache appends of a decode step go through runtime sites over one
    symbol (kv_bank0) at different static offsets; the plan leaves them
    unordered on the assumption that those sites hold one value, and checks
    it: unequal values are reported (TAC_E_RECOMPILE), not executed."""
    import ctypes as C
    b = load_bundle("tiny_l2_d128")
    sites = _sites(b, "decode")
    kv = [i for i, (s, m) in enumerate(zip(sites, [x for x in b.runtime_patch_sites if x.stream == "decode"]))
          if s.kind == 0 and m.kind == "kv_base"]
    assert len(kv) >= 4
    p = compile_program(1, 16 << 20, b.temp_base // 16 * 16, bytes(b.instruction_region()), b.decode_pc,
                        10_000_000, L.Regs(), True, sites)
    for s in b.runtime_patch_sites:
        if s.stream == "decode":
            b.patch_runtime_site(s, {"token_embed": 3 * b.embedding_row_bytes, "pos_embed": 2 * b.embedding_row_bytes,
                                     "kv_base": 2 * b.kv_step_bytes}[s.kind])
    words = _var_words(bytes(b.instruction_region()), sites)
    out = np.zeros(len(sites), np.uint64)
    f = L.Fault()
    assert L.lib.tac_encode_params(p.handle, 1, words.ctypes.data, out.ctypes.data, C.byref(f)) == L.OK
    # move one KV site by one row (still inside its range and aligned)
    site = b.runtime_patch_sites[[x for x in b.runtime_patch_sites if x.stream == "decode"].index(
        [x for x in b.runtime_patch_sites if x.stream == "decode"][kv[-1]])]
    b.patch_runtime_site(site, 3 * b.kv_step_bytes)
    words = _var_words(bytes(b.instruction_region()), sites)
    assert L.lib.tac_encode_params(p.handle, 1, words.ctypes.data, out.ctypes.data, C.byref(f)) == L.E_RECOMPILE


def _words(*insns):
    from types import SimpleNamespace
    from llm_accelerator_b200 import isa
    return b"".join(isa.encode(SimpleNamespace(**d)) for d in insns)


@pytest.mark.parametrize("reverse", [False, True], ids=["level-order", "level-reversed"])
@pytest.mark.parametrize("then", ["halt", "overwrite-then-read"])
def test_load_aliases_dram_until_it_is_overwritten(then, reverse):
    """A LOAD from writable DRAM reads the DRAM bytes in place; a later write
    of those bytes (here the end-of-run flush of a STORE, or a STORE followed
    by a LOAD of the same bytes) must not change what the LOAD saw."""
    X = 8192 // 16   # DRAM unit of the data
    prog = [dict(opcode=0x05, addr_reg=0, imm28=0), dict(opcode=0x06, addr_reg=0, imm28=0),
            dict(opcode=0x07, buf_id=0, sram_off=0, xfer_len=4, addr_reg=0, dram_off=X),     # ABUF[0:64] <- X
            dict(opcode=0x08, buf_id=1, sram_off=0, xfer_len=4, addr_reg=0, dram_off=X)]     # X <- WBUF[0:64]
    if then == "overwrite-then-read":
        prog.append(dict(opcode=0x07, buf_id=2, sram_off=0, xfer_len=4, addr_reg=0, dram_off=X))  # ACCUM <- X
    prog.append(dict(opcode=0x01))
    region = _words(*prog)
    p = compile_program(1, DRAM, 0, region, 0, 100, L.Regs(), True, ())
    assert not p.info.faulted
    rng = np.random.default_rng(7)
    img = np.zeros(DRAM, np.uint8)
    img[:len(region)] = np.frombuffer(region, np.uint8)
    old = rng.integers(0, 256, 64, dtype=np.uint8)
    new = rng.integers(0, 256, 64, dtype=np.uint8)
    img[8192:8256] = old
    m = PE.PlanMachine(img.tobytes(), 0, int(p.info.arena_bytes), int(p.info.n_slots))
    m.block[131072:131072 + 64] = new
    ops, segs, tasks, lv = p.dump()
    PE.run_plan(m, ops, segs, lv, reverse=reverse)
    f = PE.final_state(m)
    assert f["abuf"][:64] == old.tobytes()
    assert f["dram"][8192:8256] == new.tobytes()
    if then == "overwrite-then-read":
        assert f["accum"][:64] == new.tobytes()


def test_self_modifying_store_is_rejected():
    # SET_ADDR R1 = 0 ; STORE ABUF[0..16) -> DRAM[0] (the instruction region) ; HALT
    words = [(0x05 << 59) | (1 << 57), (0x06 << 59) | (1 << 57),
             (0x08 << 59) | (1 << 25) | (1 << 23), 0x01 << 59]
    region = b"".join(w.to_bytes(8, "big") for w in words)
    with pytest.raises(Exception, match="self-modifying"):
        compile_program(1, DRAM, 0, region, 0, 100, L.Regs(), True, ())


def test_pc_past_end_and_halt_counts():
    words = [0x00 << 59, 0x02 << 59]   # NOP, SYNC, no HALT
    region = b"".join(w.to_bytes(8, "big") for w in words)
    p = compile_program(1, DRAM, 0, region, 0, 100, L.Regs(), True, ())
    assert p.info.faulted and int(p.fault.status) == L.E_SIMULATOR
    assert int(p.info.executed) == 2 and int(p.info.cycles) == 2
    p = compile_program(1, DRAM, 0, region, 0, 1, L.Regs(), True, ())   # watchdog stops first
    assert not p.info.faulted and int(p.info.executed) == 1


@pytest.mark.parametrize("batch", [1, 3, 5, 8])
def test_tasks_cover_every_sequence_and_element_once(batch):
    """Element-wise tasks either take one chunk of one sequence or pack whole
    sequences; across an op's tasks every (sequence, element) appears once,
    counting the tasks a chain head runs for its sequence."""
    b = load_bundle("tiny_l2_d128")
    region = bytes(b.instruction_region())
    p = compile_program(batch, 16 << 20, b.temp_base // 16 * 16, region, b.decode_pc, 10_000_000, L.Regs(), True,
                        _sites(b, "decode"))
    ops, segs, tasks, lv = p.dump()
    EW_TASK = 8192
    ew_kinds = set(range(7, 18)) | {19, 27}
    task_elems = lambda kind: 4096 if kind in (19, 27) else (2 * EW_TASK if kind == 16 else EW_TASK)  # noqa: E731
    seen = {}
    run = []   # the tasks the executor runs: leveled tasks, chain heads expanded into their templates
    for t in tasks[:int(lv[-1])]:
        if int(ops[t["op"]]["flags2"]) & 128:   # FX_CHAINHEAD: templates tile .. tile + aux, this sequence
            for k in range(int(t["aux"])):
                tt = tasks[int(t["tile"]) + k].copy()
                assert int(tt["nseq"]) == 1
                tt["seq0"] = t["seq0"]
                run.append(tt)
        else:
            run.append(t)
    for t in run:
        op = ops[t["op"]]
        if int(op["kind"]) not in ew_kinds:
            continue
        MN = int(op["M"]) * int(op["N"])
        cov = seen.setdefault(int(t["op"]), np.zeros((batch, MN), np.int32))
        s0, n = int(t["seq0"]), int(t["nseq"])
        assert s0 + n <= batch
        te = 4096 if int(op["flags"]) & 32 else task_elems(int(op["kind"]))   # F_SEGA: 512 operand units
        if n > 1:
            assert n * MN <= te and int(t["tile"]) == 0
            cov[s0:s0 + n] += 1
        else:
            lo = int(t["tile"]) * te
            cov[s0, lo:lo + te] += 1
    assert seen, "no element-wise ops in the plan"
    for opi, cov in seen.items():
        assert (cov == 1).all(), f"op {opi}: coverage {np.unique(cov)}"



@pytest.mark.parametrize("reverse", [False, True], ids=["level-order", "level-reversed"])
@pytest.mark.parametrize("commute", [False, True], ids=["sum-first", "sum-second"])
@pytest.mark.parametrize("produced", [False, True], ids=["loaded", "produced"])
@pytest.mark.parametrize("shape,parts", [((16, 32), 8), ((16, 256), 8), ((16, 256), 11)],
                         ids=["16x32", "16x256", "16x256-11-parts"])
def test_running_fp16_sum_becomes_one_chain_op(shape, parts, produced, commute, reverse):
    """FP16 vectors summed by VADD_FP32s into one accumulator (the partial
    sums of a K-split projection) compile to K_VADD_CHAIN ops of at most 8
    operands, one level each; the plan, including an intermediate sum a
    STORE reads and an in-place accumulator, equals the oracle bit-for-bit.
    With produced vectors the ops that compute them follow the chain op in
    the plan, and dead-op elimination must keep them."""
    from types import SimpleNamespace
    words, img, _ = vadd_chain_program(*shape, parts=parts, commute=commute, produced=produced)
    region = b"".join(int(w).to_bytes(8, "big") for w in words)
    p = compile_program(1, len(img), 0, region, 0, 1000, L.Regs(), True, ())
    assert not p.info.faulted
    ops, segs, tasks, lv = p.dump()
    chains = ops[ops["kind"] == PE.K["VADD_CHAIN"]]
    # at most 8 operands a chain: the sum so far starts the next one
    assert [int(c["nseg"]) for c in chains] == ([8, parts - 8 + 1] if parts > 8 else [parts])
    assert not (ops["kind"] == PE.K["VADD_F16"]).any()
    m = PE.PlanMachine(img.tobytes(), 0, int(p.info.arena_bytes), int(p.info.n_slots))
    PE.run_plan(m, ops, segs, lv, reverse=reverse)
    f = PE.final_state(m)
    orc = G.OracleSimulator()
    orc.load_program(SimpleNamespace(instructions=region, data_base=0, data=img.tobytes(), entry_point=0,
                                     insn_count=len(words)))
    assert orc.run(1000) == int(p.info.executed)
    st = orc.state
    assert f["abuf"] == bytes(st.abuf) and f["wbuf"] == bytes(st.wbuf)
    assert f["dram"] == bytes(st.dram[:len(f["dram"])])


def test_segment_list_tasks_name_the_segments_they_read():
    """A segment-list element-wise task covers 512 operand units and stages
    only the segments holding them (Task.aux = first | count << 16); together
    those segments cover the task's units and nothing outside one segment on
    either side."""
    from llm_accelerator_b200.recipe import load_recipe
    b = load_recipe(GOLDEN / "recipe_gpt2_small.npz")
    p = compile_program(2, 1 << 30, b.temp_base // 16 * 16, bytes(b.instruction_region()), b.decode_pc,
                        10_000_000, L.Regs(), True, _sites(b, "decode"))
    ops, segs, tasks, lv = p.dump()
    seen = 0
    for i, t in enumerate(tasks):
        op = ops[int(t["op"])]
        if not int(op["flags"]) & 32 or int(op["kind"]) == PE.K["MAX_ABS"]:
            continue
        if i < int(lv[-1]) and int(op["flags2"]) & 128:
            continue   # a chain head's task points at the chain's templates (after the last level)
        units = int(op["M"]) * int(op["N"]) // 8
        u0 = int(t["tile"]) * 512
        u1 = min(units, u0 + 512)
        first, count = int(t["aux"]) & 0xFFFF, int(t["aux"]) >> 16
        assert count >= 1 and first + count <= int(op["nseg"])
        sl = segs[int(op["seg0"]) + first:int(op["seg0"]) + first + count]
        assert int(sl[0]["dst"]) <= u0 < int(sl[0]["dst"]) + int(sl[0]["n"])
        assert int(sl[-1]["dst"]) < u1 <= int(sl[-1]["dst"]) + int(sl[-1]["n"])
        assert all(int(a["dst"]) + int(a["n"]) == int(c["dst"]) for a, c in zip(sl[:-1], sl[1:]))
        seen += 1
    assert seen > 0


class _NoEngine:
    """Stands in for the GPU engine while BatchedRunner compiles its plans."""

    def __init__(self, *args, **kwargs):
        pass

    def write_dram(self, *args, **kwargs):
        pass


FX_PV, FX_ATTNGRP, HALVES = 4, 2048, 296


@pytest.mark.parametrize("batch,group", [(8, 1), (80, 2), (150, 4), (300, 4)])
def test_attention_head_groups_cover_every_pair_once(monkeypatch, batch, group):
    """Row-attention pairs (FX_PV QK^T ops of one query row) of a level run
    once per sequence: in a task of their own, or as templates of a head
    group (FX_ATTNGRP) task of one sequence.  A group holds pairs of one
    shape, its head op first; groups take the least size that fits the
    level's pairs into one round over the executor's 296 halves (all of a
    level's pairs per sequence, up to 8, when none does)."""
    from llm_accelerator_b200 import runner as R
    monkeypatch.setattr(R, "Engine", _NoEngine)
    r = R.BatchedRunner(load_bundle("tiny_l2_d128"), batch)
    ops, segs, tasks, lv = r.plans["decode"].dump()
    n_leveled = int(lv[-1])
    row_pairs = [i for i, op in enumerate(ops)
                 if int(op["flags2"]) & FX_PV and int(op["M"]) == 1 and int(op["flags"]) & 64]
    assert row_pairs
    runs = {}
    sizes = set()
    for L_ in range(len(lv) - 1):
        level = tasks[int(lv[L_]):int(lv[L_ + 1])]
        attn_tasks = 0
        for t in level:
            op = ops[int(t["op"])]
            if int(op["flags2"]) & FX_ATTNGRP:
                first, count = int(t["tile"]), int(t["aux"])
                assert n_leveled <= first and first + count <= len(tasks) and 1 <= count <= 8
                temps = tasks[first:first + count]
                assert int(temps[0]["op"]) == int(t["op"])
                assert len({(int(ops[o]["K"]), int(ops[o]["N"]), int(ops[int(ops[o]["seg0"])]["N"]))
                            for o in temps["op"]}) == 1
                assert all(int(ops[o]["level"]) == int(op["level"]) for o in temps["op"])
                for o in temps["op"]:
                    runs[(int(o), int(t["seq0"]))] = runs.get((int(o), int(t["seq0"])), 0) + 1
                sizes.add(count)
                attn_tasks += 1
            elif int(t["op"]) in row_pairs:
                runs[(int(t["op"]), int(t["seq0"]))] = runs.get((int(t["op"]), int(t["seq0"])), 0) + 1
                attn_tasks += 1
        if batch <= HALVES:
            assert attn_tasks <= HALVES
    assert runs == {(o, s): 1 for o in row_pairs for s in range(batch)}
    assert max(sizes, default=1) == group
    heads = {int(o) for o in np.nonzero(ops["flags2"] & FX_ATTNGRP)[0]}
    assert all(int(ops[o]["flags2"]) & FX_PV for o in heads)


def test_gpt2_medium_batch64_groups_run_every_op_once(monkeypatch):
    """At batch 64 the GPT-2 medium decode plan runs its attention pairs in
    head groups of four and its GELU MAX_ABS + QUANT ops in pairs
    (FX_MAXGRP, one task per pair and sequence, the second op a template);
    every such op runs exactly once per sequence, and each of those levels
    takes one round over the executor's 296 halves."""
    from llm_accelerator_b200 import runner as R
    from llm_accelerator_b200.recipe import load_recipe
    monkeypatch.setattr(R, "Engine", _NoEngine)
    B = 64
    r = R.BatchedRunner(load_recipe(GOLDEN / "recipe_gpt2_medium.npz"), B)
    ops, segs, tasks, lv = r.plans["decode"].dump()
    FX_MAXQ, FX_CHAINED, FX_MAXGRP, F_SEGA = 2, 64, 4096, 32
    grouped = [i for i, op in enumerate(ops)
               if (int(op["flags2"]) & FX_PV and int(op["M"]) == 1 and int(op["flags"]) & 64) or
               (int(op["kind"]) == PE.K["MAX_ABS"] and int(op["flags"]) & F_SEGA and int(op["flags2"]) & FX_MAXQ
                and not int(op["flags2"]) & FX_CHAINED)]
    runs, sizes = {}, {FX_ATTNGRP: set(), FX_MAXGRP: set()}
    for L_ in range(len(lv) - 1):
        level = tasks[int(lv[L_]):int(lv[L_ + 1])]
        n_group_tasks = 0
        for t in level:
            op = ops[int(t["op"])]
            f2 = int(op["flags2"])
            if f2 & (FX_ATTNGRP | FX_MAXGRP):
                temps = tasks[int(t["tile"]):int(t["tile"]) + int(t["aux"])]
                assert int(temps[0]["op"]) == int(t["op"])
                sizes[f2 & (FX_ATTNGRP | FX_MAXGRP)].add(int(t["aux"]))
                members = [int(o) for o in temps["op"]]
                n_group_tasks += 1
            elif int(t["op"]) in grouped:
                members = [int(t["op"])]
            else:
                continue
            for o in members:
                assert int(ops[o]["level"]) == int(op["level"])
                runs[(o, int(t["seq0"]))] = runs.get((o, int(t["seq0"])), 0) + 1
        assert n_group_tasks <= HALVES
    assert runs == {(o, s): 1 for o in grouped for s in range(B)}
    assert sizes == {FX_ATTNGRP: {4}, FX_MAXGRP: {2}}
