"""Shared test helpers: golden fixture loading and oracle drivers."""
from __future__ import annotations

from pathlib import Path

import numpy as np

import op_cases as oc
from oracle import golden as G
from oracle import isa as OI

GOLDEN = Path(__file__).resolve().parent / "golden"


def load_op_golden():
    z = np.load(GOLDEN / "op_cases.npz")
    n = int(z["n_cases"][0])
    out = []
    for i in range(n):
        p = f"c{i:03d}_"
        err = bytes(z[p + "err"]).decode()
        rec = dict(err="" if err == "-" else err, cycles=int(z[p + "cycles"][0]), pc=int(z[p + "cycles"][1]))
        for nm in ("abuf", "wbuf", "accum", "sregs", "dram"):
            if p + nm + "_sha" not in z:
                continue
            offs, lens, data = z[p + nm + "_off"], z[p + nm + "_len"], bytes(z[p + nm + "_data"])
            spans, pos = [], 0
            for o, l in zip(offs, lens):
                spans.append((int(o), data[pos:pos + int(l)]))
                pos += int(l)
            rec[nm] = (bytes(z[p + nm + "_sha"]).hex(), spans)
        out.append(rec)
    return out


def apply_spans(pre: np.ndarray, spans):
    post = pre.copy()
    for o, d in spans:
        post[o:o + len(d)] = np.frombuffer(d, np.uint8)
    return post


class ProgramStub:
    """ProgramBinary-like container for short hand-built programs."""

    def __init__(self, words):
        self.instructions = b"".join(int(w).to_bytes(8, "big") for w in words)
        self.data = b""
        self.entry_point = 0
        self.insn_count = len(words)
        self.data_base = 0
        self.trace_manifest = {}


def vadd_chain_program(M: int, N: int, parts: int = 8, commute: bool = False, produced: bool = False,
                       seed: int = 11):
    """(instruction words, DRAM image, parts): `parts` FP16 [M, N] vectors
    summed into WBUF[0] by VADD_FP32s, the accumulator as src1 (commute=False)
    or src2; the sum after the fourth vector is STOREd to DRAM.  The vectors
    are LOADed from DRAM into ABUF, or (produced=True) each is computed just
    before it is added: an INT32 tile LOADed into ACCUM and dequantised by
    DEQUANT_ACCUM_FP32 into the same ABUF scratch every time, as the K-split
    projections of the compiler's decode streams do."""
    from llm_accelerator_b200 import isa
    from types import SimpleNamespace
    units = M * N * 2 // 16
    X = 8192 // 16                       # DRAM unit of the inputs
    rng = np.random.default_rng(seed)
    prog = [dict(opcode=0x05, addr_reg=0, imm28=0), dict(opcode=0x06, addr_reg=0, imm28=0),
            dict(opcode=0x03, M=M // 16 - 1, N=N // 16 - 1, K=0)]

    def add(k, part_buf, part_off):      # WBUF[0] <- WBUF[0] + part (or part + WBUF[0])
        srcs = (dict(src1_buf=part_buf, src1_off=part_off, src2_buf=1, src2_off=0) if commute else
                dict(src1_buf=1, src1_off=0, src2_buf=part_buf, src2_off=part_off))
        prog.append(dict(opcode=0x19, dst_buf=1, dst_off=0, **srcs))
        if k == 3:
            prog.append(dict(opcode=0x08, buf_id=1, sram_off=0, xfer_len=units, addr_reg=0, dram_off=Y))

    if produced:
        iunits = M * N * 4 // 16
        S = X + parts * iunits           # DRAM unit of the FP16 scale row
        Y = S + N * 2 // 16 + 64         # DRAM unit of the stored partial sum
        data = [(S, (rng.random(N) * 2e-3 + 1e-4).astype(np.float16)),
                (X, rng.integers(-(1 << 20), 1 << 20, parts * M * N).astype(np.int32))]
        prog.append(dict(opcode=0x07, buf_id=1, sram_off=units, xfer_len=N * 2 // 16, addr_reg=0, dram_off=S))
        for k in range(parts):
            prog.append(dict(opcode=0x07, buf_id=2, sram_off=0, xfer_len=iunits, addr_reg=0, dram_off=X + k * iunits))
            dst = dict(dst_buf=1, dst_off=0) if k == 0 else dict(dst_buf=0, dst_off=0)
            prog.append(dict(opcode=0x17, src1_buf=2, src1_off=0, src2_buf=1, src2_off=units, **dst))
            if k:
                add(k, 0, 0)
    else:
        Y = X + parts * units + 64
        data = [(X, (rng.standard_normal(parts * M * N) * 4).astype(np.float16))]
        for k in range(parts):   # ABUF[k * units] <- p_k
            prog.append(dict(opcode=0x07, buf_id=0, sram_off=k * units, xfer_len=units, addr_reg=0,
                             dram_off=X + k * units))
        prog.append(dict(opcode=0x19, src1_buf=0, src1_off=0, src2_buf=0, src2_off=units, dst_buf=1, dst_off=0))
        for k in range(2, parts):
            add(k, 0, k * units)
    prog.append(dict(opcode=0x01))
    words = [isa.word_of(isa.encode(SimpleNamespace(**d))) for d in prog]
    img = np.zeros((Y + units) * 16 + 4096, np.uint8)
    img[:len(words) * 8] = np.frombuffer(b"".join(int(w).to_bytes(8, "big") for w in words), np.uint8)
    for at, v in data:
        img[at * 16:at * 16 + v.nbytes] = v.view(np.uint8)
    return words, img, parts


def run_oracle_case(case):
    """Runs an op case on the oracle; returns (err name, post dict, cycles, pc)."""
    abuf, wbuf, accum, sregs, dram = oc.pre_state(case)
    st = G.OracleState()
    st.abuf[:] = abuf.tobytes()
    st.wbuf[:] = wbuf.tobytes()
    st.accum[:] = accum.view(np.int32)
    st.scale_regs[:] = sregs.view(np.float16)
    if dram is not None:
        st.dram[:len(dram)] = dram.tobytes()
    if case["tile"] is not None:
        st.tile_config = tuple(case["tile"])
    v, q, k, m = case["attn"]
    if v:
        st.attn_context = {"is_valid": True, "query_row_base": q, "valid_kv_len": k, "mode": m}
    sim = G.OracleSimulator(st)
    err = ""
    try:
        if case["kind"] == "program":
            sim.load_program(ProgramStub(case["words"]))
            sim.run()
        else:
            sim._execute(OI.decode_word(int(case["words"][0])))
    except Exception as e:
        err = type(e).__name__
    post = dict(abuf=np.frombuffer(bytes(st.abuf), np.uint8), wbuf=np.frombuffer(bytes(st.wbuf), np.uint8),
                accum=st.accum.view(np.uint8).copy(), sregs=st.scale_regs.view(np.uint8).copy())
    if dram is not None:
        post["dram"] = np.frombuffer(bytes(st.dram[:len(dram)]), np.uint8)
    return err, post, st.cycle_count, st.pc


def expected_post(case, rec):
    abuf, wbuf, accum, sregs, dram = oc.pre_state(case)
    pre = dict(abuf=abuf, wbuf=wbuf, accum=accum, sregs=sregs.view(np.uint8))
    if dram is not None:
        pre["dram"] = dram
    return {nm: apply_spans(pre[nm], rec[nm][1]) for nm in pre}


def fp16_ulp_diff(a_bytes: np.ndarray, b_bytes: np.ndarray) -> np.ndarray:
    """|ulp distance| between two FP16 arrays given as bytes (same sign class)."""
    a = a_bytes.view(np.uint16).astype(np.int32)
    b = b_bytes.view(np.uint16).astype(np.int32)
    ai = np.where(a & 0x8000, -(a & 0x7FFF), a)
    bi = np.where(b & 0x8000, -(b & 0x7FFF), b)
    return np.abs(ai - bi)


def load_bundle(name):
    from llm_accelerator_b200.bundle import ProgramBundle
    return ProgramBundle.load(GOLDEN / f"bundle_{name}.npz")


def load_run(name):
    z = np.load(GOLDEN / f"run_{name}.npz")
    return {k: z[k] for k in z.files}


def run_bundle_sequence(sim_factory, bundle, prompt, n_steps, vocab, runner_cls):
    """prefill(prompt[0]) then decode with teacher forcing over the prompt and
    greedy tokens afterwards; returns (tokens, logits per step, sim)."""
    sim = sim_factory()
    r = runner_cls(bundle, simulator=sim, logits_dtype=np.float16)
    logits = [r.run_prefill([int(prompt[0])])]
    toks = [int(t) for t in prompt]
    for pos in range(1, n_steps):
        tok = int(prompt[pos]) if pos < len(prompt) else int(np.argmax(logits[-1][:vocab]))
        if pos >= len(prompt):
            toks.append(tok)
        logits.append(r.run_decode_step(tok, pos))
    return toks, np.stack(logits), sim


def import_reference() -> bool:
    """Puts the reference's ``taccel`` package on sys.path when it is present:
    an install under ``baseline/_ref`` beside the repository, else the
    checkout named by TACCEL_REFERENCE (default: the conftest's path).
    Returns whether ``taccel`` imports."""
    import importlib
    import sys
    from conftest import REFERENCE, ROOT
    for p in (ROOT / "baseline" / "_ref", REFERENCE / "software"):
        if (p / "taccel").is_dir() and str(p) not in sys.path:
            sys.path.insert(0, str(p))
            break
    sys.dont_write_bytecode = True
    try:
        importlib.import_module("taccel.runtime.host_runner")
        return True
    except ImportError:
        return False


def to_reference_bundle(b):
    """The reference's own ProgramBundle object with b's fields
    (taccel/assembler/assembler.py:163), built through its constructor."""
    from taccel.assembler.assembler import ProgramBundle as RefBundle
    from taccel.assembler.assembler import RelocationSite as RS, RuntimeConfigAttnSite as RC, RuntimePatchSite as RP
    return RefBundle(prefill_instrs=b.prefill_instrs, decode_instrs=b.decode_instrs,
                     shared_data=bytes(b.shared_data), temp_size=b.temp_size, logits_size=b.logits_size,
                     kv_cache_size=b.kv_cache_size, input_offset=b.input_offset,
                     prefill_logits_offset=b.prefill_logits_offset, decode_logits_offset=b.decode_logits_offset,
                     symbol_offsets=dict(b.symbol_offsets), symbol_regions=dict(b.symbol_regions),
                     relocation_sites=[RS(**vars(x)) for x in b.relocation_sites],
                     runtime_patch_sites=[RP(**vars(x)) for x in b.runtime_patch_sites],
                     runtime_config_attn_sites=[RC(**vars(x)) for x in b.runtime_config_attn_sites],
                     embedding_row_bytes=b.embedding_row_bytes, kv_step_bytes=b.kv_step_bytes)
