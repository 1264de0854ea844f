"""Generates the golden fixtures under tests/golden/ by running the reference.

Needs the reference checkout (SayatAbdikul/LLM_accelerator) at
/root/reference (or $TACCEL_REFERENCE) and runs on CPU:

    python tests/golden/make_fixtures.py

Writes
  * ``op_cases.npz``      single-instruction cases: random machine-state inputs,
                          one instruction word, and the reference simulator's
                          resulting bytes / registers (or its exception);
  * ``bundle_<name>.npz`` tiny random-init GPT-2 decoder bundles compiled by the
                          reference toolchain (ProgramBundle.save format);
  * ``run_<name>.npz``    the reference HostRunner on that bundle: prompt, token
                          stream, logits of every step and final-state digests.
"""
from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

REF = Path(os.environ.get("TACCEL_REFERENCE", "/root/reference"))
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(REF / "software"))
sys.path.insert(0, str(REF / "software" / "tools"))
sys.path.insert(0, str(HERE.parent.parent))
sys.path.insert(0, str(HERE))
sys.dont_write_bytecode = True

from taccel.golden_model import memory as rmem  # noqa: E402
from taccel.golden_model.simulator import Simulator  # noqa: E402
from taccel.golden_model.state import MachineState  # noqa: E402
from taccel.isa.encoding import decode as rdecode  # noqa: E402

from llm_accelerator_b200.bundle import ProgramBundle  # noqa: E402
import op_cases as oc  # noqa: E402

# ---------------------------------------------------------------------------
# single-instruction cases (definitions in op_cases.py)
# ---------------------------------------------------------------------------
def run_reference_case(case):
    """Runs one case on the reference simulator; returns its golden record."""
    from taccel.assembler.assembler import ProgramBinary
    abuf, wbuf, accum, sregs, dram = oc.pre_state(case)
    st = MachineState()
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
    sim = Simulator(st)
    err = ""
    try:
        if case["kind"] == "program":
            ins = b"".join(int(w).to_bytes(8, "big") for w in case["words"])
            sim.load_program(ProgramBinary(instructions=ins, data=b"", entry_point=0, insn_count=len(case["words"])))
            sim.run()
        else:
            sim._execute(rdecode(int(case["words"][0]).to_bytes(8, "big")))
    except Exception as e:  # the fault is part of the golden record
        err = type(e).__name__
    post = dict(abuf=np.frombuffer(bytes(st.abuf), np.uint8), wbuf=np.frombuffer(bytes(st.wbuf), np.uint8),
                accum=st.accum.view(np.uint8).copy(), sregs=st.scale_regs.view(np.uint8).copy())
    pre = dict(abuf=abuf, wbuf=wbuf, accum=accum, sregs=sregs.view(np.uint8))
    if dram is not None:
        post["dram"] = np.frombuffer(bytes(st.dram[:len(dram)]), np.uint8)
        pre["dram"] = dram
    rec = dict(err=err, cycles=int(st.cycle_count), pc=int(st.pc))
    for nm in post:
        rec[nm] = (oc.sha(post[nm]), oc.diff_ranges(pre[nm], post[nm]))
    return rec


def save_op_cases(records, path):
    out = {"n_cases": np.asarray([len(records)])}
    for i, r in enumerate(records):
        p = f"c{i:03d}_"
        out[p + "err"] = np.frombuffer((r["err"] or "-").encode(), np.uint8)
        out[p + "cycles"] = np.asarray([r["cycles"], r["pc"]], np.int64)
        for nm in ("abuf", "wbuf", "accum", "sregs", "dram"):
            if nm not in r:
                continue
            digest_hex, spans = r[nm]
            out[p + nm + "_sha"] = np.frombuffer(bytes.fromhex(digest_hex), np.uint8)
            out[p + nm + "_off"] = np.asarray([a for a, _ in spans], np.int64)
            out[p + nm + "_len"] = np.asarray([len(d) for _, d in spans], np.int64)
            out[p + nm + "_data"] = np.frombuffer(b"".join(d for _, d in spans) or b"\0", np.uint8)
    np.savez_compressed(path, **out)


# ---------------------------------------------------------------------------
# tiny GPT-2 bundles + reference runs
# ---------------------------------------------------------------------------
TINY = {
    # name: (n_layer, n_embd, n_head, vocab, n_positions, decode steps)
    "tiny_l2_d128": (2, 128, 4, 512, 64, 15),
    "tiny_l1_d64": (1, 64, 1, 128, 32, 5),
}


def build_bundle(n_layer, d, h, vocab, npos, steps, seed=0):
    import torch
    from transformers import GPT2Config, GPT2LMHeadModel
    from convert_hf_gpt2_to_nanogpt import convert_hf_state_dict_to_nanogpt
    from taccel.runtime.tiny_fixture import build_stage3_tiny_decoder_bundle
    torch.manual_seed(seed)
    cfg = GPT2Config(n_layer=n_layer, n_embd=d, n_head=h, n_positions=npos, vocab_size=vocab)
    payload = convert_hf_state_dict_to_nanogpt(GPT2LMHeadModel(cfg).state_dict(), cfg)
    return build_stage3_tiny_decoder_bundle(payload, smoke_decode_steps=steps, ptq_preset="weight_only_int8").build.bundle


def digest(b: bytes) -> np.ndarray:
    return np.frombuffer(hashlib.sha256(bytes(b)).digest(), np.uint8).copy()


def reference_run(bundle, vocab, prompt_len, new_tokens, seed):
    """prefill(prompt[0]) + teacher-forced prompt + greedy tokens, like the
    GPT-2 perplexity harness (runtime/gpt2_perplexity.py:129-147)."""
    from taccel.runtime.host_runner import HostRunner
    sim = Simulator()
    r = HostRunner(bundle, simulator=sim, logits_dtype=np.float16)
    prompt = np.random.default_rng(seed).integers(0, vocab, prompt_len).tolist()
    logits = [r.run_prefill([prompt[0]])]
    toks = list(prompt)
    digests = []
    for pos in range(1, prompt_len + new_tokens):
        tok = prompt[pos] if pos < prompt_len else int(np.argmax(logits[-1][:vocab]))
        if pos >= prompt_len:
            toks.append(tok)
        logits.append(r.run_decode_step(tok, pos))
        st = sim.state
        digests.append(np.concatenate([digest(st.abuf), digest(st.wbuf), digest(st.accum.tobytes()),
                                       digest(st.dram[bundle.temp_base:bundle.required_dram_bytes]),
                                       digest(st.scale_regs.tobytes())]))
    return prompt, toks, np.stack(logits), np.stack(digests), sim.state.cycle_count


def main():
    cases = oc.case_list()
    save_op_cases([run_reference_case(c) for c in cases], HERE / "op_cases.npz")
    print("op cases:", len(cases))
    for name, cfg in TINY.items():
        b = build_bundle(*cfg)
        ProgramBundle.from_any(b).save(HERE / f"bundle_{name}.npz")
        vocab = cfg[3]
        prompt_len, new = 4, cfg[5] + 1 - 4
        prompt, toks, logits, dig, cyc = reference_run(b, vocab, prompt_len, new, seed=7)
        np.savez_compressed(HERE / f"run_{name}.npz", prompt=np.asarray(prompt), tokens=np.asarray(toks),
                            logits=logits, digests=dig, cycles=np.asarray([cyc]), vocab=np.asarray([vocab]))
        print(name, "tokens", toks)


if __name__ == "__main__":
    main()
