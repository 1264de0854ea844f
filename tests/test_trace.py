"""Trace capture at the boundary: enable_trace / get_trace_payload
(reference: software/taccel/golden_model/simulator.py:208-236 and the capture
in step(), :299-474).

A program carries a trace manifest (pc -> events naming a tile of ABUF, WBUF
or ACCUM); after the instruction at that pc completes, the simulator reads
the tile back and records raw values, dequantised values, INT8 saturation
counts and per-node metadata.  B200Simulator executes the straight-line
stream in segments that end at the traced pcs and reads the tiles from the
device.

Checked on the CPU with the plan engine (tests/plan_engine.py) and on the
GPU: the payload of a short program equals the one the reference's own
simulator returns (when the reference package is importable) and, always,
the tiles of the oracle's state at the same pcs.
"""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest

from helpers import ProgramStub, import_reference, vadd_chain_program
from oracle import golden as G

M, N = 16, 64


def _manifest(words):
    """Events on the instructions of the VADD chain program: the int32 tile
    each LOAD into ACCUM brings, the FP16 running sum after each VADD_FP32, an
    INT8 view of ABUF, a LayerNorm-input node whose padding is cleared, and an
    ACCUM node the reference reports as zeros."""
    man = {}
    units = M * N * 2 // 16
    for pc, w in enumerate(words):
        op = int(w) >> 59
        ev = dict(mem_rows=M, mem_cols=N, logical_rows=M, logical_cols=N, full_rows=M, full_cols=N, row_start=0,
                  when="after")
        if op == 0x07 and ((int(w) >> 57) & 3) == 2:           # LOAD into ACCUM
            man.setdefault(pc, []).append(dict(ev, node_name=f"acc_pc{pc}", buf_id=2, offset_units=0,
                                               dtype="int32", scale=0.25))
        elif op == 0x19:                                          # VADD_FP32 into WBUF[0]
            man.setdefault(pc, []).append(dict(ev, node_name="running_sum", buf_id=1, offset_units=0,
                                               dtype="fp32", scale=1.0, row_start=0))
            man[pc].append(dict(ev, node_name="abuf_i8", buf_id=0, offset_units=units, dtype="int8", scale=0.5,
                                mem_rows=4, logical_rows=3, full_rows=3))
            man[pc].append(dict(ev, node_name="block0_ln1__input_padded", buf_id=0, offset_units=0,
                                dtype="int8", scale=0.125))
            man[pc].append(dict(ev, node_name="block0_ln1", buf_id=0, offset_units=0, dtype="int8",
                                scale=0.125, logical_rows=5, logical_cols=40, mem_rows=5))
            man[pc].append(dict(ev, node_name="block0_head0_qkt__accum_pre_matmul", buf_id=2, offset_units=0,
                                dtype="int32", scale=0.5))
    return man


def _program():
    words, img, _ = vadd_chain_program(M, N, parts=4, produced=True)
    return words, img


def _expected_tiles(words, img, man):
    """(pc, event index) -> the raw tile of the oracle's state after that pc."""
    orc = G.OracleSimulator()
    stub = ProgramStub(words)
    orc.load_program(SimpleNamespace(instructions=stub.instructions, data_base=0, data=img.tobytes(), entry_point=0,
                                     insn_count=stub.insn_count))
    out = {}
    while not orc.state.halted:
        pc = orc.state.pc
        orc.step()
        for i, ev in enumerate(man.get(pc, [])):
            at, r, c = ev["offset_units"] * 16, ev["mem_rows"], ev["mem_cols"]
            if ev["dtype"] == "int32":
                t = orc.state.accum.view(np.uint8)[at:at + r * c * 4].view(np.int32).reshape(r, c)
            elif ev["dtype"] == "fp32":
                t = np.frombuffer(bytes(orc.state.wbuf)[at:at + r * c * 2], np.float16).astype(np.float32)
                t = t.reshape(r, c)
            else:
                t = np.frombuffer(bytes(orc.state.abuf)[at:at + r * c], np.int8).reshape(r, c)
            out[(pc, i)] = t[:ev["logical_rows"], :ev["logical_cols"]].copy()
    return out


def _run_b200(words, img, man, names=None):
    from llm_accelerator_b200.simulator import B200Simulator
    sim = B200Simulator()
    prog = ProgramStub(words)
    prog.trace_manifest = man
    sim.load_program(prog)
    sim.state.dram[:len(img)] = img.tobytes()
    sim.enable_trace(names)
    n = sim.run()
    return sim, n


def _check(plan_mode: bool):
    words, img = _program()
    man = _manifest(words)
    sim, n = _run_b200(words, img, man)
    assert n == len(words) and sim.state.halted
    pay = sim.get_trace_payload()
    tiles = _expected_tiles(words, img, man)
    ev_by_key = {(e["pc"], e["event_index"]): e for e in pay["raw_events"]}
    assert set(ev_by_key) == set(tiles)
    for key, want in tiles.items():
        ev = ev_by_key[key]
        node = ev["node_name"]
        got = np.asarray(ev["raw"])
        if node.endswith("__accum_pre_matmul"):
            want = np.zeros_like(want)
        if node == "block0_ln1__input_padded":     # logical shape of block0_ln1: 5 x 40
            want = want.copy()
            want[5:, :] = 0
            want[:, 40:] = 0
        np.testing.assert_array_equal(got, want, err_msg=f"{node} at pc {key[0]}")
    last_sum = max(pc for pc, i in tiles if man[pc][i]["node_name"] == "running_sum")
    np.testing.assert_array_equal(pay["raw_tensors"]["running_sum"], tiles[(last_sum, 0)])
    st = pay["stats"]["abuf_i8"]
    assert 0.0 <= st["saturation_rate"] <= 1.0 and 0.0 <= st["zero_fraction"] <= 1.0
    assert pay["meta"]["running_sum"]["dtype"] == "fp32" and pay["meta"]["abuf_i8"]["raw_available"] is True
    if import_reference():
        from taccel.golden_model.simulator import Simulator
        ref = Simulator()
        stub = ProgramStub(words)
        ref.load_program(SimpleNamespace(instructions=stub.instructions, data_base=0, data=img.tobytes(),
                                         entry_point=0, insn_count=stub.insn_count, trace_manifest=man,
                                         get_instruction_bytes=lambda pc: stub.instructions[pc * 8:pc * 8 + 8]))
        ref.trace_manifest = man
        ref.enable_trace()
        ref.run()
        want = ref.get_trace_payload()
        assert [{k: v for k, v in e.items()} for e in pay["raw_events"]] == want["raw_events"]
        assert pay["meta"] == want["meta"] and pay["stats"] == want["stats"]
        for k in want["raw_tensors"]:
            np.testing.assert_array_equal(pay["raw_tensors"][k], want["raw_tensors"][k])
            np.testing.assert_array_equal(pay["tensors"][k], want["tensors"][k])


def test_trace_payload_cpu_plan(monkeypatch):
    import llm_accelerator_b200.simulator as S
    from plan_engine import PlanEngine
    monkeypatch.setattr(S, "Engine", PlanEngine)
    _check(plan_mode=True)


def test_trace_node_filter_cpu_plan(monkeypatch):
    import llm_accelerator_b200.simulator as S
    from plan_engine import PlanEngine
    monkeypatch.setattr(S, "Engine", PlanEngine)
    words, img = _program()
    sim, _ = _run_b200(words, img, _manifest(words), names=["abuf_i8"])
    pay = sim.get_trace_payload()
    assert set(pay["raw_tensors"]) == {"abuf_i8"} and {e["node_name"] for e in pay["raw_events"]} == {"abuf_i8"}


@pytest.mark.gpu
def test_trace_payload_gpu():
    _check(plan_mode=False)
