"""The C ABI library loads and exports every entry point include/*.h declares
(no compute calls; runs without a GPU)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

from llm_accelerator_b200 import _lib as L

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names.update(re.findall(r"^\s*(?:int|uint32_t|uint64_t|void)\s+(tac_\w+)\s*\(", text, flags=re.M))
    return names


def test_every_declared_symbol_is_exported():
    names = declared_symbols()
    assert len(names) >= 20
    lib = ctypes.CDLL(str(L.LIB_PATH))
    for n in sorted(names):
        assert hasattr(lib, n), n


def test_python_binding_covers_the_header():
    assert declared_symbols() == set(L.SIGNATURES)


def test_plan_record_layouts():
    from llm_accelerator_b200.engine import DEVOP_DTYPE, SEGMENT_DTYPE, TASK_DTYPE
    assert L.lib.tac_program_record_size(0) == DEVOP_DTYPE.itemsize
    assert L.lib.tac_program_record_size(1) == SEGMENT_DTYPE.itemsize
    assert L.lib.tac_program_record_size(2) == TASK_DTYPE.itemsize


def test_struct_sizes_match_header():
    assert ctypes.sizeof(L.Regs) == 64
    assert ctypes.sizeof(L.ExecInfo) == 152
    assert ctypes.sizeof(L.Fault) == 368
