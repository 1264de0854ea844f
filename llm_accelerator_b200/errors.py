"""Fault classes raised by the B200 engine.

Names, hierarchy and constructor arguments follow the golden simulator
(``software/taccel/golden_model/simulator.py:53-65`` and
``software/taccel/golden_model/memory.py:11-26``), so callers written against
the reference keep working.  When the reference package ``taccel`` is
importable, each class also derives from the reference class of the same
name, so ``except taccel...ConfigError`` catches engine faults too.
"""
from __future__ import annotations


def _reference_bases():
    try:  # optional interoperability only; the engine never needs taccel
        from taccel.golden_model import memory as _m  # type: ignore
        from taccel.golden_model import simulator as _s  # type: ignore
        return {
            "SimulatorError": (_s.SimulatorError,), "IllegalOpcodeError": (_s.IllegalOpcodeError,),
            "IllegalBufferError": (_s.IllegalBufferError,), "ConfigError": (_s.ConfigError,),
            "SRAMAccessError": (_m.SRAMAccessError,), "DRAMAccessError": (_m.DRAMAccessError,),
        }
    except Exception:
        return {}


_REF = _reference_bases()
_BUF_NAMES = {0: "ABUF", 1: "WBUF", 2: "ACCUM"}


class SimulatorError(*_REF.get("SimulatorError", ()), Exception):
    def __init__(self, *args):
        Exception.__init__(self, *args)


class IllegalOpcodeError(SimulatorError, *_REF.get("IllegalOpcodeError", ())):
    def __init__(self, pc, raw_bytes):
        Exception.__init__(self, f"Illegal opcode at PC={pc}: {bytes(raw_bytes).hex()}")
        self.pc = pc


class IllegalBufferError(SimulatorError, *_REF.get("IllegalBufferError", ())):
    def __init__(self, buf_id):
        Exception.__init__(self, f"Illegal buffer ID: {buf_id}")
        self.buf_id = buf_id


class ConfigError(SimulatorError, *_REF.get("ConfigError", ())):
    def __init__(self, *args):
        Exception.__init__(self, *args)


class SRAMAccessError(*_REF.get("SRAMAccessError", ()), Exception):
    def __init__(self, buf_id, offset, limit):
        Exception.__init__(self, f"SRAM access out of bounds: {_BUF_NAMES.get(buf_id, f'BUF{buf_id}')}[{offset}] "
                                 f"exceeds limit {limit}")
        self.buf_id, self.offset, self.limit = buf_id, offset, limit


class DRAMAccessError(*_REF.get("DRAMAccessError", ()), Exception):
    def __init__(self, addr):
        Exception.__init__(self, f"DRAM access out of bounds: address {addr:#x}")
        self.addr = addr


class EngineError(RuntimeError):
    """The CUDA engine itself failed (CUDA error, device check, bad argument)."""
