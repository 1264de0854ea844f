"""Test helper: an Engine stand-in that executes compiled plans on the CPU.

``PlanEngine`` has the methods ``B200Simulator`` calls on its engine
(DRAM / SRAM / scale-register reads and writes, ``run``, ``close``) and runs
each compiled plan with ``plan_exec`` (NumPy, the oracle's arithmetic).  With
it the host side of the simulator — bundle upload, stream patching, site
handling, planning, read-back — runs end to end without a GPU, so the
reference's own callers (its ``HostRunner``) can be driven against it on the
CPU.  Test infrastructure only; the library never uses it.
"""
from __future__ import annotations

import numpy as np

import plan_exec as PE
from llm_accelerator_b200 import _lib as L
from llm_accelerator_b200 import isa

SRAM_BYTES = PE.SRAM_UNITS * 16
BUF_BASE = (0, 131072, 393216)


class PlanEngine:
    def __init__(self, batch: int, dram_bytes: int, shared_bytes: int = 0, device: int = 0):
        assert batch == 1
        self.batch, self.dram_bytes, self.shared_bytes, self.device = batch, dram_bytes, shared_bytes, device
        self.shared = np.zeros(shared_bytes, np.uint8)
        self.block = np.zeros(SRAM_BYTES + dram_bytes - shared_bytes, np.uint8)
        self.sregs = np.zeros(16, np.uint16)
        self.runs = 0
        self.uploads = []          # (seq, addr, nbytes, type of the source buffer)
        self._last_fault = L.Fault()

    def close(self):
        pass

    # ---- memory ----------------------------------------------------------------------
    def _dram(self, addr: int, n: int):
        assert 0 <= addr and addr + n <= self.dram_bytes
        parts = []
        if addr < self.shared_bytes:
            k = min(n, self.shared_bytes - addr)
            parts.append(self.shared[addr:addr + k])
            addr, n = addr + k, n - k
        if n:
            a = SRAM_BYTES + addr - self.shared_bytes
            parts.append(self.block[a:a + n])
        return parts

    def write_dram(self, seq: int, addr: int, data) -> None:
        self.uploads.append((seq, addr, len(data), type(data).__name__))
        src = np.frombuffer(bytes(data), np.uint8)
        at = 0
        for p in self._dram(addr, len(src)):
            p[:] = src[at:at + len(p)]
            at += len(p)

    def read_dram(self, seq: int, addr: int, n: int) -> bytes:
        return b"".join(bytes(p) for p in self._dram(addr, n))

    def write_sram(self, seq: int, buf: int, off: int, data) -> None:
        d = np.frombuffer(bytes(data), np.uint8)
        self.block[BUF_BASE[buf] + off:BUF_BASE[buf] + off + len(d)] = d

    def read_sram(self, seq: int, buf: int, off: int, n: int) -> bytes:
        return bytes(self.block[BUF_BASE[buf] + off:BUF_BASE[buf] + off + n])

    def read_sregs(self, seq: int) -> np.ndarray:
        return self.sregs.copy()

    def write_sregs(self, seq: int, bits) -> None:
        self.sregs[:] = np.asarray(bits, np.uint16).reshape(16)

    # ---- execution --------------------------------------------------------------------
    @staticmethod
    def _params(words):
        """Plan parameters from the runtime words (SET_ADDR_LO/HI pairs -> the
        28+28-bit address, CONFIG_ATTN -> its packed context), in site order."""
        out, i = [], 0
        words = [] if words is None else [int(w) for w in np.asarray(words, np.uint64).ravel()]
        while i < len(words):
            w = words[i]
            if (w >> 59) == isa.SET_ADDR_LO:
                hi = words[i + 1]
                out.append((((hi >> 29) & 0xFFFFFFF) << 28) | ((w >> 29) & 0xFFFFFFF))
                i += 2
            else:
                out.append(((w >> 47) & 0xFFF) | (((w >> 35) & 0xFFF) << 16) | (((w >> 33) & 3) << 32))
                i += 1
        return out

    def run(self, prog, var_words=None) -> int:
        self.runs += 1
        if prog.info.faulted:
            raise NotImplementedError("PlanEngine runs only plans of streams that do not fault")
        ops, segs, _, lv = prog.dump()
        m = PE.PlanMachine(bytes(self.shared) + bytes(self.block[SRAM_BYTES:]), self.shared_bytes,
                           int(prog.info.arena_bytes), int(prog.info.n_slots))
        m.block[:SRAM_BYTES] = self.block[:SRAM_BYTES]
        m.sregs[:16] = self.sregs
        PE.run_plan(m, ops, segs, lv, self._params(var_words))
        self.block[:] = m.block[:len(self.block)]
        self.sregs[:] = m.sregs[:16]
        self._last_fault = L.Fault()
        return L.OK
