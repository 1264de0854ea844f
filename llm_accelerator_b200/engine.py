"""Thin object wrapper over the C ABI: an engine (device machine state for a
batch of sequences) and compiled programs."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from .errors import EngineError

_lib = L.lib

# numpy views of the plan records (layout of tac::DevOp / Segment / Task)
DEVOP_DTYPE = np.dtype([
    ("kind", "<u2"), ("flags", "<u2"), ("M", "<u4"), ("N", "<u4"), ("K", "<u4"),
    ("a", "<u8"), ("b", "<u8"), ("c", "<u8"), ("d", "<u8"), ("s", "<u4", (4,)),
    ("out_slot", "<u4"), ("seg0", "<u4"), ("nseg", "<u4"), ("param", "<i4"), ("attn_mode", "<u4"),
    ("flags2", "<u4"), ("dconst", "<i8"), ("nbytes", "<u8"), ("attn_qrb", "<u4"), ("attn_vkl", "<u4"),
    ("pc", "<u4"), ("level", "<u4"), ("m_decl", "<u4"), ("q_rows", "<u4")])
SEGMENT_DTYPE = np.dtype([("src", "<u8"), ("dst", "<u8"), ("n", "<u8")])
TASK_DTYPE = np.dtype([("op", "<u4"), ("seq0", "<u4"), ("nseq", "<u4"), ("tile", "<u4"), ("aux", "<u4"),
                       ("pf_units", "<u4"), ("pf_phys", "<u8")])


@dataclass
class Site:
    """A runtime-patched word: kind 0 = SET_ADDR pair, 1 = CONFIG_ATTN."""
    kind: int
    addr_reg: int
    lo_pc: int
    hi_pc: int = 0
    range_lo: int = 0
    range_hi: int = 0


class Program:
    def __init__(self, handle, info: L.ExecInfo, fault: L.Fault, n_var_words: int):
        self.handle = handle
        self.info = info
        self.fault = fault
        self.n_var_words = n_var_words

    def __del__(self):
        h, self.handle = getattr(self, "handle", None), None
        if h:
            _lib.tac_program_destroy(h)

    def attn_key_cols(self) -> int:
        """Fewest key columns of a runtime-configured masked softmax (0 if none)."""
        return int(_lib.tac_program_attn_key_cols(self.handle))

    def set_var_formula(self, base, tok_mul, pos_mul, mode) -> None:
        """Per runtime site (site order): an address site holds base + token *
        tok_mul + position * pos_mul; an attention site the position's context
        with `mode` (see tac_program_set_var_formula)."""
        arrs = [np.ascontiguousarray(np.asarray(a, dtype=np.uint64)) for a in (base, tok_mul, pos_mul)]
        md = np.ascontiguousarray(np.asarray(mode, dtype=np.uint32))
        n = len(md)
        L.check(_lib.tac_program_set_var_formula(self.handle, n, *(a.ctypes.data for a in arrs), md.ctypes.data),
                "tac_program_set_var_formula")

    def dump(self):
        """(ops, segments, tasks, level_offsets) as numpy structured arrays."""
        i = self.info
        assert _lib.tac_program_record_size(0) == DEVOP_DTYPE.itemsize
        ops = np.zeros(i.n_ops, DEVOP_DTYPE)
        segs = np.zeros(i.n_segments, SEGMENT_DTYPE)
        tasks = np.zeros(i.n_tasks, TASK_DTYPE)
        lv = np.zeros(i.n_levels + 1, np.uint32)
        L.check(_lib.tac_program_dump(self.handle, ops.ctypes.data, segs.ctypes.data, tasks.ctypes.data,
                                      lv.ctypes.data), "tac_program_dump")
        return ops, segs, tasks, lv


def compile_program(batch: int, dram_bytes: int, shared_bytes: int, region: bytes, entry_pc: int,
                    max_insns: int, regs: L.Regs, sregs_reset: bool, sites=(), *, live=None,
                    sram_live: bool = True, sregs_live: bool = True, pack: bool = True) -> Program:
    """Plans an instruction region; raises only when the stream cannot be
    planned at all (a faulting stream still yields a program).  ``live``:
    DRAM byte ranges that must hold their final values after a run (None =
    all of DRAM); ``sram_live`` / ``sregs_live``: keep SRAM / scale registers;
    ``pack=False`` keeps every intermediate in its own arena extent."""
    n = len(region) // 8
    buf = C.create_string_buffer(bytes(region), len(region))
    arr = (L.VarSite * max(1, len(sites)))()
    for k, s in enumerate(sites):
        arr[k] = L.VarSite(s.kind, s.addr_reg, s.lo_pc, s.hi_pc, s.range_lo, s.range_hi)
    h = C.c_void_p()
    info, fault = L.ExecInfo(), L.Fault()
    opts = None
    if live is not None or not sram_live or not sregs_live or not pack:
        rng = np.asarray(list(live or []), dtype=np.uint64).reshape(-1, 2)
        if live is not None and len(rng) == 0:
            rng = np.zeros((1, 2), np.uint64)   # nothing in DRAM stays live
        rng = np.ascontiguousarray(rng)
        opts = L.CompileOpts(len(rng), int(sram_live), int(sregs_live), 0 if pack else L.COMPILE_NO_PACK,
                             rng.ctypes.data if len(rng) else None)
        opts._keep = rng
    st = _lib.tac_compile_ex(batch, dram_bytes, shared_bytes, buf, n, entry_pc, max_insns, C.byref(regs),
                             1 if sregs_reset else 0, arr, len(sites), None if opts is None else C.byref(opts),
                             C.byref(h), C.byref(info), C.byref(fault))
    if st != L.OK:
        raise L.fault_to_exception(fault, st)
    return Program(h, info, fault, int(info.n_var_words))


def home_reads(prog: Program):
    """(DRAM byte ranges, reads SRAM, reads scale registers) that a run of
    ``prog`` reads before writing them, i.e. state an earlier run left."""
    n = C.c_uint32()
    sr, gr = C.c_int32(), C.c_int32()
    L.check(_lib.tac_program_home_reads(prog.handle, None, 0, C.byref(n), C.byref(sr), C.byref(gr)),
            "tac_program_home_reads")
    arr = np.zeros((max(1, n.value), 2), np.uint64)
    L.check(_lib.tac_program_home_reads(prog.handle, arr.ctypes.data, n.value, C.byref(n), C.byref(sr),
                                        C.byref(gr)), "tac_program_home_reads")
    return [tuple(int(v) for v in r) for r in arr[:n.value]], bool(sr.value), bool(gr.value)


class Engine:
    """Device machine state for `batch` sequences (one GPU)."""

    def __init__(self, batch: int, dram_bytes: int, shared_bytes: int = 0, device: int = 0):
        h = C.c_void_p()
        st = _lib.tac_engine_create(device, batch, dram_bytes, shared_bytes, C.byref(h))
        if st != L.OK:
            raise EngineError(f"tac_engine_create failed with status {st} (no usable sm_100 GPU?)")
        self.handle = h
        self.batch, self.dram_bytes, self.shared_bytes, self.device = batch, dram_bytes, shared_bytes, device

    def close(self):
        h, self.handle = getattr(self, "handle", None), None
        if h:
            _lib.tac_engine_destroy(h)

    __del__ = close

    # ---- memory ----------------------------------------------------------------------
    def write_dram(self, seq: int, addr: int, data) -> None:
        """Copies bytes (any buffer: bytes, bytearray, a NumPy array or a view
        of a mapped file) to DRAM without an intermediate host copy; seq -1
        writes every sequence (the shared region is written once)."""
        if isinstance(data, (bytes, bytearray, memoryview, np.ndarray)):
            a = np.frombuffer(data, np.uint8) if not isinstance(data, np.ndarray) else data.reshape(-1).view(np.uint8)
            if not a.flags.c_contiguous:
                a = np.ascontiguousarray(a)
        else:
            a = np.frombuffer(bytes(data), np.uint8)
        if a.size:
            L.check(_lib.tac_dram_write(self.handle, seq, addr, a.ctypes.data, a.size), "tac_dram_write")

    def read_dram(self, seq: int, addr: int, n: int) -> bytes:
        out = C.create_string_buffer(n)
        L.check(_lib.tac_dram_read(self.handle, seq, addr, out, n), "tac_dram_read")
        return out.raw

    def write_sram(self, seq: int, buf: int, off: int, data) -> None:
        b = bytes(data)
        L.check(_lib.tac_sram_write(self.handle, seq, buf, off, b, len(b)), "tac_sram_write")

    def read_sram(self, seq: int, buf: int, off: int, n: int) -> bytes:
        out = C.create_string_buffer(n)
        L.check(_lib.tac_sram_read(self.handle, seq, buf, off, out, n), "tac_sram_read")
        return out.raw

    def read_sregs(self, seq: int) -> np.ndarray:
        a = np.zeros(16, np.uint16)
        L.check(_lib.tac_sregs_read(self.handle, seq, a.ctypes.data), "tac_sregs_read")
        return a

    def write_sregs(self, seq: int, bits) -> None:
        a = np.ascontiguousarray(np.asarray(bits, dtype=np.uint16).reshape(16))
        L.check(_lib.tac_sregs_write(self.handle, seq, a.ctypes.data), "tac_sregs_write")

    # ---- execution --------------------------------------------------------------------
    def run(self, prog: Program, var_words=None) -> int:
        """Runs a program on every sequence; returns the status (0 or the
        stream's own fault) and raises on engine / device failures."""
        vw = None
        if prog.n_var_words:
            vw = np.ascontiguousarray(np.asarray(var_words, dtype=np.uint64).reshape(self.batch, prog.n_var_words))
        f = L.Fault()
        st = _lib.tac_run(self.handle, prog.handle, None if vw is None else vw.ctypes.data, C.byref(f))
        self._last_fault = f
        return st

    def run_async(self, prog: Program, var_words, stream=None) -> None:
        vw = None
        if prog.n_var_words:
            vw = np.ascontiguousarray(np.asarray(var_words, dtype=np.uint64).reshape(self.batch, prog.n_var_words))
        f = L.Fault()
        st = _lib.tac_run_async(self.handle, prog.handle, None if vw is None else vw.ctypes.data, stream, C.byref(f))
        if st != L.OK and not (prog.info.faulted and st == prog.fault.status):
            raise L.fault_to_exception(f, st)

    def encode_params(self, prog: Program, var_words) -> np.ndarray:
        """Decodes and range-checks runtime words into the [batch, n_params]
        parameter block a run consumes (host only)."""
        n = int(_lib.tac_program_param_count(prog.handle))
        out = np.zeros((self.batch, n), np.uint64)
        vw = None
        if prog.n_var_words:
            vw = np.ascontiguousarray(np.asarray(var_words, dtype=np.uint64).reshape(self.batch, prog.n_var_words))
        f = L.Fault()
        st = _lib.tac_encode_params(prog.handle, self.batch, None if vw is None else vw.ctypes.data,
                                    out.ctypes.data, C.byref(f))
        if st != L.OK:
            raise L.fault_to_exception(f, st)
        return out

    def encode_params_tp(self, prog: Program, tokens, positions) -> np.ndarray:
        """encode_params for the words the program's site formulas give
        (Program.set_var_formula) for these tokens and positions."""
        n = int(_lib.tac_program_param_count(prog.handle))
        out = np.zeros((self.batch, n), np.uint64)
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64).reshape(self.batch))
        pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int64).reshape(self.batch))
        f = L.Fault()
        st = _lib.tac_encode_params_tp(prog.handle, self.batch, tok.ctypes.data, pos.ctypes.data, out.ctypes.data,
                                       C.byref(f))
        if st != L.OK:
            raise L.fault_to_exception(f, st)
        return out

    def run_async_tp(self, prog: Program, tokens, positions, stream=None) -> None:
        """run_async with the runtime words given by the site formulas."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64).reshape(self.batch))
        pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int64).reshape(self.batch))
        f = L.Fault()
        st = _lib.tac_run_async_tp(self.handle, prog.handle, tok.ctypes.data, pos.ctypes.data, stream, C.byref(f))
        if st != L.OK and not (prog.info.faulted and st == prog.fault.status):
            raise L.fault_to_exception(f, st)

    def run_async_params(self, prog: Program, params_dev_ptr: int, stream=None) -> None:
        """Runs with a parameter block already in device memory."""
        f = L.Fault()
        st = _lib.tac_run_async_params(self.handle, prog.handle, params_dev_ptr, stream, C.byref(f))
        if st != L.OK and not (prog.info.faulted and st == prog.fault.status):
            raise L.fault_to_exception(f, st)

    def check_device(self) -> None:
        f = L.Fault()
        st = _lib.tac_check_device_status(self.handle, C.byref(f))
        if st != L.OK:
            raise L.fault_to_exception(f, st)

    def argmax_f16(self, addr: int, count: int, out_dev_ptr: int, stream=None) -> None:
        L.check(_lib.tac_argmax_f16(self.handle, addr, count, out_dev_ptr, stream), "tac_argmax_f16")

    def set_profiling(self, on, tasks: bool = False) -> None:
        """Level timestamps (on); with tasks=True also each task's SM cycles."""
        mode = (2 if tasks else 1) if on else 0
        L.check(_lib.tac_set_profiling(self.handle, mode), "tac_set_profiling")

    def read_task_profile(self) -> np.ndarray:
        """SM cycles of each task of the last run (tasks in level order)."""
        n = C.c_uint64()
        L.check(_lib.tac_read_task_profile(self.handle, None, 0, C.byref(n)), "tac_read_task_profile")
        out = np.zeros(n.value, np.uint32)
        if n.value:
            L.check(_lib.tac_read_task_profile(self.handle, out.ctypes.data, n.value, C.byref(n)),
                    "tac_read_task_profile")
        return out

    def read_profile(self) -> np.ndarray:
        """Device time (ns) at the end of each level of the last run; entry 0 is the start."""
        n = C.c_uint32()
        L.check(_lib.tac_read_profile(self.handle, None, 0, C.byref(n)), "tac_read_profile")
        out = np.zeros(n.value, np.uint64)
        if n.value:
            L.check(_lib.tac_read_profile(self.handle, out.ctypes.data, n.value, C.byref(n)), "tac_read_profile")
        return out

    def grid(self) -> int:
        """CTAs of the persistent executor launch."""
        return int(_lib.tac_engine_grid(self.handle))

    def layout(self):
        sb, ss, sh = C.c_void_p(), C.c_uint64(), C.c_void_p()
        L.check(_lib.tac_engine_layout(self.handle, C.byref(sb), C.byref(ss), C.byref(sh)), "tac_engine_layout")
        return sb.value, ss.value, sh.value
