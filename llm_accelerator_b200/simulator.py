"""Drop-in replacement for the golden simulator, executing on a B200.

``B200Simulator`` keeps the interface of ``taccel.golden_model.simulator.Simulator``
(``software/taccel/golden_model/simulator.py:68-322``): ``load_bundle``,
``load_program``, ``run_program``, ``run``, ``step``, ``_execute``,
``enable_trace`` / ``get_trace_payload`` and a ``state`` whose buffers
(``abuf``, ``wbuf``, ``accum``, ``dram``, ``scale_regs``) read and write the
device copy.  ``HostRunner(bundle, simulator=B200Simulator())`` works
unchanged.  Instead of decoding and dispatching instruction by instruction,
each stream is planned once by the C++ compiler and executed by the CUDA
engine; the registers that the stream fixes (address registers, tile shape,
attention context, pc, cycle count) are kept on the host.
"""
from __future__ import annotations

import hashlib
from typing import Optional

import numpy as np

from . import _lib as L
from . import errors as E
from . import isa
from .bundle import ProgramBundle, instruction_region, symbol_extent
from .engine import Engine, Site, compile_program

DRAM_MIN_BYTES = 16 * 1024 * 1024
BUF_BYTES = (128 * 1024, 256 * 1024, 64 * 1024)


def _fresh_attn():
    return {"is_valid": False, "query_row_base": 0, "valid_kv_len": 0, "mode": 0}


class _SramView:
    """bytearray-like view of one SRAM buffer of sequence 0."""

    def __init__(self, sim: "B200Simulator", buf: int):
        self._sim, self._buf = sim, buf

    def __len__(self):
        return BUF_BYTES[self._buf]

    def _span(self, key):
        if isinstance(key, slice):
            a, b, step = key.indices(len(self))
            if step != 1:
                raise ValueError("strided SRAM access is not supported")
            return a, max(a, b)
        k = key + len(self) if key < 0 else key
        if not 0 <= k < len(self):
            raise IndexError("SRAM index out of range")
        return k, k + 1

    def __getitem__(self, key):
        a, b = self._span(key)
        data = self._sim._eng().read_sram(0, self._buf, a, b - a) if b > a else b""
        return data if isinstance(key, slice) else data[0]

    def __setitem__(self, key, value):
        a, b = self._span(key)
        data = bytes([value]) if isinstance(value, int) else bytes(value)
        if len(data) != b - a:
            raise ValueError("SRAM views cannot change size")
        if data:
            self._sim._eng().write_sram(0, self._buf, a, data)

    def __bytes__(self):
        return self[:]

    def __eq__(self, other):
        return bytes(self) == bytes(other)

    def tobytes(self):
        return bytes(self)


class _AccumView:
    """int32 array-like view of ACCUM (sequence 0)."""

    def __init__(self, sim):
        self._sim = sim
        self.dtype = np.dtype(np.int32)

    def __len__(self):
        return BUF_BYTES[2] // 4

    @property
    def shape(self):
        return (len(self),)

    def __array__(self, dtype=None, copy=None):
        a = np.frombuffer(self._sim._eng().read_sram(0, 2, 0, BUF_BYTES[2]), dtype=np.int32).copy()
        return a if dtype is None else a.astype(dtype)

    def __getitem__(self, key):
        return np.asarray(self)[key]

    def __setitem__(self, key, value):
        a = np.asarray(self)
        a[key] = value
        self._sim._eng().write_sram(0, 2, 0, a.tobytes())

    def view(self, dtype):
        if np.dtype(dtype) == np.uint8:
            return _SramView(self._sim, 2)
        return np.asarray(self).view(dtype)

    def copy(self):
        return np.asarray(self)


class _DramView:
    """bytearray-like view of the DRAM of sequence 0."""

    def __init__(self, sim):
        self._sim = sim

    def __len__(self):
        return self._sim._dram_bytes

    def _span(self, key):
        if isinstance(key, slice):
            a, b, step = key.indices(len(self))
            if step != 1:
                raise ValueError("strided DRAM access is not supported")
            return a, max(a, b)
        k = key + len(self) if key < 0 else key
        if not 0 <= k < len(self):
            raise IndexError("DRAM index out of range")
        return k, k + 1

    def __getitem__(self, key):
        a, b = self._span(key)
        data = self._sim._eng().read_dram(0, a, b - a) if b > a else b""
        return data if isinstance(key, slice) else data[0]

    def __setitem__(self, key, value):
        a, b = self._span(key)
        data = bytes([value]) if isinstance(value, int) else bytes(value)
        if len(data) != b - a:
            raise ValueError("DRAM views cannot change size")
        if data:
            self._sim._eng().write_dram(0, a, data)
            self._sim._note_dram_write(a, data)

    def __eq__(self, other):
        return self[:] == bytes(other)


class _ScaleRegs:
    """float16[16] array-like view of the scale registers (sequence 0)."""

    def __init__(self, sim):
        self._sim = sim
        self.dtype = np.dtype(np.float16)

    def __array__(self, dtype=None, copy=None):
        a = self._sim._eng().read_sregs(0).view(np.float16).copy()
        return a if dtype is None else a.astype(dtype)

    def __len__(self):
        return 16

    def __getitem__(self, key):
        return np.asarray(self)[key]

    def __setitem__(self, key, value):
        a = np.asarray(self)
        a[key] = value
        self._sim._eng().write_sregs(0, a.view(np.uint16))

    def tobytes(self):
        return np.asarray(self).tobytes()


class B200State:
    """MachineState-compatible view (golden_model/state.py:19-108)."""

    def __init__(self, sim: "B200Simulator"):
        self._sim = sim
        self.abuf = _SramView(sim, 0)
        self.wbuf = _SramView(sim, 1)
        self.accum = _AccumView(sim)
        self.dram = _DramView(sim)
        self.scale_regs = _ScaleRegs(sim)
        self.addr_regs = np.zeros(4, dtype=np.uint64)
        self.tile_config = None
        self.attn_context = _fresh_attn()
        self.pc = 0
        self.current_pc = 0
        self.halted = False
        self.cycle_count = 0
        self.runtime_twin_specs = {}

    def get_buffer(self, buf_id: int):
        if buf_id == 0:
            return self.abuf
        if buf_id == 1:
            return self.wbuf
        if buf_id == 2:
            raise ValueError("Use get_accum() for ACCUM buffer")
        raise E.IllegalBufferError(buf_id)

    def get_buffer_or_accum(self, buf_id: int):
        if buf_id == 2:
            return self.accum
        return self.get_buffer(buf_id)

    def reset(self):
        sim = self._sim
        for b in range(3):
            sim._eng().write_sram(0, b, 0, bytes(BUF_BYTES[b]))
        sim._eng().write_sregs(0, np.zeros(16, np.uint16))
        self.addr_regs[:] = 0
        self.tile_config = None
        self.attn_context = _fresh_attn()
        self.pc = self.current_pc = 0
        self.halted = False
        self.cycle_count = 0
        self.runtime_twin_specs = {}

    # host register snapshot for the compiler
    def _regs(self) -> L.Regs:
        r = L.Regs()
        for i in range(4):
            r.addr_regs[i] = int(self.addr_regs[i])
        if self.tile_config is not None:
            r.tile_valid = 1
            r.tile[0], r.tile[1], r.tile[2] = (int(v) for v in self.tile_config)
        ctx = self.attn_context or {}
        if ctx.get("is_valid", False):
            r.attn_valid = 1
            r.attn_qrb, r.attn_vkl, r.attn_mode = int(ctx["query_row_base"]), int(ctx["valid_kv_len"]), int(ctx["mode"])
        return r

    def _apply_regs(self, r: L.Regs) -> None:
        for i in range(4):
            self.addr_regs[i] = np.uint64(r.addr_regs[i])
        self.tile_config = (int(r.tile[0]), int(r.tile[1]), int(r.tile[2])) if r.tile_valid else None
        if r.attn_valid:
            self.attn_context = {"is_valid": True, "query_row_base": int(r.attn_qrb),
                                 "valid_kv_len": int(r.attn_vkl), "mode": int(r.attn_mode)}


class B200Simulator:
    """Golden-simulator interface backed by the CUDA engine (one sequence)."""

    def __init__(self, state=None, *, device: int = 0):
        if state is not None and not isinstance(state, B200State):
            raise TypeError("B200Simulator manages its own device state; pass state=None")
        self.device = device
        self._engine: Optional[Engine] = None
        self._dram_bytes = DRAM_MIN_BYTES
        self._shared_bytes = 0
        self._insn: Optional[bytearray] = None   # host copy of the instruction region
        self._insn_from_dram = True
        self.state = B200State(self)
        self.bundle = None
        self.program = None
        self.trace_manifest = {}
        self.runtime_twin_specs = {}
        self.trace_enabled = False
        self.trace_node_names = None
        self._cache = {}
        self.last_plan = None

    # ---- engine management ---------------------------------------------------------
    def _eng(self) -> Engine:
        if self._engine is None:
            self._engine = Engine(1, self._dram_bytes, self._shared_bytes, self.device)
        return self._engine

    def _relayout(self, dram_bytes: int, shared_bytes: int) -> None:
        """Recreates the engine for a new DRAM size / shared region, keeping SRAM,
        scale registers and the DRAM prefix that survives."""
        if (self._engine is not None and dram_bytes == self._dram_bytes and
                shared_bytes == self._shared_bytes):
            return
        keep = None
        if self._engine is not None:
            e = self._engine
            keep = ([e.read_sram(0, b, 0, BUF_BYTES[b]) for b in range(3)], e.read_sregs(0))
            e.close()
        self._engine = None
        self._cache.clear()
        self._dram_bytes, self._shared_bytes = dram_bytes, shared_bytes
        e = self._eng()
        if keep is not None:
            for b in range(3):
                e.write_sram(0, b, 0, keep[0][b])
            e.write_sregs(0, keep[1])

    def _note_dram_write(self, addr: int, data: bytes) -> None:
        if self._insn is not None and self._insn_from_dram and addr < len(self._insn):
            n = min(len(data), len(self._insn) - addr)
            self._insn[addr:addr + n] = data[:n]

    # ---- program loading (simulator.py:85-179) ------------------------------------------
    def load_bundle(self, bundle, *, strict_dram_size: bool = False, max_dram_bytes: int = 1 << 30) -> None:
        """Loads the bundle's image (simulator.py:162-179): the relocated
        streams, the shared data and a zeroed writable tail.  The shared data
        goes to the device straight from the bundle's own buffer (bytes, or a
        view of a mapped bundle file from ProgramBundle.load_mapped); no
        materialised host copy of the image is made."""
        region = instruction_region(bundle, reset_runtime=True)
        need = bundle.required_dram_bytes
        size = self._dram_bytes
        if need > size:
            if strict_dram_size:
                raise E.SimulatorError(f"Program requires {need} DRAM bytes, but strict DRAM size is {size} bytes")
            if need > max_dram_bytes:
                raise E.SimulatorError(f"Program requires {need} DRAM bytes, exceeding cap {max_dram_bytes}")
            size = need
        # instructions + shared data form one read-only image shared by all sequences
        self._relayout(size, (bundle.temp_base // 16) * 16)
        e = self._eng()
        e.write_dram(-1, 0, region)
        e.write_dram(-1, bundle.data_base, bundle.shared_data)
        end = bundle.data_base + len(bundle.shared_data)
        if need > end:
            e.write_dram(-1, end, np.zeros(need - end, np.uint8))
        self._insn = region
        self._insn_from_dram = True
        self.bundle = self.program = bundle
        self.trace_manifest, self.runtime_twin_specs = {}, {}
        self._reset_volatile(bundle.prefill_pc)

    def load_program(self, program) -> None:
        """ProgramBinary: instructions at 0 and data at data_base (or legacy
        data at 0 with instructions outside DRAM)."""
        self.program, self.bundle = program, None
        if program.data_base > 0:
            img = bytes(program.instructions) + bytes(program.data_base - len(program.instructions)) + bytes(program.data)
        else:
            img = bytes(program.data)
        size = self._dram_bytes
        if len(img) > size:
            size = len(img) + 1024 * 1024
        self._relayout(size, 0)
        if img:
            self._eng().write_dram(0, 0, img)
        if program.data_base > 0:
            self._insn = bytearray(img[:len(program.instructions)])
            self._insn_from_dram = True
        else:
            self._insn = bytearray(program.instructions)
            self._insn_from_dram = False
        self.state.pc = program.entry_point
        self.state.halted = False
        self.trace_manifest = getattr(program, "trace_manifest", {}) or {}

    def _reset_volatile(self, entry_pc: int) -> None:
        st = self.state
        st.pc = st.current_pc = int(entry_pc)
        st.halted = False
        st.tile_config = None
        st.attn_context = _fresh_attn()
        st.addr_regs[:] = 0
        self._sregs_zero_pending = True

    # ---- execution ----------------------------------------------------------------------
    def run_program(self, bundle, name: str, max_instructions: int = 10_000_000) -> int:
        if name not in ("prefill", "decode"):
            raise ValueError("ProgramBundle stream name must be 'prefill' or 'decode'")
        if self.bundle is not bundle:
            self.load_bundle(bundle)
        stream = bundle.stream_bytes(name)
        off = bundle.prefill_instrs_offset if name == "prefill" else bundle.decode_instrs_offset
        self._write_stream(off, stream)
        self.program = bundle
        self._reset_volatile(bundle.prefill_pc if name == "prefill" else bundle.decode_pc)
        return self._execute_region(sites=self._bundle_sites(bundle), max_instructions=max_instructions,
                                    sregs_reset=True)

    def _write_stream(self, off: int, stream: bytes) -> None:
        """Copies a stream into DRAM, uploading only the words that changed."""
        cur = np.frombuffer(bytes(self._insn[off:off + len(stream)]), dtype=np.uint64)
        new = np.frombuffer(stream, dtype=np.uint64)
        diff = np.flatnonzero(cur != new)
        if diff.size:
            # contiguous runs
            breaks = np.flatnonzero(np.diff(diff) != 1)
            starts = np.concatenate(([diff[0]], diff[breaks + 1]))
            ends = np.concatenate((diff[breaks], [diff[-1]])) + 1
            for s, e in zip(starts, ends):
                a, b = off + int(s) * 8, off + int(e) * 8
                self._eng().write_dram(-1, a, stream[a - off:b - off])
        self._insn[off:off + len(stream)] = stream

    def _bundle_sites(self, bundle):
        key = id(bundle)
        cached = getattr(self, "_sites_cache", None)
        if cached and cached[0] == key:
            return cached[1]
        sites = []
        for s in bundle.runtime_patch_sites:
            lo, hi = symbol_extent(bundle, s.base_symbol)
            sites.append(Site(0, s.addr_reg, s.absolute_lo_pc, s.absolute_hi_pc, lo, hi))
        for s in bundle.runtime_config_attn_sites:
            sites.append(Site(1, 0, s.absolute_pc))
        self._sites_cache = (key, sites)
        return sites

    def run(self, max_instructions: int = 10_000_000) -> int:
        if self.trace_enabled and self.trace_manifest:
            return self._run_traced(max_instructions)
        return self._execute_region(sites=(), max_instructions=max_instructions, sregs_reset=False)

    def step(self) -> None:
        if self.state.halted:
            return
        pc = self.state.pc
        self._execute_region(sites=(), max_instructions=1, sregs_reset=False)
        self._capture_trace_events(pc)

    def _run_traced(self, max_instructions: int) -> int:
        """run() with trace capture: the stream is straight-line code, so it
        executes in segments that end at each traced pc, and the manifest's
        tiles are read back after that instruction has completed, as the
        reference's step() captures them (simulator.py:299-322)."""
        import bisect
        pcs = sorted(int(p) for p in self.trace_manifest)
        count = 0
        while not self.state.halted and count < max_instructions:
            pc = int(self.state.pc)
            i = bisect.bisect_left(pcs, pc)
            nxt = pcs[i] if i < len(pcs) else None
            n = max_instructions - count if nxt is None else min(nxt - pc + 1, max_instructions - count)
            done = self._execute_region(sites=(), max_instructions=n, sregs_reset=False)
            count += done
            if nxt is not None and done == nxt - pc + 1:
                self._capture_trace_events(nxt)
            if done == 0:
                break
        return count

    def _execute(self, insn) -> None:
        """Executes one instruction object (reference dataclass or compatible)
        against the current state, without moving pc."""
        word = isa.encode(insn)
        pc, halted = self.state.pc, self.state.halted
        saved = (self._insn, self._insn_from_dram, self.program)
        try:
            self._insn, self._insn_from_dram = bytearray(word), False
            self.program = None
            self.state.pc, self.state.halted = 0, False
            self._execute_region(sites=(), max_instructions=1, sregs_reset=False, bump_pc=False)
        finally:
            self._insn, self._insn_from_dram, self.program = saved
            now_halted = self.state.halted
            self.state.pc = pc
            self.state.halted = halted or now_halted

    def _masked_region(self, sites) -> bytes:
        if not sites:
            return bytes(self._insn)
        m = bytearray(self._insn)
        for s in sites:
            for pc in ((s.lo_pc, s.hi_pc) if s.kind == 0 else (s.lo_pc,)):
                # keep the opcode / register bits, clear the payload
                w = isa.word_of(m[pc * 8:pc * 8 + 8]) & (0x7F << 57)
                m[pc * 8:pc * 8 + 8] = isa.bytes_of(w)
        return bytes(m)

    def _var_words(self, sites) -> np.ndarray:
        words = []
        for s in sites:
            for pc in ((s.lo_pc, s.hi_pc) if s.kind == 0 else (s.lo_pc,)):
                words.append(isa.word_of(self._insn[pc * 8:pc * 8 + 8]))
        return np.asarray(words, dtype=np.uint64)

    def _plan(self, region: bytes, sites, max_instructions: int, sregs_reset: bool):
        st = self.state
        regs = st._regs()
        key = (hashlib.blake2b(region, digest_size=16).digest(), st.pc, max_instructions, sregs_reset,
               bytes(regs), tuple((s.kind, s.addr_reg, s.lo_pc, s.hi_pc, s.range_lo, s.range_hi) for s in sites),
               self._dram_bytes, self._shared_bytes)
        prog = self._cache.get(key)
        if prog is None:
            try:
                prog = compile_program(1, self._dram_bytes, self._shared_bytes, region, st.pc, max_instructions,
                                       regs, sregs_reset, sites)
            except E.EngineError:
                raise
            if len(self._cache) > 64:
                self._cache.clear()
            self._cache[key] = prog
        return prog

    def _execute_region(self, *, sites, max_instructions: int, sregs_reset: bool, bump_pc: bool = True) -> int:
        st = self.state
        if st.halted:
            return 0
        if self._insn is None:
            self._insn = bytearray(0)
        if sregs_reset and getattr(self, "_sregs_zero_pending", False):
            self._sregs_zero_pending = False
        try:
            prog = self._plan(self._masked_region(sites), sites, max_instructions, sregs_reset)
        except E.EngineError:
            raise
        except Exception as exc:
            if getattr(exc, "args", None) and sites and "shared" in str(exc):
                raise
            raise
        words = self._var_words(sites) if prog.n_var_words else None
        status = self._eng().run(prog, words)
        if status == L.E_RECOMPILE:
            # runtime words outside the planned ranges: plan this exact stream
            prog = self._plan(bytes(self._insn), (), max_instructions, sregs_reset)
            status = self._eng().run(prog, None)
        self.last_plan = prog
        info = prog.info
        st.cycle_count += int(info.cycles)
        st._apply_regs(info.final_regs)
        st.pc = int(info.final_pc) if bump_pc else st.pc
        st.current_pc = int(info.final_pc) if info.faulted else max(int(info.final_pc) - 1, 0)
        st.halted = bool(info.halted)
        if status != L.OK:
            f = self._eng()._last_fault
            if prog.info.faulted and status == prog.fault.status:
                raise L.fault_to_exception(prog.fault)
            raise L.fault_to_exception(f, status)
        return int(info.executed)

    # ---- tracing (simulator.py:208-236, 324-474) --------------------------------------------
    def enable_trace(self, node_names=None):
        """Capture the trace manifest's tensors after their instructions."""
        self.trace_enabled = True
        self.trace_node_names = set(node_names) if node_names else None
        self.trace_tensors, self.trace_raw_tensors = {}, {}
        self.trace_saturation, self.trace_meta, self.trace_raw_events = {}, {}, []

    def get_trace_payload(self):
        """Traced tensors, raw tiles, events, INT8 saturation statistics and
        per-node metadata, in the reference's payload layout."""
        stats = {}
        for node, c in getattr(self, "trace_saturation", {}).items():
            total = c.get("total", 0)
            stats[node] = {"saturation_rate": (c.get("sat", 0) / total) if total else 0.0,
                           "zero_fraction": (c.get("zero", 0) / total) if total else 0.0}
        return {"tensors": getattr(self, "trace_tensors", {}), "raw_tensors": getattr(self, "trace_raw_tensors", {}),
                "raw_events": getattr(self, "trace_raw_events", []), "stats": stats,
                "meta": getattr(self, "trace_meta", {})}

    def _node_shape(self, node: str):
        rows = cols = 0
        for events in self.trace_manifest.values():
            for ev in events:
                if ev["node_name"] == node:
                    rows = max(rows, int(ev.get("row_start", 0)) + int(ev["logical_rows"]))
                    cols = max(cols, int(ev["logical_cols"]))
        return rows, cols

    def _zero_padding(self, node: str, view: np.ndarray) -> np.ndarray:
        """The reference's padding clean-up of two node kinds before capture:
        the padded LayerNorm-1 input of a block and the padded projection
        tiles of the per-head query / key / value matmuls keep only their
        logical rows and columns (simulator.py:243-297)."""
        base = None
        if node.endswith("__input_padded") and node.startswith("block") and "_ln1__" in node:
            base = node[:-len("__input_padded")]
        else:
            for suffix, cut in (("__act_input_padded", 7), ("__accum_pre_bias_padded", 7), ("__accum_padded", 7),
                                ("__output_padded", 15)):
                if node.endswith(suffix):
                    cand = node[:-cut]
                    if cand.split("__", 1)[0].endswith(("_query", "_key", "_value")):
                        base = cand
                    break
        if base is None:
            return view
        rows, cols = self._node_shape(base)
        out = view.copy()
        if rows < out.shape[0]:
            out[rows:, :] = 0
        if cols < out.shape[1]:
            out[:, cols:] = 0
        return out

    def _read_tile(self, dtype: str, buf_id: int, off_units: int, rows: int, cols: int) -> np.ndarray:
        st = self.state
        at = int(off_units) * 16
        if dtype == "int32":
            if buf_id == 2:
                return np.frombuffer(st.accum.view(np.uint8)[at:at + rows * cols * 4], np.int32).reshape(rows, cols)
            return np.frombuffer(st.get_buffer(buf_id)[at:at + rows * cols * 4], np.int32).reshape(rows, cols)
        if dtype == "fp32":      # FP16 storage widened to FP32
            return np.frombuffer(st.get_buffer(buf_id)[at:at + rows * cols * 2],
                                 np.float16).astype(np.float32).reshape(rows, cols)
        return np.frombuffer(st.get_buffer(buf_id)[at:at + rows * cols], np.int8).reshape(rows, cols)

    def _capture_trace_events(self, pc: int) -> None:
        if not self.trace_enabled:
            return
        for idx, ev in enumerate(self.trace_manifest.get(pc, [])):
            node = ev["node_name"]
            if self.trace_node_names is not None and node not in self.trace_node_names:
                continue
            rows, cols = int(ev["logical_rows"]), int(ev["logical_cols"])
            full_rows, full_cols = int(ev["full_rows"]), int(ev["full_cols"])
            row_start = int(ev.get("row_start", 0))
            scale = np.float32(ev["scale"])
            source = str(ev.get("source", "architectural"))
            meta = self.trace_meta.setdefault(node, {"scale": float(scale), "dtype": ev["dtype"], "source": source,
                                                     "full_rows": full_rows, "full_cols": full_cols,
                                                     "row_start": row_start, "fragments": [],
                                                     "raw_available": source != "virtual"})
            meta.update(scale=float(scale), dtype=ev["dtype"], source=source, full_rows=full_rows,
                        full_cols=full_cols)
            meta["raw_available"] = bool(meta.get("raw_available", False) or source != "virtual")
            meta["fragments"].append({"pc": int(pc), "event_index": idx, "row_start": row_start,
                                      "logical_rows": rows, "logical_cols": cols})
            raw_ev = {"pc": int(pc), "event_index": idx, "node_name": node, "dtype": ev["dtype"],
                      "scale": float(scale), "source": source,
                      "capture_phase": str(ev.get("capture_phase", "retire_cycle")), "row_start": row_start,
                      "logical_rows": rows, "logical_cols": cols, "full_rows": full_rows, "full_cols": full_cols}
            if source == "virtual":
                # the fused legacy SOFTMAX_ATTNV ops keep no side payload on the device
                raw_ev["raw_available"] = False
                self.trace_raw_events.append(raw_ev)
                continue
            dtype = ev["dtype"]
            if dtype == "int32" and node.endswith(("__accum_pre_matmul", "__accum_pre_matmul_next")):
                view = np.zeros((rows, cols), np.int32)
            else:
                tile = self._read_tile(dtype, int(ev["buf_id"]), int(ev["offset_units"]), int(ev["mem_rows"]),
                                       int(ev["mem_cols"]))
                view = tile[:rows, :cols]
                if dtype != "fp32" and not (dtype == "int32" and
                                            node.endswith(("__accum_pre_softmax", "__accum_pre_softmax_next"))):
                    view = self._zero_padding(node, view)
            deq = view.astype(np.float32) if dtype == "fp32" else view.astype(np.float32) * scale
            raw_ev["raw_available"] = True
            raw_ev["raw"] = view.tolist()
            if node not in self.trace_tensors:
                self.trace_tensors[node] = np.zeros((full_rows, full_cols), np.float32)
            self.trace_tensors[node][row_start:row_start + rows, :cols] = deq
            if node not in self.trace_raw_tensors:
                rt = {"int32": np.int32, "fp32": np.float32}.get(dtype, np.int8)
                self.trace_raw_tensors[node] = np.zeros((full_rows, full_cols), rt)
            self.trace_raw_tensors[node][row_start:row_start + rows, :cols] = view
            self.trace_raw_events.append(raw_ev)
            if dtype not in ("int32", "fp32"):
                c = self.trace_saturation.setdefault(node, {"sat": 0, "zero": 0, "total": 0})
                c["sat"] += int(np.count_nonzero((view == 127) | (view == -128)))
                c["zero"] += int(np.count_nonzero(view == 0))
                c["total"] += int(view.size)
