"""CPU restatement of the taccel golden simulator (NumPy).

TEST INFRASTRUCTURE ONLY.  This is the oracle the CUDA engine is checked
against.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
legs of ``bench.py`` may import it; the product path in
``llm_accelerator_b200`` never calls it.

Each handler restates one reference handler, cited by file:line inside
``software/taccel/golden_model`` of SayatAbdikul/LLM_accelerator:

* machine state ........................ ``state.py:19-108``
* SRAM access + bounds faults ........... ``memory.py:29-366``
* fetch / decode / run loop ............. ``simulator.py:162-206,299-322``
* dispatch ............................... ``simulator.py:476-565``
* MATMUL ................................. ``systolic.py:31-71``
* LOAD / STORE / BUF_COPY ................ ``dma.py:27-97``
* REQUANT(_PC), SCALE_MUL, VADD, DEQUANT_ADD ``simulator.py:629-788``
* W8A16 FP ops (0x17-0x1F) ............... ``simulator.py:808-1140``
* legacy INT8 SFU ops .................... ``sfu.py:97-443``

Floating-point expressions use the same NumPy operations, in the same order,
as the reference, so on a host with the same NumPy build the oracle is
bit-identical to the reference (checked against the reference's own
``rtl/verilator/fixtures/gen2`` vectors and by lock-step runs on compiled
GPT-2 bundles; see ``tests/test_oracle_pin.py``).

One deliberate divergence: an SRAM write that runs past the end of ABUF or
WBUF raises ``SRAMAccessError`` here, where the reference's Python
``bytearray`` slice assignment silently grows the buffer
(``memory.py:356-366``).  Fixed-size SRAM cannot grow, so the engine and the
oracle both fault.
"""
from __future__ import annotations

import numpy as np

from . import isa as I

UNIT = 16
DRAM_MIN_BYTES = 16 * 1024 * 1024
_BUF_NAMES = {0: "ABUF", 1: "WBUF", 2: "ACCUM"}


# --------------------------------------------------------------------------
# Fault classes (same names and meaning as the reference's)
# --------------------------------------------------------------------------
class SimulatorError(Exception):
    pass


class IllegalOpcodeError(SimulatorError):
    def __init__(self, pc, raw):
        super().__init__(f"Illegal opcode at PC={pc}: {bytes(raw).hex()}")
        self.pc = pc


class IllegalBufferError(SimulatorError):
    def __init__(self, buf_id):
        super().__init__(f"Illegal buffer ID: {buf_id}")
        self.buf_id = buf_id


class ConfigError(SimulatorError):
    pass


class SRAMAccessError(Exception):
    def __init__(self, buf_id, offset, limit):
        super().__init__(f"SRAM access out of bounds: {_BUF_NAMES.get(buf_id, buf_id)}[{offset}] "
                         f"exceeds limit {limit}")
        self.buf_id, self.offset, self.limit = buf_id, offset, limit


class DRAMAccessError(Exception):
    def __init__(self, addr):
        super().__init__(f"DRAM access out of bounds: address {addr:#x}")
        self.addr = addr


# --------------------------------------------------------------------------
# Machine state
# --------------------------------------------------------------------------
def _fresh_attn():
    return {"is_valid": False, "query_row_base": 0, "valid_kv_len": 0, "mode": 0}


class OracleState:
    """SRAM buffers, DRAM, registers.  Multi-byte data is little-endian."""

    def __init__(self, dram_bytes: int = DRAM_MIN_BYTES):
        self.abuf = bytearray(I.BUF_BYTES[I.ABUF])
        self.wbuf = bytearray(I.BUF_BYTES[I.WBUF])
        self.accum = np.zeros(I.BUF_BYTES[I.ACCUM] // 4, dtype=np.int32)
        self.dram = bytearray(max(DRAM_MIN_BYTES, dram_bytes))
        self.scale_regs = np.zeros(16, dtype=np.float16)
        self.addr_regs = np.zeros(4, dtype=np.uint64)
        self.tile_config = None
        self.attn_context = _fresh_attn()
        self.pc = 0
        self.current_pc = 0
        self.halted = False
        self.cycle_count = 0

    def raw(self, buf: int):
        """Byte view of an SRAM buffer (ACCUM viewed as bytes)."""
        if buf == I.ABUF:
            return self.abuf
        if buf == I.WBUF:
            return self.wbuf
        if buf == I.ACCUM:
            return self.accum.view(np.uint8)
        raise IllegalBufferError(buf)


# --------------------------------------------------------------------------
# SRAM access helpers (memory.py:29-366)
# --------------------------------------------------------------------------
def _start_ok(buf: int, off: int) -> None:
    lim = I.MAX_OFF.get(buf)
    if lim is None or off > lim:
        raise SRAMAccessError(buf, off, 0 if lim is None else lim)


def _span(st: OracleState, buf: int, off: int, nbytes: int):
    _start_ok(buf, off)
    a = off * UNIT
    if a + nbytes > I.BUF_BYTES[buf]:
        raise SRAMAccessError(buf, off, I.MAX_OFF[buf])
    return a, a + nbytes


def rd_bytes(st, buf, off, n) -> bytes:
    a, b = _span(st, buf, off, n)
    return bytes(st.raw(buf)[a:b])


def wr_bytes(st, buf, off, data) -> None:
    a, b = _span(st, buf, off, len(data))
    if buf == I.ACCUM:
        st.raw(buf)[a:b] = np.frombuffer(bytes(data), dtype=np.uint8)
    else:
        st.raw(buf)[a:b] = data


def rd_i8(st, buf, off, rows, cols) -> np.ndarray:
    _start_ok(buf, off)
    if buf == I.ACCUM:
        raise ValueError("Use read_int32_tile for ACCUM buffer")
    a, b = _span(st, buf, off, rows * cols)
    return np.frombuffer(bytes(st.raw(buf)[a:b]), dtype=np.int8).reshape(rows, cols)


def wr_i8(st, buf, off, arr) -> None:
    _start_ok(buf, off)
    if buf == I.ACCUM:
        raise ValueError("Use write_int32_tile for ACCUM buffer")
    data = np.ascontiguousarray(arr, dtype=np.int8).tobytes()
    a, b = _span(st, buf, off, len(data))
    st.raw(buf)[a:b] = data


def rd_i32(st, buf, off, rows, cols) -> np.ndarray:
    a, b = _span(st, buf, off, rows * cols * 4)
    return np.frombuffer(bytes(st.raw(buf)[a:b]), dtype=np.int32).reshape(rows, cols).copy()


def wr_i32(st, buf, off, arr) -> None:
    data = np.ascontiguousarray(arr, dtype=np.int32).tobytes()
    a, b = _span(st, buf, off, len(data))
    wr = st.raw(buf)
    if buf == I.ACCUM:
        wr[a:b] = np.frombuffer(data, dtype=np.uint8)
    else:
        wr[a:b] = data


def rd_f16(st, buf, off, rows, cols) -> np.ndarray:
    """FP16 tile widened to float32 (FP16 storage, FP32 datapath)."""
    if buf == I.ACCUM:
        raise ValueError("ACCUM buffer is INT32-only")
    a, b = _span(st, buf, off, rows * cols * 2)
    return np.frombuffer(bytes(st.raw(buf)[a:b]), dtype=np.float16).astype(np.float32).reshape(rows, cols)


def wr_f16(st, buf, off, arr) -> None:
    if buf == I.ACCUM:
        raise ValueError("ACCUM buffer is INT32-only")
    data = np.asarray(arr).astype(np.float16).tobytes()
    a, b = _span(st, buf, off, len(data))
    st.raw(buf)[a:b] = data


def rd_f16_vec(st, buf, off, n) -> np.ndarray:
    if buf == I.ACCUM:
        raise ValueError("ACCUM buffer is INT32-only")
    a, b = _span(st, buf, off, n * 2)
    return np.frombuffer(bytes(st.raw(buf)[a:b]), dtype=np.float16).astype(np.float32)


def _tile(st):
    if st.tile_config is None:
        raise ConfigError("CONFIG_TILE not set")
    m, n, k = st.tile_config
    return (m + 1) * 16, (n + 1) * 16, (k + 1) * 16


def _sat8(x):
    return np.clip(np.round(x), -128, 127).astype(np.int8)


# --------------------------------------------------------------------------
# Opcode handlers
# --------------------------------------------------------------------------
def op_matmul(sim, x):                                   # systolic.py:31-71
    st = sim.state
    M, N, K = _tile(st)
    a = rd_i8(st, x.src1_buf, x.src1_off, M, K)
    b = rd_i8(st, x.src2_buf, x.src2_off, K, N)
    acc = rd_i32(st, x.dst_buf, x.dst_off, M, N) if x.flags & 1 else np.zeros((M, N), np.int32)
    acc += np.matmul(a.astype(np.int32), b.astype(np.int32))
    wr_i32(st, x.dst_buf, x.dst_off, acc)
    st.cycle_count += (M // 16) * (N // 16) * (K // 16) * 16


def op_load(sim, x):                                     # dma.py:27-44
    st = sim.state
    addr = int(st.addr_regs[x.addr_reg]) + x.dram_off * UNIT
    n = x.xfer_len * UNIT
    if addr + n > len(st.dram):
        raise DRAMAccessError(addr + n)
    wr_bytes(st, x.buf_id, x.sram_off, bytes(st.dram[addr:addr + n]))
    st.cycle_count += x.xfer_len


def op_store(sim, x):                                    # dma.py:47-64
    st = sim.state
    addr = int(st.addr_regs[x.addr_reg]) + x.dram_off * UNIT
    n = x.xfer_len * UNIT
    data = rd_bytes(st, x.buf_id, x.sram_off, n)
    if addr + n > len(st.dram):
        raise DRAMAccessError(addr + n)
    st.dram[addr:addr + n] = data
    st.cycle_count += x.xfer_len


def op_buf_copy(sim, x):                                 # dma.py:67-97
    st = sim.state
    n = x.length * UNIT
    if not x.transpose:
        wr_bytes(st, x.dst_buf, x.dst_off, rd_bytes(st, x.src_buf, x.src_off, n))
    else:
        rows = x.src_rows * 16
        if rows == 0:
            return
        cols = n // rows
        if cols == 0:
            return
        src = np.frombuffer(rd_bytes(st, x.src_buf, x.src_off, n), dtype=np.int8).reshape(rows, cols)
        wr_bytes(st, x.dst_buf, x.dst_off, np.ascontiguousarray(src.T).tobytes())
    st.cycle_count += x.length


def op_set_scale(sim, x):                                # simulator.py:605-617
    st = sim.state
    if x.src_mode == 0:
        st.scale_regs[x.sreg] = np.frombuffer(x.imm16.to_bytes(2, "little"), dtype=np.float16)[0]
    else:
        buf = {1: I.ABUF, 2: I.WBUF, 3: I.ACCUM}[x.src_mode]
        st.scale_regs[x.sreg] = np.frombuffer(rd_bytes(st, buf, x.imm16, 2), dtype=np.float16)[0]


def op_set_addr_lo(sim, x):                              # simulator.py:619-622
    r = sim.state.addr_regs
    r[x.addr_reg] = (int(r[x.addr_reg]) & ~0xFFFFFFF) | x.imm28


def op_set_addr_hi(sim, x):                              # simulator.py:624-627
    r = sim.state.addr_regs
    r[x.addr_reg] = (int(r[x.addr_reg]) & 0xFFFFFFF) | (x.imm28 << 28)


def op_config_attn(sim, x):                              # simulator.py:567-580
    st = sim.state
    if st.tile_config is None:
        raise ConfigError("CONFIG_TILE not set")
    if x.mode == 0:
        raise ConfigError("CONFIG_ATTN mode 0b00 is reserved")
    if x.valid_kv_len == 0:
        raise ConfigError("CONFIG_ATTN valid_kv_len must be > 0")
    st.attn_context = {"is_valid": True, "query_row_base": int(x.query_row_base),
                       "valid_kv_len": int(x.valid_kv_len), "mode": int(x.mode)}


def check_attn_for_key_cols(st, key_cols: int) -> None:  # simulator.py:582-603
    if st.tile_config is None:
        raise ConfigError("CONFIG_TILE not set")
    ctx = st.attn_context or {}
    if not ctx.get("is_valid", False):
        raise ConfigError("CONFIG_ATTN not set")
    mode, vkl = int(ctx.get("mode", 0)), int(ctx.get("valid_kv_len", 0))
    if mode == 0:
        raise ConfigError("CONFIG_ATTN mode 0b00 is reserved")
    if vkl == 0:
        raise ConfigError("CONFIG_ATTN valid_kv_len must be > 0")
    if mode in (1, 3) and key_cols < vkl:
        raise ConfigError(f"CONFIG_ATTN valid_kv_len={vkl} exceeds softmax key columns {key_cols}")
    if mode == 2 and key_cols != vkl:
        raise ConfigError(f"CONFIG_ATTN pure-causal mode requires softmax key columns {key_cols} "
                          f"to equal valid_kv_len={vkl}")


def op_requant(sim, x):                                  # simulator.py:629-659
    st = sim.state
    M, N, _ = _tile(st)
    s = np.float32(st.scale_regs[x.sreg])
    src = rd_i32(st, x.src1_buf, x.src1_off, M, N)
    wr_i8(st, x.dst_buf, x.dst_off, _sat8(src.astype(np.float32) * s))
    st.cycle_count += M * N


def _need_accum_src1(x):
    if x.src1_buf != I.ACCUM:
        raise IllegalBufferError(x.src1_buf)
    if x.src2_buf == I.ACCUM:
        raise IllegalBufferError(x.src2_buf)
    if x.dst_buf == I.ACCUM:
        raise IllegalBufferError(x.dst_buf)


def op_requant_pc(sim, x):                               # simulator.py:661-688
    st = sim.state
    M, N, _ = _tile(st)
    _need_accum_src1(x)
    src = rd_i32(st, x.src1_buf, x.src1_off, M, N)
    sc = np.frombuffer(rd_bytes(st, x.src2_buf, x.src2_off, N * 2), dtype=np.float16)
    sc = sc.astype(np.float32).reshape(1, N)
    wr_i8(st, x.dst_buf, x.dst_off, _sat8(src.astype(np.float32) * sc))
    st.cycle_count += M * N


def op_scale_mul(sim, x):                                # simulator.py:690-722
    st = sim.state
    M, N, _ = _tile(st)
    s = np.float32(st.scale_regs[x.sreg])
    if x.src1_buf == I.ACCUM:
        src = rd_i32(st, x.src1_buf, x.src1_off, M, N)
        v = np.round(src.astype(np.float32) * s)
        with np.errstate(invalid="ignore"):
            out = np.clip(v, np.iinfo(np.int32).min, np.iinfo(np.int32).max).astype(np.int32)
        wr_i32(st, x.dst_buf, x.dst_off, out)
    else:
        src = rd_i8(st, x.src1_buf, x.src1_off, M, N)
        wr_i8(st, x.dst_buf, x.dst_off, _sat8(src.astype(np.float32) * s))
    st.cycle_count += M * N


def op_vadd(sim, x):                                     # simulator.py:724-760
    st = sim.state
    M, N, _ = _tile(st)
    if x.src1_buf == I.ABUF:
        a = rd_i8(st, x.src1_buf, x.src1_off, M, N).astype(np.int16)
        b = rd_i8(st, x.src2_buf, x.src2_off, M, N).astype(np.int16)
        wr_i8(st, x.dst_buf, x.dst_off, np.clip(a + b, -128, 127).astype(np.int8))
    elif x.src1_buf == I.ACCUM:
        a = rd_i32(st, x.src1_buf, x.src1_off, M, N)
        row = rd_i32(st, x.src2_buf, x.src2_off, 1, N)
        wr_i32(st, x.dst_buf, x.dst_off, a + np.tile(row, (M, 1)))
    else:
        raise IllegalBufferError(x.src1_buf)
    st.cycle_count += M * N


def op_dequant_add(sim, x):                              # simulator.py:762-788
    st = sim.state
    M, N, _ = _tile(st)
    _need_accum_src1(x)
    if x.sreg >= 15:
        raise ConfigError("DEQUANT_ADD sreg+1 out of range")
    ra = np.float32(st.scale_regs[x.sreg])
    rs = np.float32(st.scale_regs[x.sreg + 1])
    acc = rd_i32(st, x.src1_buf, x.src1_off, M, N).astype(np.float32)
    skip = rd_i8(st, x.src2_buf, x.src2_off, M, N).astype(np.float32)
    wr_i8(st, x.dst_buf, x.dst_off, _sat8(acc * ra + skip * rs))
    st.cycle_count += M * N


def op_dequant_accum_fp32(sim, x):                       # simulator.py:808-833
    st = sim.state
    M, N, _ = _tile(st)
    _need_accum_src1(x)
    src = rd_i32(st, x.src1_buf, x.src1_off, M, N)
    sc = rd_f16_vec(st, x.src2_buf, x.src2_off, N).reshape(1, N)
    wr_f16(st, x.dst_buf, x.dst_off, (src.astype(np.float32) * sc).astype(np.float32))
    st.cycle_count += M * N


def op_quant_fp32_int8(sim, x):                          # simulator.py:835-867
    st = sim.state
    M, N, _ = _tile(st)
    if x.src1_buf == I.ACCUM:
        raise IllegalBufferError(x.src1_buf)
    if x.dst_buf == I.ACCUM:
        raise IllegalBufferError(x.dst_buf)
    s = np.float32(st.scale_regs[x.sreg])
    v = np.round(rd_f16(st, x.src1_buf, x.src1_off, M, N) * s)
    out = np.where(np.isnan(v), np.float32(0.0), np.clip(v, -128, 127)).astype(np.int8)
    wr_i8(st, x.dst_buf, x.dst_off, out)
    st.cycle_count += M * N


def _fp_operands_not_accum(x, *srcs):
    for s in srcs:
        if s == I.ACCUM:
            raise IllegalBufferError(I.ACCUM)
    if x.dst_buf == I.ACCUM:
        raise IllegalBufferError(x.dst_buf)


def op_vadd_fp32(sim, x):                                # simulator.py:869-891
    st = sim.state
    M, N, _ = _tile(st)
    _fp_operands_not_accum(x, x.src1_buf, x.src2_buf)
    a = rd_f16(st, x.src1_buf, x.src1_off, M, N)
    b = rd_f16(st, x.src2_buf, x.src2_off, M, N)
    wr_f16(st, x.dst_buf, x.dst_off, (a + b).astype(np.float32))
    st.cycle_count += M * N


def op_layernorm_fp32(sim, x):                           # simulator.py:893-934
    st = sim.state
    M, N, _ = _tile(st)
    _fp_operands_not_accum(x, x.src1_buf, x.src2_buf)
    src = rd_f16(st, x.src1_buf, x.src1_off, M, N)
    gb = rd_f16_vec(st, x.src2_buf, x.src2_off, 2 * N)
    gamma, beta = gb[:N].reshape(1, N), gb[N:].reshape(1, N)
    mean = src.mean(axis=-1, keepdims=True).astype(np.float32)
    var = src.var(axis=-1, keepdims=True).astype(np.float32)
    y = (src - mean) / np.sqrt(var + np.float32(1e-5))
    wr_f16(st, x.dst_buf, x.dst_off, (y * gamma + beta).astype(np.float32))
    st.cycle_count += M * N


def _gelu_tanh(xf):
    c = np.float32(np.sqrt(2.0 / np.pi))
    inner = c * (xf + np.float32(0.044715) * xf ** 3)
    return xf * np.float32(0.5) * (np.float32(1.0) + np.tanh(inner))


def op_gelu_fp32(sim, x):                                # simulator.py:936-962
    st = sim.state
    M, N, _ = _tile(st)
    if x.src1_buf == I.ACCUM:
        raise IllegalBufferError(x.src1_buf)
    if x.dst_buf == I.ACCUM:
        raise IllegalBufferError(x.dst_buf)
    xf = rd_f16(st, x.src1_buf, x.src1_off, M, N).astype(np.float32)
    wr_f16(st, x.dst_buf, x.dst_off, _gelu_tanh(xf).astype(np.float32))
    st.cycle_count += M * N


def op_softmax_fp32(sim, x):                             # simulator.py:964-988
    st = sim.state
    M, N, _ = _tile(st)
    if x.src1_buf == I.ACCUM:
        raise IllegalBufferError(x.src1_buf)
    if x.dst_buf == I.ACCUM:
        raise IllegalBufferError(x.dst_buf)
    src = rd_f16(st, x.src1_buf, x.src1_off, M, N)
    e = np.exp((src - src.max(axis=-1, keepdims=True)).astype(np.float32))
    wr_f16(st, x.dst_buf, x.dst_off, (e / e.sum(axis=-1, keepdims=True)).astype(np.float32))
    st.cycle_count += M * N


def op_masked_softmax_fp32(sim, x):                      # simulator.py:990-1037
    st = sim.state
    M, N, _ = _tile(st)
    check_attn_for_key_cols(st, N)
    if x.src1_buf == I.ACCUM:
        raise IllegalBufferError(x.src1_buf)
    if x.dst_buf == I.ACCUM:
        raise IllegalBufferError(x.dst_buf)
    qrb = int(st.attn_context["query_row_base"])
    vkl = int(st.attn_context["valid_kv_len"])
    src = rd_f16(st, x.src1_buf, x.src1_off, M, N)
    out = np.zeros((M, N), dtype=np.float32)
    for i in range(M):
        last = min(i + qrb, vkl - 1)
        if last < 0:
            continue
        row = src[i].astype(np.float32).copy()
        if last + 1 < N:
            row[last + 1:] = -np.inf
        e = np.exp((row - float(row.max())).astype(np.float32))
        if last + 1 < N:
            e[last + 1:] = 0.0
        denom = float(e.sum())
        out[i] = e / denom if denom > 0.0 else 0.0
    wr_f16(st, x.dst_buf, x.dst_off, out.astype(np.float32))
    st.cycle_count += M * N


def op_dequant_accum_fp32_scaled(sim, x):                # simulator.py:1043-1086
    st = sim.state
    M, N, _ = _tile(st)
    _need_accum_src1(x)
    src = rd_i32(st, x.src1_buf, x.src1_off, M, N)
    pb = rd_f16_vec(st, x.src2_buf, x.src2_off, 2 * N)
    w, bias = pb[:N].reshape(1, N), pb[N:].reshape(1, N)
    act = np.float32(st.scale_regs[x.sreg])
    wr_f16(st, x.dst_buf, x.dst_off, (src.astype(np.float32) * w * act + bias).astype(np.float32))
    st.cycle_count += M * N


MAX_ABS_FLOOR = 2.0 ** -9                    # keeps 127/max finite in FP16
MAX_ABS_CEIL = 65504.0 * 127.0 / 2.0         # keeps max/127 finite in FP16


def max_abs_scales(max_abs: float):
    """The two FP16 scale-register values MAX_ABS_REDUCE_FP32 derives.

    The divisions run in float64 and convert float64 -> float16 directly
    (simulator.py:1124-1136)."""
    m = min(max(max_abs, MAX_ABS_FLOOR), MAX_ABS_CEIL)
    return np.float16(127.0 / m), np.float16(m / 127.0)


def op_max_abs_reduce_fp32(sim, x):                      # simulator.py:1088-1140
    st = sim.state
    M, N, _ = _tile(st)
    if x.src1_buf == I.ACCUM:
        raise IllegalBufferError(x.src1_buf)
    if x.sreg >= 15:
        raise ConfigError("MAX_ABS_REDUCE_FP32 sreg+1 out of range (must be 0..14)")
    src = rd_f16(st, x.src1_buf, x.src1_off, M, N)
    inv, fwd = max_abs_scales(float(np.max(np.abs(src.astype(np.float32)))))
    st.scale_regs[x.sreg] = inv
    st.scale_regs[x.sreg + 1] = fwd
    st.cycle_count += M * N


# ---- legacy INT8-I/O SFU ops (sfu.py) -------------------------------------
SFU_CYCLES = 2


def _dual(st, sreg):                                     # sfu.py:67-78
    if sreg >= 15:
        raise ConfigError("SFU sreg+1 out of range")
    return np.float32(st.scale_regs[sreg]), np.float32(st.scale_regs[sreg + 1])


def _quad(st, sreg):                                     # sfu.py:81-86
    if sreg >= 13:
        raise ConfigError("SFU sreg+3 out of range")
    return tuple(np.float32(st.scale_regs[sreg + i]) for i in range(4))


def _requant_out(v, out_scale):                          # sfu.py:97-101
    if out_scale == np.float32(0):
        return np.zeros(v.shape, dtype=np.int8)
    return _sat8(v / out_scale)


def _sfu_input(st, x, M, N, in_scale):
    if x.src1_buf == I.ACCUM:
        return rd_i32(st, I.ACCUM, x.src1_off, M, N).astype(np.float32) * in_scale
    return rd_i8(st, x.src1_buf, x.src1_off, M, N).astype(np.float32) * in_scale


def _attn_ctx(st):                                       # sfu.py:137-146
    ctx = st.attn_context or {}
    if not ctx.get("is_valid", False):
        raise ConfigError("CONFIG_ATTN not set")
    return int(ctx["query_row_base"]), int(ctx["valid_kv_len"]), int(ctx["mode"])


def _visible(M, N, qrb, vkl, mode):                      # sfu.py:104-120
    if vkl <= 0:
        raise ConfigError("CONFIG_ATTN valid_kv_len must be > 0")
    r = np.arange(M, dtype=np.int32).reshape(M, 1)
    c = np.arange(N, dtype=np.int32).reshape(1, N)
    vis = np.ones((M, N), dtype=bool)
    if mode & 0b10:
        vis &= c <= (qrb + r)
    if mode & 0b01:
        vis &= c < vkl
    dead = ~vis.any(axis=1)
    if np.any(dead):
        raise ConfigError(f"CONFIG_ATTN produced a fully masked row at local row {int(np.flatnonzero(dead)[0])}")
    return vis


def _masked_probs(v, qrb, vkl, mode):                    # sfu.py:123-134
    vis = _visible(v.shape[0], v.shape[1], qrb, vkl, mode)
    m = np.where(vis, v, np.float32(-np.inf)).astype(np.float32)
    e = np.exp(m - m.max(axis=-1, keepdims=True)).astype(np.float32)
    e = np.where(vis, e, np.float32(0.0))
    d = e.sum(axis=-1, keepdims=True)
    if np.any(d == np.float32(0)):
        raise ConfigError("CONFIG_ATTN produced zero softmax denominator")
    return (e / d).astype(np.float32)


def op_layernorm(sim, x):                                # sfu.py:149-190
    st = sim.state
    M, N, _ = _tile(st)
    si, so = _dual(st, x.sreg)
    inp = rd_i8(st, x.src1_buf, x.src1_off, M, N)
    gb = rd_bytes(st, x.src2_buf, x.src2_off, N * 4)
    g = np.frombuffer(gb[:N * 2], dtype=np.float16).astype(np.float32)
    b = np.frombuffer(gb[N * 2:], dtype=np.float16).astype(np.float32)
    v = inp.astype(np.float32) * si
    y = (v - v.mean(axis=-1, keepdims=True)) / np.sqrt(v.var(axis=-1, keepdims=True) + np.float32(1e-6))
    y = y * g + b
    out = np.zeros_like(inp) if so == np.float32(0) else _sat8(y / so)
    wr_i8(st, x.dst_buf, x.dst_off, out)
    st.cycle_count += M * N * SFU_CYCLES


def op_softmax(sim, x):                                  # sfu.py:193-235
    st = sim.state
    M, N, _ = _tile(st)
    si, so = _dual(st, x.sreg)
    v = _sfu_input(st, x, M, N, si)
    e = np.exp(v - v.max(axis=-1, keepdims=True)).astype(np.float32)
    y = e / e.sum(axis=-1, keepdims=True)
    out = np.zeros((M, N), dtype=np.int8) if so == np.float32(0) else _sat8(y / so)
    wr_i8(st, x.dst_buf, x.dst_off, out)
    st.cycle_count += M * N * SFU_CYCLES


def op_masked_softmax(sim, x):                           # simulator.py:521-525, sfu.py:238-272
    st = sim.state
    if st.tile_config is None:
        raise ConfigError("CONFIG_TILE not set")
    check_attn_for_key_cols(st, (st.tile_config[1] + 1) * 16)
    M, N, _ = _tile(st)
    si, so = _dual(st, x.sreg)
    qrb, vkl, mode = _attn_ctx(st)
    v = _sfu_input(st, x, M, N, si)
    wr_i8(st, x.dst_buf, x.dst_off, _requant_out(_masked_probs(v, qrb, vkl, mode), so))
    st.cycle_count += M * N * SFU_CYCLES


def op_gelu(sim, x):                                     # sfu.py:275-320
    st = sim.state
    M, N, _ = _tile(st)
    si, so = _dual(st, x.sreg)
    v = _sfu_input(st, x, M, N, si)
    y = _gelu_tanh(v)
    out = np.zeros((M, N), dtype=np.int8) if so == np.float32(0) else _sat8(y / so)
    wr_i8(st, x.dst_buf, x.dst_off, out)
    st.cycle_count += M * N * SFU_CYCLES


def _attnv_common(sim, x, masked):                       # sfu.py:323-443
    st = sim.state
    if st.tile_config is None:
        raise ConfigError("CONFIG_TILE not set")
    if masked:
        check_attn_for_key_cols(st, (st.tile_config[2] + 1) * 16)
    M, N, K = _tile(st)
    _need_accum_src1(x)
    if masked:
        qrb, vkl, mode = _attn_ctx(st)
    s_qkt, s_v, s_out, s_trace = _quad(st, x.sreg)
    qkt = rd_i32(st, I.ACCUM, x.src1_off, M, K).astype(np.float32) * s_qkt
    v = rd_i8(st, x.src2_buf, x.src2_off, K, N).astype(np.float32) * s_v
    if masked:
        p = _masked_probs(qkt, qrb, vkl, mode)
    else:
        e = np.exp(qkt - qkt.max(axis=-1, keepdims=True)).astype(np.float32)
        p = e / e.sum(axis=-1, keepdims=True)
    av = np.matmul(p, v).astype(np.float32)
    wr_i8(st, x.dst_buf, x.dst_off, _requant_out(av, s_out))
    st.cycle_count += M * K * SFU_CYCLES + (M // 16) * (N // 16) * (K // 16) * 16 + M * N


def op_softmax_attnv(sim, x):
    _attnv_common(sim, x, masked=False)


def op_masked_softmax_attnv(sim, x):
    _attnv_common(sim, x, masked=True)


def _op_nop(sim, x):
    sim.state.cycle_count += 1


def _op_halt(sim, x):
    sim.state.halted = True


def _op_config_tile(sim, x):
    sim.state.tile_config = (x.M, x.N, x.K)


HANDLERS = {
    I.NOP: _op_nop, I.HALT: _op_halt, I.SYNC: _op_nop, I.CONFIG_TILE: _op_config_tile,
    I.CONFIG_ATTN: op_config_attn, I.SET_SCALE: op_set_scale,
    I.SET_ADDR_LO: op_set_addr_lo, I.SET_ADDR_HI: op_set_addr_hi,
    I.LOAD: op_load, I.STORE: op_store, I.BUF_COPY: op_buf_copy, I.MATMUL: op_matmul,
    I.REQUANT: op_requant, I.REQUANT_PC: op_requant_pc, I.SCALE_MUL: op_scale_mul,
    I.VADD: op_vadd, I.DEQUANT_ADD: op_dequant_add, I.SOFTMAX: op_softmax,
    I.MASKED_SOFTMAX: op_masked_softmax, I.SOFTMAX_ATTNV: op_softmax_attnv,
    I.MASKED_SOFTMAX_ATTNV: op_masked_softmax_attnv, I.LAYERNORM: op_layernorm,
    I.GELU: op_gelu, I.DEQUANT_ACCUM_FP32: op_dequant_accum_fp32,
    I.QUANT_FP32_INT8: op_quant_fp32_int8, I.VADD_FP32: op_vadd_fp32,
    I.LAYERNORM_FP32: op_layernorm_fp32, I.GELU_FP32: op_gelu_fp32,
    I.SOFTMAX_FP32: op_softmax_fp32, I.MASKED_SOFTMAX_FP32: op_masked_softmax_fp32,
    I.DEQUANT_ACCUM_FP32_SCALED: op_dequant_accum_fp32_scaled,
    I.MAX_ABS_REDUCE_FP32: op_max_abs_reduce_fp32,
}


# --------------------------------------------------------------------------
# Simulator front-end (simulator.py:68-206,299-322)
# --------------------------------------------------------------------------
class OracleSimulator:
    """Sequential fetch-decode-execute over one machine state."""

    def __init__(self, state: OracleState | None = None):
        self.state = state or OracleState()
        self.bundle = None
        self.program = None

    # ---- program loading ---------------------------------------------------
    def _ensure_dram(self, need: int, strict: bool = False, cap: int = 1 << 30) -> None:
        if need <= len(self.state.dram):
            return
        if strict:
            raise SimulatorError(f"Program requires {need} DRAM bytes, but strict DRAM size is "
                                 f"{len(self.state.dram)} bytes")
        if need > cap:
            raise SimulatorError(f"Program requires {need} DRAM bytes, exceeding cap {cap}")
        self.state.dram = bytearray(need)

    def _reset_volatile(self, entry_pc: int) -> None:
        st = self.state
        st.pc = st.current_pc = int(entry_pc)
        st.halted = False
        st.tile_config = None
        st.attn_context = _fresh_attn()
        st.scale_regs[:] = 0
        st.addr_regs[:] = 0

    def load_bundle(self, bundle, *, strict_dram_size: bool = False, max_dram_bytes: int = 1 << 30):
        image = bundle.materialize(reset_runtime=True)
        self._ensure_dram(bundle.required_dram_bytes, strict_dram_size, max_dram_bytes)
        self.state.dram[:bundle.required_dram_bytes] = image
        self.bundle = self.program = bundle
        self._reset_volatile(bundle.prefill_pc)

    def load_program(self, program):
        """Load a ProgramBinary-style object (instructions + data)."""
        self.program, self.bundle = program, None
        self.state.pc = program.entry_point
        self.state.halted = False
        if program.data_base > 0:
            img = bytes(program.instructions) + bytes(program.data_base - len(program.instructions)) \
                + bytes(program.data)
        else:
            img = bytes(program.data)
        if len(img) > len(self.state.dram):
            self.state.dram = bytearray(len(img) + 1024 * 1024)
        self.state.dram[:len(img)] = img

    def run_program(self, bundle, name: str, max_instructions: int = 10_000_000) -> int:
        if name not in ("prefill", "decode"):
            raise ValueError("ProgramBundle stream name must be 'prefill' or 'decode'")
        if self.bundle is not bundle:
            self.load_bundle(bundle)
        stream = bundle.stream_bytes(name)
        off = bundle.prefill_instrs_offset if name == "prefill" else bundle.decode_instrs_offset
        self.state.dram[off:off + len(stream)] = stream
        self.program = bundle
        self._reset_volatile(bundle.prefill_pc if name == "prefill" else bundle.decode_pc)
        return self.run(max_instructions)

    # ---- execution -----------------------------------------------------------
    def run(self, max_instructions: int = 10_000_000) -> int:
        n = 0
        while not self.state.halted and n < max_instructions:
            self.step()
            n += 1
        return n

    def fetch(self, pc: int) -> bytes:
        if self.program.data_base > 0:
            return bytes(self.state.dram[pc * 8:pc * 8 + 8])
        return bytes(self.program.instructions[pc * 8:pc * 8 + 8])

    def step(self) -> None:
        st = self.state
        if st.halted:
            return
        pc = st.current_pc = st.pc
        if pc >= self.program.insn_count:
            raise SimulatorError(f"PC={pc} past end of program ({self.program.insn_count} insns)")
        raw = self.fetch(pc)
        try:
            insn = I.decode_bytes(raw)
        except ValueError:
            raise IllegalOpcodeError(pc, raw)
        self._execute(insn)
        st.pc += 1

    def _execute(self, insn) -> None:
        HANDLERS[insn.opcode](self, insn)
