"""Instruction-word encoding helpers used by the host runtime.

Field positions follow the reference ISA (``software/taccel/isa/opcodes.py:173-266``,
``software/taccel/isa/encoding.py:336-392``).  Decoding for execution happens
in the C++ compiler; Python only builds and patches words.
"""
from __future__ import annotations

import struct

OPCODES = {
    "NOP": 0x00, "HALT": 0x01, "SYNC": 0x02, "CONFIG_TILE": 0x03, "SET_SCALE": 0x04,
    "SET_ADDR_LO": 0x05, "SET_ADDR_HI": 0x06, "LOAD": 0x07, "STORE": 0x08, "BUF_COPY": 0x09,
    "MATMUL": 0x0A, "REQUANT": 0x0B, "SCALE_MUL": 0x0C, "VADD": 0x0D, "SOFTMAX": 0x0E,
    "LAYERNORM": 0x0F, "GELU": 0x10, "REQUANT_PC": 0x11, "SOFTMAX_ATTNV": 0x12,
    "DEQUANT_ADD": 0x13, "CONFIG_ATTN": 0x14, "MASKED_SOFTMAX": 0x15,
    "MASKED_SOFTMAX_ATTNV": 0x16, "DEQUANT_ACCUM_FP32": 0x17, "QUANT_FP32_INT8": 0x18,
    "VADD_FP32": 0x19, "LAYERNORM_FP32": 0x1A, "GELU_FP32": 0x1B, "SOFTMAX_FP32": 0x1C,
    "MASKED_SOFTMAX_FP32": 0x1D, "DEQUANT_ACCUM_FP32_SCALED": 0x1E, "MAX_ABS_REDUCE_FP32": 0x1F,
}
SET_ADDR_LO, SET_ADDR_HI, CONFIG_ATTN = 0x05, 0x06, 0x14
M28 = 0xFFFFFFF


def word_of(raw: bytes) -> int:
    return struct.unpack(">Q", bytes(raw))[0]


def bytes_of(word: int) -> bytes:
    return struct.pack(">Q", word)


def set_addr_word(hi: bool, addr_reg: int, imm28: int) -> int:
    return ((SET_ADDR_HI if hi else SET_ADDR_LO) << 59) | ((addr_reg & 3) << 57) | ((imm28 & M28) << 29)


def set_addr_pair(addr_reg: int, value: int) -> tuple[int, int]:
    """The SET_ADDR_LO / SET_ADDR_HI words that load a 56-bit address."""
    if not 0 <= value < (1 << 56):
        raise ValueError(f"byte_addr must fit in 56 bits, got {value:#x}")
    return set_addr_word(False, addr_reg, value & M28), set_addr_word(True, addr_reg, (value >> 28) & M28)


def config_attn_word(query_row_base: int, valid_kv_len: int, mode: int) -> int:
    for v, n, lim in ((query_row_base, "query_row_base", 0xFFF), (valid_kv_len, "valid_kv_len", 0xFFF),
                      (mode, "mode", 3)):
        if not 0 <= v <= lim:
            raise ValueError(f"{n} must be 0-{lim}, got {v}")
    return (CONFIG_ATTN << 59) | (query_row_base << 47) | (valid_kv_len << 35) | (mode << 33)


def _opcode_of(insn) -> int:
    op = getattr(insn, "opcode")
    return int(op)


def encode(insn) -> bytes:
    """Encodes an instruction object (reference dataclass or any object with
    the same field names) to its 8 big-endian bytes."""
    op = _opcode_of(insn)
    g = lambda n: int(getattr(insn, n, 0))  # noqa: E731
    w = (op & 0x1F) << 59
    if op in (0x07, 0x08):
        w |= (g("buf_id") & 3) << 57 | (g("sram_off") & 0xFFFF) << 41 | (g("xfer_len") & 0xFFFF) << 25
        w |= (g("addr_reg") & 3) << 23 | (g("dram_off") & 0xFFFF) << 7 | (g("stride_log2") & 0xF) << 3
        w |= g("flags") & 7
    elif op == 0x09:
        w |= (g("src_buf") & 3) << 57 | (g("src_off") & 0xFFFF) << 41 | (g("dst_buf") & 3) << 39
        w |= (g("dst_off") & 0xFFFF) << 23 | (g("length") & 0xFFFF) << 7 | (g("src_rows") & 0x3F) << 1
        w |= g("transpose") & 1
    elif op in (0x05, 0x06):
        w |= (g("addr_reg") & 3) << 57 | (g("imm28") & M28) << 29
    elif op == 0x03:
        w |= (g("M") & 0x3FF) << 49 | (g("N") & 0x3FF) << 39 | (g("K") & 0x3FF) << 29
    elif op == 0x14:
        w |= (g("query_row_base") & 0xFFF) << 47 | (g("valid_kv_len") & 0xFFF) << 35 | (g("mode") & 3) << 33
    elif op == 0x04:
        w |= (g("sreg") & 0xF) << 55 | (g("src_mode") & 3) << 53 | (g("imm16") & 0xFFFF) << 37
    elif op == 0x02:
        w |= (g("resource_mask") & 7) << 56
    elif op in (0x00, 0x01):
        pass
    else:  # R-type
        w |= (g("src1_buf") & 3) << 57 | (g("src1_off") & 0xFFFF) << 41 | (g("src2_buf") & 3) << 39
        w |= (g("src2_off") & 0xFFFF) << 23 | (g("dst_buf") & 3) << 21 | (g("dst_off") & 0xFFFF) << 5
        w |= (g("sreg") & 0xF) << 1 | (g("flags") & 1)
    return bytes_of(w)
