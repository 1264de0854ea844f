"""Oracle-side decoder for the 64-bit taccel instruction word.

TEST INFRASTRUCTURE ONLY.  This module is part of the CPU oracle: only the
test suite, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it.  It is written
independently of the product decoder (the C++ engine in
``llm_accelerator_b200/csrc``) so that the two can check each other.

Field layout and validation follow the reference ISA:
  * opcode in bits [63:59] (``software/taccel/isa/opcodes.py:86-123``);
  * per-format bit positions (``software/taccel/isa/opcodes.py:194-247``);
  * word decode and CONFIG_ATTN reserved-bit rule
    (``software/taccel/isa/encoding.py:395-479``);
  * field validation that turns a malformed word into an illegal-opcode
    fault (``software/taccel/isa/instructions.py:8-19,38-49,216-229,253-263``).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

# Opcode numbers (reference: software/taccel/isa/opcodes.py:86-123)
NOP, HALT, SYNC, CONFIG_TILE, SET_SCALE, SET_ADDR_LO, SET_ADDR_HI = range(7)
LOAD, STORE, BUF_COPY, MATMUL, REQUANT, SCALE_MUL, VADD = range(7, 14)
SOFTMAX, LAYERNORM, GELU, REQUANT_PC, SOFTMAX_ATTNV, DEQUANT_ADD = range(14, 20)
CONFIG_ATTN, MASKED_SOFTMAX, MASKED_SOFTMAX_ATTNV = 20, 21, 22
DEQUANT_ACCUM_FP32, QUANT_FP32_INT8, VADD_FP32, LAYERNORM_FP32 = 23, 24, 25, 26
GELU_FP32, SOFTMAX_FP32, MASKED_SOFTMAX_FP32 = 27, 28, 29
DEQUANT_ACCUM_FP32_SCALED, MAX_ABS_REDUCE_FP32 = 30, 31

OPCODE_NAMES = {
    0: "NOP", 1: "HALT", 2: "SYNC", 3: "CONFIG_TILE", 4: "SET_SCALE",
    5: "SET_ADDR_LO", 6: "SET_ADDR_HI", 7: "LOAD", 8: "STORE", 9: "BUF_COPY",
    10: "MATMUL", 11: "REQUANT", 12: "SCALE_MUL", 13: "VADD", 14: "SOFTMAX",
    15: "LAYERNORM", 16: "GELU", 17: "REQUANT_PC", 18: "SOFTMAX_ATTNV",
    19: "DEQUANT_ADD", 20: "CONFIG_ATTN", 21: "MASKED_SOFTMAX",
    22: "MASKED_SOFTMAX_ATTNV", 23: "DEQUANT_ACCUM_FP32", 24: "QUANT_FP32_INT8",
    25: "VADD_FP32", 26: "LAYERNORM_FP32", 27: "GELU_FP32", 28: "SOFTMAX_FP32",
    29: "MASKED_SOFTMAX_FP32", 30: "DEQUANT_ACCUM_FP32_SCALED",
    31: "MAX_ABS_REDUCE_FP32",
}

R_TYPE = frozenset({MATMUL, REQUANT, SCALE_MUL, VADD, SOFTMAX, LAYERNORM, GELU,
                    REQUANT_PC, SOFTMAX_ATTNV, DEQUANT_ADD, MASKED_SOFTMAX,
                    MASKED_SOFTMAX_ATTNV, DEQUANT_ACCUM_FP32, QUANT_FP32_INT8,
                    VADD_FP32, LAYERNORM_FP32, GELU_FP32, SOFTMAX_FP32,
                    MASKED_SOFTMAX_FP32, DEQUANT_ACCUM_FP32_SCALED,
                    MAX_ABS_REDUCE_FP32})

ABUF, WBUF, ACCUM = 0, 1, 2
# Highest legal 16-byte-unit offset per buffer (128 KB / 256 KB / 64 KB).
MAX_OFF = {ABUF: 8191, WBUF: 16383, ACCUM: 4095}
BUF_BYTES = {ABUF: 128 * 1024, WBUF: 256 * 1024, ACCUM: 64 * 1024}


class DecodeError(ValueError):
    """A word that does not decode to a legal instruction."""


@dataclass(frozen=True)
class Insn:
    """One decoded instruction; unused fields stay zero."""
    opcode: int
    # R-type
    src1_buf: int = 0
    src1_off: int = 0
    src2_buf: int = 0
    src2_off: int = 0
    dst_buf: int = 0
    dst_off: int = 0
    sreg: int = 0
    flags: int = 0
    # M-type (LOAD / STORE)
    buf_id: int = 0
    sram_off: int = 0
    xfer_len: int = 0
    addr_reg: int = 0
    dram_off: int = 0
    stride_log2: int = 0
    # B-type (BUF_COPY)
    src_buf: int = 0
    src_off: int = 0
    length: int = 0
    src_rows: int = 0
    transpose: int = 0
    # A-type
    imm28: int = 0
    # C-type
    M: int = 0
    N: int = 0
    K: int = 0
    # CONFIG_ATTN
    query_row_base: int = 0
    valid_kv_len: int = 0
    mode: int = 0
    # SET_SCALE
    src_mode: int = 0
    imm16: int = 0
    # SYNC
    resource_mask: int = 0

    @property
    def name(self) -> str:
        return OPCODE_NAMES[self.opcode]


def _bits(word: int, shift: int, width: int) -> int:
    return (word >> shift) & ((1 << width) - 1)


def _check_buf_off(buf: int, off: int) -> None:
    if buf not in MAX_OFF:
        raise DecodeError(f"buffer id {buf} is reserved")
    if off > MAX_OFF[buf]:
        raise DecodeError(f"offset {off} exceeds {MAX_OFF[buf]} for buffer {buf}")


def decode_word(word: int) -> Insn:
    """Decode one 64-bit instruction word (already in host integer form)."""
    op = _bits(word, 59, 5)
    if op in R_TYPE:
        f = dict(src1_buf=_bits(word, 57, 2), src1_off=_bits(word, 41, 16),
                 src2_buf=_bits(word, 39, 2), src2_off=_bits(word, 23, 16),
                 dst_buf=_bits(word, 21, 2), dst_off=_bits(word, 5, 16),
                 sreg=_bits(word, 1, 4), flags=_bits(word, 0, 1))
        _check_buf_off(f["src1_buf"], f["src1_off"])
        _check_buf_off(f["src2_buf"], f["src2_off"])
        _check_buf_off(f["dst_buf"], f["dst_off"])
        return Insn(op, **f)
    if op in (LOAD, STORE):
        f = dict(buf_id=_bits(word, 57, 2), sram_off=_bits(word, 41, 16),
                 xfer_len=_bits(word, 25, 16), addr_reg=_bits(word, 23, 2),
                 dram_off=_bits(word, 7, 16), stride_log2=_bits(word, 3, 4),
                 flags=_bits(word, 0, 3))
        _check_buf_off(f["buf_id"], f["sram_off"])
        return Insn(op, **f)
    if op == BUF_COPY:
        f = dict(src_buf=_bits(word, 57, 2), src_off=_bits(word, 41, 16),
                 dst_buf=_bits(word, 39, 2), dst_off=_bits(word, 23, 16),
                 length=_bits(word, 7, 16), src_rows=_bits(word, 1, 6),
                 transpose=_bits(word, 0, 1))
        _check_buf_off(f["src_buf"], f["src_off"])
        _check_buf_off(f["dst_buf"], f["dst_off"])
        return Insn(op, **f)
    if op in (SET_ADDR_LO, SET_ADDR_HI):
        return Insn(op, addr_reg=_bits(word, 57, 2), imm28=_bits(word, 29, 28))
    if op == CONFIG_TILE:
        return Insn(op, M=_bits(word, 49, 10), N=_bits(word, 39, 10), K=_bits(word, 29, 10))
    if op == CONFIG_ATTN:
        if word & ((1 << 33) - 1):
            raise DecodeError("CONFIG_ATTN reserved bits [32:0] must be zero")
        return Insn(op, query_row_base=_bits(word, 47, 12),
                    valid_kv_len=_bits(word, 35, 12), mode=_bits(word, 33, 2))
    if op == SET_SCALE:
        return Insn(op, sreg=_bits(word, 55, 4), src_mode=_bits(word, 53, 2),
                    imm16=_bits(word, 37, 16))
    if op == SYNC:
        return Insn(op, resource_mask=_bits(word, 56, 3))
    # NOP / HALT carry no payload
    return Insn(op)


def decode_bytes(raw: bytes) -> Insn:
    """Decode 8 big-endian bytes."""
    if len(raw) != 8:
        raise DecodeError(f"expected 8 bytes, got {len(raw)}")
    return decode_word(struct.unpack(">Q", raw)[0])


def encode(insn: Insn) -> bytes:
    """Encode an instruction back to 8 big-endian bytes (used to build tests)."""
    op = insn.opcode
    w = (op & 0x1F) << 59
    if op in R_TYPE:
        w |= (insn.src1_buf & 3) << 57 | (insn.src1_off & 0xFFFF) << 41
        w |= (insn.src2_buf & 3) << 39 | (insn.src2_off & 0xFFFF) << 23
        w |= (insn.dst_buf & 3) << 21 | (insn.dst_off & 0xFFFF) << 5
        w |= (insn.sreg & 0xF) << 1 | (insn.flags & 1)
    elif op in (LOAD, STORE):
        w |= (insn.buf_id & 3) << 57 | (insn.sram_off & 0xFFFF) << 41
        w |= (insn.xfer_len & 0xFFFF) << 25 | (insn.addr_reg & 3) << 23
        w |= (insn.dram_off & 0xFFFF) << 7 | (insn.stride_log2 & 0xF) << 3 | (insn.flags & 7)
    elif op == BUF_COPY:
        w |= (insn.src_buf & 3) << 57 | (insn.src_off & 0xFFFF) << 41
        w |= (insn.dst_buf & 3) << 39 | (insn.dst_off & 0xFFFF) << 23
        w |= (insn.length & 0xFFFF) << 7 | (insn.src_rows & 0x3F) << 1 | (insn.transpose & 1)
    elif op in (SET_ADDR_LO, SET_ADDR_HI):
        w |= (insn.addr_reg & 3) << 57 | (insn.imm28 & 0xFFFFFFF) << 29
    elif op == CONFIG_TILE:
        w |= (insn.M & 0x3FF) << 49 | (insn.N & 0x3FF) << 39 | (insn.K & 0x3FF) << 29
    elif op == CONFIG_ATTN:
        w |= (insn.query_row_base & 0xFFF) << 47 | (insn.valid_kv_len & 0xFFF) << 35
        w |= (insn.mode & 3) << 33
    elif op == SET_SCALE:
        w |= (insn.sreg & 0xF) << 55 | (insn.src_mode & 3) << 53 | (insn.imm16 & 0xFFFF) << 37
    elif op == SYNC:
        w |= (insn.resource_mask & 7) << 56
    return struct.pack(">Q", w)
