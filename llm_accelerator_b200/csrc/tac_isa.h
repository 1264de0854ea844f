// Instruction-word decoder for the taccel 64-bit ISA (host side).
//
// Bit layout, buffer limits and field validation follow the reference ISA:
//   software/taccel/isa/opcodes.py:86-266   (opcodes, buffer sizes, bit fields)
//   software/taccel/isa/encoding.py:395-479 (decode, CONFIG_ATTN reserved bits)
//   software/taccel/isa/instructions.py:8-345 (field validation -> illegal opcode)
#pragma once
#include <cstdint>

namespace tac {

enum Opcode : uint8_t {
  OP_NOP = 0x00, OP_HALT = 0x01, OP_SYNC = 0x02, OP_CONFIG_TILE = 0x03, OP_SET_SCALE = 0x04,
  OP_SET_ADDR_LO = 0x05, OP_SET_ADDR_HI = 0x06, OP_LOAD = 0x07, OP_STORE = 0x08,
  OP_BUF_COPY = 0x09, OP_MATMUL = 0x0A, OP_REQUANT = 0x0B, OP_SCALE_MUL = 0x0C,
  OP_VADD = 0x0D, OP_SOFTMAX = 0x0E, OP_LAYERNORM = 0x0F, OP_GELU = 0x10,
  OP_REQUANT_PC = 0x11, OP_SOFTMAX_ATTNV = 0x12, OP_DEQUANT_ADD = 0x13,
  OP_CONFIG_ATTN = 0x14, OP_MASKED_SOFTMAX = 0x15, OP_MASKED_SOFTMAX_ATTNV = 0x16,
  OP_DEQUANT_ACCUM_FP32 = 0x17, OP_QUANT_FP32_INT8 = 0x18, OP_VADD_FP32 = 0x19,
  OP_LAYERNORM_FP32 = 0x1A, OP_GELU_FP32 = 0x1B, OP_SOFTMAX_FP32 = 0x1C,
  OP_MASKED_SOFTMAX_FP32 = 0x1D, OP_DEQUANT_ACCUM_FP32_SCALED = 0x1E,
  OP_MAX_ABS_REDUCE_FP32 = 0x1F,
};

enum Buf : uint8_t { BUF_ABUF = 0, BUF_WBUF = 1, BUF_ACCUM = 2 };

constexpr uint32_t kUnit = 16;                         // bytes per addressing unit
constexpr uint32_t kBufUnits[3] = {8192, 16384, 4096}; // 128 KB, 256 KB, 64 KB
constexpr uint32_t kBufUnitBase[3] = {0, 8192, 8192 + 16384};
constexpr uint32_t kSramUnits = 8192 + 16384 + 4096;   // 448 KB per sequence

inline bool is_rtype(uint8_t op) {
  switch (op) {
    case OP_MATMUL: case OP_REQUANT: case OP_SCALE_MUL: case OP_VADD: case OP_SOFTMAX:
    case OP_LAYERNORM: case OP_GELU: case OP_REQUANT_PC: case OP_SOFTMAX_ATTNV:
    case OP_DEQUANT_ADD: case OP_MASKED_SOFTMAX: case OP_MASKED_SOFTMAX_ATTNV:
    case OP_DEQUANT_ACCUM_FP32: case OP_QUANT_FP32_INT8: case OP_VADD_FP32:
    case OP_LAYERNORM_FP32: case OP_GELU_FP32: case OP_SOFTMAX_FP32:
    case OP_MASKED_SOFTMAX_FP32: case OP_DEQUANT_ACCUM_FP32_SCALED: case OP_MAX_ABS_REDUCE_FP32:
      return true;
    default:
      return false;
  }
}

struct Insn {
  uint8_t op = 0;
  // R-type
  uint8_t src1_buf = 0, src2_buf = 0, dst_buf = 0, sreg = 0, flags = 0;
  uint32_t src1_off = 0, src2_off = 0, dst_off = 0;
  // M-type
  uint8_t buf_id = 0, addr_reg = 0;
  uint32_t sram_off = 0, xfer_len = 0, dram_off = 0;
  // B-type
  uint8_t src_buf = 0, dst_buf_b = 0, src_rows = 0, transpose = 0;
  uint32_t src_off = 0, dst_off_b = 0, length = 0;
  // A-type
  uint32_t imm28 = 0;
  // C-type (encoded, 0-based tile counts)
  uint32_t tm = 0, tn = 0, tk = 0;
  // CONFIG_ATTN
  uint32_t qrb = 0, vkl = 0, mode = 0;
  // SET_SCALE
  uint8_t src_mode = 0;
  uint32_t imm16 = 0;
};

inline uint64_t bits(uint64_t w, int shift, int width) {
  return (w >> shift) & ((1ull << width) - 1);
}

inline bool buf_off_ok(uint32_t buf, uint32_t off) {
  return buf < 3 && off < kBufUnits[buf];
}

// Decodes one instruction word (host integer form, i.e. after the big-endian
// byte swap).  Returns false when the word is illegal: a reserved buffer id,
// an SRAM offset beyond the buffer, or non-zero CONFIG_ATTN reserved bits.
inline bool decode(uint64_t w, Insn& x) {
  x = Insn();
  x.op = static_cast<uint8_t>(bits(w, 59, 5));
  if (is_rtype(x.op)) {
    x.src1_buf = bits(w, 57, 2); x.src1_off = bits(w, 41, 16);
    x.src2_buf = bits(w, 39, 2); x.src2_off = bits(w, 23, 16);
    x.dst_buf = bits(w, 21, 2);  x.dst_off = bits(w, 5, 16);
    x.sreg = bits(w, 1, 4);      x.flags = bits(w, 0, 1);
    return buf_off_ok(x.src1_buf, x.src1_off) && buf_off_ok(x.src2_buf, x.src2_off) &&
           buf_off_ok(x.dst_buf, x.dst_off);
  }
  switch (x.op) {
    case OP_LOAD: case OP_STORE:
      x.buf_id = bits(w, 57, 2); x.sram_off = bits(w, 41, 16);
      x.xfer_len = bits(w, 25, 16); x.addr_reg = bits(w, 23, 2);
      x.dram_off = bits(w, 7, 16);
      return buf_off_ok(x.buf_id, x.sram_off);
    case OP_BUF_COPY:
      x.src_buf = bits(w, 57, 2); x.src_off = bits(w, 41, 16);
      x.dst_buf_b = bits(w, 39, 2); x.dst_off_b = bits(w, 23, 16);
      x.length = bits(w, 7, 16); x.src_rows = bits(w, 1, 6); x.transpose = bits(w, 0, 1);
      return buf_off_ok(x.src_buf, x.src_off) && buf_off_ok(x.dst_buf_b, x.dst_off_b);
    case OP_SET_ADDR_LO: case OP_SET_ADDR_HI:
      x.addr_reg = bits(w, 57, 2); x.imm28 = bits(w, 29, 28);
      return true;
    case OP_CONFIG_TILE:
      x.tm = bits(w, 49, 10); x.tn = bits(w, 39, 10); x.tk = bits(w, 29, 10);
      return true;
    case OP_CONFIG_ATTN:
      if (w & ((1ull << 33) - 1)) return false;
      x.qrb = bits(w, 47, 12); x.vkl = bits(w, 35, 12); x.mode = bits(w, 33, 2);
      return true;
    case OP_SET_SCALE:
      x.sreg = bits(w, 55, 4); x.src_mode = bits(w, 53, 2); x.imm16 = bits(w, 37, 16);
      return true;
    default:  // NOP, HALT, SYNC
      return true;
  }
}

inline uint64_t load_be64(const uint8_t* p) {
  uint64_t w = 0;
  for (int i = 0; i < 8; ++i) w = (w << 8) | p[i];
  return w;
}

}  // namespace tac
