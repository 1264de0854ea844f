// Execution plan shared by the host compiler (tac_compile.cpp) and the device
// executor (tac_exec.cu).
//
// A taccel instruction stream is straight-line code (the ISA has no branches),
// so every address, tile shape and register value except a few runtime-patched
// words is known before execution.  The compiler walks the stream once and
// tracks, for every 16-byte unit of SRAM and of writable DRAM, the physical
// location that holds its current value:
//   * LOAD / STORE / flat BUF_COPY only move pointers (no device work),
//   * every compute instruction writes a fresh extent of a per-sequence arena
//     (so SRAM reuse never creates write-after-read hazards),
//   * reads whose units are not physically contiguous get one gather op.
// Device ops are then grouped into dependency levels; ops in one level are
// independent and run concurrently, levels are separated by a grid barrier.
#pragma once
#include <cstdint>

namespace tac {

// Physical addresses are counted in 16-byte units.  Bit 63 set: the shared
// read-only DRAM image (weights, tables), identical for every sequence.
// Otherwise: an offset inside the per-sequence block, laid out as
//   [SRAM home: ABUF | WBUF | ACCUM][writable DRAM home][arena].
constexpr uint64_t kSharedBit = 1ull << 63;

// Scale-register operands.  Bit 31 set: an FP16 constant in the low 16 bits.
// Otherwise an index into the per-sequence register file: 0..15 are the
// architectural registers, 16.. are renamed slots written during the run.
constexpr uint32_t kSregConst = 1u << 31;
constexpr uint32_t kSregSlotBase = 16;

enum DevKind : uint16_t {
  K_GATHER = 1,            // copy a list of unit segments
  K_DYN_LOAD,              // arena <- DRAM at (runtime register + constant)
  K_DYN_STORE,             // writable DRAM at (runtime register + constant) <- arena
  K_SREG_LOAD,             // register slot <- 2 bytes of SRAM (SET_SCALE from buffer)
  K_SREG_FINAL,            // write the architectural registers at the end of a run
  K_MATMUL,                // int8 x int8 -> int32 (optionally + previous int32)
  K_REQUANT,               // int32 * scalar -> int8
  K_REQUANT_PC,            // int32 * per-column FP16 -> int8
  K_SCALE_MUL_I32,         // int32 * scalar -> int32
  K_SCALE_MUL_I8,          // int8 * scalar -> int8
  K_VADD_I8,               // saturating int8 add
  K_VADD_I32,              // int32 + broadcast int32 row
  K_DEQUANT_ADD,           // int32*s0 + int8*s1 -> int8
  K_DEQUANT_ACCUM,         // int32 * per-column FP16 -> FP16
  K_DEQUANT_SCALED,        // int32 * per-column FP16 * scalar + bias -> FP16
  K_QUANT,                 // FP16 * scalar -> int8 (NaN -> 0)
  K_VADD_F16,              // FP16 + FP16 -> FP16
  K_LAYERNORM_F16,         // row LayerNorm, eps 1e-5
  K_GELU_F16,              // tanh GELU
  K_SOFTMAX_F16,           // row softmax
  K_MASKED_SOFTMAX_F16,    // causal / padded row softmax
  K_MAX_ABS,               // max |x| -> two FP16 scale slots
  K_TRANSPOSE,             // int8 [rows, cols] -> [cols, rows]
  K_LN_I8,                 // legacy INT8-I/O LayerNorm (eps 1e-6)
  K_SOFTMAX_I8,            // legacy INT8-I/O softmax (src int8 or int32)
  K_MASKED_SOFTMAX_I8,     // legacy INT8-I/O masked softmax
  K_GELU_I8,               // legacy INT8-I/O GELU
  K_SOFTMAX_ATTNV,         // legacy fused softmax(QK^T) @ V -> int8
  K_MASKED_SOFTMAX_ATTNV,  // legacy fused masked softmax(QK^T) @ V -> int8
  K_DYN_STORE_MULTI,       // the runtime-addressed stores of one level: segment k copies n bytes
                           // from src to DRAM at params[dst >> 32] + (dst & 0xFFFFFFFF)
  K_VADD_CHAIN,            // FP16 running sum of the segments' operands in order: s0 = seg 0, sk =
                           // f16(sk-1 + seg k); sk stored at seg k's dst unless that is 0
  K_NUM_KINDS
};

// Flags on DevOp::flags.
constexpr uint16_t F_ACCUMULATE = 1;   // MATMUL adds the previous int32 tile (operand c)
constexpr uint16_t F_SRC_I32 = 2;      // legacy SFU input is int32 (ACCUM) rather than int8
constexpr uint16_t F_ATTN_DYN = 4;     // masked softmax context comes from a runtime parameter
constexpr uint16_t F_TC = 8;           // MATMUL with shared weights on tcgen05, TMA maps pair seg0
constexpr uint16_t F_SPLIT = 16;       // DEQUANT_SCALED / LAYERNORM: second half of the [scale|bias]
                                       // ([gamma|beta]) vector at operand c instead of b + N
constexpr uint16_t F_SEGA = 32;        // MAX_ABS / QUANT / VADD_F16: operand a is the segment list
constexpr uint16_t F_WIDE = 64;        // MATMUL (per-sequence operands, M <= 32, K <= 128, N <= 256):
                                       // one task per sequence covers every column
constexpr uint16_t F_BT = 128;         // MATMUL: operand b holds B transposed, [N][K] row-major
constexpr uint16_t F_TC128 = 256;      // F_TC MATMUL with N >= 128: 128-column tasks (else 64)
constexpr uint16_t F_QB = 512;         // wide MATMUL: operand b is FP16 and is quantised on load
                                       // (rint(x * s[1]), NaN -> 0, clipped to int8), as QUANT does
constexpr uint16_t F_QA = 1024;        // wide MATMUL: operand a is FP16, quantised on load with s[0]
constexpr uint16_t F_DQ = 2048;        // wide MATMUL: also writes DEQUANT_ACCUM's FP16 result,
                                       // f16(f32(acc) * f32(c[col])), to the unit address in dconst
constexpr uint16_t F_NOI32 = 4096;     // F_DQ MATMUL whose int32 result nothing reads: not stored
constexpr uint16_t F_SM = 8192;        // F_DQ MATMUL: also the FP16 softmax of the dequantised rows
                                       // (attention context in attn_* / param, output unit in nbytes)
constexpr uint16_t F_SMMASK = 16384;   // F_SM: the masked softmax
constexpr uint16_t F_NODQ = 32768;     // F_SM MATMUL whose dequantised rows nothing reads: not stored

// Flags on DevOp::flags2.
constexpr uint32_t FX_DQS = 1;         // tcgen05 MATMUL (no accumulate) also writes DEQUANT_SCALED's FP16
                                       // result f16((f32(acc) * scale[col]) * s[0] + bias[col]) to the unit
                                       // address in dconst; scale row at c, bias row at nbytes
constexpr uint32_t FX_MAXQ = 2;        // MAX_ABS also writes QUANT's int8 result of its input with the
                                       // inverse scale it derives, to the unit address in d
constexpr uint32_t FX_PV = 4;          // wide F_SM MATMUL (QK^T) whose task also runs the wide MATMUL at op
                                       // index seg0 (P.V), that op's A being these softmax rows quantised
                                       // straight into its shared-memory A tile
constexpr uint32_t FX_PVY = 8;         // the P.V op of an FX_PV pair: same level, no tasks of its own
constexpr uint32_t FX_SMSKIP = 16;     // FX_PV op whose softmax rows only its P.V op reads: not stored
constexpr uint32_t FX_PVPF = 32;       // FX_PV op that stages its P.V op's FP16 B (V) in shared memory once
                                       // its own operand tiles are quantised; the P.V op skips that load
constexpr uint32_t FX_CHAINED = 64;    // per-sequence row op that runs in the task of the op before it (same
                                       // level), after every tile of that op for the sequence
constexpr uint32_t FX_CHAINHEAD = 128; // first op of such a chain: its tasks (one per sequence) hold, in tile
                                       // and aux, the first and count of the chain's task templates, stored
                                       // after the last level's tasks (seq0 taken from the head's task)
constexpr uint32_t FX_GELUSEG = 512;   // F_SEGA MAX_ABS some of whose segments (dst | kSegGelu) read a GELU's
                                       // input: the value is f16(gelu(x)) of the unit read, as the GELU op
                                       // would have stored it
constexpr uint64_t kSegGelu = 1ull << 62;   // Segment.dst flag of such a segment (dst & ~kSegGelu is the offset)
constexpr uint32_t FX_DSTORE = 1024;   // FX_DQS tcgen05 MATMUL that also stores the first attn_vkl rows of its
                                       // FP16 result to writable DRAM at params[param] + attn_qrb (a STORE
                                       // through a runtime register, e.g. a KV-cache append, absorbed)
constexpr uint32_t FX_ATTNGRP = 2048;  // FX_PV op heading a group of attention pairs of one sequence (the
                                       // heads of a layer) run as row attention in one task, the next pair's
                                       // copies overlapped: its tasks hold, in tile and aux, the first and
                                       // count of the group's task templates (after the last level's tasks)
constexpr uint32_t FX_MAXGRP = 4096;   // F_SEGA FX_MAXQ MAX_ABS heading a pair of such ops of one level and
                                       // shape run in one task per sequence, each on half the threads: its
                                       // tasks hold, in tile and aux, the first and count (2) of the pair's
                                       // task templates (after the last level's tasks)
constexpr uint32_t FX_TCRES = 256;     // tcgen05 MATMUL (64-column tasks) whose every K chunk fits in shared
                                       // memory at once: A boxes of q_rows rows packed back to back, then B;
                                       // no stage is reused

                                       // [seg0, seg0 + nseg) (Segment.dst = offset in the operand, units)

// Most runs an operand read through a segment list may have (longer lists are gathered).
constexpr uint32_t kMaxSegRuns = 256;
constexpr uint32_t kSegTaskUnits = 512;   // operand units (4096 FP16 elements) of one QUANT / VADD_F16 task
// MAX_ABS pairs (FX_MAXGRP): ops of at most kMaxGrpElems FP16 elements read
// through at most kMaxSegRuns segments, each on half the threads of a task.
constexpr uint32_t kMaxGrpElems = 8192;
                                          // whose first operand is a segment list

struct DevOp {
  uint16_t kind;
  uint16_t flags;
  uint32_t M, N, K;        // element dimensions (rows, cols, reduction)
  uint64_t a, b, c, d;     // physical unit addresses: src1, src2, extra input, destination
  uint32_t s[4];           // scale-register operands
  uint32_t out_slot;       // first renamed register slot written (MAX_ABS, SET_SCALE)
  uint32_t seg0, nseg;     // K_GATHER: segment range; K_SREG_FINAL: unused
  int32_t param;           // runtime parameter index (dynamic address / attention context)
  uint32_t attn_mode;
  uint32_t flags2;         // more flags (FX_*)
  int64_t dconst;          // byte constant added to the runtime address
  uint64_t nbytes;         // bytes moved by dynamic copies
  uint32_t attn_qrb, attn_vkl;
  uint32_t pc;             // instruction that produced the op (for error reports)
  uint32_t level;
  uint32_t m_decl;         // row-wise op narrowed to the rows some later op reads: the instruction's
                           // tile rows (M then holds the rows computed); 0 = not narrowed
  uint32_t q_rows;         // FX_MAXQ MAX_ABS: rows of the QUANT result stored (0 = all M); the
                           // reduction still reads every row.  FX_TCRES MATMUL: rows of a task's A
                           // box (its sequences' rows rounded up to 8)
};
static_assert(sizeof(DevOp) == 128, "DevOp is a 128-byte record");

struct Segment {
  uint64_t src;   // physical unit address
  uint64_t dst;   // physical unit address
  uint64_t n;     // units
};

struct Task {
  uint32_t op;
  uint32_t seq0;   // first sequence
  uint32_t nseq;   // sequences covered
  uint32_t tile;   // op-specific tile index (K_GATHER: first segment, relative to seg0)
  uint32_t aux;    // K_GATHER: one past the last segment (relative to seg0)
  uint32_t pf_units;   // prefetch hint: 16-byte units the task reads first (0 = none)
  uint64_t pf_phys;    // prefetch hint: their physical start (sequence seq0)
};
static_assert(sizeof(Task) == 32, "Task is a 32-byte record");
// Task.aux of a tcgen05 MATMUL task: this bit | the op's tensor-map pair index
// (seg0), so a prefetcher holding only the task record reaches its maps.
constexpr uint32_t kTaskTcMap = 1u << 31;

// Gathers split their segments into pieces of at most this many units, and a
// gather task copies a run of whole segments of about this size.
constexpr uint64_t kGatherChunkUnits = 4096;

// Elements of one sequence an element-wise task covers (256 threads x 4 groups of 8).
constexpr uint64_t kEwTaskElems = 8192;

#ifdef __CUDACC__
#define TAC_HD __host__ __device__
#else
#define TAC_HD
#endif

// MATMULs that run on tcgen05: shared weights (B), per-sequence A of fewer
// than 128 rows (128 / M sequences fill one 128-row tile): a 16-multiple, or
// a divisor of 128 (a MATMUL narrowed to the rows some op reads), N and K
// 16-multiples.
TAC_HD constexpr bool max_pair_ok(uint32_t M, uint32_t N, uint32_t nseg, uint32_t flags, uint32_t flags2) {
  return (flags & F_SEGA) && (flags2 & FX_MAXQ) && M * N <= kMaxGrpElems && (M * N) % 8 == 0 && nseg >= 1 &&
         nseg <= kMaxSegRuns;
}
TAC_HD constexpr bool tc_rows_ok(uint32_t M) { return M > 0 && M < 128 && (M % 16 == 0 || 128 % M == 0); }
// Shared memory of the tcgen05 stages (after the 1024-byte alignment) and
// the resident layout: every K chunk's A box (rows x 128 B) then every B box
// (128 K rows x 64 columns); the MMA of the last chunk reads 128 A rows from
// its box on, which must stay inside the stage region.
constexpr uint32_t kTcStageRegion = 73728;
constexpr uint32_t kTcSplitRows = 32;   // rows of a ring-fed (non-resident) tcgen05 task with more sequences
TAC_HD constexpr bool tc_resident_fits(uint32_t rows, uint32_t K) {
  const uint32_t nchunks = (K + 127) / 128;
  return rows % 8 == 0 && rows <= 128 && nchunks * (rows * 128 + 8192) <= kTcStageRegion &&
         (nchunks - 1) * rows * 128 + 16384 <= kTcStageRegion;
}
TAC_HD constexpr bool tc_eligible(uint64_t a, uint64_t b, uint32_t M, uint32_t N, uint32_t K) {
  return (b & kSharedBit) && !(a & kSharedBit) && tc_rows_ok(M) && N > 0 && N % 16 == 0 && K > 0 && K % 16 == 0;
}

// Element-wise task size by op kind: GELU (float64 tanh per element) takes
// 4096-element tasks (two groups of 8 per thread) so its work spreads over
// more SMs; QUANT (FP16 in, staged in shared memory, 32 KB per task) takes
// twice kEwTaskElems to halve its per-task overhead; the rest take
// kEwTaskElems.
constexpr uint32_t kVaddChainMax = 8;     // operands of one K_VADD_CHAIN op at most
constexpr uint32_t kVaddChainTask = 4096;  // elements of one K_VADD_CHAIN task (all operands staged: 64 KB)

TAC_HD constexpr uint32_t ew_task_elems(uint32_t kind) {
  return (kind == K_GELU_F16 || kind == K_GELU_I8) ? 4096u
         : kind == K_QUANT                         ? 2u * uint32_t(kEwTaskElems)
                                                   : uint32_t(kEwTaskElems);
}

// Shared memory of a wide MATMUL task (op_matmul_wide): A and B^T rows of K
// bytes padded to 32 plus 16, raw B [K][N] unless B arrives transposed, and
// the FP16 B when it is quantised on load.
constexpr uint32_t kWideMmSmem = 73 * 1024;
// The FP16 A (F_QA) shares the B^T area when B is not transposed on arrival
// and it fits there: B^T is written only after A has been quantised.
TAC_HD constexpr bool wide_mm_a_in_bt(uint32_t M, uint32_t N, uint32_t K, bool bt) {
  return !bt && M * K * 2 <= (((N + 7) / 8) * 8) * (((K + 31) & ~31u) + 16);
}
TAC_HD constexpr uint32_t wide_mm_smem(uint32_t M, uint32_t N, uint32_t K, bool bt, bool qb, bool qa = false) {
  return (((M + 15) / 16) * 16) * (((K + 31) & ~31u) + 16) + (((N + 7) / 8) * 8) * (((K + 31) & ~31u) + 16) +
         (bt ? 0u : ((K + 31) & ~31u) * N) + (qb ? K * N * 2 : 0u) +
         ((qa && !wide_mm_a_in_bt(M, N, K, bt)) ? M * K * 2 : 0u) + 512u;   // + the F_DQ scale row
}
TAC_HD constexpr bool wide_mm_ok(uint32_t M, uint32_t N, uint32_t K, bool bt, bool qb, bool qa = false) {
  return M > 0 && M <= 32 && K > 0 && K <= 256 && N > 0 && N <= 256 && M % 16 == 0 && K % 16 == 0 &&
         N % 16 == 0 && wide_mm_smem(M, N, K, bt, qb, qa) <= kWideMmSmem;
}
// Offset of the FP16 B (F_QB) in the wide MATMUL layout: after the A and B^T
// tiles and, when B is not read transposed, the raw int8 B.
TAC_HD constexpr uint32_t wide_mm_bh_off(uint32_t M, uint32_t N, uint32_t K, bool bt) {
  return ((M + 15) / 16) * 16 * (((K + 31) & ~31u) + 16) + ((N + 7) / 8) * 8 * (((K + 31) & ~31u) + 16) +
         (bt ? 0u : ((K + 31) & ~31u) * N);
}

// Shared memory of an FX_PV task (QK^T [M x K] x [K x N], then P.V with
// K' = N): the P.V op's int8 A tile at 0, then the softmax scratch (the
// dequantised rows [M][N] FP16, two row buffers of N floats per warp, the
// pairwise-sum scratch); the QK^T op's F_DQ scale row keeps the last 512
// bytes.  With FX_PVPF, V lands at the P.V op's FP16-B offset, which must
// clear the softmax scratch and the QK^T op's A and B^T tiles (read by its
// MMAs while V is in flight).
constexpr uint32_t kExecWarps = 8;                           // warps of one half
constexpr uint32_t kPwScratchBytes = kExecWarps * 3 * 64 * 4;   // pairwise-sum scratch of every warp
TAC_HD constexpr uint32_t pv_a_bytes(uint32_t M, uint32_t N) { return ((M + 15) / 16) * 16 * (((N + 31) & ~31u) + 16); }
TAC_HD constexpr uint32_t pv_scratch_end(uint32_t M, uint32_t N) {
  return pv_a_bytes(M, N) + M * N * 2 + 2 * kExecWarps * N * 4 + kPwScratchBytes;
}
TAC_HD constexpr bool pv_ok(uint32_t M, uint32_t N) { return pv_scratch_end(M, N) <= kWideMmSmem - 512; }
// Row attention: one query row of an FX_PV pair (QK^T op x, P.V op y) on
// CUDA cores.  Q, the scores, P and the scratch sit below kAttnRowVOff, the
// visible K rows (as many as fit) and V rows above it; in a head group
// (FX_ATTNGRP) the next pair's rows land there while this pair computes.
// Groups are sized for one round over kTargetHalves executor halves (148 SMs
// x 2).
constexpr uint32_t kAttnRowVOff = 8192;
constexpr uint32_t kTargetHalves = 296;
constexpr uint32_t kAttnGroupMax = 8;   // pairs of one head group
TAC_HD constexpr bool attn_row_shape_ok(uint32_t xM, uint32_t xK, uint32_t xN, uint32_t xflags, uint32_t xflags2,
                                        uint32_t yM, uint32_t yK, uint32_t yN, uint32_t yflags) {
  return xM == 1 && (xflags & (F_WIDE | F_QA | F_QB | F_BT | F_DQ | F_SM | F_NOI32 | F_NODQ)) ==
                        uint32_t(F_WIDE | F_QA | F_QB | F_BT | F_DQ | F_SM | F_NOI32 | F_NODQ) &&
         !(xflags & F_ACCUMULATE) && (xflags2 & FX_PV) && (xflags2 & FX_SMSKIP) && xK % 8 == 0 && xK <= 128 &&
         xN % 8 == 0 && xN <= 1024 && yM == 1 &&
         (yflags & (F_WIDE | F_QB | F_DQ | F_NOI32)) == uint32_t(F_WIDE | F_QB | F_DQ | F_NOI32) &&
         !(yflags & (F_BT | F_ACCUMULATE | F_NODQ)) && yK == xN && yN % 8 == 0 && yN <= 64 &&
         kAttnRowVOff + xN * yN * 2 <= kWideMmSmem;
}
TAC_HD constexpr bool pvpf_ok(uint32_t M, uint32_t N, uint32_t K, uint32_t n_pv, bool bt_pv) {
  return pv_scratch_end(M, N) <= wide_mm_bh_off(M, n_pv, N, bt_pv) &&
         ((M + 15) / 16) * 16 * (((K + 31) & ~31u) + 16) + ((N + 7) / 8) * 8 * (((K + 31) & ~31u) + 16) <=
             wide_mm_bh_off(M, n_pv, N, bt_pv) &&
         wide_mm_bh_off(M, n_pv, N, bt_pv) + N * n_pv * 2 <= kWideMmSmem - 512;
}

// Rows of a row-op task: FP16 softmaxes of at most 1024 columns take 16 rows
// (two per warp, both rows' loads in flight together); the rest take 8.
TAC_HD constexpr uint32_t row_task_rows(uint32_t kind, uint32_t n) {
  return ((kind == K_SOFTMAX_F16 || kind == K_MASKED_SOFTMAX_F16) && n <= 1024) ? 16u : 8u;
}

// Parameters decoded from runtime-patched instruction words, one set per
// sequence.  Address parameters hold the 56-bit register value; attention
// parameters pack query_row_base | valid_kv_len << 16 | mode << 32.
struct RunParam {
  uint64_t value;
};

}  // namespace tac
