// Device executor: one persistent cooperative kernel runs a compiled plan.
//
// The grid walks the plan's dependency levels in order.  Inside a level the
// tasks (op x tile x sequence group) are independent and are spread over the
// CTAs; a bounded grid barrier separates levels.  Every op reproduces the
// golden model's arithmetic (see tac_numerics.cuh) on the physical operands
// the compiler resolved.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

#include "tac_isa.h"
#include "tac_numerics.cuh"
#include "tac_sm100.cuh"
#include "tac_plan.h"

namespace tac {

// The executor runs one 512-thread CTA per SM made of two independent halves
// of 256 threads.  Each half walks its own share of a level's tasks with its
// own shared memory, TMEM columns and mbarriers, and synchronizes on its own
// named barrier; the halves meet only at the grid barrier between levels.
// (A kernel that issues tcgen05 instructions gets one CTA per SM, so the
// halves provide the task concurrency that two CTAs per SM would.)
constexpr int kThreads = 256;                    // threads of one half
constexpr int kWarps = kThreads / 32;
constexpr int kHalves = 2;
constexpr int kCtaThreads = kThreads * kHalves;
constexpr uint32_t kBarrierSpinLimit = 1u << 22;   // polls of L2 (~0.5 us each): a few seconds

__device__ __forceinline__ uint32_t htid() { return threadIdx.x & (kThreads - 1); }   // thread in its half
__device__ __forceinline__ uint32_t hidx() { return threadIdx.x / kThreads; }         // which half
__device__ __forceinline__ void hsync() {
  asm volatile("bar.sync %0, %1;\n" ::"r"(1 + hidx()), "n"(kThreads) : "memory");
}

// Device-side fault codes (status word 0).
enum DevFault : uint32_t {
  DF_NONE = 0,
  DF_BARRIER_TIMEOUT = 1,
  DF_DYN_ADDRESS = 2,
  DF_ZERO_DENOM = 3,
  DF_BAD_OP = 4,
  DF_MMA_TIMEOUT = 5,
  DF_STAGE_TIMEOUT = 6,
};

struct ExecArgs {
  const CUtensorMap* tmaps;  // two per F_TC MATMUL (A, B), indexed by op.seg0
  const DevOp* ops;
  const Segment* segs;
  const Task* tasks;
  const uint32_t* level_off;
  uint32_t n_levels;
  uint32_t n_params;
  uint8_t* seq_base;
  uint64_t seq_stride;       // bytes
  const uint8_t* shared_base;
  uint16_t* sregs;           // [batch][sreg_stride]
  uint32_t sreg_stride;
  const uint64_t* params;    // [batch][n_params]
  uint32_t* status;          // [0] fault, [1] op, [2] seq, [3] level
  uint32_t* barrier;         // [0] arrivals, [1] generation
  uint64_t shared_bytes;
  uint64_t dram_bytes;
  uint64_t* prof;            // optional: globaltimer at the end of each level (n_levels + 1)
  uint32_t* task_prof;       // optional: SM cycles of each task
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint8_t* pptr(const ExecArgs& A, uint64_t phys, uint32_t seq) {
  if (phys & kSharedBit) return const_cast<uint8_t*>(A.shared_base) + ((phys & ~kSharedBit) << 4);
  return A.seq_base + uint64_t(seq) * A.seq_stride + (phys << 4);
}

__device__ __forceinline__ uint16_t sreg_bits(const ExecArgs& A, uint32_t enc, uint32_t seq) {
  if (enc & kSregConst) return static_cast<uint16_t>(enc & 0xFFFF);
  // slots are written by other CTAs earlier in the launch: read through L2
  return __ldcg(&A.sregs[uint64_t(seq) * A.sreg_stride + enc]);
}
__device__ __forceinline__ float sreg_f32(const ExecArgs& A, uint32_t enc, uint32_t seq) {
  return h2f(sreg_bits(A, enc, seq));
}

__device__ __forceinline__ void raise_fault(const ExecArgs& A, uint32_t code, uint32_t op, uint32_t seq) {
  if (atomicCAS(A.status, 0u, code) == 0u) {
    A.status[1] = op;
    A.status[2] = seq;
  }
}

// Address of DRAM byte `addr` for sequence `seq` (runtime-addressed copies).
__device__ __forceinline__ uint8_t* dram_ptr(const ExecArgs& A, uint64_t addr, uint32_t seq) {
  if (addr < A.shared_bytes) return const_cast<uint8_t*>(A.shared_base) + addr;
  return A.seq_base + uint64_t(seq) * A.seq_stride + uint64_t(kSramUnits) * 16 + (addr - A.shared_bytes);
}

// ---------------------------------------------------------------------------------
// Data movement
// ---------------------------------------------------------------------------------
// Copies segments [t.tile, t.aux) of the op.  A task with fewer segments
// than warps gives each segment several warps; every lane keeps four 16-byte
// loads in flight before it stores.
__device__ __noinline__ void op_gather(const ExecArgs& A, const DevOp& op, const Task& t) {
  const uint32_t warp = htid() >> 5, lane = htid() & 31;
  const uint32_t nseg = t.aux - t.tile;
  const uint32_t wps = nseg >= uint32_t(kWarps) ? 1u : uint32_t(kWarps) / nseg;   // warps per segment
  const uint32_t groups = uint32_t(kWarps) / wps;
  const uint32_t gi = warp / wps;
  if (gi >= groups) return;
  const uint32_t stride = wps * 32, start = (warp % wps) * 32 + lane;
  for (uint32_t k = t.tile + gi; k < t.aux; k += groups) {
    const Segment sg = A.segs[op.seg0 + k];
    const uint4* __restrict__ src = reinterpret_cast<const uint4*>(pptr(A, sg.src, t.seq0));
    uint4* __restrict__ dst = reinterpret_cast<uint4*>(pptr(A, sg.dst, t.seq0));
    const uint64_t n = sg.n;
    for (uint64_t u0 = start; u0 < n; u0 += 4 * stride) {
      uint4 v[4];
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j)
        if (u0 + j * stride < n) v[j] = __ldcg(src + u0 + j * stride);
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j)
        if (u0 + j * stride < n) dst[u0 + j * stride] = v[j];
    }
  }
}

__device__ __noinline__ void op_dyn_copy(const ExecArgs& A, const DevOp& op, const Task& t, uint32_t opi) {
  const uint32_t seq = t.seq0;
  const uint64_t addr = A.params[uint64_t(seq) * A.n_params + op.param] + op.dconst;
  if ((addr & 15) || addr + op.nbytes > A.dram_bytes) {
    if (htid() == 0) raise_fault(A, DF_DYN_ADDRESS, opi, seq);
    return;
  }
  const uint64_t n = op.nbytes / 16;
  const uint4* src;
  uint4* dst;
  if (op.kind == K_DYN_LOAD) {
    src = reinterpret_cast<const uint4*>(dram_ptr(A, addr, seq));
    dst = reinterpret_cast<uint4*>(pptr(A, op.d, seq));
  } else {
    if (addr < A.shared_bytes) {
      if (htid() == 0) raise_fault(A, DF_DYN_ADDRESS, opi, seq);
      return;
    }
    src = reinterpret_cast<const uint4*>(pptr(A, op.a, seq));
    dst = reinterpret_cast<uint4*>(dram_ptr(A, addr, seq));
  }
  for (uint64_t u = htid(); u < n; u += kThreads) dst[u] = __ldcg(src + u);
}

// The runtime-addressed stores of one level for one sequence: eight threads
// per store, each taking 16-byte units of it; the address checks of
// op_dyn_copy apply to every store.
__device__ __noinline__ void op_dyn_store_multi(const ExecArgs& A, const DevOp& op, const Task& t, uint32_t opi) {
  const uint32_t seq = t.seq0;
  for (uint32_t k = htid() / 8; k < op.nseg; k += kThreads / 8) {
    const Segment sg = A.segs[op.seg0 + k];
    const uint64_t addr = A.params[uint64_t(seq) * A.n_params + (sg.dst >> 32)] + (sg.dst & 0xFFFFFFFFull);
    if ((addr & 15) || addr + sg.n > A.dram_bytes || addr < A.shared_bytes) {
      if ((htid() & 7) == 0) raise_fault(A, DF_DYN_ADDRESS, opi, seq);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(pptr(A, sg.src, seq));
    uint4* dst = reinterpret_cast<uint4*>(dram_ptr(A, addr, seq));
    for (uint64_t u = htid() & 7; u < sg.n / 16; u += 8) dst[u] = __ldcg(src + u);
  }
}

// int8 [rows, cols] -> [cols, rows].  A matrix of at most kTransposeSmem bytes
// (one task) is staged in shared memory: 16-byte coalesced loads, then each
// thread gathers 16 consecutive output bytes of one column.  Larger matrices
// take the element loop, 16384 output bytes per task.
constexpr uint32_t kTransposeSmem = 16384;

__device__ __noinline__ void op_transpose(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem) {
  const int8_t* __restrict__ src = reinterpret_cast<const int8_t*>(pptr(A, op.a, t.seq0));
  int8_t* __restrict__ dst = reinterpret_cast<int8_t*>(pptr(A, op.d, t.seq0));
  const uint32_t rows = op.M, cols = op.N, total = rows * cols;
  if (t.tile == 0 && total <= kTransposeSmem && rows % 16 == 0 && cols % 16 == 0) {
    const uint32_t nv = total / 16;
    const uint4* __restrict__ s4 = reinterpret_cast<const uint4*>(src);
    uint4* sm4 = reinterpret_cast<uint4*>(smem);
    for (uint32_t i0 = htid(); i0 < nv; i0 += 4 * kThreads) {
      uint4 v[4];
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j)
        if (i0 + j * kThreads < nv) v[j] = __ldcg(s4 + i0 + j * kThreads);
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j)
        if (i0 + j * kThreads < nv) sm4[i0 + j * kThreads] = v[j];
    }
    hsync();
    const uint32_t rchunks = rows / 16;
    uint4* __restrict__ d4 = reinterpret_cast<uint4*>(dst);
    for (uint32_t o = htid(); o < nv; o += kThreads) {
      const uint32_t c = o % cols, r0 = (o / cols) * 16;   // output column c, rows r0 .. r0+15
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t x = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) x |= uint32_t(smem[(r0 + 4 * q + j) * cols + c]) << (8 * j);
        w[q] = x;
      }
      d4[c * rchunks + r0 / 16] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    return;
  }
  const uint64_t lo = uint64_t(t.tile) * 16384, hi = lo + 16384 < total ? lo + 16384 : total;
  for (uint64_t i0 = lo + htid(); i0 < hi; i0 += 4 * kThreads) {
    int8_t v[4];
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
      const uint64_t i = i0 + j * kThreads;
      if (i < hi) v[j] = src[(i % rows) * cols + i / rows];   // dst element i = (i / rows, i % rows)
    }
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j)
      if (i0 + j * kThreads < hi) dst[i0 + j * kThreads] = v[j];
  }
}

__device__ __noinline__ void op_sreg_load(const ExecArgs& A, const DevOp& op, const Task& t) {
  for (uint32_t s = t.seq0 + htid(); s < t.seq0 + t.nseq; s += kThreads) {
    const uint16_t v = *reinterpret_cast<const uint16_t*>(pptr(A, op.a, s));
    A.sregs[uint64_t(s) * A.sreg_stride + op.out_slot] = v;
  }
}

__device__ __noinline__ void op_sreg_final(const ExecArgs& A, const DevOp& op, const Task& t) {
  for (uint32_t s = t.seq0 + htid(); s < t.seq0 + t.nseq; s += kThreads) {
    uint16_t vals[16];
    for (uint32_t k = 0; k < op.nseg && k < 16; ++k)
      vals[k] = sreg_bits(A, static_cast<uint32_t>(A.segs[op.seg0 + k].src), s);
    for (uint32_t k = 0; k < op.nseg && k < 16; ++k)
      A.sregs[uint64_t(s) * A.sreg_stride + A.segs[op.seg0 + k].dst] = vals[k];
  }
}

// ---------------------------------------------------------------------------------
// MATMUL: int8 x int8 -> int32 on the tensor cores (mma.sync m16n8k32).
// A task covers up to 128 rows (whole sequences when B is shared) x 64 columns.
// ---------------------------------------------------------------------------------
constexpr int kMmKc = 128;             // K chunk (bytes of A rows / rows of B)
constexpr int kMmStages = 2;           // cp.async pipeline depth (per-sequence operands: K <= 256 in decoder programs)
constexpr int kMmAStride = kMmKc + 16; // A row stride in shared memory: 144 B keeps the 8 rows
                                       // of an mma fragment load on distinct banks
constexpr int kMmAStage = 128 * kMmAStride; // 8 row blocks x 16 rows x K chunk
constexpr int kMmBStage = kMmKc * 64;  // K chunk x 64 columns, raw [k][n]
constexpr int kMmBStride = kMmKc + 16; // transposed B row stride [n][k] (bytes)
constexpr size_t kMmSmem = size_t(kMmStages) * (kMmAStage + kMmBStage) + 64 * kMmBStride;

__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                       uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, uint32_t src_bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gsrc), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __noinline__ void op_matmul(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem) {
  const uint32_t M = op.M, N = op.N, K = op.K;
  const uint32_t ntile = (N + 63) / 64;
  const bool grouped = (op.b & kSharedBit) && M < 128;
  uint32_t n0, nblocks;
  uint32_t blk_seq[8], blk_row[8];
  if (grouped) {
    n0 = t.tile * 64;
    const uint32_t bps = M / 16;
    nblocks = 0;
    for (uint32_t s = 0; s < t.nseq; ++s)
      for (uint32_t b = 0; b < bps && nblocks < 8; ++b) {
        blk_seq[nblocks] = t.seq0 + s;
        blk_row[nblocks] = b * 16;
        ++nblocks;
      }
  } else {
    n0 = (t.tile % ntile) * 64;
    const uint32_t r0 = (t.tile / ntile) * 128;
    nblocks = 0;
    for (uint32_t r = r0; r < M && nblocks < 8; r += 16) {
      blk_seq[nblocks] = t.seq0;
      blk_row[nblocks] = r;
      ++nblocks;
    }
  }
  const uint32_t ncols = N - n0 < 64 ? N - n0 : 64;
  uint8_t* As = smem;                                    // [stage][blk*16 + row][kMmAStride]
  uint8_t* Bs = smem + kMmStages * kMmAStage;            // [stage][k][64] raw
  uint8_t* Bt = Bs + kMmStages * kMmBStage;              // [n][kMmBStride] transposed
  const int warp = htid() >> 5, lane = htid() & 31;
  const int g = lane >> 2, q = lane & 3;
  int acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0;

  const uint8_t* Bg = pptr(A, op.b, t.seq0);
  const uint8_t* Ag[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) Ag[i] = i < int(nblocks) ? pptr(A, op.a, blk_seq[i]) + uint64_t(blk_row[i]) * K : nullptr;
  const uint32_t nchunks = (K + kMmKc - 1) / kMmKc;

  // issues the cp.async copies of chunk c into pipeline slot c % kMmStages
  auto issue = [&](uint32_t c) {
    const uint32_t k0 = c * kMmKc;
    const uint32_t kc = K - k0 < uint32_t(kMmKc) ? K - k0 : uint32_t(kMmKc);
    uint8_t* as = As + (c % kMmStages) * kMmAStage;
    uint8_t* bs = Bs + (c % kMmStages) * kMmBStage;
    // A: nblocks*16 rows x 8 vectors of 16 bytes
    for (uint32_t i = htid(); i < nblocks * 16 * (kMmKc / 16); i += kThreads) {
      const uint32_t v = i % (kMmKc / 16), row = i / (kMmKc / 16);
      const bool in = v * 16 < kc;
      const uint8_t* src = Ag[row / 16] + uint64_t(row % 16) * K + k0 + (in ? v * 16 : 0);
      cp_async16(as + row * kMmAStride + v * 16, src, in ? 16u : 0u);
    }
    // B: kMmKc rows x 4 vectors of 16 bytes (64 columns)
    for (uint32_t i = htid(); i < uint32_t(kMmKc) * 4; i += kThreads) {
      const uint32_t v = i % 4, kk = i / 4;
      const bool in = kk < kc && v * 16 < ncols;
      const uint8_t* src = Bg + (in ? uint64_t(k0 + kk) * N + n0 + v * 16 : 0);
      cp_async16(bs + kk * 64 + v * 16, src, in ? 16u : 0u);
    }
  };

#pragma unroll
  for (int sidx = 0; sidx < kMmStages - 1; ++sidx) {
    if (uint32_t(sidx) < nchunks) issue(sidx);
    cp_async_commit();
  }
  for (uint32_t c = 0; c < nchunks; ++c) {
    cp_async_wait<kMmStages - 2>();
    hsync();   // chunk c landed; every warp finished chunk c-1 (slot and Bt free)
    if (c + kMmStages - 1 < nchunks) issue(c + kMmStages - 1);
    cp_async_commit();
    const uint32_t k0 = c * kMmKc;
    const uint32_t kc = K - k0 < uint32_t(kMmKc) ? K - k0 : uint32_t(kMmKc);
    const uint32_t kc32 = (kc + 31) & ~31u;
    const uint8_t* as = As + (c % kMmStages) * kMmAStage;
    const uint8_t* bs = Bs + (c % kMmStages) * kMmBStage;
    // transpose B [k][n] -> Bt [n][k], 4x4 byte blocks
    for (uint32_t i = htid(); i < (kc32 / 4) * 16; i += kThreads) {
      const uint32_t kb = (i / 16) * 4, nb = (i % 16) * 4;
      uint32_t r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = *reinterpret_cast<const uint32_t*>(bs + (kb + j) * 64 + nb);
      const uint32_t t0 = __byte_perm(r[0], r[1], 0x5140), t1 = __byte_perm(r[2], r[3], 0x5140);
      const uint32_t t2 = __byte_perm(r[0], r[1], 0x7362), t3 = __byte_perm(r[2], r[3], 0x7362);
      *reinterpret_cast<uint32_t*>(Bt + (nb + 0) * kMmBStride + kb) = __byte_perm(t0, t1, 0x5410);
      *reinterpret_cast<uint32_t*>(Bt + (nb + 1) * kMmBStride + kb) = __byte_perm(t0, t1, 0x7632);
      *reinterpret_cast<uint32_t*>(Bt + (nb + 2) * kMmBStride + kb) = __byte_perm(t2, t3, 0x5410);
      *reinterpret_cast<uint32_t*>(Bt + (nb + 3) * kMmBStride + kb) = __byte_perm(t2, t3, 0x7632);
    }
    hsync();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t p = warp + 8 * i;
      const uint32_t blk = p / 8, ns = p % 8;
      if (blk >= nblocks || ns * 8 >= ncols) continue;
      const uint8_t* a_row0 = as + (blk * 16 + g) * kMmAStride;
      const uint8_t* a_row8 = as + (blk * 16 + g + 8) * kMmAStride;
      const uint8_t* b_col = Bt + (ns * 8 + g) * kMmBStride;
      for (uint32_t ks = 0; ks < kc32; ks += 32) {
        const uint32_t a0 = *reinterpret_cast<const uint32_t*>(a_row0 + ks + q * 4);
        const uint32_t a1 = *reinterpret_cast<const uint32_t*>(a_row8 + ks + q * 4);
        const uint32_t a2 = *reinterpret_cast<const uint32_t*>(a_row0 + ks + 16 + q * 4);
        const uint32_t a3 = *reinterpret_cast<const uint32_t*>(a_row8 + ks + 16 + q * 4);
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(b_col + ks + q * 4);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(b_col + ks + 16 + q * 4);
        mma_s8(acc[i], a0, a1, a2, a3, b0, b1);
      }
    }
  }
  cp_async_wait<0>();
  // epilogue
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t p = warp + 8 * i;
    const uint32_t blk = p / 8, ns = p % 8;
    if (blk >= nblocks || ns * 8 >= ncols) continue;
    const uint32_t col = n0 + ns * 8 + q * 2;
    const uint32_t seq = blk_seq[blk];
    int32_t* D = reinterpret_cast<int32_t*>(pptr(A, op.d, seq));
    const int32_t* C = (op.flags & F_ACCUMULATE) ? reinterpret_cast<const int32_t*>(pptr(A, op.c, seq)) : nullptr;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint64_t row = blk_row[blk] + g + 8 * h;
      int2 v = make_int2(acc[i][2 * h], acc[i][2 * h + 1]);
      if (C) {
        const int2 c = __ldcg(reinterpret_cast<const int2*>(C + row * N + col));
        v.x = static_cast<int32_t>(static_cast<uint32_t>(v.x) + static_cast<uint32_t>(c.x));
        v.y = static_cast<int32_t>(static_cast<uint32_t>(v.y) + static_cast<uint32_t>(c.y));
      }
      *reinterpret_cast<int2*>(D + row * N + col) = v;
    }
  }
  hsync();
}

// ---------------------------------------------------------------------------------
// Small vector helpers: 16-byte loads through L2 and lane views of packed values.
// ---------------------------------------------------------------------------------
struct V8 { uint4 lo, hi; };   // 8 x 32-bit values

// Operands are written by other CTAs in earlier levels of the same launch, so
// loads go through L2 (ld.global.cg), never the non-coherent read-only path.
__device__ __forceinline__ uint4 ld16(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint2 ld8(const void* p) { return __ldcg(reinterpret_cast<const uint2*>(p)); }
__device__ __forceinline__ V8 ld32(const void* p) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  return V8{__ldcg(q), __ldcg(q + 1)};
}
__device__ __forceinline__ uint16_t h_at(const uint4& v, int j) {
  const uint32_t w = j < 2 ? v.x : j < 4 ? v.y : j < 6 ? v.z : v.w;
  return static_cast<uint16_t>(j & 1 ? w >> 16 : w & 0xFFFF);
}
__device__ __forceinline__ int32_t i_at(const V8& v, int j) {
  const uint4& q = j < 4 ? v.lo : v.hi;
  const int k = j & 3;
  return static_cast<int32_t>(k == 0 ? q.x : k == 1 ? q.y : k == 2 ? q.z : q.w);
}
__device__ __forceinline__ int8_t b_at(const uint2& v, int j) {
  const uint32_t w = j < 4 ? v.x : v.y;
  return static_cast<int8_t>((w >> (8 * (j & 3))) & 0xFF);
}
__device__ __forceinline__ uint4 pack_h(const uint16_t (&h)[8]) {
  return make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                    h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
}
__device__ __forceinline__ uint2 pack_b(const int8_t (&q)[8]) {
  uint32_t x = 0, y = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    x |= uint32_t(uint8_t(q[j])) << (8 * j);
    y |= uint32_t(uint8_t(q[j + 4])) << (8 * j);
  }
  return make_uint2(x, y);
}

// One FP16 softmax row (SOFTMAX_FP32 / MASKED_SOFTMAX_FP32, simulator.py:964-1037)
// held as floats in rowbuf (n a multiple of 8): columns after `last` are
// masked (last = n - 1 for the plain softmax).  exp in float64 rounded once,
// NumPy's pairwise row sum, f16(e / sum); a masked row whose sum is zero, or
// with no visible column (masked and last < 0), writes zeros.
__device__ __forceinline__ void softmax_row_f16(float* rowbuf, uint32_t n, bool masked, int64_t last,
                                                uint16_t* out, uint32_t* pw, int lane, int8_t* qout = nullptr,
                                                float qs = 0.f) {
  if (masked && last < 0) {
    for (uint32_t g = lane; g < n / 8; g += 32) {
      if (out) reinterpret_cast<uint4*>(out)[g] = make_uint4(0, 0, 0, 0);
      if (qout) reinterpret_cast<uint2*>(qout)[g] = make_uint2(0, 0);
    }
    return;
  }
  const uint32_t lst = masked ? static_cast<uint32_t>(last) : n - 1;
  float mx = -INFINITY;
  for (uint32_t j = lane; j <= lst && j < n; j += 32) mx = fmaxf(mx, rowbuf[j]);
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  __syncwarp();
  for (uint32_t j = lane; j < n; j += 32) rowbuf[j] = j <= lst ? exp_f32(__fsub_rn(rowbuf[j], mx)) : 0.f;
  __syncwarp();
  const float denom = warp_pairwise_sum_smem(rowbuf, n, pw, false, 0.f, lst + 1);
  if (!out && qout) {   // only the quantised rows: column j on lane j % 32; masked columns are zero
    for (uint32_t j0 = 0; j0 < n; j0 += 32) {
      const uint32_t j = j0 + lane;
      int8_t q8 = 0;
      if (j0 <= lst && j <= lst) {
        const float e = rowbuf[j];
        const uint16_t h = f2h(!masked ? __fdiv_rn(e, denom) : (denom > 0.f ? __fdiv_rn(e, denom) : 0.f));
        q8 = sat8(__fmul_rn(h2f(h), qs));
      }
      if (j < n) qout[j] = q8;
    }
    return;
  }
  for (uint32_t g = lane; g < n / 8; g += 32) {
    uint16_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float e = rowbuf[g * 8 + j];
      h[j] = f2h(!masked ? __fdiv_rn(e, denom) : (denom > 0.f ? __fdiv_rn(e, denom) : 0.f));
    }
    if (out) reinterpret_cast<uint4*>(out)[g] = pack_h(h);
    if (qout) {   // QUANT's rule on the FP16 value: rint(x * s), NaN -> 0, clipped to int8
      int8_t q8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        q8[j] = sat8(__fmul_rn(h2f(h[j]), qs));
      }
      reinterpret_cast<uint2*>(qout)[g] = pack_b(q8);
    }
  }
}

constexpr int kTcStages = 3;                            // stage slots (64-column tasks use 3, 128-column 2)

// Per-half state of the TMA / tcgen05 stages and of the bulk-copy stage
// barrier: mbarriers, the half's TMEM columns and the next phase parities.
struct TcShared {
  uint64_t full[kTcStages];    // TMA bytes of a stage landed
  uint64_t empty[kTcStages];   // the MMAs reading a stage completed
  uint64_t stage;              // bulk-copied element-wise operands landed
  uint64_t stage2;             // row attention: its V rows landed
  uint32_t tmem;
  uint32_t phase_full;         // bit s: parity of the next phase of full[s]
  uint32_t phase_empty;
  uint32_t phase_stage;        // parity of the next phase of `stage`
  uint32_t phase_stage2;       // parity of the next phase of `stage2`
  uint32_t pv_phase;           // FX_PVPF: parity of the `stage` phase that brings V
};

// Two softmax rows of one warp quantised for the P.V A tile only (rows in
// rb0 / rb1 as floats, last visible columns last0 / last1, -1 for none): the
// bytes two softmax_row_f16 calls with out == nullptr write, the two rows'
// chains interleaved.
__device__ __forceinline__ void softmax_rows2_q(float* rb0, float* rb1, uint32_t n, bool masked, int64_t last0,
                                                int64_t last1, uint32_t* pw0, uint32_t* pw1, int lane, int8_t* q0,
                                                int8_t* q1, float qs) {
  const int64_t l0 = masked ? last0 : int64_t(n) - 1, l1 = masked ? last1 : int64_t(n) - 1;
  float m0 = -INFINITY, m1 = -INFINITY;
  for (uint32_t j = lane; j < n; j += 32) {
    if (int64_t(j) <= l0) m0 = fmaxf(m0, rb0[j]);
    if (int64_t(j) <= l1) m1 = fmaxf(m1, rb1[j]);
  }
  for (int o = 16; o; o >>= 1) {
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
  }
  __syncwarp();
  for (uint32_t j = lane; j < n; j += 32) {
    rb0[j] = int64_t(j) <= l0 ? exp_f32(__fsub_rn(rb0[j], m0)) : 0.f;
    rb1[j] = int64_t(j) <= l1 ? exp_f32(__fsub_rn(rb1[j], m1)) : 0.f;
  }
  __syncwarp();
  float d0, d1;
  warp_pairwise_sum2_smem(rb0, rb1, n, pw0, pw1, uint32_t(l0 + 1), uint32_t(l1 + 1), d0, d1);
  for (uint32_t j0 = 0; j0 < n; j0 += 32) {
    const uint32_t j = j0 + lane;
    int8_t a = 0, b = 0;
    if (int64_t(j0) <= l0 && int64_t(j) <= l0) {
      const float e = rb0[j];
      a = sat8(__fmul_rn(h2f(f2h(!masked ? __fdiv_rn(e, d0) : (d0 > 0.f ? __fdiv_rn(e, d0) : 0.f))), qs));
    }
    if (int64_t(j0) <= l1 && int64_t(j) <= l1) {
      const float e = rb1[j];
      b = sat8(__fmul_rn(h2f(f2h(!masked ? __fdiv_rn(e, d1) : (d1 > 0.f ? __fdiv_rn(e, d1) : 0.f))), qs));
    }
    if (j < n) {
      q0[j] = a;
      q1[j] = b;
    }
  }
}

// ---------------------------------------------------------------------------------
// MATMUL with per-sequence operands in the wide shape (F_WIDE: M <= 32,
// K <= 256, N <= 256, shared memory by wide_mm_smem): one task computes every
// column of one sequence (QK^T and P.V of a head).  A and B^T land in shared
// memory as rows of K bytes padded to the MMA's 32 plus 16 (so the eight rows
// of a fragment load sit on distinct banks).  B^T is copied row by row when
// the op holds it (F_BT), else B [K][N] is loaded and transposed in 4 x 4 byte
// blocks.  With F_QB, B arrives as FP16 and is quantised on the way in, with
// QUANT's rule.  Padding bytes are zero.  a_staged: the int8 A tile is
// already in shared memory (the P.V op of an FX_PV pair, whose QK^T softmax
// wrote it there); b_staged: so are the FP16 B copies (FX_PVPF).
// ---------------------------------------------------------------------------------
__device__ __noinline__ uint32_t op_matmul_wide(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem,
                                                TcShared* tc, bool a_staged, bool b_staged,
                                                uint32_t k_used = 0xFFFFFFFFu) {
  const uint32_t M = op.M, N = op.N, K = op.K, seq = t.seq0;
  const uint32_t kc32 = (K + 31) & ~31u;
  // K rows that can be nonzero in A (the P.V op: P is zero past the QK^T
  // op's key columns kept), rounded up to the MMA's 32; zeros times any int8
  // add nothing, so the rows past them are neither quantised nor multiplied
  const uint32_t kr = k_used < K ? ((k_used + 31) & ~31u) : kc32;
  const uint32_t bts = kc32 + 16;
  const uint32_t nblocks = (M + 15) / 16, n8 = (N + 7) / 8;
  const bool bt = (op.flags & F_BT) != 0, qb = (op.flags & F_QB) != 0;
  const bool qa = !a_staged && (op.flags & F_QA) != 0;
  uint8_t* As = smem;                               // [nblocks * 16][bts]
  uint8_t* Bt = As + nblocks * 16 * bts;            // [n8 * 8][bts]
  uint8_t* Braw = Bt + n8 * 8 * bts;                // [kc32][N] (not F_BT)
  uint8_t* Bh = Braw + (bt ? 0u : kc32 * N);        // FP16 B (F_QB)
  uint8_t* Ah = wide_mm_a_in_bt(M, N, K, bt) ? Bt : Bh + (qb ? K * N * 2 : 0u);   // FP16 A (F_QA)
  uint8_t* Pc = smem + kWideMmSmem - 512;   // F_DQ scale row: the last 512 bytes (the budget's reserve)
  const bool dq = (op.flags & F_DQ) != 0;
  const uint8_t* Ag = pptr(A, op.a, seq);
  const uint8_t* Bg = pptr(A, op.b, seq);
  const uint32_t kv = kc32 / 16;                    // 16-byte vectors per padded row
  // the contiguous operands (FP16 A and B, quantised on load, and the F_DQ
  // scale row) arrive by bulk copies that one thread issues on the half's
  // stage barrier; padded int8 tiles take 16-byte copies per thread
  const bool bulk_b = qb && !b_staged, bulk_pc = dq && !b_staged;
  const uint32_t bulk_bytes = (qa ? M * K * 2 : 0u) + (bulk_b ? K * N * 2 : 0u) + (bulk_pc ? N * 2 : 0u);
  uint32_t par = 0;
  if (bulk_bytes) {
    par = tc->phase_stage;
    hsync();   // every thread has the parity before it flips
    if (htid() == 0) {
      tc->phase_stage = par ^ 1u;
      sm100::fence_proxy_async();
      sm100::mbar_arrive_expect_tx(&tc->stage, bulk_bytes);
      if (qa) sm100::bulk_g2s(Ah, Ag, M * K * 2, &tc->stage);
      if (bulk_b) sm100::bulk_g2s(Bh, Bg, K * N * 2, &tc->stage);
      if (bulk_pc) sm100::bulk_g2s(Pc, pptr(A, op.c, seq), N * 2, &tc->stage);
    }
  }
  if (!qa && !a_staged) {
    for (uint32_t i = htid(); i < nblocks * 16 * kv; i += kThreads) {
      const uint32_t r = i / kv, v = i % kv;
      const bool in = r < M && v * 16 < K;
      cp_async16(As + r * bts + v * 16, Ag + (in ? uint64_t(r) * K + v * 16 : 0), in ? 16u : 0u);
    }
  }
  if (qb) {
    // bulk copy above, or already staged
  } else if (bt) {
    for (uint32_t i = htid(); i < n8 * 8 * kv; i += kThreads) {
      const uint32_t n = i / kv, v = i % kv;
      const bool in = n < N && v * 16 < K;
      cp_async16(Bt + n * bts + v * 16, Bg + (in ? uint64_t(n) * K + v * 16 : 0), in ? 16u : 0u);
    }
  } else {
    const uint32_t nv = N / 16;
    for (uint32_t i = htid(); i < kc32 * nv; i += kThreads) {
      const uint32_t k = i / nv, v = i % nv;
      const bool in = k < K;
      cp_async16(Braw + k * N + v * 16, Bg + (in ? uint64_t(k) * N + v * 16 : 0), in ? 16u : 0u);
    }
  }
  if (dq && !bulk_pc) {
    const uint8_t* pg = pptr(A, op.c, seq);
    for (uint32_t i = htid(); i < N / 8; i += kThreads) cp_async16(Pc + i * 16, pg + uint64_t(i) * 16, 16u);
  }
  cp_async_commit();
  const uint16_t sb = qb ? sreg_bits(A, op.s[1], seq) : uint16_t(0);
  const uint16_t sa = qa ? sreg_bits(A, op.s[0], seq) : uint16_t(0);
  const bool sm = (op.flags & F_SM) != 0;
  uint32_t qrb = op.attn_qrb, vkl = op.attn_vkl;
  if (sm && (op.flags & F_ATTN_DYN)) {
    const uint64_t pv = A.params[uint64_t(seq) * A.n_params + op.param];
    qrb = pv & 0xFFFF;
    vkl = (pv >> 16) & 0xFFFF;
  }
  // masked softmax whose int32 and dequantised scores nothing reads: key
  // columns past every row's last visible one (min(M - 1 + qrb, vkl - 1))
  // are zero after the softmax whatever their scores, so only the first nk
  // keys (B^T rows) are quantised, multiplied and dequantised
  uint32_t nk = N;
  if (sm && bt && (op.flags & F_SMMASK) && (op.flags & F_NOI32) && (op.flags & F_NODQ) &&
      !(op.flags & F_ACCUMULATE)) {
    const int64_t lmax = int64_t(M) - 1 + qrb < int64_t(vkl) - 1 ? int64_t(M) - 1 + qrb : int64_t(vkl) - 1;
    nk = lmax < 0 ? 0u : min(N, (uint32_t(lmax) + 8) & ~7u);
  }
  cp_async_wait<0>();
  // the bulk copies of this op, then (FX_PVPF) V, issued by its QK^T op
  const bool bulk_ok = !bulk_bytes || sm100::mbar_wait(&tc->stage, par, nullptr, 0);
  if (!bulk_ok || (b_staged && !sm100::mbar_wait(&tc->stage, tc->pv_phase, nullptr, 0))) {
    sm100::mbar_wait(&tc->stage, bulk_ok ? tc->pv_phase : par, nullptr, 0);   // bounded: let copies land
    if (htid() == 0) raise_fault(A, DF_STAGE_TIMEOUT, t.op, seq);
    return 0xFFFFFFFFu;
  }
  hsync();
  if (qa) {
    // QUANT's rule into the padded A rows; padding rows and columns are zero
    const float s0 = h2f(sa);
    for (uint32_t i = htid(); i < nblocks * 16 * (kc32 / 8); i += kThreads) {
      const uint32_t r = i / (kc32 / 8), k = (i % (kc32 / 8)) * 8;
      int8_t q8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (r < M && k < K) {
        const uint4 x = *reinterpret_cast<const uint4*>(Ah + (uint64_t(r) * K + k) * 2);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          q8[j] = sat8(__fmul_rn(h2f(h_at(x, j)), s0));
        }
      }
      *reinterpret_cast<uint2*>(As + r * bts + k) = pack_b(q8);
    }
    if (!qb) hsync();
  }
  if (qb) {
    // QUANT's rule: rint(x * s), NaN -> 0, clipped to int8; 8 elements per step
    const float s1 = h2f(sb);
    const uint32_t qn = bt ? nk * K / 8 : min(K, kr) * N / 8;   // B^T rows of the kept keys, or B's K rows < kr
    for (uint32_t i = htid(); i < qn; i += kThreads) {
      const uint4 x = *reinterpret_cast<const uint4*>(Bh + i * 16);
      int8_t q8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        q8[j] = sat8(__fmul_rn(h2f(h_at(x, j)), s1));
      }
      const uint32_t e = i * 8;
      uint8_t* dst = bt ? Bt + (e / K) * bts + (e % K) : Braw + e;   // [N][K] rows or [K][N]
      *reinterpret_cast<uint2*>(dst) = pack_b(q8);
    }
    // zero padding: B^T columns K .. kc32 of every row, or raw rows K .. kc32
    if (kc32 > K) {
      if (bt) {
        for (uint32_t i = htid(); i < n8 * 8 * ((kc32 - K) / 16); i += kThreads) {
          const uint32_t n = i / ((kc32 - K) / 16), v = i % ((kc32 - K) / 16);
          *reinterpret_cast<uint4*>(Bt + n * bts + K + v * 16) = make_uint4(0, 0, 0, 0);
        }
      } else {
        for (uint32_t i = htid(); i < (kc32 - K) * N / 16; i += kThreads)
          *reinterpret_cast<uint4*>(Braw + K * N + i * 16) = make_uint4(0, 0, 0, 0);
      }
    }
    hsync();
  }
  if (!bt) {
    const uint32_t nb4 = N / 4;
    for (uint32_t i = htid(); i < (kr / 4) * nb4; i += kThreads) {
      const uint32_t kb = (i / nb4) * 4, nb = (i % nb4) * 4;
      uint32_t r[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) r[j] = *reinterpret_cast<const uint32_t*>(Braw + (kb + j) * N + nb);
      const uint32_t t0 = __byte_perm(r[0], r[1], 0x5140), t1 = __byte_perm(r[2], r[3], 0x5140);
      const uint32_t t2 = __byte_perm(r[0], r[1], 0x7362), t3 = __byte_perm(r[2], r[3], 0x7362);
      *reinterpret_cast<uint32_t*>(Bt + (nb + 0) * bts + kb) = __byte_perm(t0, t1, 0x5410);
      *reinterpret_cast<uint32_t*>(Bt + (nb + 1) * bts + kb) = __byte_perm(t0, t1, 0x7632);
      *reinterpret_cast<uint32_t*>(Bt + (nb + 2) * bts + kb) = __byte_perm(t2, t3, 0x5410);
      *reinterpret_cast<uint32_t*>(Bt + (nb + 3) * bts + kb) = __byte_perm(t2, t3, 0x7632);
    }
    hsync();
  }
  if ((op.flags2 & FX_PVPF) && htid() == 0) {
    // V for the P.V op, one bulk copy in flight while this op multiplies and
    // takes the softmax; its region was last read before the barrier above
    const DevOp& y = A.ops[op.seg0];
    const uint32_t vpar = tc->phase_stage;
    tc->pv_phase = vpar;
    tc->phase_stage = vpar ^ 1u;
    sm100::fence_proxy_async();
    sm100::mbar_arrive_expect_tx(&tc->stage, y.K * y.N * 2);
    sm100::bulk_g2s(smem + wide_mm_bh_off(y.M, y.N, y.K, (y.flags & F_BT) != 0), pptr(A, y.b, seq),
                    y.K * y.N * 2, &tc->stage);
  }
  const int warp = htid() >> 5, lane = htid() & 31;
  const int g = lane >> 2, q = lane & 3;
  const uint32_t pairs = nblocks * n8;
  int acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t p = warp + 8 * i;
    if (p >= pairs || (p % n8) * 8 >= nk) continue;
    const uint32_t blk = p / n8, ns = p % n8;
    const uint8_t* a_row0 = As + (blk * 16 + g) * bts;
    const uint8_t* a_row8 = a_row0 + 8 * bts;
    const uint8_t* b_col = Bt + (ns * 8 + g) * bts;
    for (uint32_t ks = 0; ks < kr; ks += 32) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(a_row0 + ks + q * 4);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(a_row8 + ks + q * 4);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(a_row0 + ks + 16 + q * 4);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(a_row8 + ks + 16 + q * 4);
      const uint32_t b0 = *reinterpret_cast<const uint32_t*>(b_col + ks + q * 4);
      const uint32_t b1 = *reinterpret_cast<const uint32_t*>(b_col + ks + 16 + q * 4);
      mma_s8(acc[i], a0, a1, a2, a3, b0, b1);
    }
  }
  if (sm) hsync();   // every warp is done with the operand tiles: the rows reuse the space
  // F_SM: the dequantised rows [M][N] FP16 in shared memory, then per-warp
  // float row buffers and pairwise-sum scratch behind them (FX_PV: packed
  // behind the P.V op's A tile, which the softmax rows are quantised into)
  const bool pv = (op.flags2 & FX_PV) != 0;
  uint8_t* sbase = smem + (pv ? pv_a_bytes(M, N) : 0u);
  uint16_t* Sc = reinterpret_cast<uint16_t*>(sbase);
  float* rows = reinterpret_cast<float*>(sbase + (pv ? M * N * 2 : 32u * 256 * 2));
  // (FX_PV: two row buffers per warp, for the two-row softmax)
  uint32_t* pws = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(rows) + kWarps * (pv ? 2 * N : 256u) * 4);
  int32_t* D = reinterpret_cast<int32_t*>(pptr(A, op.d, seq));
  const int32_t* C = (op.flags & F_ACCUMULATE) ? reinterpret_cast<const int32_t*>(pptr(A, op.c, seq)) : nullptr;
  const bool store_i32 = !(op.flags & F_NOI32);
  const bool store_dq = dq && !(op.flags & F_NODQ);
  uint16_t* D16 = dq ? reinterpret_cast<uint16_t*>(pptr(A, static_cast<uint64_t>(op.dconst), seq)) : nullptr;
  // the F_DQ scale row: read from shared memory before the rows overwrite it
  const uint8_t* Pcs = Pc;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t p = warp + 8 * i;
    if (p >= pairs) continue;
    const uint32_t blk = p / n8, ns = p % n8;
    const uint32_t col = ns * 8 + q * 2;
    if (col >= nk) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint64_t row = blk * 16 + g + 8 * h;
      if (row >= M) continue;
      int2 v = make_int2(acc[i][2 * h], acc[i][2 * h + 1]);
      if (C) {
        const int2 c = __ldcg(reinterpret_cast<const int2*>(C + row * N + col));
        v.x = static_cast<int32_t>(static_cast<uint32_t>(v.x) + static_cast<uint32_t>(c.x));
        v.y = static_cast<int32_t>(static_cast<uint32_t>(v.y) + static_cast<uint32_t>(c.y));
      }
      if (store_i32) *reinterpret_cast<int2*>(D + row * N + col) = v;
      if (dq) {   // DEQUANT_ACCUM: f16(f32(acc) * f32(scale[col]))
        const uint32_t sc = *reinterpret_cast<const uint32_t*>(Pcs + col * 2);
        const uint16_t lo = f2h(__fmul_rn(__int2float_rn(v.x), h2f(static_cast<uint16_t>(sc & 0xFFFF))));
        const uint16_t hi = f2h(__fmul_rn(__int2float_rn(v.y), h2f(static_cast<uint16_t>(sc >> 16))));
        const uint32_t pr = uint32_t(lo) | (uint32_t(hi) << 16);
        if (store_dq) *reinterpret_cast<uint32_t*>(D16 + row * N + col) = pr;
        if (sm) *reinterpret_cast<uint32_t*>(Sc + row * N + col) = pr;
      }
    }
  }
  if (sm) {
    hsync();
    uint16_t* out = (op.flags2 & FX_SMSKIP) ? nullptr : reinterpret_cast<uint16_t*>(pptr(A, op.nbytes, seq));
    int8_t* qout = nullptr;
    float qs = 0.f;
    const uint32_t qstride = ((N + 31) & ~31u) + 16;   // the P.V op's A rows: K = N bytes, padded
    if (pv) {
      qout = reinterpret_cast<int8_t*>(smem);
      qs = h2f(sreg_bits(A, A.ops[op.seg0].s[0], seq));
    }
    const bool masked = (op.flags & F_SMMASK) != 0;
    float* rb = rows + warp * (pv ? 2 * N : N);
    uint32_t* pw = pws + warp * (3 * kPwMaxLeaves);
    auto row_last = [&](uint32_t r) -> int64_t {
      return int64_t(r) + qrb < int64_t(vkl) - 1 ? int64_t(r) + qrb : int64_t(vkl) - 1;
    };
    auto zero_pad = [&](uint32_t r) {   // the A row's padding columns N .. (N rounded up to 32) are zero
      for (uint32_t g = N / 16 + lane; g < (qstride - 16) / 16; g += 32)
        reinterpret_cast<uint4*>(qout + uint64_t(r) * qstride)[g] = make_uint4(0, 0, 0, 0);
    };
    uint32_t r_single = 0;   // first row left to the one-row loop below
    if (qout && !out) {      // rows r and r + kWarps of this warp together
      float* rb1 = rb + N;
      for (uint32_t r = warp; r + kWarps < M; r += 2 * kWarps) {
        const uint32_t r1 = r + kWarps;
        const int64_t lt0 = masked ? row_last(r) : int64_t(N) - 1, lt1 = masked ? row_last(r1) : int64_t(N) - 1;
        const uint32_t n0 = lt0 < 0 ? 0u : min(N, uint32_t(lt0) + 1), n1 = lt1 < 0 ? 0u : min(N, uint32_t(lt1) + 1);
        for (uint32_t j = lane; j < n0 || j < n1; j += 32) {
          if (j < n0) rb[j] = h2f(Sc[r * N + j]);
          if (j < n1) rb1[j] = h2f(Sc[r1 * N + j]);
        }
        __syncwarp();
        softmax_rows2_q(rb, rb1, N, masked, lt0, lt1, pw, pw, lane, qout + uint64_t(r) * qstride,
                        qout + uint64_t(r1) * qstride, qs);
        zero_pad(r);
        zero_pad(r1);
        __syncwarp();
      }
      r_single = M - M % (2 * kWarps);   // rows past the last full pair of passes
    }
    for (uint32_t r = r_single + warp; r < M; r += kWarps) {
      const int64_t lt = row_last(r);
      const uint32_t nr = masked ? (lt < 0 ? 0u : min(N, uint32_t(lt) + 1)) : N;   // columns the row reads
      for (uint32_t j = lane; j < nr; j += 32) rb[j] = h2f(Sc[r * N + j]);
      __syncwarp();
      softmax_row_f16(rb, N, masked, masked ? lt : int64_t(N) - 1, out ? out + uint64_t(r) * N : nullptr, pw, lane,
                      qout ? qout + uint64_t(r) * qstride : nullptr, qs);
      if (qout) zero_pad(r);
      __syncwarp();
    }
  }
  return nk;
}

// NumPy's pairwise sum of x[0..N) (or of (x - mean)^2), for a balanced tree
// of nl <= 8 leaves of L elements, by every warp of the half: warp w sums
// leaf w (lanes 0..7 one accumulator chain each, combined by xor shuffles),
// the leaf sums combine level by level.  `part` holds 8 floats; every thread
// returns the sum.  Contains one hsync.
__device__ __forceinline__ float ln_pairwise(const float* x, uint32_t nl, uint32_t L, bool sq, float mean,
                                             float* part) {
  const uint32_t warp = htid() >> 5, lane = htid() & 31;
  float v = 0.f;
  if (warp < nl && lane < 8) {
    const float* q = x + warp * L + lane;
    float r;
    if (sq) {
      const float d0 = __fsub_rn(q[0], mean);
      r = __fmul_rn(d0, d0);
      for (uint32_t i = 8; i < L; i += 8) {
        const float d = __fsub_rn(q[i], mean);
        r = __fadd_rn(r, __fmul_rn(d, d));
      }
    } else {
      r = q[0];
      for (uint32_t i = 8; i < L; i += 8) r = __fadd_rn(r, q[i]);
    }
    v = r;
  }
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 4));
  if (lane == 0 && warp < nl) part[warp] = v;
  hsync();
  float t8[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) t8[k] = part[k < int(nl) ? k : 0];
  for (uint32_t w = nl; w > 1; w >>= 1)
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k)
      if (k < w / 2) t8[k] = __fadd_rn(t8[2 * k], t8[2 * k + 1]);
  return t8[0];
}

// mean and denominator sqrt(var + eps) of the row in x (float32, N
// elements, balanced tree), as NumPy's mean and var compute them.  Uses
// part[0..16); contains two hsyncs.
__device__ __forceinline__ void ln_stats(const float* x, uint32_t N, float* part, float& mean, float& denom) {
  uint32_t nl, L;
  pw_balanced(N, nl, L);
  mean = div_count(ln_pairwise(x, nl, L, false, 0.f, part), N);
  const float var = div_count(ln_pairwise(x, nl, L, true, mean, part + 8), N);
  denom = __fsqrt_rn(__fadd_rn(var, 1e-5f));
}

// The LayerNorm output of 4 elements (x as floats, gamma and beta as FP16
// pairs in uint2), row_one's arithmetic.
__device__ __forceinline__ uint2 ln_out4(const float (&xs)[4], float mean, float denom, uint2 gv, uint2 bv) {
  const uint16_t* g16 = reinterpret_cast<const uint16_t*>(&gv);
  const uint16_t* b16 = reinterpret_cast<const uint16_t*>(&bv);
  uint16_t h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float y = __fdiv_rn(__fsub_rn(xs[j], mean), denom);
    h[j] = f2h(__fadd_rn(__fmul_rn(y, h2f(g16[j])), h2f(b16[j])));
  }
  return make_uint2(uint32_t(h[0]) | (uint32_t(h[1]) << 16), uint32_t(h[2]) | (uint32_t(h[3]) << 16));
}

// ---------------------------------------------------------------------------------
// Row attention: one query row of an attention pair, an FX_PV QK^T op and its
// P.V op, both narrowed to row 0 (a decode step).  The scores, the masked
// softmax and P.V run on CUDA cores with the wide path's arithmetic element
// for element: the QUANT rule on Q, K, P and V, exact int32 dot products
// (dp4a), the F_DQ dequantisation of scores and output, softmax_row_f16.
// Keys past the row's last visible one get P = 0 there and are skipped here.
// A task runs one pair, or the pairs of a head group (FX_ATTNGRP) of one
// sequence one after another.  The visible K and V rows arrive by bulk copy
// into shared memory; in a group the next pair's K rows are copied once this
// pair's scores are out and its V rows once this pair's P.V is done.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ bool attn_row_ok(const ExecArgs& A, const DevOp& x) {
  if (x.M != 1 || !(x.flags2 & FX_PV)) return false;
  const DevOp& y = A.ops[x.seg0];
  return attn_row_shape_ok(x.M, x.K, x.N, x.flags, x.flags2, y.M, y.K, y.N, y.flags);
}

// L2 prefetch of a task's hinted operand bytes.  L2 is the point of
// coherence, so a prefetch can never expose a stale value.
__device__ __forceinline__ void prefetch_task_operand(const ExecArgs& A, const Task& t) {
  if (!t.pf_units) return;
  const uint8_t* p = pptr(A, t.pf_phys, t.seq0);
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(t.pf_units * 16u) : "memory");
}

__device__ __forceinline__ void prefetch_l2_bytes(const void* p, uint32_t bytes) {
  if (bytes) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// The last key a query row sees: its row in the KV window (F_SMMASK),
// bounded by the window's valid length; every key when unmasked.
__device__ __forceinline__ int64_t attn_row_last(const ExecArgs& A, const DevOp& x, uint32_t seq) {
  uint32_t qrb = x.attn_qrb, vkl = x.attn_vkl;
  if (x.flags & F_ATTN_DYN) {
    const uint64_t pv = A.params[uint64_t(seq) * A.n_params + x.param];
    qrb = pv & 0xFFFF;
    vkl = (pv >> 16) & 0xFFFF;
  }
  if (!(x.flags & F_SMMASK)) return int64_t(x.N) - 1;
  return int64_t(qrb) < int64_t(vkl) - 1 ? int64_t(qrb) : int64_t(vkl) - 1;
}

// An attention pair resolved for one sequence: its operand addresses, scale
// registers and visible keys.  A task resolves each of its pairs once, into
// shared memory, so that loading a pair's rows waits on no chain of record
// reads.
struct __align__(16) AttnDesc {
  const uint8_t* k;     // K rows [N][Kd], FP16
  const uint8_t* v;     // V rows [N][Ny], FP16
  const uint16_t* sx;   // score scales [N]
  const uint16_t* sy;   // output scales [Ny]
  const uint8_t* q;     // the query row [Kd], FP16
  uint16_t* out;        // the output row [Ny], FP16
  int32_t lt;           // last visible key, within [-1, N - 1]
  uint32_t nvis;        // visible keys (lt + 1)
  uint16_t kd, n, ny, masked;
  uint16_t sqb, skb, svb, qsb;   // Q's, K's, V's and P's quantisation registers
};
static_assert(sizeof(AttnDesc) == 80, "AttnDesc is an 80-byte record");

__device__ __forceinline__ AttnDesc attn_desc(const ExecArgs& A, const DevOp& x, uint32_t seq) {
  const DevOp& y = A.ops[x.seg0];
  const int64_t lt = attn_row_last(A, x, seq);
  AttnDesc d;
  d.k = pptr(A, x.b, seq);
  d.v = pptr(A, y.b, seq);
  d.sx = reinterpret_cast<const uint16_t*>(pptr(A, x.c, seq));
  d.sy = reinterpret_cast<const uint16_t*>(pptr(A, y.c, seq));
  d.q = pptr(A, x.a, seq);
  d.out = reinterpret_cast<uint16_t*>(pptr(A, static_cast<uint64_t>(y.dconst), seq));
  // a last key at or past N - 1 sees every key, below 0 none: the same rows
  d.lt = lt < 0 ? -1 : int32_t(lt < int64_t(x.N) - 1 ? lt : int64_t(x.N) - 1);
  d.nvis = uint32_t(d.lt + 1);
  d.kd = static_cast<uint16_t>(x.K);
  d.n = static_cast<uint16_t>(x.N);
  d.ny = static_cast<uint16_t>(y.N);
  d.masked = (x.flags & F_SMMASK) != 0;
  d.sqb = sreg_bits(A, x.s[0], seq);
  d.skb = sreg_bits(A, x.s[1], seq);
  d.svb = sreg_bits(A, y.s[1], seq);
  d.qsb = sreg_bits(A, y.s[0], seq);
  return d;
}

// L2 prefetch of what task ti reads first: for a row-attention task its
// (first) pair's visible K and V rows, scales and query row, whose extent
// the static hint cannot know; for any other task its hint.  Resolving the
// pair also pulls its records, position word and registers into this SM's
// L1 for the task.
__device__ void prefetch_next_attn(const ExecArgs& A, uint32_t ti) {
  const Task tn = A.tasks[ti];
  const DevOp& x = A.ops[tn.op];
  if (!(x.kind == K_MATMUL && (x.flags & F_WIDE) && attn_row_ok(A, x))) {
    prefetch_task_operand(A, tn);
    return;
  }
  const AttnDesc d = attn_desc(A, x, tn.seq0);
  prefetch_l2_bytes(d.k, d.nvis * d.kd * 2u);
  prefetch_l2_bytes(d.v, d.nvis * d.ny * 2u);
  prefetch_l2_bytes(d.sx, d.n * 2u);
  prefetch_l2_bytes(d.sy, d.ny * 2u);
  prefetch_l2_bytes(d.q, d.kd * 2u);
}

// An op the dispatcher may run as row attention (attn_row_ok decides), judged
// from its own record.
__device__ __forceinline__ bool attn_row_candidate(const DevOp& x) {
  return x.kind == K_MATMUL && (x.flags & F_WIDE) && !(x.flags & F_TC) && (x.flags2 & FX_PV);
}

// One pair's per-thread operands: this thread's key's score scale, its word
// of Q (threads < K / 4) and its column's output scale (threads < N of P.V).
struct AttnLoads {
  uint2 qv;
  uint16_t sxb, syb;
};

__device__ __forceinline__ void attn_load(const AttnDesc& d, AttnLoads& L) {
  L.sxb = htid() < d.nvis ? d.sx[htid()] : uint16_t(0);
  L.syb = htid() < d.ny ? d.sy[htid()] : uint16_t(0);
  if (htid() < d.kd / 4u) L.qv = __ldcg(reinterpret_cast<const uint2*>(d.q) + htid());
}

// Thread 0: the first `rows` rows of K or V (rb bytes each) by one bulk copy
// into dst, completing a phase of bar (none for no rows).
__device__ __forceinline__ void attn_issue_rows(const uint8_t* src, uint32_t rows, uint32_t rb, void* dst,
                                                uint64_t* bar) {
  const uint32_t bytes = rows * rb;
  if (!bytes) return;
  sm100::fence_proxy_async();
  sm100::mbar_arrive_expect_tx(bar, bytes);
  sm100::bulk_g2s(dst, src, bytes, bar);
}

// Shared memory of row attention: Q words at 0, scores / exp values at 128,
// P at 4224, P.V partial sums at 5248, cross-warp reductions at 6272, warp
// 0's pairwise scratch from 6400, the task's resolved pairs at kAttnTabOff;
// from kAttnRowVOff the first visible K rows (as many as fit beside the
// window's V rows), then the visible V rows.
constexpr uint32_t kAttnTabOff = 7168;
static_assert(128 + 4096 + 1024 + kThreads * 4 + 128 + 3 * kPwMaxLeaves * 4 <= kAttnTabOff &&
                  kAttnTabOff + sizeof(AttnDesc) * kAttnGroupMax <= kAttnRowVOff,
              "row attention scratch overlaps its pair table or K rows");

// The int32 dot of a key row read from global memory (every word in flight)
// with the quantised Q words, the row quantised with sk (QUANT's rule): the
// keys row attention could not stage in shared memory, kept out of line.
__device__ __noinline__ int32_t attn_dot_global(const uint4* row, const int32_t* q8w, uint32_t nw, float sk) {
  uint4 kw[16];
#pragma unroll
  for (uint32_t g = 0; g < 16; ++g)
    if (g < nw) kw[g] = __ldcg(row + g);
  int32_t acc = 0;
#pragma unroll
  for (uint32_t g = 0; g < 16; ++g) {
    if (g >= nw) break;
    int8_t q[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) q[e] = sat8(__fmul_rn(h2f(h_at(kw[g], e)), sk));
    const uint2 pk = pack_b(q);
    acc = __dp4a(static_cast<int32_t>(pk.x), q8w[2 * g], acc);
    acc = __dp4a(static_cast<int32_t>(pk.y), q8w[2 * g + 1], acc);
  }
  return acc;
}

__device__ __noinline__ void op_attn_rows(const ExecArgs& A, const Task& t, uint32_t npairs, bool grouped,
                                          uint8_t* smem, TcShared* tc, uint32_t next_ti) {
  const uint32_t seq = t.seq0;
  const uint32_t warp = htid() >> 5, lane = htid() & 31;
  int32_t* q8w = reinterpret_cast<int32_t*>(smem);                 // Q quantised, 4 per word (K <= 128)
  float* rb = reinterpret_cast<float*>(smem + 128);                // scores, then exp values (N <= 1024)
  int8_t* p8 = reinterpret_cast<int8_t*>(smem + 128 + 4096);       // P quantised for P.V
  int32_t* part = reinterpret_cast<int32_t*>(smem + 128 + 4096 + 1024);   // P.V partial sums
  float* red = reinterpret_cast<float*>(smem + 128 + 4096 + 1024 + kThreads * 4);   // 16 floats
  uint32_t* pw = reinterpret_cast<uint32_t*>(red + 32);            // warp 0's pairwise scratch
  AttnDesc* tab = reinterpret_cast<AttnDesc*>(smem + kAttnTabOff);
  const DevOp& x0 = A.ops[t.op];
  // the first kr K rows at kAttnRowVOff (every pair of a group has the
  // head's shape), V rows after them; keys from kr on are read from global
  // memory.  `stage` brings K, `stage2` V, one phase a pair.
  const uint32_t vwin = x0.N * A.ops[x0.seg0].N * 2;
  const uint32_t kr = min(x0.N, (kWideMmSmem - kAttnRowVOff - vwin) / (x0.K * 2));
  uint16_t* ks = reinterpret_cast<uint16_t*>(smem + kAttnRowVOff);
  uint16_t* vs = reinterpret_cast<uint16_t*>(smem + kAttnRowVOff + kr * x0.K * 2);
  uint32_t kpar = tc->phase_stage, vpar = tc->phase_stage2;   // read before thread 0 stores the final ones
  // the task's pairs resolved once, lane h of the last warp for pair h (a
  // group's first pair is its head op); every thread also resolves the first
  // pair for itself: thread 0 starts its copies, every thread its loads
  if (warp == kWarps - 1 && lane < npairs) {
    const uint32_t xi = lane == 0 ? t.op : A.tasks[t.tile + lane].op;
    const DevOp& xh = A.ops[xi];
    const bool ok = lane == 0 || (attn_row_ok(A, xh) && xh.K == x0.K && xh.N == x0.N &&
                                  A.ops[xh.seg0].N == A.ops[x0.seg0].N);
    AttnDesc d = attn_desc(A, xh, seq);
    if (!ok) {
      raise_fault(A, DF_BAD_OP, xi, seq);
      d.lt = -1;
      d.nvis = 0;
    }
    tab[lane] = d;
  }
  AttnLoads L;
  {
    const AttnDesc d0 = attn_desc(A, x0, seq);
    if (htid() == 0) {
      attn_issue_rows(d0.k, min(d0.nvis, kr), d0.kd * 2u, ks, &tc->stage);
      attn_issue_rows(d0.v, d0.nvis, d0.ny * 2u, vs, &tc->stage2);
    }
    attn_load(d0, L);
  }
  if (warp == kWarps - 2 && lane == 31 && next_ti != 0xFFFFFFFFu) prefetch_next_attn(A, next_ti);
  hsync();
  for (uint32_t h = 0; h < npairs; ++h) {
    const AttnDesc& D = tab[h];
    const uint32_t Kd = D.kd, N = D.n, Ny = D.ny, nvis = D.nvis;
    const bool masked = D.masked != 0;
    const int64_t lt = D.lt;
    // 1. Q quantised with its register (QUANT's rule), four values a word
    if (htid() < Kd / 4) {
      const float sq = h2f(D.sqb);
      uint32_t w = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint16_t hv = static_cast<uint16_t>((j < 2 ? L.qv.x : L.qv.y) >> (16 * (j & 1)));
        w |= uint32_t(uint8_t(sat8(__fmul_rn(h2f(hv), sq)))) << (8 * j);
      }
      q8w[htid()] = static_cast<int32_t>(w);
    }
    hsync();
    if (min(nvis, kr)) {
      if (!sm100::mbar_wait(&tc->stage, kpar, nullptr, 0)) {
        // bounded: let the K and V copies land, then fault
        sm100::mbar_wait(&tc->stage, kpar, nullptr, 0);
        sm100::mbar_wait(&tc->stage2, vpar, nullptr, 0);
        if (htid() == 0) raise_fault(A, DF_STAGE_TIMEOUT, t.op, seq);
        return;
      }
      kpar ^= 1u;
    }
    // 2. scores: each key row quantised (QUANT's rule) and dotted with Q, the
    //    int32 dot dequantised to FP16 (F_DQ).  A row in shared memory is
    //    read from its word (j mod K/8) on, so the rows of a quarter warp
    //    fall in different banks; the int32 sum is exact in any order.
    const float sk = h2f(D.skb);
    const uint32_t nw = Kd / 8;
    auto dot_word = [&](const uint4& w, uint32_t g, int32_t acc) {
      int8_t q[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) q[e] = sat8(__fmul_rn(h2f(h_at(w, e)), sk));
      const uint2 pk = pack_b(q);
      acc = __dp4a(static_cast<int32_t>(pk.x), q8w[2 * g], acc);
      return __dp4a(static_cast<int32_t>(pk.y), q8w[2 * g + 1], acc);
    };
    auto score = [&](uint32_t j, uint16_t scb) {
      int32_t acc = 0;
      if (j < kr) {
        const uint4* row = reinterpret_cast<const uint4*>(ks + j * Kd);
        uint32_t g = j % nw;
        for (uint32_t i = 0; i < nw; ++i) {
          acc = dot_word(row[g], g, acc);
          g = g + 1 == nw ? 0u : g + 1;
        }
      } else {   // past the staged rows: the row from global memory
        acc = attn_dot_global(reinterpret_cast<const uint4*>(D.k + uint64_t(j) * Kd * 2), q8w, nw, sk);
      }
      return h2f(f2h(__fmul_rn(__int2float_rn(acc), h2f(scb))));
    };
    const uint32_t j0 = htid();
    if (j0 < nvis) rb[j0] = score(j0, L.sxb);
    for (uint32_t j = j0 + kThreads; j < nvis; j += kThreads) rb[j] = score(j, D.sx[j]);   // keys past kThreads
    const uint16_t syb = L.syb;
    if (h + 1 < npairs) attn_load(tab[h + 1], L);   // the next pair's small operands
    hsync();
    // the K rows are read: the next pair's land there
    if (h + 1 < npairs && htid() == 0)
      attn_issue_rows(tab[h + 1].k, min(tab[h + 1].nvis, kr), Kd * 2u, ks, &tc->stage);
    // 3. the masked softmax row, softmax_row_f16's arithmetic: max over the
    //    visible columns, exp in float64 rounded once, NumPy's pairwise sum,
    //    f16(e / sum) quantised with the P.V op's register
    const float qs = h2f(D.qsb);
    uint32_t nl = 0, Lv = 0;
    if (!pw_balanced(N, nl, Lv) || nvis == 0) {
      if (warp == 0) softmax_row_f16(rb, N, masked, masked ? lt : int64_t(N) - 1, nullptr, pw, lane, p8, qs);
    } else {
      float mx = -INFINITY;
      for (uint32_t j = htid(); j < nvis; j += kThreads) mx = fmaxf(mx, rb[j]);
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) red[warp] = mx;
      hsync();
#pragma unroll
      for (int w = 0; w < kWarps; ++w) mx = fmaxf(mx, red[w]);
      for (uint32_t j = htid(); j < N; j += kThreads) rb[j] = j < nvis ? exp_f32(__fsub_rn(rb[j], mx)) : 0.f;
      hsync();
      const float denom = ln_pairwise(rb, nl, Lv, false, 0.f, red + 8);
      for (uint32_t j = htid(); j < N; j += kThreads) {
        int8_t q8 = 0;
        if (j < nvis) {
          const float e = rb[j];
          const uint16_t hq = f2h(!masked ? __fdiv_rn(e, denom) : (denom > 0.f ? __fdiv_rn(e, denom) : 0.f));
          q8 = sat8(__fmul_rn(h2f(hq), qs));
        }
        p8[j] = q8;
      }
    }
    hsync();
    // 4. P.V: column n, four keys per dp4a (P's bytes of keys j..j+3, zero
    //    past the visible ones, against V's quantised column entries; rows
    //    past the copy hold whatever is there and meet P = 0, a NaN
    //    quantises to 0)
    const uint32_t nq = kThreads / Ny, n = htid() % Ny, kq = htid() / Ny;
    if (nvis) {
      if (!sm100::mbar_wait(&tc->stage2, vpar, nullptr, 0)) {
        sm100::mbar_wait(&tc->stage2, vpar, nullptr, 0);   // bounded: let the copies land, then fault
        if (h + 1 < npairs && min(tab[h + 1].nvis, kr)) sm100::mbar_wait(&tc->stage, kpar, nullptr, 0);
        if (htid() == 0) raise_fault(A, DF_STAGE_TIMEOUT, t.op, seq);
        return;
      }
      vpar ^= 1u;
    }
    const float sv = h2f(D.svb);
    int32_t acc = 0;
    if (kq < nq) {
      const uint32_t nv4 = (nvis + 3) & ~3u;
#pragma unroll 2
      for (uint32_t j = 4 * kq; j < nv4; j += 4 * nq) {
        const int32_t pw4 = *reinterpret_cast<const int32_t*>(p8 + j);
        uint32_t vw = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          vw |= uint32_t(uint8_t(sat8(__fmul_rn(h2f(vs[(j + e) * Ny + n]), sv)))) << (8 * e);
        acc = __dp4a(pw4, static_cast<int32_t>(vw), acc);
      }
    }
    part[htid()] = acc;
    hsync();
    if (htid() < Ny) {
      int32_t sum = 0;
      for (uint32_t k = 0; k < nq; ++k) sum += part[k * Ny + htid()];   // int32 sums are exact in any order
      D.out[htid()] = f2h(__fmul_rn(__int2float_rn(sum), h2f(syb)));
    }
    // the V rows are read: the next pair's land there
    if (h + 1 < npairs && htid() == 0) attn_issue_rows(tab[h + 1].v, tab[h + 1].nvis, Ny * 2u, vs, &tc->stage2);
  }
  if (htid() == 0) {
    tc->phase_stage = kpar;
    tc->phase_stage2 = vpar;
  }
}

// ---------------------------------------------------------------------------------
// MATMUL with shared weights on the 5th-generation tensor cores (ops flagged
// F_TC).  A task is up to 128 rows (the M rows of up to 128/M sequences) x 64
// columns.  Per 128-byte K block, TMA brings A as one [128/M sequences][M
// rows][128 B] box (128-byte swizzle, K-major) and the weights as a [128 K
// rows][64 B] box (64-byte swizzle, MN-major) into one of three
// shared-memory stages; thread 0 issues tcgen05.mma.kind::i8 (M 128, N 64,
// K 32) into this CTA's 64 TMEM columns and recycles a stage once the MMAs
// that read it have committed.  The eight warps read the int32 accumulator
// back with tcgen05.ld.  Waits are bounded (DF_MMA_TIMEOUT).
// ---------------------------------------------------------------------------------
constexpr uint32_t kTcAStage = 128 * 128;
constexpr uint32_t kTcBStage = 128 * 64;                // 64 columns x 128 K rows
constexpr uint32_t kTcStage = kTcAStage + kTcBStage;    // a multiple of 1024
constexpr uint32_t kTcStage128 = kTcAStage + 128 * 128; // 128-column stage
constexpr uint32_t kTcCols = 128;                       // TMEM columns per half
constexpr uint32_t kTcIdesc = sm100::idesc_i8(128, 64, 1);
constexpr uint32_t kTcIdesc128 = sm100::idesc_i8(128, 128, 1);



// shared-memory descriptor, 64-byte swizzle (layout type 4)
__device__ __forceinline__ uint64_t desc_sw64(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr >> 4) & 0x3FFF) | (uint64_t((lbo >> 4) & 0x3FFF) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFF) << 32) | (uint64_t(1) << 46) | (uint64_t(4) << 61);
}

// One warp's slice of the tcgen05 MATMUL epilogue: TMEM lanes 32q..32q+31,
// columns 32h..32h+31 of the task's tile, to int32 rows (plus the previous
// int32 tile when F_ACCUMULATE).
// Shared memory the tcgen05 task's epilogue reads, past its operand stages:
// the DEQUANT_SCALED scale and bias of the tile's columns (FP16, 128 each)
// and the activation-scale register of each of the 128 rows.
constexpr uint32_t kTcEpiBytes = 768;

__device__ __forceinline__ void tc_epilogue_slice(const ExecArgs& A, const DevOp& op, const Task& t, TcShared* tc,
                                                  uint32_t q, uint32_t lane, uint32_t h, uint32_t n0,
                                                  uint32_t ncols, uint32_t rows, const uint8_t* epi) {
  const uint32_t M = op.M, N = op.N;
  uint32_t v[32];
  __syncwarp();
  sm100::tmem_ld32(tc->tmem + ((q * 32) << 16) + h * 32, v);
  const uint32_t r = q * 32 + lane;
  if (r < rows && h * 32 < ncols) {
    const uint32_t seq = t.seq0 + r / M, row = r % M;
    const uint32_t col0 = n0 + h * 32;
    const uint32_t nc = ncols - h * 32 < 32 ? ncols - h * 32 : 32;
    int32_t* D = reinterpret_cast<int32_t*>(pptr(A, op.d, seq)) + uint64_t(row) * N + col0;
    if (op.flags2 & FX_DQS) {
      // DEQUANT_ACCUM_FP32_SCALED: f16((f32(acc) * scale[col]) * s0 + bias[col]); the rows are the same
      // for every lane of the warp
      // scale, bias and this row's activation scale staged in shared memory
      // (epi) when the vectors are shared, else read for the row's sequence
      const bool staged = epi != nullptr;
      const float s0 = h2f(staged ? reinterpret_cast<const uint16_t*>(epi + 512)[r] : sreg_bits(A, op.s[0], seq));
      const uint16_t* sc = staged ? reinterpret_cast<const uint16_t*>(epi) + h * 32
                                  : reinterpret_cast<const uint16_t*>(pptr(A, op.c, seq)) + col0;
      const uint16_t* bi = staged ? reinterpret_cast<const uint16_t*>(epi + 256) + h * 32
                                  : reinterpret_cast<const uint16_t*>(pptr(A, op.nbytes, seq)) + col0;
      uint16_t* O = reinterpret_cast<uint16_t*>(pptr(A, static_cast<uint64_t>(op.dconst), seq)) +
                    uint64_t(row) * N + col0;
      // FX_DSTORE: the absorbed store of the first attn_vkl rows to the runtime address
      uint16_t* Ost = nullptr;
      if ((op.flags2 & FX_DSTORE) && row < op.attn_vkl) {
        const uint64_t addr = A.params[uint64_t(seq) * A.n_params + op.param] + op.attn_qrb +
                              (uint64_t(row) * N + col0) * 2;
        if ((addr & 15) || addr + nc * 2 > A.dram_bytes || addr < A.shared_bytes) raise_fault(A, DF_DYN_ADDRESS, t.op, seq);
        else Ost = reinterpret_cast<uint16_t*>(dram_ptr(A, addr, seq));
      }
#pragma unroll
      for (uint32_t j = 0; j < 32; j += 8) {
        if (j < nc) {
          const uint4 s8 = staged ? *reinterpret_cast<const uint4*>(sc + j) : __ldcg(reinterpret_cast<const uint4*>(sc + j));
          const uint4 b8 = staged ? *reinterpret_cast<const uint4*>(bi + j) : __ldcg(reinterpret_cast<const uint4*>(bi + j));
          uint16_t hh[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            float x = __fmul_rn(__int2float_rn(int(v[j + k])), h2f(h_at(s8, k)));
            x = __fmul_rn(x, s0);
            hh[k] = f2h(__fadd_rn(x, h2f(h_at(b8, k))));
          }
          *reinterpret_cast<uint4*>(O + j) = pack_h(hh);
          if (Ost) *reinterpret_cast<uint4*>(Ost + j) = pack_h(hh);
        }
      }
      if (op.flags & F_NOI32) return;
    }
    const int32_t* C = (op.flags & F_ACCUMULATE)
                           ? reinterpret_cast<const int32_t*>(pptr(A, op.c, seq)) + uint64_t(row) * N + col0
                           : nullptr;
#pragma unroll
    for (uint32_t j = 0; j < 32; j += 4) {
      if (j < nc) {
        int4 val = make_int4(int(v[j]), int(v[j + 1]), int(v[j + 2]), int(v[j + 3]));
        if (C) {
          const int4 cv = __ldcg(reinterpret_cast<const int4*>(C + j));
          val.x = int32_t(uint32_t(val.x) + uint32_t(cv.x));
          val.y = int32_t(uint32_t(val.y) + uint32_t(cv.y));
          val.z = int32_t(uint32_t(val.z) + uint32_t(cv.z));
          val.w = int32_t(uint32_t(val.w) + uint32_t(cv.w));
        }
        *reinterpret_cast<int4*>(D + j) = val;
      }
    }
  }
}

// The FX_DQS + F_NOI32 slice with its vectors staged and all 32 columns
// valid: each lane computes its row's 32 FP16 results into the warp's own
// 2.5 KB of shared memory (scr), and after a warp barrier each store
// instruction writes 8 rows' 64 bytes (4 lanes a row) instead of 32 rows'
// 16 bytes, the rows being different sequences.
__device__ __forceinline__ void tc_epilogue_slice_t(const ExecArgs& A, const DevOp& op, const Task& t, TcShared* tc,
                                                    uint32_t q, uint32_t lane, uint32_t h, uint32_t n0,
                                                    uint32_t rows, const uint8_t* epi, uint8_t* scr) {
  const uint32_t M = op.M, N = op.N;
  uint32_t v[32];
  __syncwarp();
  sm100::tmem_ld32(tc->tmem + ((q * 32) << 16) + h * 32, v);
  const uint32_t r = q * 32 + lane, col0 = n0 + h * 32;
  uint64_t ost = 0;   // this row's absorbed store address (FX_DSTORE), else 0
  if (r < rows) {
    const uint32_t seq = t.seq0 + r / M, row = r % M;
    const float s0 = h2f(reinterpret_cast<const uint16_t*>(epi + 512)[r]);
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(epi) + h * 32;
    const uint16_t* bi = reinterpret_cast<const uint16_t*>(epi + 256) + h * 32;
    if ((op.flags2 & FX_DSTORE) && row < op.attn_vkl) {
      const uint64_t addr = A.params[uint64_t(seq) * A.n_params + op.param] + op.attn_qrb +
                            (uint64_t(row) * N + col0) * 2;
      if ((addr & 15) || addr + 64 > A.dram_bytes || addr < A.shared_bytes) raise_fault(A, DF_DYN_ADDRESS, t.op, seq);
      else ost = reinterpret_cast<uint64_t>(dram_ptr(A, addr, seq));
    }
#pragma unroll
    for (uint32_t j = 0; j < 32; j += 8) {
      const uint4 s8 = *reinterpret_cast<const uint4*>(sc + j);
      const uint4 b8 = *reinterpret_cast<const uint4*>(bi + j);
      uint16_t hh[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float x = __fmul_rn(__int2float_rn(int(v[j + k])), h2f(h_at(s8, k)));
        x = __fmul_rn(x, s0);
        hh[k] = f2h(__fadd_rn(x, h2f(h_at(b8, k))));
      }
      *reinterpret_cast<uint4*>(scr + lane * 80 + j * 2) = pack_h(hh);
    }
  }
  __syncwarp();
#pragma unroll
  for (uint32_t i = 0; i < 4; ++i) {
    const uint32_t rr = 8 * i + (lane >> 2), c = lane & 3, rg = q * 32 + rr;   // the row and 16-byte word
    const uint64_t o2 = __shfl_sync(0xffffffffu, ost, rr);
    if (rg < rows) {
      const uint4 w = *reinterpret_cast<const uint4*>(scr + rr * 80 + c * 16);
      const uint32_t seq = t.seq0 + rg / M, row = rg % M;
      uint16_t* O = reinterpret_cast<uint16_t*>(pptr(A, static_cast<uint64_t>(op.dconst), seq)) + uint64_t(row) * N + col0;
      *reinterpret_cast<uint4*>(O + c * 8) = w;
      if (o2) *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(o2) + c * 8) = w;
    }
  }
  __syncwarp();   // the scratch is free for the warp's next slice
}

// The weight tiles a tcgen05 MATMUL task streams (its B column slice over
// every K chunk), pulled into L2 by TMA prefetches, and its tensor maps into
// the descriptor cache; other tasks need nothing here.
__device__ __forceinline__ void prefetch_task_weights(const ExecArgs& A, const Task& t) {
  const DevOp& op = A.ops[t.op];
  if (op.kind != K_MATMUL || !(op.flags & F_TC)) return;
  const CUtensorMap* ma = A.tmaps + 2 * op.seg0;
  sm100::prefetch_tmap(ma);
  sm100::prefetch_tmap(ma + 1);
  const uint32_t tn = (op.flags & F_TC128) ? 128u : 64u;
  for (uint32_t c = 0; c * 128 < op.K; ++c) sm100::tma_prefetch_2d(ma + 1, int32_t(t.tile * tn), int32_t(c * 128));
}

__device__ __noinline__ void op_matmul_tc(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem,
                                          TcShared* tc, uint32_t opi, uint32_t next_ti) {
  const uint32_t M = op.M, N = op.N, K = op.K;
  // tile width: 128 columns (B box 128 x 128, 128-byte swizzle, two 32 KB
  // stages) or 64 (B box 64 x 128, 64-byte swizzle, three 24 KB stages)
  const bool w128 = (op.flags & F_TC128) != 0;
  const uint32_t tn = w128 ? 128u : 64u;
  const uint32_t nst = w128 ? 2u : uint32_t(kTcStages);
  const uint32_t stage_bytes = w128 ? kTcStage128 : kTcStage;
  const uint32_t n0 = t.tile * tn;
  const uint32_t ncols = N - n0 < tn ? N - n0 : tn;
  const uint32_t rows = t.nseq * M;                       // <= 128
  const uint32_t nchunks = (K + 127) / 128;
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem) + 1023) & ~uintptr_t(1023));
  const CUtensorMap* ma = A.tmaps + 2 * op.seg0;
  const CUtensorMap* mb = ma + 1;
  // Chunk c uses stage c % nst for the (c / nst)-th time in this task: its
  // full and empty barriers complete the phase of that parity relative to
  // the task's start, whichever thread waits.  Each stage advances by one
  // phase per chunk that uses it.
  const uint32_t warp = htid() >> 5, lane = htid() & 31, q = warp & 3;
  // The DEQUANT_SCALED scale and bias of the tile's columns (when shared by
  // every sequence) and each row's activation scale go to shared memory from
  // warps 3 and 4, idle while the K loop runs.
  uint8_t* epi = (op.flags2 & FX_DQS) && (op.c & kSharedBit) && (op.nbytes & kSharedBit)
                     ? base + kTcStageRegion : nullptr;
  if (epi && warp == 3) {
    const uint32_t nv = (ncols + 7) / 8;   // 16-byte vectors of each row
    for (uint32_t i = lane; i < 2 * nv; i += 32) {
      const uint8_t* src = i < nv ? pptr(A, op.c, t.seq0) + (uint64_t(n0) + i * 8) * 2
                                  : pptr(A, op.nbytes, t.seq0) + (uint64_t(n0) + (i - nv) * 8) * 2;
      *reinterpret_cast<uint4*>(epi + (i < nv ? i * 16 : 256 + (i - nv) * 16)) = __ldcg(reinterpret_cast<const uint4*>(src));
    }
  } else if (epi && warp == 4) {
    for (uint32_t r = lane; r < rows; r += 32)
      reinterpret_cast<uint16_t*>(epi + 512)[r] = sreg_bits(A, op.s[0], t.seq0 + r / M);
  }
  const uint32_t pf0 = tc->phase_full, pe0 = tc->phase_empty;
  auto parity = [&](uint32_t ph0, uint32_t c) { return ((ph0 >> (c % nst)) ^ (c / nst)) & 1u; };
  uint32_t flip = 0;
  for (uint32_t st = 0; st < nst; ++st)
    if (((nchunks + nst - 1 - st) / nst) & 1u) flip |= 1u << st;
  const bool res = (op.flags2 & FX_TCRES) != 0;
  if (res) {
    // every K chunk resident at once: A boxes of q_rows rows back to back,
    // then the B boxes; chunks [0, h) complete on full[0], the rest on
    // full[1], so the first MMAs overlap the second half's transfer; one
    // commit on empty[0] when all MMAs are done
    const uint32_t abytes = op.q_rows * 128, h = (nchunks + 1) / 2;
    uint8_t* bbase = base + nchunks * abytes;
    if (htid() == 32) {
      sm100::fence_proxy_async();   // A was written by generic stores in earlier levels
      sm100::mbar_arrive_expect_tx(&tc->full[0], h * (abytes + 8192));
      if (nchunks > h) sm100::mbar_arrive_expect_tx(&tc->full[1], (nchunks - h) * (abytes + 8192));
      for (uint32_t c = 0; c < nchunks; ++c) {
        uint64_t* bar = &tc->full[c < h ? 0 : 1];
        sm100::tma_load_3d(base + c * abytes, ma, int32_t(c * 128), 0, int32_t(t.seq0), bar);
        sm100::tma_load_2d(bbase + c * 8192, mb, int32_t(n0), int32_t(c * 128), bar);
      }
    } else if (htid() == 0) {
      bool ok = true;
      for (uint32_t c = 0; c < nchunks; ++c) {
        if ((c == 0 || c == h) && !sm100::mbar_wait(&tc->full[c < h ? 0 : 1], (pf0 >> (c < h ? 0 : 1)) & 1u, nullptr, 0))
          ok = false;
        sm100::tc_fence_after();
        const uint32_t a_addr = sm100::smem_u32(base + c * abytes), b_addr = sm100::smem_u32(bbase + c * 8192);
        const uint32_t kc = K - c * 128 < 128 ? K - c * 128 : 128;
        for (uint32_t ks = 0; ks * 32 < kc; ++ks)
          sm100::mma_i8(tc->tmem, sm100::smem_desc_sw128(a_addr + ks * 32, 16, 1024), desc_sw64(b_addr + ks * 2048, 16, 512),
                        kTcIdesc, (c | ks) != 0);
      }
      sm100::mma_commit(&tc->empty[0]);
      if (!sm100::mbar_wait(&tc->empty[0], pe0 & 1u, nullptr, 0)) ok = false;
      if (!ok) raise_fault(A, DF_MMA_TIMEOUT, opi, t.seq0);
    } else if (htid() == 64 && next_ti != 0xFFFFFFFFu) {
      prefetch_task_weights(A, A.tasks[next_ti]);
    }
  } else if (htid() == 32) {
    // producer (warp 1): TMA loads; a stage is refilled once the MMAs of the
    // chunk before it in that stage have completed
    const uint32_t bytes = (op.q_rows ? op.q_rows : (128 / M) * M) * 128 + tn * 128;   // the A box's rows
    bool ok = true;
    sm100::fence_proxy_async();   // A was written by generic stores in earlier levels
    for (uint32_t c = 0; c < nchunks; ++c) {
      const uint32_t st = c % nst;
      if (c >= nst && !sm100::mbar_wait(&tc->empty[st], parity(pe0, c - nst), nullptr, 0)) ok = false;
      uint8_t* as = base + st * stage_bytes;
      sm100::mbar_arrive_expect_tx(&tc->full[st], bytes);
      sm100::tma_load_3d(as, ma, int32_t(c * 128), 0, int32_t(t.seq0), &tc->full[st]);
      sm100::tma_load_2d(as + kTcAStage, mb, int32_t(n0), int32_t(c * 128), &tc->full[st]);
    }
    if (!ok) raise_fault(A, DF_MMA_TIMEOUT, opi, t.seq0);
  } else if (htid() == 0) {
    // MMA issuer (warp 0)
    bool ok = true;
    for (uint32_t c = 0; c < nchunks; ++c) {
      const uint32_t st = c % nst;
      if (!sm100::mbar_wait(&tc->full[st], parity(pf0, c), nullptr, 0)) ok = false;
      sm100::tc_fence_after();
      const uint32_t a_addr = sm100::smem_u32(base + st * stage_bytes), b_addr = a_addr + kTcAStage;
      const uint32_t kc = K - c * 128 < 128 ? K - c * 128 : 128;
      for (uint32_t ks = 0; ks * 32 < kc; ++ks) {
        // B: MN-major rows (one per K) of 64 or 128 bytes, 8-K groups of 512 or 1024 B;
        // a step of 32 K rows is 2 or 4 KB
        const uint64_t db = w128 ? sm100::smem_desc_sw128(b_addr + ks * 4096, 16384, 1024)
                                 : desc_sw64(b_addr + ks * 2048, 16, 512);
        sm100::mma_i8(tc->tmem, sm100::smem_desc_sw128(a_addr + ks * 32, 16, 1024), db,
                      w128 ? kTcIdesc128 : kTcIdesc, (c | ks) != 0);
      }
      sm100::mma_commit(&tc->empty[st]);
    }
    // the commits the producer does not wait for: every MMA of the task is done after these
    for (uint32_t c = nchunks > nst ? nchunks - nst : 0; c < nchunks; ++c)
      if (!sm100::mbar_wait(&tc->empty[c % nst], parity(pe0, c), nullptr, 0)) ok = false;
    if (!ok) raise_fault(A, DF_MMA_TIMEOUT, opi, t.seq0);
  } else if (htid() == 64 && next_ti != 0xFFFFFFFFu && !res) {
    prefetch_task_weights(A, A.tasks[next_ti]);   // warp 2 is idle during the K loop
  }
  hsync();
  sm100::tc_fence_after();
  if (htid() == 0) {   // every thread has read the parities at the start (before the hsync above)
    tc->phase_full = pf0 ^ (res ? (nchunks > (nchunks + 1) / 2 ? 3u : 1u) : flip);
    tc->phase_empty = pe0 ^ (res ? 1u : flip);
  }
  // epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31; with 64 columns it
  // takes columns 32 (w / 4) .. +31, with 128 columns two such slices
  // (with the DEQUANT_SCALED vectors staged and no int32 result, through the
  // warp's own scratch in the stage region, free once the MMAs are done)
  for (uint32_t hh = warp >> 2; hh * 32 < tn; hh += 2) {
    if (epi && (op.flags & F_NOI32) && hh * 32 + 32 <= ncols)
      tc_epilogue_slice_t(A, op, t, tc, q, lane, hh, n0, rows, epi, base + warp * 2560);
    else
      tc_epilogue_slice(A, op, t, tc, q, lane, hh, n0, ncols, rows, epi);
  }
  // the next tcgen05 MATMUL overwrites the accumulator only after every warp read it
  sm100::tc_fence_before();
  hsync();
}


// ---------------------------------------------------------------------------------
// Element-wise ops.  A task covers kEwTask elements of one sequence; each
// thread owns groups of 8 consecutive elements (8 never straddle a row: N is
// a multiple of 16) and issues every load of its groups before computing, so
// the memory latency is paid once per task rather than once per element.
// ---------------------------------------------------------------------------------
constexpr uint32_t kEwGroups = 4;                       // groups of 8 per thread
constexpr uint32_t kEwTask = kThreads * kEwGroups * 8;   // 8192 elements per task
static_assert(kEwTask == kEwTaskElems, "host and device element-wise task sizes differ");



// A task covers kEwTask elements of one sequence (t.nseq == 1, chunk t.tile)
// or, for small ops, t.nseq whole sequences (t.nseq * M * N <= kEwTask) whose
// elements are numbered consecutively.  Operands of sequence seq0 + k sit
// k * seq_stride bytes after those of seq0 (0 for the shared region).
template <int KIND>
__device__ __noinline__ void ew_kernel(const ExecArgs& A, const DevOp& op, const Task& t) {
  const uint32_t N = op.N;
  const uint32_t MN = op.M * N;
  constexpr uint32_t kTask = ew_task_elems(KIND);
  // a task larger than kEwTask runs as consecutive chunks of kEwTask elements
  constexpr uint32_t kChunk = kTask < kEwTask ? kTask : kEwTask;
  constexpr uint32_t kGroups = kChunk / (kThreads * 8);   // groups of 8 per thread
  static_assert(kGroups >= 1 && kGroups <= kEwGroups && kTask % kChunk == 0, "element-wise task size");
  const bool packed = t.nseq > 1;
  const uint32_t task_base = packed ? 0u : t.tile * kTask;
  const uint32_t span = packed ? t.nseq * MN : MN;
  const uint8_t* __restrict__ a0 = pptr(A, op.a, t.seq0);
  const uint8_t* __restrict__ b0 = pptr(A, op.b, t.seq0);
  uint8_t* __restrict__ d0 = pptr(A, op.d, t.seq0);
  const uint64_t sa = (op.a & kSharedBit) ? 0 : A.seq_stride;
  const uint64_t sb = (op.b & kSharedBit) ? 0 : A.seq_stride;
  const uint64_t sd = (op.d & kSharedBit) ? 0 : A.seq_stride;
  for (uint32_t base = task_base; base < task_base + kTask && base < span; base += kChunk) {
    // phase 1: loads
    uint4 ra[kEwGroups], rb[kEwGroups], rc[kEwGroups];
    V8 ia[kEwGroups];
    uint2 qa[kEwGroups], qb[kEwGroups];
    uint32_t e0[kEwGroups], sq[kEwGroups];
    // raw FP16 register bits: converted only in phase 2, so no load of phase 1
    // waits for another
    uint16_t s0b[kEwGroups], s1b[kEwGroups];
  #pragma unroll
    for (uint32_t g = 0; g < kGroups; ++g) {
      const uint32_t e = base + (g * kThreads + htid()) * 8;
      sq[g] = packed ? e / MN : 0u;
      e0[g] = e - sq[g] * MN;
      if (e >= span || e0[g] >= MN) {
        e0[g] = MN;   // marks the group empty
        continue;
      }
      const uint32_t seq = t.seq0 + sq[g];
      s0b[g] = sreg_bits(A, op.s[0], seq);
      s1b[g] = sreg_bits(A, op.s[1], seq);
      const uint8_t* __restrict__ a = a0 + sq[g] * sa;
      const uint8_t* __restrict__ b = b0 + sq[g] * sb;
      const uint32_t col = e0[g] % N;
      if constexpr (KIND == K_QUANT || KIND == K_GELU_F16) {
        ra[g] = ld16(a + e0[g] * 2);
      } else if constexpr (KIND == K_VADD_F16) {
        ra[g] = ld16(a + e0[g] * 2);
        rb[g] = ld16(b + e0[g] * 2);
      } else if constexpr (KIND == K_DEQUANT_SCALED) {
        ia[g] = ld32(a + e0[g] * 4);
        rb[g] = ld16(b + uint64_t(col) * 2);
        rc[g] = (op.flags & F_SPLIT) ? ld16(pptr(A, op.c, seq) + uint64_t(col) * 2) : ld16(b + uint64_t(N + col) * 2);
      } else if constexpr (KIND == K_DEQUANT_ACCUM || KIND == K_REQUANT_PC) {
        ia[g] = ld32(a + e0[g] * 4);
        rb[g] = ld16(b + uint64_t(col) * 2);
      } else if constexpr (KIND == K_REQUANT || KIND == K_SCALE_MUL_I32) {
        ia[g] = ld32(a + e0[g] * 4);
      } else if constexpr (KIND == K_VADD_I32) {
        ia[g] = ld32(a + e0[g] * 4);
        const uint4* q = reinterpret_cast<const uint4*>(b + uint64_t(col) * 4);
        rb[g] = __ldcg(q);
        rc[g] = __ldcg(q + 1);
      } else if constexpr (KIND == K_SCALE_MUL_I8) {
        qa[g] = ld8(a + e0[g]);
      } else if constexpr (KIND == K_VADD_I8) {
        qa[g] = ld8(a + e0[g]);
        qb[g] = ld8(b + e0[g]);
      } else if constexpr (KIND == K_DEQUANT_ADD) {
        ia[g] = ld32(a + e0[g] * 4);
        qb[g] = ld8(b + e0[g]);
      } else if constexpr (KIND == K_GELU_I8) {
        if (op.flags & F_SRC_I32) ia[g] = ld32(a + e0[g] * 4);
        else qa[g] = ld8(a + e0[g]);
      }
    }
    // phase 2: compute and store
  #pragma unroll
    for (uint32_t g = 0; g < kGroups; ++g) {
      if (e0[g] >= MN) continue;
      uint8_t* __restrict__ d = d0 + sq[g] * sd;
      const float s0 = h2f(s0b[g]), s1 = h2f(s1b[g]);
      if constexpr (KIND == K_QUANT) {
        int8_t q[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) {
          q[j] = sat8(__fmul_rn(h2f(h_at(ra[g], j)), s0));
        }
        *reinterpret_cast<uint2*>(d + e0[g]) = pack_b(q);
      } else if constexpr (KIND == K_GELU_F16) {
        uint16_t h[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = f2h(gelu_f32(h2f(h_at(ra[g], j))));
        *reinterpret_cast<uint4*>(d + e0[g] * 2) = pack_h(h);
      } else if constexpr (KIND == K_VADD_F16) {
        uint16_t h[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = f2h(__fadd_rn(h2f(h_at(ra[g], j)), h2f(h_at(rb[g], j))));
        *reinterpret_cast<uint4*>(d + e0[g] * 2) = pack_h(h);
      } else if constexpr (KIND == K_DEQUANT_SCALED) {
        uint16_t h[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) {
          float v = __fmul_rn(__int2float_rn(i_at(ia[g], j)), h2f(h_at(rb[g], j)));
          v = __fmul_rn(v, s0);
          h[j] = f2h(__fadd_rn(v, h2f(h_at(rc[g], j))));
        }
        *reinterpret_cast<uint4*>(d + e0[g] * 2) = pack_h(h);
      } else if constexpr (KIND == K_DEQUANT_ACCUM) {
        uint16_t h[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = f2h(__fmul_rn(__int2float_rn(i_at(ia[g], j)), h2f(h_at(rb[g], j))));
        *reinterpret_cast<uint4*>(d + e0[g] * 2) = pack_h(h);
      } else if constexpr (KIND == K_REQUANT_PC) {
        int8_t q[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = sat8(__fmul_rn(__int2float_rn(i_at(ia[g], j)), h2f(h_at(rb[g], j))));
        *reinterpret_cast<uint2*>(d + e0[g]) = pack_b(q);
      } else if constexpr (KIND == K_REQUANT) {
        int8_t q[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = sat8(__fmul_rn(__int2float_rn(i_at(ia[g], j)), s0));
        *reinterpret_cast<uint2*>(d + e0[g]) = pack_b(q);
      } else if constexpr (KIND == K_SCALE_MUL_I32) {
        int32_t o[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = sat32(__fmul_rn(__int2float_rn(i_at(ia[g], j)), s0));
        uint4* q = reinterpret_cast<uint4*>(d + e0[g] * 4);
        q[0] = make_uint4(o[0], o[1], o[2], o[3]);
        q[1] = make_uint4(o[4], o[5], o[6], o[7]);
      } else if constexpr (KIND == K_VADD_I32) {
        const V8 rv{rb[g], rc[g]};
        uint32_t o[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = static_cast<uint32_t>(i_at(ia[g], j)) + static_cast<uint32_t>(i_at(rv, j));
        uint4* q = reinterpret_cast<uint4*>(d + e0[g] * 4);
        q[0] = make_uint4(o[0], o[1], o[2], o[3]);
        q[1] = make_uint4(o[4], o[5], o[6], o[7]);
      } else if constexpr (KIND == K_SCALE_MUL_I8) {
        int8_t q[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = sat8(__fmul_rn(static_cast<float>(b_at(qa[g], j)), s0));
        *reinterpret_cast<uint2*>(d + e0[g]) = pack_b(q);
      } else if constexpr (KIND == K_VADD_I8) {
        int8_t q[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int v = int(b_at(qa[g], j)) + int(b_at(qb[g], j));
          q[j] = static_cast<int8_t>(v < -128 ? -128 : (v > 127 ? 127 : v));
        }
        *reinterpret_cast<uint2*>(d + e0[g]) = pack_b(q);
      } else if constexpr (KIND == K_DEQUANT_ADD) {
        int8_t q[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float accv = __fmul_rn(__int2float_rn(i_at(ia[g], j)), s0);
          const float skip = __fmul_rn(static_cast<float>(b_at(qb[g], j)), s1);
          q[j] = sat8(__fadd_rn(accv, skip));
        }
        *reinterpret_cast<uint2*>(d + e0[g]) = pack_b(q);
      } else if constexpr (KIND == K_GELU_I8) {
        int8_t q[8];
  #pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float x = (op.flags & F_SRC_I32) ? __fmul_rn(__int2float_rn(i_at(ia[g], j)), s0)
                                                 : __fmul_rn(static_cast<float>(b_at(qa[g], j)), s0);
          const float y = gelu_f32(x);
          q[j] = s1 == 0.f ? int8_t(0) : sat8(__fdiv_rn(y, s1));
        }
        *reinterpret_cast<uint2*>(d + e0[g]) = pack_b(q);
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// QUANT, GELU_F16, VADD_F16 and DEQUANT_SCALED with their operands staged in
// shared memory: one thread bulk-copies the task's slice of a (and of b for
// VADD, the [scale | bias] rows for DEQUANT_SCALED) for every sequence of the
// task, the half waits once on an mbarrier, then computes from shared memory.
// No operand register is held across the memory latency, and the latency is
// paid once per task.  Requires MN and N multiples of 8 (every copy is whole
// 16-byte units) and a staged size of at most kStageBytes.
// ---------------------------------------------------------------------------------
constexpr uint32_t kStageBytes = 64 * 1024;

template <int KIND>
__device__ __forceinline__ uint32_t staged_bytes(const DevOp& op, const Task& t) {
  const uint32_t N = op.N, MN = op.M * N;
  constexpr uint32_t kTask = ew_task_elems(KIND);
  constexpr uint32_t ea = KIND == K_DEQUANT_SCALED ? 4 : 2;
  const uint32_t nseq = t.nseq > 1 ? t.nseq : 1;
  const uint32_t e_begin = t.nseq > 1 ? 0 : t.tile * kTask;
  const uint32_t e_count = t.nseq > 1 ? MN : min(kTask, MN - e_begin);
  uint32_t bytes = nseq * e_count * ea;
  if (KIND == K_VADD_F16) bytes += nseq * e_count * 2;
  if (KIND == K_DEQUANT_SCALED) bytes += ((op.b & kSharedBit) ? 1u : nseq) * N * 4;
  return bytes;
}

template <int KIND>
__device__ __noinline__ void ew_staged(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem,
                                       TcShared* tc, uint32_t opi) {
  const uint32_t N = op.N, MN = op.M * N;
  constexpr uint32_t kTask = ew_task_elems(KIND);
  constexpr uint32_t ea = KIND == K_DEQUANT_SCALED ? 4 : 2;   // bytes of an a element
  const uint32_t nseq = t.nseq > 1 ? t.nseq : 1;
  const uint32_t e_begin = t.nseq > 1 ? 0 : t.tile * kTask;
  const uint32_t e_count = t.nseq > 1 ? MN : min(kTask, MN - e_begin);   // elements per sequence
  const bool row_shared = (op.b & kSharedBit) != 0;
  uint8_t* sa = smem;                                   // [nseq][e_count] a
  uint8_t* sb = sa + nseq * e_count * ea;               // VADD: [nseq][e_count] b; DEQ: [seq][scale N | bias N]
  const uint32_t par = tc->phase_stage;
  hsync();   // every thread has the parity before it flips
  if (htid() == 0) {
    tc->phase_stage = par ^ 1u;
    sm100::fence_proxy_async();
    sm100::mbar_arrive_expect_tx(&tc->stage, staged_bytes<KIND>(op, t));
    for (uint32_t s = 0; s < nseq; ++s) {
      const uint32_t seq = t.seq0 + s;
      sm100::bulk_g2s(sa + s * e_count * ea, pptr(A, op.a, seq) + uint64_t(e_begin) * ea, e_count * ea, &tc->stage);
      if (KIND == K_VADD_F16)
        sm100::bulk_g2s(sb + s * e_count * 2, pptr(A, op.b, seq) + uint64_t(e_begin) * 2, e_count * 2, &tc->stage);
      if (KIND == K_DEQUANT_SCALED && (s == 0 || !row_shared)) {
        uint8_t* rows = sb + s * N * 4;
        const uint8_t* scale = pptr(A, op.b, seq);
        const uint8_t* bias = (op.flags & F_SPLIT) ? pptr(A, op.c, seq) : scale + uint64_t(N) * 2;
        sm100::bulk_g2s(rows, scale, N * 2, &tc->stage);
        sm100::bulk_g2s(rows + N * 2, bias, N * 2, &tc->stage);
      }
    }
  }
  // the registers' raw bits load while the copies are in flight
  uint16_t s0b = 0;
  if (KIND == K_QUANT || KIND == K_DEQUANT_SCALED) s0b = sreg_bits(A, op.s[0], t.seq0);
  if (!sm100::mbar_wait(&tc->stage, par, nullptr, 0)) {
    // the copies did not land in time: wait (bounded) for them once more, then fault
    sm100::mbar_wait(&tc->stage, par, nullptr, 0);
    if (htid() == 0) raise_fault(A, DF_STAGE_TIMEOUT, opi, t.seq0);
    return;
  }
  const uint32_t total = nseq * e_count;
  uint32_t cur_seq = 0xFFFFFFFFu;
  float s0 = 0.f;
  for (uint32_t i = htid() * 8; i < total; i += kThreads * 8) {
    const uint32_t s = i / e_count, e = e_begin + (i - s * e_count);
    const uint32_t seq = t.seq0 + s;
    if (KIND == K_QUANT || KIND == K_DEQUANT_SCALED) {
      if (seq != cur_seq) {
        s0 = h2f(seq == t.seq0 ? s0b : sreg_bits(A, op.s[0], seq));
        cur_seq = seq;
      }
    }
    uint8_t* d = pptr(A, op.d, seq);
    if constexpr (KIND == K_QUANT) {
      const uint4 x = *reinterpret_cast<const uint4*>(sa + uint64_t(i) * 2);
      int8_t q[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        q[j] = sat8(__fmul_rn(h2f(h_at(x, j)), s0));
      }
      *reinterpret_cast<uint2*>(d + e) = pack_b(q);
    } else if constexpr (KIND == K_GELU_F16) {
      const uint4 x = *reinterpret_cast<const uint4*>(sa + uint64_t(i) * 2);
      uint16_t h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = f2h(gelu_f32(h2f(h_at(x, j))));
      *reinterpret_cast<uint4*>(d + uint64_t(e) * 2) = pack_h(h);
    } else if constexpr (KIND == K_VADD_F16) {
      const uint4 x = *reinterpret_cast<const uint4*>(sa + uint64_t(i) * 2);
      const uint4 y = *reinterpret_cast<const uint4*>(sb + uint64_t(i) * 2);
      uint16_t h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = f2h(__fadd_rn(h2f(h_at(x, j)), h2f(h_at(y, j))));
      *reinterpret_cast<uint4*>(d + uint64_t(e) * 2) = pack_h(h);
    } else {   // K_DEQUANT_SCALED
      const uint4 lo = *reinterpret_cast<const uint4*>(sa + uint64_t(i) * 4);
      const uint4 hi = *reinterpret_cast<const uint4*>(sa + uint64_t(i) * 4 + 16);
      const uint32_t col = e % N;
      const uint8_t* rows = sb + (row_shared ? 0u : s) * N * 4;
      const uint4 sc = *reinterpret_cast<const uint4*>(rows + col * 2);
      const uint4 bi = *reinterpret_cast<const uint4*>(rows + N * 2 + col * 2);
      const int32_t acc[8] = {int32_t(lo.x), int32_t(lo.y), int32_t(lo.z), int32_t(lo.w),
                              int32_t(hi.x), int32_t(hi.y), int32_t(hi.z), int32_t(hi.w)};
      uint16_t h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float v = __fmul_rn(__int2float_rn(acc[j]), h2f(h_at(sc, j)));
        v = __fmul_rn(v, s0);
        h[j] = f2h(__fadd_rn(v, h2f(h_at(bi, j))));
      }
      *reinterpret_cast<uint4*>(d + uint64_t(e) * 2) = pack_h(h);
    }
  }
}

// K_VADD_CHAIN: the running FP16 sum of the op's segment operands over
// kVaddChainTask elements of one sequence.  One thread stages every operand's
// slice in shared memory with bulk copies on the stage barrier, then each
// thread adds 8 elements at a time, rounding to FP16 after each add in the
// program's order, and stores each partial sum whose segment names a dst.
static_assert(kVaddChainMax * kVaddChainTask * 2 <= kStageBytes, "chain operands exceed the staging area");
__device__ __noinline__ void op_vadd_chain(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem,
                                           TcShared* tc, uint32_t opi) {
  const uint32_t MN = op.M * op.N;
  const uint32_t e_begin = t.tile * kVaddChainTask;
  if (e_begin >= MN) return;   // the same for every thread of the half
  const uint32_t e_count = min(kVaddChainTask, MN - e_begin);
  const uint32_t n = op.nseg < kVaddChainMax ? op.nseg : kVaddChainMax;
  const Segment* sg = A.segs + op.seg0;
  const uint32_t par = tc->phase_stage;
  hsync();   // every thread has the parity before it flips
  if (htid() == 0) {
    tc->phase_stage = par ^ 1u;
    sm100::fence_proxy_async();
    sm100::mbar_arrive_expect_tx(&tc->stage, n * e_count * 2);
    for (uint32_t k = 0; k < n; ++k)
      sm100::bulk_g2s(smem + k * e_count * 2, pptr(A, sg[k].src, t.seq0) + uint64_t(e_begin) * 2, e_count * 2,
                      &tc->stage);
  }
  if (!sm100::mbar_wait(&tc->stage, par, nullptr, 0)) {
    sm100::mbar_wait(&tc->stage, par, nullptr, 0);   // bounded: let copies in flight land, then fault
    if (htid() == 0) raise_fault(A, DF_STAGE_TIMEOUT, opi, t.seq0);
    return;
  }
  for (uint32_t i = htid() * 8; i < e_count; i += kThreads * 8) {
    const uint4 x0 = *reinterpret_cast<const uint4*>(smem + uint64_t(i) * 2);
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = h2f(h_at(x0, j));
    for (uint32_t k = 1; k < n; ++k) {
      const uint4 x = *reinterpret_cast<const uint4*>(smem + (uint64_t(k) * e_count + i) * 2);
      uint16_t h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        h[j] = f2h(__fadd_rn(acc[j], h2f(h_at(x, j))));
        acc[j] = h2f(h[j]);
      }
      const uint64_t d = sg[k].dst;
      if (d) *reinterpret_cast<uint4*>(pptr(A, d, t.seq0) + (uint64_t(e_begin) + i) * 2) = pack_h(h);
    }
  }
}

// Whether a task can take the staged path.
template <int KIND>
__device__ __forceinline__ bool can_stage(const DevOp& op, const Task& t) {
  if (op.N % 8 || (op.M * op.N) % 8) return false;
  return staged_bytes<KIND>(op, t) <= kStageBytes;
}

__device__ __noinline__ void op_elementwise(const ExecArgs& A, const DevOp& op, const Task& t) {
  switch (op.kind) {
    case K_QUANT: ew_kernel<K_QUANT>(A, op, t); break;
    case K_GELU_F16: ew_kernel<K_GELU_F16>(A, op, t); break;
    case K_VADD_F16: ew_kernel<K_VADD_F16>(A, op, t); break;
    case K_DEQUANT_SCALED: ew_kernel<K_DEQUANT_SCALED>(A, op, t); break;
    case K_DEQUANT_ACCUM: ew_kernel<K_DEQUANT_ACCUM>(A, op, t); break;
    case K_REQUANT_PC: ew_kernel<K_REQUANT_PC>(A, op, t); break;
    case K_REQUANT: ew_kernel<K_REQUANT>(A, op, t); break;
    case K_SCALE_MUL_I32: ew_kernel<K_SCALE_MUL_I32>(A, op, t); break;
    case K_VADD_I32: ew_kernel<K_VADD_I32>(A, op, t); break;
    case K_SCALE_MUL_I8: ew_kernel<K_SCALE_MUL_I8>(A, op, t); break;
    case K_VADD_I8: ew_kernel<K_VADD_I8>(A, op, t); break;
    case K_DEQUANT_ADD: ew_kernel<K_DEQUANT_ADD>(A, op, t); break;
    case K_GELU_I8: ew_kernel<K_GELU_I8>(A, op, t); break;
    default: break;
  }
}

// ---------------------------------------------------------------------------------
// MAX_ABS_REDUCE_FP32 (simulator.py:1088-1140): one task per sequence.
// ---------------------------------------------------------------------------------
// Operands read through a segment list (F_SEGA): the op's segments give, in
// order, runs of physically contiguous 16-byte units; Segment.dst is the run's
// offset in the operand.  The table is staged in shared memory past the first
// kSegTableOff bytes and each unit found by binary search, so every thread
// keeps four 16-byte loads in flight however the runs are sized.
constexpr uint32_t kSegTableOff = 4096;
constexpr uint32_t kMaxQStage = 8192;   // MAX_ABS + QUANT: the reduced input, 16384 FP16 at most

// A task whose units touch only part of the list names that part in
// Task::aux (first segment | count << 16); aux 0 stands for the whole list.
// Returns the number of segments staged.
__device__ __forceinline__ uint32_t seg_stage(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem) {
  uint32_t* ofs = reinterpret_cast<uint32_t*>(smem + kSegTableOff);
  uint64_t* src = reinterpret_cast<uint64_t*>(smem + kSegTableOff + kMaxSegRuns * 4);
  uint8_t* gelu = smem + kSegTableOff + kMaxSegRuns * 12;   // kSegGelu flag of each segment
  const uint32_t first = t.aux ? (t.aux & 0xFFFFu) : 0u, count = t.aux ? (t.aux >> 16) : op.nseg;
  for (uint32_t k = htid(); k < count; k += kThreads) {
    const Segment sg = A.segs[op.seg0 + first + k];
    ofs[k] = static_cast<uint32_t>(sg.dst);   // the offset (the flag bit lies above 32 bits)
    src[k] = sg.src;
    gelu[k] = (sg.dst & kSegGelu) ? 1 : 0;
  }
  hsync();
  return count;
}

// The staged segment (index) holding operand unit u (nseg segments staged).
__device__ __forceinline__ uint32_t seg_index(uint32_t nseg, const uint8_t* smem, uint32_t u) {
  const uint32_t* ofs = reinterpret_cast<const uint32_t*>(smem + kSegTableOff);
  uint32_t lo = 0, hi = nseg;   // last k with ofs[k] <= u
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) >> 1;
    if (ofs[mid] <= u) lo = mid;
    else hi = mid;
  }
  return lo;
}

// Address of operand unit u (segments staged by seg_stage; nseg of them).
__device__ __forceinline__ const uint4* seg_unit(const ExecArgs& A, uint32_t nseg, const uint8_t* smem,
                                                 uint32_t seq, uint32_t u) {
  const uint32_t* ofs = reinterpret_cast<const uint32_t*>(smem + kSegTableOff);
  const uint64_t* src = reinterpret_cast<const uint64_t*>(smem + kSegTableOff + kMaxSegRuns * 4);
  const uint32_t lo = seg_index(nseg, smem, u);
  return reinterpret_cast<const uint4*>(pptr(A, src[lo], seq)) + (u - ofs[lo]);
}

// QUANT / VADD_F16 / GELU with a segment-list first operand; a task takes
// operand units [tile * kSegTaskUnits, +kSegTaskUnits) of one sequence.
__device__ __noinline__ void op_seg_ew(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem) {
  const uint32_t seq = t.seq0;
  const uint32_t u_begin = t.tile * kSegTaskUnits;
  const uint32_t units = min(op.M * op.N / 8, u_begin + kSegTaskUnits);   // FP16 operand: 8 elements per unit
  // the register's raw bits load while the segment table is staged; they are
  // converted at their first use, after the operand loads are in flight
  const uint16_t s0b = op.kind == K_QUANT ? sreg_bits(A, op.s[0], seq) : uint16_t(0);
  const uint32_t nseg = seg_stage(A, op, t, smem);
  const uint4* b = reinterpret_cast<const uint4*>(pptr(A, op.b, seq));
  uint8_t* d = pptr(A, op.d, seq);
  for (uint32_t u0 = u_begin + htid(); u0 < units; u0 += 4 * kThreads) {
    uint4 va[4], vb[4];
#pragma unroll
    for (uint32_t q = 0; q < 4; ++q) {
      const uint32_t u = u0 + q * kThreads;
      if (u < units) {
        va[q] = __ldcg(seg_unit(A, nseg, smem, seq, u));
        if (op.kind == K_VADD_F16) vb[q] = __ldcg(b + u);
      }
    }
#pragma unroll
    for (uint32_t q = 0; q < 4; ++q) {
      const uint32_t u = u0 + q * kThreads;
      if (u >= units) continue;
      if (op.kind == K_QUANT) {
        const float s0 = h2f(s0b);
        int8_t o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] = sat8(__fmul_rn(h2f(h_at(va[q], j)), s0));
        }
        *reinterpret_cast<uint2*>(d + uint64_t(u) * 8) = pack_b(o);
      } else if (op.kind == K_GELU_F16) {
        uint16_t h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = f2h(gelu_f32(h2f(h_at(va[q], j))));
        *reinterpret_cast<uint4*>(d + uint64_t(u) * 16) = pack_h(h);
      } else {
        uint16_t h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = f2h(__fadd_rn(h2f(h_at(va[q], j)), h2f(h_at(vb[q], j))));
        *reinterpret_cast<uint4*>(d + uint64_t(u) * 16) = pack_h(h);
      }
    }
  }
}

// The scale pair MAX_ABS derives from max |x| (m: its FP16 bit pattern,
// 0xFFFF for a NaN): inverse 127 / max and forward max / 127, max clamped to
// [2^-9, 65504 * 127 / 2], both rounded once from float64.
__device__ __forceinline__ void max_abs_scales(uint32_t m, uint16_t& inv, uint16_t& fwd) {
  if (m == 0xFFFFu) {
    inv = fwd = 0x7E00u;
    return;
  }
  double mx = static_cast<double>(h2f(static_cast<uint16_t>(m)));
  mx = mx > 0.001953125 ? mx : 0.001953125;         // 2^-9
  mx = mx < 4159504.0 ? mx : 4159504.0;             // 65504 * 127 / 2
  inv = d2h(127.0 / mx);
  fwd = d2h(mx / 127.0);
}

__device__ __noinline__ void op_max_abs(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem) {
  const uint32_t seq = t.seq0;
  const uint64_t MN = uint64_t(op.M) * op.N;
  const uint16_t* x = reinterpret_cast<const uint16_t*>(pptr(A, op.a, seq));
  // |x| of FP16 values compared as bit patterns (monotone for non-NaN);
  // any NaN wins, as np.max propagates NaN.
  uint32_t m = 0;
  const uint4* xv = reinterpret_cast<const uint4*>(x);
  const uint64_t ng = MN / 8;   // MN is a multiple of 256
  const bool seg = op.flags & F_SEGA;
  const bool maxq = (op.flags2 & FX_MAXQ) != 0;   // also QUANT's result (MN <= 16384)
  uint4* keep = reinterpret_cast<uint4*>(smem + kMaxQStage);   // the input, kept for the QUANT
  const uint32_t nseg = seg ? seg_stage(A, op, t, smem) : 0u;
  for (uint64_t g0 = htid(); g0 < ng; g0 += uint64_t(kThreads) * 8) {
    uint4 v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint64_t g = g0 + uint64_t(k) * kThreads;
      v[k] = g < ng ? __ldcg(seg ? seg_unit(A, nseg, smem, seq, uint32_t(g)) : xv + g) : make_uint4(0, 0, 0, 0);
    }
    if (op.flags2 & FX_GELUSEG) {
      // segments that read a GELU's input: the value the GELU op would have stored
      const uint8_t* gelu = smem + kSegTableOff + kMaxSegRuns * 12;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint64_t g = g0 + uint64_t(k) * kThreads;
        if (g < ng && gelu[seg_index(nseg, smem, uint32_t(g))]) {
          uint16_t h[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) h[j] = f2h(gelu_f32(h2f(h_at(v[k], j))));
          v[k] = pack_h(h);
        }
      }
    }
    if (maxq) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint64_t g = g0 + uint64_t(k) * kThreads;
        if (g < ng) keep[g] = v[k];
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t h = h_at(v[k], j) & 0x7FFFu;
        if (h > 0x7C00u) h = 0xFFFFu;  // NaN
        m = h > m ? h : m;
      }
  }
  for (int o = 16; o; o >>= 1) {
    uint32_t w = __shfl_xor_sync(0xffffffffu, m, o);
    m = w > m ? w : m;
  }
  uint32_t* red = reinterpret_cast<uint32_t*>(smem);
  if ((htid() & 31) == 0) red[htid() >> 5] = m;
  hsync();
  if (htid() == 0) {
    for (int w = 1; w < kWarps; ++w) m = red[w] > m ? red[w] : m;
    uint16_t inv, fwd;
    max_abs_scales(m, inv, fwd);
    A.sregs[uint64_t(seq) * A.sreg_stride + op.out_slot] = inv;
    A.sregs[uint64_t(seq) * A.sreg_stride + op.out_slot + 1] = fwd;
    red[kWarps] = inv;
  }
  hsync();
  if (maxq) {
    // QUANT's rule with the inverse scale just derived: rint(x * inv), NaN -> 0, clipped to int8
    const float s0 = h2f(static_cast<uint16_t>(red[kWarps]));
    int8_t* out = reinterpret_cast<int8_t*>(pptr(A, op.d, seq));
    const uint64_t nq = op.q_rows ? uint64_t(op.q_rows) * op.N / 8 : ng;   // rows of the result some op reads
    for (uint64_t g = htid(); g < nq; g += kThreads) {
      const uint4 x8 = keep[g];
      int8_t q8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        q8[j] = sat8(__fmul_rn(h2f(h_at(x8, j)), s0));
      }
      *reinterpret_cast<uint2*>(out + g * 8) = pack_b(q8);
    }
  }
}

// ---------------------------------------------------------------------------------
// A pair of MAX_ABS + QUANT ops (FX_MAXGRP: two ops of one level and shape,
// segment-list input, FX_MAXQ) of one sequence in one task: each op on half
// the threads (128) with a shared-memory region of its own, op_max_abs's
// arithmetic.  Both halves pass the same barriers.
// ---------------------------------------------------------------------------------
constexpr uint32_t kMaxGrpRegion = 24576;   // per op: reductions, segment table, the kept input
constexpr uint32_t kMaxGrpSegs = 64;        // segment table at 64
constexpr uint32_t kMaxGrpKeep = 4096;      // the kept input (kMaxGrpElems FP16)
static_assert(kMaxGrpSegs + kMaxSegRuns * 13 <= kMaxGrpKeep && kMaxGrpKeep + kMaxGrpElems * 2 <= kMaxGrpRegion,
              "MAX_ABS pair region layout");

__device__ __noinline__ void op_max_abs_pair(const ExecArgs& A, const Task& t, uint8_t* smem) {
  const uint32_t seq = t.seq0;
  const uint32_t g = htid() >> 7, gt = htid() & 127, gw = gt >> 5, lane = htid() & 31;
  const uint32_t opi = g == 0 ? t.op : A.tasks[t.tile + 1].op;
  const DevOp& op = A.ops[opi];
  uint8_t* base = smem + g * kMaxGrpRegion;
  uint32_t* red = reinterpret_cast<uint32_t*>(base);
  uint32_t* ofs = reinterpret_cast<uint32_t*>(base + kMaxGrpSegs);
  uint64_t* src = reinterpret_cast<uint64_t*>(base + kMaxGrpSegs + kMaxSegRuns * 4);
  uint8_t* gel = base + kMaxGrpSegs + kMaxSegRuns * 12;
  uint4* keep = reinterpret_cast<uint4*>(base + kMaxGrpKeep);
  const uint32_t nseg = op.nseg;
  for (uint32_t k = gt; k < nseg; k += 128) {
    const Segment sg = A.segs[op.seg0 + k];
    ofs[k] = static_cast<uint32_t>(sg.dst);   // the offset (the flag bit lies above 32 bits)
    src[k] = sg.src;
    gel[k] = (sg.dst & kSegGelu) ? 1 : 0;
  }
  hsync();
  auto seg_of = [&](uint32_t u) {   // last segment k with ofs[k] <= u
    uint32_t lo = 0, hi = nseg;
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) >> 1;
      if (ofs[mid] <= u) lo = mid;
      else hi = mid;
    }
    return lo;
  };
  const uint32_t ng = op.M * op.N / 8;
  uint32_t m = 0;
  for (uint32_t g0 = gt; g0 < ng; g0 += 128 * 8) {
    uint4 v[8];
    uint32_t si[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t u = g0 + k * 128;
      si[k] = 0;
      v[k] = make_uint4(0, 0, 0, 0);
      if (u < ng) {
        si[k] = seg_of(u);
        v[k] = __ldcg(reinterpret_cast<const uint4*>(pptr(A, src[si[k]], seq)) + (u - ofs[si[k]]));
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const uint32_t u = g0 + k * 128;
      if (u >= ng) continue;
      if (gel[si[k]]) {   // a GELU's input: the value the GELU op would have stored
        uint16_t h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) h[j] = f2h(gelu_f32(h2f(h_at(v[k], j))));
        v[k] = pack_h(h);
      }
      keep[u] = v[k];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t h = h_at(v[k], j) & 0x7FFFu;
        if (h > 0x7C00u) h = 0xFFFFu;  // NaN
        m = h > m ? h : m;
      }
    }
  }
  for (int o = 16; o; o >>= 1) {
    const uint32_t w = __shfl_xor_sync(0xffffffffu, m, o);
    m = w > m ? w : m;
  }
  if (lane == 0) red[gw] = m;
  hsync();
  if (gt == 0) {
    for (int w = 1; w < 4; ++w) m = red[w] > m ? red[w] : m;
    uint16_t inv, fwd;
    max_abs_scales(m, inv, fwd);
    A.sregs[uint64_t(seq) * A.sreg_stride + op.out_slot] = inv;
    A.sregs[uint64_t(seq) * A.sreg_stride + op.out_slot + 1] = fwd;
    red[4] = inv;
  }
  hsync();
  // QUANT's rule with the inverse scale just derived: rint(x * inv), NaN -> 0, clipped to int8
  const float s0 = h2f(static_cast<uint16_t>(red[4]));
  int8_t* out = reinterpret_cast<int8_t*>(pptr(A, op.d, seq));
  const uint32_t nq = op.q_rows ? op.q_rows * op.N / 8 : ng;   // rows of the result some op reads
  for (uint32_t u = gt; u < nq; u += 128) {
    const uint4 x8 = keep[u];
    int8_t q8[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) q8[j] = sat8(__fmul_rn(h2f(h_at(x8, j)), s0));
    *reinterpret_cast<uint2*>(out + uint64_t(u) * 8) = pack_b(q8);
  }
}

// ---------------------------------------------------------------------------------
// Row ops: one warp per row, 8 rows per task.
// ---------------------------------------------------------------------------------
struct RowCtx {
  float* row;            // per-warp float row buffer (capacity kRowCap) or null
  uint32_t* pw;          // per-warp pairwise scratch
};
constexpr uint32_t kRowCap = 2048;

// float32 value of element j of row r of the op's first input.
__device__ __forceinline__ float in_val(const ExecArgs& A, const DevOp& op, uint32_t seq, uint64_t idx,
                                        float in_scale) {
  const uint8_t* a = pptr(A, op.a, seq);
  switch (op.kind) {
    case K_LAYERNORM_F16: case K_SOFTMAX_F16: case K_MASKED_SOFTMAX_F16:
      return h2f(reinterpret_cast<const uint16_t*>(a)[idx]);
    case K_LN_I8:
      return __fmul_rn(static_cast<float>(reinterpret_cast<const int8_t*>(a)[idx]), in_scale);
    default:  // legacy softmax variants: int8 or int32 input times in_scale
      if (op.flags & F_SRC_I32)
        return __fmul_rn(__int2float_rn(reinterpret_cast<const int32_t*>(a)[idx]), in_scale);
      return __fmul_rn(static_cast<float>(reinterpret_cast<const int8_t*>(a)[idx]), in_scale);
  }
}


// One row of a row op (op_rows); a buffered FP16 row is already in rowbuf.
__device__ __forceinline__ void row_one(const ExecArgs& A, const DevOp& op, uint32_t seq, uint32_t r, float* rowbuf,
                                       uint32_t* pw, bool buffered, bool fp16_in, float in_scale, float out_scale,
                                       int lane, uint32_t qrb, uint32_t vkl, uint32_t mode) {
  const uint32_t N = op.N;
  const uint64_t base = uint64_t(r) * N;
  auto x_at = [&](uint32_t j) -> float {
    return buffered ? rowbuf[j] : in_val(A, op, seq, base + j, in_scale);
  };
  if (!fp16_in && buffered) {
    for (uint32_t j = lane; j < N; j += 32) rowbuf[j] = in_val(A, op, seq, base + j, in_scale);
    __syncwarp();
  }
  uint8_t* d = pptr(A, op.d, seq);

  if (op.kind == K_LAYERNORM_F16 || op.kind == K_LN_I8) {
    const float eps = op.kind == K_LN_I8 ? 1e-6f : 1e-5f;
    const float sum = buffered ? warp_pairwise_sum_smem(rowbuf, N, pw)
                               : warp_pairwise_sum([&](uint32_t j) { return x_at(j); }, N, pw);
    const float mean = div_count(sum, N);
    const float sq =
        buffered ? warp_pairwise_sum_smem(rowbuf, N, pw, true, mean)
                 : warp_pairwise_sum(
                       [&](uint32_t j) { const float dd = __fsub_rn(x_at(j), mean); return __fmul_rn(dd, dd); }, N, pw);
    const float var = div_count(sq, N);
    const float denom = __fsqrt_rn(__fadd_rn(var, eps));
    const uint8_t* gb = pptr(A, op.b, seq);
    const uint8_t* be = (op.flags & F_SPLIT) ? pptr(A, op.c, seq) : gb + uint64_t(N) * 2;   // beta
    if (op.kind == K_LAYERNORM_F16 && buffered) {
      const uint32_t ng = N / 8;
      for (uint32_t half = 0; half < kRowCap / 256; half += 4) {
      uint4 gv[4], bv[4];
#pragma unroll
      for (uint32_t k = 0; k < 4; ++k) {
        const uint32_t g = lane + 32 * (half + k);
        if (g < ng) {
          gv[k] = __ldcg(reinterpret_cast<const uint4*>(gb) + g);
          bv[k] = __ldcg(reinterpret_cast<const uint4*>(be) + g);
        }
      }
#pragma unroll
      for (uint32_t k = 0; k < 4; ++k) {
        const uint32_t g = lane + 32 * (half + k);
        if (g >= ng) continue;
        uint16_t h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float y = __fdiv_rn(__fsub_rn(rowbuf[g * 8 + j], mean), denom);
          h[j] = f2h(__fadd_rn(__fmul_rn(y, h2f(h_at(gv[k], j))), h2f(h_at(bv[k], j))));
        }
        *reinterpret_cast<uint4*>(d + (base + uint64_t(g) * 8) * 2) = pack_h(h);
      }
      }
      return;
    }
    for (uint32_t j = lane; j < N; j += 32) {
      const float y = __fdiv_rn(__fsub_rn(x_at(j), mean), denom);
      const float g = h2f(reinterpret_cast<const uint16_t*>(gb)[j]);
      const float b = h2f(reinterpret_cast<const uint16_t*>(be)[j]);
      const float o = __fadd_rn(__fmul_rn(y, g), b);
      if (op.kind == K_LAYERNORM_F16) reinterpret_cast<uint16_t*>(d)[base + j] = f2h(o);
      else reinterpret_cast<int8_t*>(d)[base + j] = out_scale == 0.f ? int8_t(0) : sat8(__fdiv_rn(o, out_scale));
    }
    return;
  }

  // softmax family
  if ((op.kind == K_SOFTMAX_F16 || op.kind == K_MASKED_SOFTMAX_F16) && buffered && N % 8 == 0) {
    const bool mk = op.kind == K_MASKED_SOFTMAX_F16;
    const int64_t lt = int64_t(r) + qrb < int64_t(vkl) - 1 ? int64_t(r) + qrb : int64_t(vkl) - 1;
    softmax_row_f16(rowbuf, N, mk, mk ? lt : int64_t(N) - 1, reinterpret_cast<uint16_t*>(d) + base, pw, lane);
    return;
  }
  uint32_t last = N - 1;        // last visible column (FP16 masked variant)
  bool masked_f16 = op.kind == K_MASKED_SOFTMAX_F16;
  bool masked_i8 = op.kind == K_MASKED_SOFTMAX_I8;
  if (masked_f16) {
    const int64_t lt = int64_t(r) + qrb < int64_t(vkl) - 1 ? int64_t(r) + qrb : int64_t(vkl) - 1;
    if (lt < 0) {
      for (uint32_t j = lane; j < N; j += 32) reinterpret_cast<uint16_t*>(d)[base + j] = 0;
      return;
    }
    last = static_cast<uint32_t>(lt);
  }
  auto visible = [&](uint32_t j) -> bool {
    if (masked_f16) return j <= last;
    if (masked_i8) {
      bool v = true;
      if (mode & 2) v = v && (j <= qrb + r);
      if (mode & 1) v = v && (j < vkl);
      return v;
    }
    return true;
  };
  float mx = -INFINITY;
  for (uint32_t j = lane; j < N; j += 32)
    if (visible(j)) mx = fmaxf(mx, x_at(j));
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  // exp values (buffered rows are overwritten in place)
  auto e_at = [&](uint32_t j) -> float {
    return visible(j) ? exp_f32(__fsub_rn(x_at(j), mx)) : 0.f;
  };
  if (buffered) {
    __syncwarp();
    for (uint32_t j = lane; j < N; j += 32) rowbuf[j] = e_at(j);
    __syncwarp();
  }
  auto ev = [&](uint32_t j) -> float { return buffered ? rowbuf[j] : e_at(j); };
  const float denom = buffered ? warp_pairwise_sum_smem(rowbuf, N, pw) : warp_pairwise_sum(ev, N, pw);
  if (masked_i8 && denom == 0.f) {
    if (lane == 0) raise_fault(A, DF_ZERO_DENOM, 0, seq);
  }
  if ((op.kind == K_SOFTMAX_F16 || masked_f16) && buffered) {
    for (uint32_t g = lane; g < N / 8; g += 32) {
      uint16_t h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float e = rowbuf[g * 8 + j];
        h[j] = f2h(op.kind == K_SOFTMAX_F16 ? __fdiv_rn(e, denom) : (denom > 0.f ? __fdiv_rn(e, denom) : 0.f));
      }
      *reinterpret_cast<uint4*>(d + (base + uint64_t(g) * 8) * 2) = pack_h(h);
    }
    return;
  }
  for (uint32_t j = lane; j < N; j += 32) {
    const float e = ev(j);
    if (op.kind == K_SOFTMAX_F16) {
      reinterpret_cast<uint16_t*>(d)[base + j] = f2h(__fdiv_rn(e, denom));
    } else if (masked_f16) {
      reinterpret_cast<uint16_t*>(d)[base + j] = f2h(denom > 0.f ? __fdiv_rn(e, denom) : 0.f);
    } else {
      const float p = __fdiv_rn(e, denom);
      reinterpret_cast<int8_t*>(d)[base + j] = out_scale == 0.f ? int8_t(0) : sat8(__fdiv_rn(p, out_scale));
    }
  }
}

// FP16 LayerNorm of one or two rows (a decode step's live row) with every warp
// of the half, for rows whose NumPy pairwise-summation tree is balanced (nl <=
// 8 leaves of L elements, pw_balanced): warp w sums leaf w, lanes 0..7 one of
// its eight accumulator chains each, combined ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7))
// by xor shuffles (IEEE addition commutes); the leaf sums then combine level
// by level, as the tree does.  Arithmetic per element is row_one's.
__device__ __forceinline__ bool ln_small_ok(const DevOp& op) {
  uint32_t nl, L;
  return op.kind == K_LAYERNORM_F16 && op.M <= 2 && op.N % 8 == 0 && op.N <= kRowCap && pw_balanced(op.N, nl, L);
}

__device__ __noinline__ void op_ln_small(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem) {
  const uint32_t seq = t.seq0, N = op.N;
  float* x = reinterpret_cast<float*>(smem);   // the row as float32
  float* part = x + kRowCap;                   // leaf sums: [0, 8) the row, [8, 16) the squares
  const uint8_t* gb = pptr(A, op.b, seq);
  const uint8_t* be = (op.flags & F_SPLIT) ? pptr(A, op.c, seq) : gb + uint64_t(N) * 2;
  const bool has4 = htid() < N / 4;   // output groups of 4 elements
  uint2 gv = make_uint2(0, 0), bv = make_uint2(0, 0);
  if (has4) {   // gamma and beta of this thread's outputs, in flight during the sums
    gv = __ldcg(reinterpret_cast<const uint2*>(gb) + htid());
    bv = __ldcg(reinterpret_cast<const uint2*>(be) + htid());
  }
  for (uint32_t r = 0; r < op.M; ++r) {
    if (r) hsync();   // the previous row's readers are done with x and part
    const uint4* src = reinterpret_cast<const uint4*>(pptr(A, op.a, seq) + uint64_t(r) * N * 2);
    for (uint32_t g = htid(); g < N / 8; g += kThreads) {
      const uint4 v = __ldcg(src + g);
#pragma unroll
      for (int j = 0; j < 8; ++j) x[g * 8 + j] = h2f(h_at(v, j));
    }
    hsync();
    float mean, denom;
    ln_stats(x, N, part, mean, denom);
    if (has4) {
      const float4 xv = *reinterpret_cast<const float4*>(x + htid() * 4);
      const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
      *reinterpret_cast<uint2*>(pptr(A, op.d, seq) + (uint64_t(r) * N + htid() * 4) * 2) = ln_out4(xs, mean, denom, gv, bv);
    }
  }
}

// A chain VADD -> LAYERNORM -> MAX_ABS + QUANT over one live row (a decode
// step's residual add, LayerNorm and activation quantisation), in one pass
// with the row kept in shared memory and registers: the sum is stored for
// later ops, the LayerNorm output is stored and reduced, the MAX_ABS
// operand's other rows (the padding the program reloads) are reduced from
// memory as they arrive, and row 0 is quantised.  Each step's arithmetic is
// its op's own (ew VADD, op_ln_small, op_max_abs).
__device__ __forceinline__ bool chain_vln_ok(const ExecArgs& A, const Task& t) {
  if (t.aux != 3) return false;
  const Task* tp = A.tasks + t.tile;
  const DevOp& v = A.ops[tp[0].op];
  const DevOp& l = A.ops[tp[1].op];
  const DevOp& m = A.ops[tp[2].op];
  const uint32_t N = v.N, ru = N / 8;
  if (v.kind != K_VADD_F16 || l.kind != K_LAYERNORM_F16 || m.kind != K_MAX_ABS || !(m.flags2 & FX_MAXQ) ||
      (m.flags2 & FX_GELUSEG) ||
      !(m.flags & F_SEGA) || v.M != 1 || l.M != 1 || l.N != N || m.N != N || N % 8 || N > 4 * kThreads ||
      !ln_small_ok(l) || l.a != v.d || m.nseg > 8 || (m.q_rows ? m.q_rows : m.M) != 1 || (v.flags & ~F_SEGA) ||
      (l.flags & ~F_SPLIT))
    return false;
  const Segment s0 = A.segs[m.seg0];
  if (s0.dst != 0 || s0.src != l.d || s0.n != ru) return false;
  for (uint32_t k = 1; k < m.nseg; ++k) {   // the other rows read neither result of the chain
    const Segment sk = A.segs[m.seg0 + k];
    if (!(sk.src & kSharedBit) && ((sk.src < l.d + ru && l.d < sk.src + sk.n) || (sk.src < v.d + ru && v.d < sk.src + sk.n)))
      return false;
  }
  return true;
}

__device__ __noinline__ void op_chain_vln(const ExecArgs& A, const Task& t, uint8_t* smem) {
  const Task* tp = A.tasks + t.tile;
  const DevOp& v = A.ops[tp[0].op];
  const DevOp& l = A.ops[tp[1].op];
  const DevOp& m = A.ops[tp[2].op];
  const uint32_t seq = t.seq0, N = v.N, ru = N / 8;
  const uint32_t warp = htid() >> 5, lane = htid() & 31;
  float* x = reinterpret_cast<float*>(smem + 8192);    // the summed row as float32
  float* part = reinterpret_cast<float*>(smem + 8192 + kRowCap * 4);   // 16 leaf sums
  uint32_t* red = reinterpret_cast<uint32_t*>(part + 16);              // per-warp maxima, then the scale
  // 1. loads in flight together: the VADD operands' units of row 0, gamma and
  //    beta of this thread's 4 outputs, the MAX_ABS operand's other rows
  const uint32_t nseg_a = (v.flags & F_SEGA) ? seg_stage(A, v, Task{tp[0].op, seq, 1, 0, 0}, smem) : 0u;
  uint4 va = make_uint4(0, 0, 0, 0), vb = make_uint4(0, 0, 0, 0);
  if (htid() < ru) {
    va = __ldcg((v.flags & F_SEGA) ? seg_unit(A, nseg_a, smem, seq, htid())
                                   : reinterpret_cast<const uint4*>(pptr(A, v.a, seq)) + htid());
    vb = __ldcg(reinterpret_cast<const uint4*>(pptr(A, v.b, seq)) + htid());
  }
  const bool has4 = htid() < N / 4;
  const uint8_t* gb = pptr(A, l.b, seq);
  const uint8_t* be = (l.flags & F_SPLIT) ? pptr(A, l.c, seq) : gb + uint64_t(N) * 2;
  uint2 gv = make_uint2(0, 0), bv = make_uint2(0, 0);
  if (has4) {
    gv = __ldcg(reinterpret_cast<const uint2*>(gb) + htid());
    bv = __ldcg(reinterpret_cast<const uint2*>(be) + htid());
  }
  // |x| of FP16 values compared as bit patterns (monotone for non-NaN); any NaN wins
  auto absmax8 = [](uint4 w, uint32_t mx) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      uint32_t h = h_at(w, j) & 0x7FFFu;
      if (h > 0x7C00u) h = 0xFFFFu;
      mx = h > mx ? h : mx;
    }
    return mx;
  };
  uint32_t mx = 0;
  for (uint32_t k = 1; k < m.nseg; ++k) {
    const Segment sk = A.segs[m.seg0 + k];
    const uint4* src = reinterpret_cast<const uint4*>(pptr(A, sk.src, seq));
    for (uint64_t u0 = htid(); u0 < sk.n; u0 += 8 * kThreads) {   // eight loads in flight per thread
      uint4 w[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint64_t u = u0 + uint64_t(j) * kThreads;
        w[j] = u < sk.n ? __ldcg(src + u) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = absmax8(w[j], mx);
    }
  }
  // 2. VADD: f16(a + b), stored for later ops and kept as float32
  if (htid() < ru) {
    uint16_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      h[j] = f2h(__fadd_rn(h2f(h_at(va, j)), h2f(h_at(vb, j))));
      x[htid() * 8 + j] = h2f(h[j]);
    }
    reinterpret_cast<uint4*>(pptr(A, v.d, seq))[htid()] = pack_h(h);
  }
  hsync();
  // 3. LayerNorm of the row
  float mean, denom;
  ln_stats(x, N, part, mean, denom);
  uint2 yv = make_uint2(0, 0);
  if (has4) {
    const float4 xv = *reinterpret_cast<const float4*>(x + htid() * 4);
    const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
    yv = ln_out4(xs, mean, denom, gv, bv);
    reinterpret_cast<uint2*>(pptr(A, l.d, seq))[htid()] = yv;
    mx = absmax8(make_uint4(yv.x, yv.y, 0, 0), mx);
  }
  // 4. MAX_ABS over every row: scales, then QUANT of row 0
  for (int o = 16; o; o >>= 1) {
    const uint32_t w = __shfl_xor_sync(0xffffffffu, mx, o);
    mx = w > mx ? w : mx;
  }
  if (lane == 0) red[warp] = mx;
  hsync();
  if (htid() == 0) {
    for (int w = 1; w < kWarps; ++w) mx = red[w] > mx ? red[w] : mx;
    uint16_t inv, fwd;
    if (mx == 0xFFFFu) {
      inv = fwd = 0x7E00u;
    } else {
      double d = static_cast<double>(h2f(static_cast<uint16_t>(mx)));
      d = d > 0.001953125 ? d : 0.001953125;         // 2^-9
      d = d < 4159504.0 ? d : 4159504.0;             // 65504 * 127 / 2
      inv = d2h(127.0 / d);
      fwd = d2h(d / 127.0);
    }
    A.sregs[uint64_t(seq) * A.sreg_stride + m.out_slot] = inv;
    A.sregs[uint64_t(seq) * A.sreg_stride + m.out_slot + 1] = fwd;
    red[kWarps] = inv;
  }
  hsync();
  if (has4) {
    const float s0 = h2f(static_cast<uint16_t>(red[kWarps]));
    uint32_t q = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint16_t h = static_cast<uint16_t>((j < 2 ? yv.x : yv.y) >> (16 * (j & 1)));
      q |= uint32_t(uint8_t(sat8(__fmul_rn(h2f(h), s0)))) << (8 * j);
    }
    reinterpret_cast<uint32_t*>(pptr(A, m.d, seq))[htid()] = q;
  }
}

__device__ __noinline__ void op_rows(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem, uint32_t opi) {
  if (ln_small_ok(op)) {
    op_ln_small(A, op, t, smem);
    return;
  }
  const int warp = htid() >> 5, lane = htid() & 31;
  const uint32_t seq = t.seq0, N = op.N;
  const uint32_t rpt = row_task_rows(op.kind, N), rpw = rpt / 8;   // rows per task, per warp
  float* rowbuf0 = reinterpret_cast<float*>(smem) + warp * kRowCap;
  uint32_t* pw = reinterpret_cast<uint32_t*>(smem + kWarps * kRowCap * 4) + warp * (3 * kPwMaxLeaves);
  if (t.tile * rpt + warp >= op.M) return;
  const bool legacy = op.kind == K_LN_I8 || op.kind == K_SOFTMAX_I8 || op.kind == K_MASKED_SOFTMAX_I8;
  const float in_scale = legacy ? sreg_f32(A, op.s[0], seq) : 0.f;
  const float out_scale = legacy ? sreg_f32(A, op.s[1], seq) : 0.f;
  const bool buffered = rpw * N <= kRowCap;
  // attention context
  uint32_t qrb = op.attn_qrb, vkl = op.attn_vkl, mode = op.attn_mode;
  if (op.flags & F_ATTN_DYN) {
    const uint64_t v = A.params[uint64_t(seq) * A.n_params + op.param];
    qrb = v & 0xFFFF;
    vkl = (v >> 16) & 0xFFFF;
    mode = (v >> 32) & 0x3;
  }
  const bool fp16_in = op.kind == K_LAYERNORM_F16 || op.kind == K_SOFTMAX_F16 || op.kind == K_MASKED_SOFTMAX_F16;
  if (buffered && fp16_in) {
    // every row of this warp: 8 FP16 per lane per load, four loads issued
    // before any conversion; row rr of the warp lands at rowbuf0 + rr * N
    const uint8_t* a = pptr(A, op.a, seq);
    const uint32_t ng = N / 8, total = rpw * ng;
    for (uint32_t k0 = 0; k0 < total; k0 += 128) {
      uint4 v[4];
#pragma unroll
      for (uint32_t k = 0; k < 4; ++k) {
        const uint32_t idx = k0 + lane + 32 * k, rr = idx / ng, g = idx - rr * ng;
        const uint32_t r = t.tile * rpt + warp + 8 * rr;
        if (idx < total && r < op.M) v[k] = __ldcg(reinterpret_cast<const uint4*>(a + uint64_t(r) * N * 2) + g);
      }
#pragma unroll
      for (uint32_t k = 0; k < 4; ++k) {
        const uint32_t idx = k0 + lane + 32 * k, rr = idx / ng, g = idx - rr * ng;
        const uint32_t r = t.tile * rpt + warp + 8 * rr;
        if (idx < total && r < op.M)
#pragma unroll
          for (int j = 0; j < 8; ++j) rowbuf0[rr * N + g * 8 + j] = h2f(h_at(v[k], j));
      }
    }
    __syncwarp();
  }
  for (uint32_t rr = 0; rr < rpw; ++rr) {
    const uint32_t r = t.tile * rpt + warp + 8 * rr;
    if (r >= op.M) break;
    row_one(A, op, seq, r, rowbuf0 + rr * N, pw, buffered, fp16_in, in_scale, out_scale, lane, qrb, vkl, mode);
  }
  (void)opi;
}


// Legacy fused softmax(QK^T)·V (sfu.py:323-443): one warp per query row.
__device__ __noinline__ void op_attnv(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem) {
  const int warp = htid() >> 5, lane = htid() & 31;
  const uint32_t seq = t.seq0, M = op.M, N = op.N, K = op.K;
  const uint32_t r = t.tile * 8 + warp;
  float* rowbuf = reinterpret_cast<float*>(smem) + warp * kRowCap;
  uint32_t* pw = reinterpret_cast<uint32_t*>(smem + kWarps * kRowCap * 4) + warp * (3 * kPwMaxLeaves);
  if (r >= M) return;
  const float s_qkt = sreg_f32(A, op.s[0], seq), s_v = sreg_f32(A, op.s[1], seq);
  const float s_out = sreg_f32(A, op.s[2], seq);
  const int32_t* q = reinterpret_cast<const int32_t*>(pptr(A, op.a, seq)) + uint64_t(r) * K;
  const int8_t* v = reinterpret_cast<const int8_t*>(pptr(A, op.b, seq));
  int8_t* d = reinterpret_cast<int8_t*>(pptr(A, op.d, seq));
  uint32_t qrb = op.attn_qrb, vkl = op.attn_vkl, mode = op.attn_mode;
  if (op.flags & F_ATTN_DYN) {
    const uint64_t pv = A.params[uint64_t(seq) * A.n_params + op.param];
    qrb = pv & 0xFFFF;
    vkl = (pv >> 16) & 0xFFFF;
    mode = (pv >> 32) & 0x3;
  }
  const bool masked = op.kind == K_MASKED_SOFTMAX_ATTNV;
  auto visible = [&](uint32_t j) -> bool {
    if (!masked) return true;
    bool vis = true;
    if (mode & 2) vis = vis && (j <= qrb + r);
    if (mode & 1) vis = vis && (j < vkl);
    return vis;
  };
  const bool buffered = K <= kRowCap;
  float mx = -INFINITY;
  for (uint32_t j = lane; j < K; j += 32)
    if (visible(j)) mx = fmaxf(mx, __fmul_rn(__int2float_rn(q[j]), s_qkt));
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  auto e_at = [&](uint32_t j) -> float {
    return visible(j) ? exp_f32(__fsub_rn(__fmul_rn(__int2float_rn(q[j]), s_qkt), mx)) : 0.f;
  };
  if (buffered) {
    for (uint32_t j = lane; j < K; j += 32) rowbuf[j] = e_at(j);
    __syncwarp();
  }
  auto ev = [&](uint32_t j) -> float { return buffered ? rowbuf[j] : e_at(j); };
  const float denom = warp_pairwise_sum(ev, K, pw);
  if (masked && denom == 0.f && lane == 0) raise_fault(A, DF_ZERO_DENOM, 0, seq);
  for (uint32_t n = lane; n < N; n += 32) {
    float accv = 0.f;
    for (uint32_t k = 0; k < K; ++k)
      accv = __fadd_rn(accv, __fmul_rn(__fdiv_rn(ev(k), denom), __fmul_rn(static_cast<float>(v[uint64_t(k) * N + n]), s_v)));
    d[uint64_t(r) * N + n] = s_out == 0.f ? int8_t(0) : sat8(__fdiv_rn(accv, s_out));
  }
}

// ---------------------------------------------------------------------------------
// Grid barrier with a bounded wait.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];\n" ::"l"(p));
}

// Brings the plan records task ti reads first into this SM's L1 by loading
// them with one warp (the values are discarded): the task record and its op
// record; for a chain, head-group or MAX_ABS-pair task its templates and
// their ops; for an attention pair the P.V op; for a segment-list op its
// first segments.  Done while the half waits at the grid barrier, so the
// task starts on L1 hits rather than a chain of L2 round trips.
__device__ __forceinline__ uint32_t touch_op(const ExecArgs& A, uint32_t opi, uint32_t sub) {
  // one word of each 32-byte sector of the 128-byte record (sub = sector)
  return reinterpret_cast<const uint32_t*>(A.ops + opi)[sub * 8];
}

__device__ void warm_task(const ExecArgs& A, uint32_t ti, uint32_t lane) {
  const Task t = A.tasks[ti];
  uint32_t sink = lane < 4 ? touch_op(A, t.op, lane) : 0u;
  const DevOp& op = A.ops[t.op];
  const uint32_t f2 = op.flags2;
  if (f2 & (FX_CHAINHEAD | FX_ATTNGRP | FX_MAXGRP)) {
    // lanes 4k .. 4k+3: template k's op record, then its P.V op or first segments
    const uint32_t k = lane >> 2, sub = lane & 3;
    if (k < t.aux && k < 8) {
      const uint32_t xo = A.tasks[t.tile + k].op;
      sink ^= touch_op(A, xo, sub);
      const DevOp& x = A.ops[xo];
      if (x.flags2 & FX_PV) sink ^= touch_op(A, x.seg0, sub);
      if ((x.flags & F_SEGA) && sub < x.nseg) sink ^= static_cast<uint32_t>(A.segs[x.seg0 + sub].src);
    }
  } else {
    if ((f2 & FX_PV) && lane < 4) sink ^= touch_op(A, op.seg0, lane);
    const uint32_t first = t.aux & 0xFFFFu;   // a segment-list task's first segment (0 for MAX_ABS)
    if ((op.flags & F_SEGA) && lane < 16 && first + lane < op.nseg)
      sink ^= static_cast<uint32_t>(A.segs[op.seg0 + first + lane].src);
  }
  asm volatile("" ::"r"(sink));   // keeps the loads
}

// Grid-wide barrier between levels.  The arrival counter only grows during a
// launch (the host zeroes it before each launch): a CTA arrives with a release
// add and waits, with acquire loads, until all gridDim.x CTAs of this level
// have arrived (target = (level + 1) * gridDim.x).  The same poll watches the
// fault word, so a fault anywhere stops every CTA at its next barrier.  The
// wait is bounded: running out raises DF_BARRIER_TIMEOUT.  Meanwhile warp 1 of
// each half loads the records that half's first task of the next level reads
// first into L1 (warm_task), and its lane 0 prefetches the task's tensor
// maps and hinted operand bytes.
__device__ __forceinline__ bool grid_barrier(const ExecArgs& A, uint32_t target, uint32_t next_level) {
  __syncthreads();
  __shared__ uint32_t ok;
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;\n" ::"l"(A.barrier) : "memory");
    uint32_t spins = 0, v = 0, st = 0;
    for (;;) {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(A.barrier) : "memory");
      st = *reinterpret_cast<volatile uint32_t*>(A.status);
      if (v >= target || st != 0) break;
      if (++spins > kBarrierSpinLimit) {
        raise_fault(A, DF_BARRIER_TIMEOUT, 0, 0);
        st = 1;
        break;
      }
      if (spins > 256) __nanosleep(32);
    }
    ok = st == 0;
  } else if ((htid() >> 5) == 1 && next_level < A.n_levels) {
    const uint32_t ti = A.level_off[next_level] + hidx() * gridDim.x + blockIdx.x;
    if (ti < A.level_off[next_level + 1]) warm_task(A, ti, htid() & 31);
    if (htid() == 32 && ti < A.level_off[next_level + 1]) {
      const Task tn = A.tasks[ti];
      prefetch_l1(A.ops + tn.op);
      prefetch_l1(reinterpret_cast<const uint8_t*>(A.ops + tn.op) + sizeof(DevOp) - 1);
      if (tn.aux & kTaskTcMap) {
        sm100::prefetch_tmap(A.tmaps + 2 * (tn.aux & ~kTaskTcMap));
        sm100::prefetch_tmap(A.tmaps + 2 * (tn.aux & ~kTaskTcMap) + 1);
      }
      prefetch_task_operand(A, tn);
      const uint32_t t2 = ti + gridDim.x * kHalves;
      if (t2 < A.level_off[next_level + 1]) prefetch_l1(A.tasks + t2);
    }
  }
  __syncthreads();
  return ok != 0;
}

// Runs one task on the calling half.  Meanwhile lane 0 of the last warp pulls the
// next task's op record into L1 (op records never change during a launch)
// and its hinted operand bytes into L2, and the record of the task after it
// into L1.
__device__ void run_op(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem, TcShared* tc,
                       uint32_t next_ti);

__device__ void run_task(const ExecArgs& A, uint32_t ti, uint8_t* smem, uint32_t next_ti, uint32_t next2_ti,
                         TcShared* tc) {
  const Task& t = A.tasks[ti];   // read in place (L1), not copied to local memory
  const DevOp& op = A.ops[t.op];
  // the last warp (not the tcgen05 producer or MMA thread, whose first
  // copies would wait behind this task-record load) prefetches for the next task
  if (htid() == kThreads - 32 && next_ti != 0xFFFFFFFFu) {
    const Task tn = A.tasks[next_ti];
    prefetch_l1(A.ops + tn.op);
    prefetch_l1(reinterpret_cast<const uint8_t*>(A.ops + tn.op) + sizeof(DevOp) - 1);
    if (tn.aux & kTaskTcMap) {   // a tcgen05 task: its tensor maps into the descriptor cache
      sm100::prefetch_tmap(A.tmaps + 2 * (tn.aux & ~kTaskTcMap));
      sm100::prefetch_tmap(A.tmaps + 2 * (tn.aux & ~kTaskTcMap) + 1);
    }
    if (!attn_row_candidate(op)) prefetch_task_operand(A, tn);   // else the attention op prefetches it
    if (next2_ti != 0xFFFFFFFFu) prefetch_l1(A.tasks + next2_ti);
  }
  if (op.flags2 & FX_ATTNGRP) {   // a head group: its attention pairs of this sequence in one task
    if (attn_row_ok(A, op) && t.aux >= 1 && t.aux <= kAttnGroupMax)
      op_attn_rows(A, t, t.aux, true, smem, tc, next_ti);
    else if (htid() == 0)
      raise_fault(A, DF_BAD_OP, t.op, t.seq0);
    hsync();
    return;
  }
  if (op.flags2 & FX_MAXGRP) {   // a pair of MAX_ABS + QUANT ops of this sequence
    if (t.aux == 2 && max_pair_ok(op.M, op.N, op.nseg, op.flags, op.flags2)) op_max_abs_pair(A, t, smem);
    else if (htid() == 0) raise_fault(A, DF_BAD_OP, t.op, t.seq0);
    hsync();
    return;
  }
  if (op.flags2 & FX_CHAINHEAD) {
    if (chain_vln_ok(A, t)) {   // VADD -> LAYERNORM -> MAX_ABS + QUANT of one row, in one pass
      op_chain_vln(A, t, smem);
      hsync();
      return;
    }
    // a chain: the templates' tasks in order for this sequence; generic
    // stores of one step are fenced against the next step's bulk copies
    for (uint32_t k = 0; k < t.aux; ++k) {
      Task tt = A.tasks[t.tile + k];
      tt.seq0 = t.seq0;
      run_op(A, A.ops[tt.op], tt, smem, tc, 0xFFFFFFFFu);
      sm100::fence_proxy_async();
      hsync();
    }
    return;
  }
  run_op(A, op, t, smem, tc, next_ti);
  hsync();
}

// The op of one task (or one chain step) on the calling half.
__device__ void run_op(const ExecArgs& A, const DevOp& op, const Task& t, uint8_t* smem, TcShared* tc,
                       uint32_t next_ti) {
  switch (op.kind) {
    case K_GATHER: op_gather(A, op, t); break;
    case K_DYN_LOAD:
    case K_DYN_STORE: op_dyn_copy(A, op, t, t.op); break;
    case K_DYN_STORE_MULTI: op_dyn_store_multi(A, op, t, t.op); break;
    case K_VADD_CHAIN: op_vadd_chain(A, op, t, smem, tc, t.op); break;
    case K_SREG_LOAD: op_sreg_load(A, op, t); break;
    case K_SREG_FINAL: op_sreg_final(A, op, t); break;
    case K_MATMUL:
      if (op.flags & F_TC) op_matmul_tc(A, op, t, smem, tc, t.op, next_ti);
      else if ((op.flags & F_WIDE) && attn_row_ok(A, op)) op_attn_rows(A, t, 1, false, smem, tc, next_ti);
      else if (op.flags & F_WIDE) {
        if (attn_row_candidate(op) && htid() == 32 && next_ti != 0xFFFFFFFFu) prefetch_task_operand(A, A.tasks[next_ti]);
        const uint32_t nk = op_matmul_wide(A, op, t, smem, tc, false, false);
        if ((op.flags2 & FX_PV) && nk != 0xFFFFFFFFu) {   // the P.V op, its A tile from the softmax above
          hsync();
          op_matmul_wide(A, A.ops[op.seg0], t, smem, tc, true, (op.flags2 & FX_PVPF) != 0, nk);
        }
      }
      else op_matmul(A, op, t, smem);
      break;
    case K_TRANSPOSE: op_transpose(A, op, t, smem); break;
    case K_MAX_ABS: op_max_abs(A, op, t, smem); break;
    case K_LAYERNORM_F16: case K_SOFTMAX_F16: case K_MASKED_SOFTMAX_F16:
    case K_LN_I8: case K_SOFTMAX_I8: case K_MASKED_SOFTMAX_I8:
      op_rows(A, op, t, smem, t.op);
      break;
    case K_SOFTMAX_ATTNV: case K_MASKED_SOFTMAX_ATTNV: op_attnv(A, op, t, smem); break;
    case K_REQUANT: case K_REQUANT_PC: case K_SCALE_MUL_I32: case K_SCALE_MUL_I8:
    case K_VADD_I8: case K_VADD_I32: case K_DEQUANT_ADD: case K_DEQUANT_ACCUM:
    case K_DEQUANT_SCALED: case K_QUANT: case K_VADD_F16: case K_GELU_F16: case K_GELU_I8:
      if (op.flags & F_SEGA) {
        op_seg_ew(A, op, t, smem);
      } else if (op.kind == K_QUANT && can_stage<K_QUANT>(op, t)) {
        ew_staged<K_QUANT>(A, op, t, smem, tc, t.op);
      } else if (op.kind == K_DEQUANT_SCALED && can_stage<K_DEQUANT_SCALED>(op, t)) {
        ew_staged<K_DEQUANT_SCALED>(A, op, t, smem, tc, t.op);
      } else if (op.kind == K_VADD_F16 && can_stage<K_VADD_F16>(op, t)) {
        ew_staged<K_VADD_F16>(A, op, t, smem, tc, t.op);
      } else if (op.kind == K_GELU_F16 && can_stage<K_GELU_F16>(op, t)) {
        ew_staged<K_GELU_F16>(A, op, t, smem, tc, t.op);
      } else {
        op_elementwise(A, op, t);
      }
      break;
    default:
      if (htid() == 0) raise_fault(A, DF_BAD_OP, t.op, t.seq0);
      break;
  }
}

// Shared memory of one half: max(MATMUL tiles, row buffers + pairwise scratch,
// tcgen05 stages); the two halves' regions are followed by their TcShared slots.
constexpr size_t kRowSmem = kWarps * kRowCap * 4 + kWarps * 3 * kPwMaxLeaves * 4;
static_assert(kTcStages * kTcStage <= kTcStageRegion && 2 * kTcStage128 <= kTcStageRegion,
              "tcgen05 stages outgrow their region");
constexpr size_t kTcSmem = kTcStageRegion + 1024 + kTcEpiBytes;   // + alignment of the swizzled stages, + the epilogue's vectors
constexpr size_t kExecOpSmem0 = kRowSmem > kMmSmem ? kRowSmem : kMmSmem;
constexpr size_t kExecOpSmem = kExecOpSmem0 > kTcSmem ? kExecOpSmem0 : kTcSmem;
constexpr size_t kExecSmem = kHalves * kExecOpSmem + kHalves * 128;
static_assert(sizeof(TcShared) <= 128, "TcShared outgrew its slot");
static_assert(kStageBytes <= kExecOpSmem, "element-wise staging exceeds the op shared memory");
static_assert(kWideMmSmem <= kExecOpSmem, "wide MATMUL exceeds the op shared memory");
static_assert(kWarps == int(kExecWarps) && kPwScratchBytes == kWarps * 3 * kPwMaxLeaves * 4,
              "FX_PV layout constants disagree with the executor");
static_assert(kSegTableOff + kMaxSegRuns * 12 <= kExecOpSmem, "segment table exceeds the op shared memory");
static_assert(2 * kMaxGrpRegion <= kExecOpSmem, "MAX_ABS pair regions exceed the op shared memory");
static_assert(kSegTableOff + kMaxSegRuns * 13 <= kMaxQStage && kMaxQStage + 16384 * 2 <= kExecOpSmem,
              "MAX_ABS staging overlaps the segment table or exceeds the op shared memory");
static_assert(kExecOpSmem % 1024 == 0 || kTcSmem <= kExecOpSmem, "half regions must keep the stage alignment slack");
static_assert(kExecSmem <= 227 * 1024, "executor shared memory exceeds one CTA's limit");

// A is a __grid_constant__ parameter: the op functions take its address
// without a per-thread copy in local memory.
__global__ void __launch_bounds__(kCtaThreads, 1) exec_kernel(const __grid_constant__ ExecArgs A) {
  extern __shared__ __align__(16) uint8_t smem_all[];
  uint8_t* smem = smem_all + hidx() * kExecOpSmem;
  TcShared* tcs = reinterpret_cast<TcShared*>(smem_all + kHalves * kExecOpSmem);
  TcShared* tc = tcs + hidx();
  if (threadIdx.x == 0) {
    for (int h = 0; h < kHalves; ++h) {
      for (int st = 0; st < kTcStages; ++st) {
        sm100::mbar_init(&tcs[h].full[st], 1);
        sm100::mbar_init(&tcs[h].empty[st], 1);
      }
      sm100::mbar_init(&tcs[h].stage, 1);
      sm100::mbar_init(&tcs[h].stage2, 1);
      tcs[h].phase_full = 0;
      tcs[h].phase_empty = 0;
      tcs[h].phase_stage = 0;
      tcs[h].phase_stage2 = 0;
    }
    sm100::mbar_fence_init();
  }
  if (threadIdx.x < 32) sm100::tmem_alloc(&tcs[0].tmem, kHalves * kTcCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (threadIdx.x == 0)
    for (int h = 1; h < kHalves; ++h) tcs[h].tmem = tcs[0].tmem + h * kTcCols;   // column offset
  __syncthreads();
  if (A.prof && blockIdx.x == 0 && threadIdx.x == 0) A.prof[0] = global_ns();
  // half-major: a level's first gridDim.x tasks take one half of every SM
  const uint32_t vid = hidx() * gridDim.x + blockIdx.x, vgrid = gridDim.x * kHalves;
  for (uint32_t L = 0; L < A.n_levels; ++L) {
    const uint32_t t0 = A.level_off[L], t1 = A.level_off[L + 1];
    // the half's first task of the next level follows its last task of this
    // one: its prefetches start a task early
    const uint32_t tn0 = L + 1 < A.n_levels && A.level_off[L + 1] + vid < A.level_off[L + 2]
                             ? A.level_off[L + 1] + vid : 0xFFFFFFFFu;
    for (uint32_t ti = t0 + vid; ti < t1; ti += vgrid) {
      const long long c0 = A.task_prof ? clock64() : 0;
      run_task(A, ti, smem, ti + vgrid < t1 ? ti + vgrid : tn0,
               ti + 2 * vgrid < t1 ? ti + 2 * vgrid : (ti + vgrid < t1 ? tn0 : 0xFFFFFFFFu), tc);
      if (A.task_prof && htid() == 0) A.task_prof[ti] = static_cast<uint32_t>(clock64() - c0);
    }
    if (L + 1 < A.n_levels) {
      if (!grid_barrier(A, (L + 1) * gridDim.x, L + 1)) break;
      if (threadIdx.x == 0 && blockIdx.x == 0) {
        A.status[3] = L + 1;
        if (A.prof) A.prof[L + 1] = global_ns();
      }
    }
  }
  if (A.prof) {
    // the last level ends when every CTA has finished it
    __syncthreads();
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned long long*>(&A.prof[A.n_levels]),
                                    static_cast<unsigned long long>(global_ns()));
  }
  // every MMA completed inside its task; release this CTA's TMEM columns
  sm100::tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tcs[0].tmem, kHalves * kTcCols);
  }
}

// Greedy argmax over FP16 logits (np.argmax: first maximal index; NaN wins).
__global__ void argmax_f16_kernel(const uint8_t* seq_base, uint64_t seq_stride, const uint8_t* shared_base,
                                  uint64_t shared_bytes, uint64_t addr, uint64_t count, int32_t* out) {
  const uint32_t seq = blockIdx.x;
  const uint16_t* x = reinterpret_cast<const uint16_t*>(
      addr < shared_bytes ? shared_base + addr
                          : seq_base + uint64_t(seq) * seq_stride + uint64_t(kSramUnits) * 16 + (addr - shared_bytes));
  float best = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  bool nan_seen = false;
  uint32_t nan_i = 0xFFFFFFFFu;
  for (uint32_t i = threadIdx.x; i < count; i += blockDim.x) {
    const float v = h2f(x[i]);
    if (v != v) {
      if (i < nan_i) nan_i = i;
      nan_seen = true;
    } else if (v > best || (v == best && i < bi)) {
      best = v;
      bi = i;
    }
  }
  __shared__ float sb[1024];
  __shared__ uint32_t si[1024], sn[1024];
  sb[threadIdx.x] = best;
  si[threadIdx.x] = bi;
  sn[threadIdx.x] = nan_seen ? nan_i : 0xFFFFFFFFu;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = -INFINITY;
    uint32_t idx = 0xFFFFFFFFu, ni = 0xFFFFFFFFu;
    for (uint32_t k = 0; k < blockDim.x; ++k) {
      if (sn[k] < ni) ni = sn[k];
      if (si[k] == 0xFFFFFFFFu) continue;
      if (sb[k] > b || (sb[k] == b && si[k] < idx)) { b = sb[k]; idx = si[k]; }
    }
    if (ni != 0xFFFFFFFFu) idx = ni;
    if (idx == 0xFFFFFFFFu) idx = 0;
    out[seq] = static_cast<int32_t>(idx);
  }
}

}  // namespace tac
