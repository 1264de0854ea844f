// tcgen05 INT8 GEMM for sm_100a: C[M,N] = A[M,K] x B[K,N], int8 inputs,
// int32 accumulation in TMEM, with the MATMUL epilogues fused into the
// TMEM read-back (plain int32, per-column FP16 requant, per-column
// multiplier + rounding shift).
//
// Layout: A row-major (K-major), B row-major [K,N] (MN-major), both moved by
// TMA with 128-byte swizzle into a ring of shared-memory stages.  One CTA per
// SM walks output tiles [128 x BN] in a static round-robin (with BN 256, the
// tiles of a last, partial wave run as half-width units); warp roles:
//   warp 0      one thread issues the TMA loads of each K block,
//   warp 1      allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN,
//               K=32 per instruction, four per 128-byte K block),
//   warps 2..5  epilogue: tcgen05.ld of their 32-lane quadrant, epilogue
//               arithmetic, stores to global memory.
// Two TMEM accumulators (2 x BN int32 columns) let the epilogue of one tile
// overlap the main loop of the next.  Out-of-range rows / columns / K bytes
// are zero-filled by TMA, so any M and any K, N that are multiples of 16 work.
#pragma once
#include <cuda.h>
#include <cstdint>

#include "tac_gemm_sync.cuh"
#include "tac_numerics.cuh"
#include "tac_sm100.cuh"

namespace tac {

// Fault codes of the tcgen05 GEMM (device flag, first one wins).
enum TcGemmFault : int { TC_OK = 0, TC_TIMEOUT_EMPTY = 1, TC_TIMEOUT_FULL = 2, TC_TIMEOUT_ACC = 3,
                         TC_TIMEOUT_DRAIN = 4 };

struct TcGemmParams {
  void* out;
  const uint16_t* scale_f16;   // EPI_REQUANT_PC
  const int32_t* mult;         // EPI_REQUANT_SHIFT
  const int32_t* shift;
  int M, N, K;
  int epi;
  int m_tiles, n_tiles, k_blocks;
  int* fault;
  const uint16_t* act_scale;   // EPI_DEQUANT_SCALED
  const uint16_t* bias;
  // Work units: tiles [0, full_units) are whole BN-wide tiles; when
  // total_units > full_units, each later tile t (the last, partial wave) is
  // two half-width units 2(t - full_units) and 2(t - full_units) + 1 (BN 256
  // only), so the last wave takes half as long.
  int full_units, total_units;
  // 0: B row-major [K, N] (MN-major, the ISA's layout); 1: B given transposed,
  // row-major [N, K] (K-major, like A)
  int b_kmajor;
};

// One unit of work: output rows [mb * 128, +128), columns [n0, n0 + width).
struct TcUnit {
  int mb, n0, width;
};

template <int BN>
__device__ __forceinline__ TcUnit tc_unit(const TcGemmParams& p, int u) {
  if (u < p.full_units) return {u % p.m_tiles, (u / p.m_tiles) * BN, BN};
  const int v = u - p.full_units, t = p.full_units + (v >> 1);
  return {t % p.m_tiles, (t / p.m_tiles) * BN + (v & 1) * (BN / 2), BN / 2};
}

template <int BN>
struct TcGemmCfg {
  static constexpr int kBM = 128;
  static constexpr int kBK = 128;                      // bytes of K per stage
  static constexpr int kABytes = kBM * kBK;            // 16 KB
  static constexpr int kBBytes = BN * kBK;             // 16 / 32 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (192 * 1024) / kStageBytes;   // 6 (BN 128) / 4 (BN 256)
  static constexpr int kTmemCols = 2 * BN;
  static constexpr int kSmem = kStages * kStageBytes + 1024;   // + alignment slack
  static constexpr int kThreads = 192;
  // kind::i8, int32 accumulate, A K-major, B MN-major
  static constexpr uint32_t kIdesc = sm100::idesc_i8(kBM, BN, 1);
  static constexpr uint32_t kIdescHalf = sm100::idesc_i8(kBM, BN / 2, 1);
  static constexpr uint32_t kIdescK = sm100::idesc_i8(kBM, BN, 0);
  static constexpr uint32_t kIdescHalfK = sm100::idesc_i8(kBM, BN / 2, 0);
};

__device__ __forceinline__ void tc_store_chunk(const TcGemmParams& p, int row, int col0, const uint32_t (&v)[32]) {
  // every lane takes part in the shuffles; only in-range rows store
  const int lane = threadIdx.x & 31;
  const bool row_ok = row < p.M;
  const bool full = col0 + 32 <= p.N;
  if (p.epi == EPI_I32) {
    if (!row_ok) return;
    int32_t* dst = static_cast<int32_t*>(p.out) + uint64_t(row) * p.N + col0;
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<int4*>(dst + j) = make_int4(int(v[j]), int(v[j + 1]), int(v[j + 2]), int(v[j + 3]));
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) dst[j] = int(v[j]);
    }
    return;
  }
  if (p.epi == EPI_DEQUANT_SCALED) {
    const int c = col0 + lane;
    const float pc_mine = c < p.N ? h2f(p.scale_f16[c]) : 0.f;
    const float b_mine = (p.bias && c < p.N) ? h2f(p.bias[c]) : 0.f;
    const float act = h2f(*p.act_scale);
    uint32_t h2[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      uint32_t w = 0;
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const float pc = __shfl_sync(0xffffffffu, pc_mine, j + t);
        const float bb = __shfl_sync(0xffffffffu, b_mine, j + t);
        float y = __fmul_rn(__fmul_rn(__int2float_rn(int(v[j + t])), pc), act);
        if (p.bias) y = __fadd_rn(y, bb);
        w |= uint32_t(f2h(y)) << (16 * t);
      }
      h2[j / 2] = w;
    }
    if (!row_ok) return;
    uint16_t* dst = static_cast<uint16_t*>(p.out) + uint64_t(row) * p.N + col0;
    if (full) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        reinterpret_cast<uint4*>(dst)[q] = make_uint4(h2[4 * q], h2[4 * q + 1], h2[4 * q + 2], h2[4 * q + 3]);
    } else {
      for (int j = 0; j < 32; ++j)
        if (col0 + j < p.N) dst[j] = uint16_t(h2[j / 2] >> (16 * (j % 2)));
    }
    return;
  }
  uint32_t packed[8];
  if (p.epi == EPI_REQUANT_PC) {
    const int c = col0 + lane;
    const float mine = c < p.N ? h2f(p.scale_f16[c]) : 0.f;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      uint32_t w = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float sc = __shfl_sync(0xffffffffu, mine, j + t);
        const int8_t q = sat8(__fmul_rn(__int2float_rn(int(v[j + t])), sc));
        w |= uint32_t(uint8_t(q)) << (8 * t);
      }
      packed[j / 4] = w;
    }
  } else {
    const int c = col0 + lane;
    const int32_t mm = c < p.N ? p.mult[c] : 0;
    const int32_t sh = c < p.N ? p.shift[c] : 0;
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      uint32_t w = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int32_t m1 = __shfl_sync(0xffffffffu, mm, j + t);
        const int32_t s1 = __shfl_sync(0xffffffffu, sh, j + t);
        w |= uint32_t(uint8_t(requant_shift(int(v[j + t]), m1, s1))) << (8 * t);
      }
      packed[j / 4] = w;
    }
  }
  if (!row_ok) return;
  int8_t* dst = static_cast<int8_t*>(p.out) + uint64_t(row) * p.N + col0;
  if (full) {
    reinterpret_cast<uint4*>(dst)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    reinterpret_cast<uint4*>(dst)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
  } else {
    for (int j = 0; j < 32; ++j)
      if (col0 + j < p.N) dst[j] = int8_t(packed[j / 4] >> (8 * (j % 4)));
  }
}

template <int BN>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   TcGemmParams p) {
  using Cfg = TcGemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S], acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&acc_full[b], 1);
      sm100::mbar_init(&acc_empty[b], 128);
    }
    sm100::mbar_init(&drain_bar, 1);
    abort_flag = 0;
    sm100::mbar_fence_init();
  }
  if (warp == 1) sm100::tmem_alloc(&tmem_base, Cfg::kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int total = p.total_units;
  volatile int* abort_v = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < total && !*abort_v; tile += gridDim.x) {
        const TcUnit un = tc_unit<BN>(p, tile);
        const int nbox = un.width / 128;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!sm100::mbar_wait(&empty_bar[s], ph ^ 1, p.fault, TC_TIMEOUT_EMPTY) || *abort_v) {
            *abort_v = 1;
            break;
          }
          uint8_t* st = smem + s * Cfg::kStageBytes;
          sm100::mbar_arrive_expect_tx(&full_bar[s], Cfg::kABytes + nbox * 128 * Cfg::kBK);
          sm100::tma_load_2d(st, &tm_a, kb * Cfg::kBK, un.mb * Cfg::kBM, &full_bar[s]);
          for (int h = 0; h < nbox; ++h) {
            // MN-major: 128 columns x 128 K rows; K-major: 128 rows of B^T x 128 K bytes
            const int c0 = p.b_kmajor ? kb * Cfg::kBK : un.n0 + h * 128;
            const int c1 = p.b_kmajor ? un.n0 + h * 128 : kb * Cfg::kBK;
            sm100::tma_load_2d(st + Cfg::kABytes + h * 128 * Cfg::kBK, &tm_b, c0, c1, &full_bar[s]);
          }
        }
        if (*abort_v) break;
      }
      // wait for the copies still in flight before the CTA may exit
      const uint32_t first = it > uint32_t(S) ? it - S : 0;
      for (uint32_t j = first; j < it; ++j)
        sm100::mbar_wait(&full_bar[j % S], (j / S) & 1, p.fault, TC_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      uint32_t it = 0, local = 0;
      for (int tile = blockIdx.x; tile < total && !*abort_v; tile += gridDim.x, ++local) {
        const uint32_t b = local & 1, aph = (local >> 1) & 1;
        if (!sm100::mbar_wait(&acc_empty[b], aph ^ 1, p.fault, TC_TIMEOUT_ACC)) {
          *abort_v = 1;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t d = tmem + b * BN;
        const uint32_t idesc = p.b_kmajor ? (tile < p.full_units ? Cfg::kIdescK : Cfg::kIdescHalfK)
                                          : (tile < p.full_units ? Cfg::kIdesc : Cfg::kIdescHalf);
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!sm100::mbar_wait(&full_bar[s], ph, p.fault, TC_TIMEOUT_FULL) || *abort_v) {
            *abort_v = 1;
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_addr = sm100::smem_u32(smem + s * Cfg::kStageBytes);
          const uint32_t b_addr = a_addr + Cfg::kABytes;
#pragma unroll
          for (int k = 0; k < Cfg::kBK / 32; ++k) {
            // A: K-major rows of 128 bytes, 8-row groups 1024 B apart; step 32 B along K
            const uint64_t da = sm100::smem_desc_sw128(a_addr + k * 32, 16, 1024);
            // B: MN-major 128-byte rows (one per K), 8-K groups 1024 B apart,
            // 128-column blocks (BN 256) 16 KB apart; step 32 K rows = 4 KB
            // K-major B: like A, 128-byte rows of B^T in 8-row groups 1024 B apart
            const uint64_t db = p.b_kmajor ? sm100::smem_desc_sw128(b_addr + k * 32, 16, 1024)
                                           : sm100::smem_desc_sw128(b_addr + k * 32 * 128, 128 * Cfg::kBK, 1024);
            sm100::mma_i8(d, da, db, idesc, (kb | k) != 0);
          }
          sm100::mma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        sm100::mma_commit(&acc_full[b]);
      }
      // every MMA issued must finish before TMEM is released
      sm100::mma_commit(&drain_bar);
      sm100::mbar_wait(&drain_bar, 0, p.fault, TC_TIMEOUT_DRAIN);
    }
  } else {
    // ---- epilogue: warps 2..5 own TMEM lane quadrants (warp % 4) ----
    const int q = warp & 3;
    uint32_t local = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++local) {
      const uint32_t b = local & 1, aph = (local >> 1) & 1;
      if (*abort_v) break;
      if (!sm100::mbar_wait(&acc_full[b], aph, p.fault, TC_TIMEOUT_ACC)) {
        *abort_v = 1;
        break;
      }
      __syncwarp();
      sm100::tc_fence_after();
      const TcUnit un = tc_unit<BN>(p, tile);
      const int row = un.mb * Cfg::kBM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < un.width / 32; ++c) {
        uint32_t v[32];
        __syncwarp();   // tcgen05.ld is warp-aligned
        sm100::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + b * BN + c * 32, v);
        tc_store_chunk(p, row, un.n0 + c * 32, v);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(&acc_empty[b]);
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace tac
