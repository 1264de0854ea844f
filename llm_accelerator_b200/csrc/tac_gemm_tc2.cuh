// tcgen05 INT8 GEMM on CTA pairs (cta_group::2): the same product and
// epilogues as tac_gemm_tc.cuh, with 256 x 256 output tiles computed by two
// SMs together.
//
// A cluster of two CTAs walks 256 x 256 tiles in a static round-robin.  CTA
// rank r stages rows [128 r, +128) of the tile's A block and columns
// [128 r, +128) of its B block (32 KB per 128-byte K block, six stages); rank
// 0 issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32), which reads
// both CTAs' stages and leaves each CTA's 128 result rows in its own TMEM.
// Per SM that is half the B bytes of a 128 x 256 single-SM tile for the same
// MMA work, which is what bounds the single-SM kernel (shared-memory fill and
// operand reads per MMA clock).
//   warp 0      (both CTAs) one thread issues the TMA loads; their bytes
//               complete on rank 0's stage barrier,
//   warp 1      (both) allocates the pair's TMEM; rank 0's thread issues the
//               MMAs and commits them to the stage-free and accumulator-ready
//               barriers of both CTAs (commit multicast),
//   warps 2..5  (both) epilogue of the CTA's 128 rows; each warp releases the
//               accumulator on rank 0's barrier (remote arrive).
// No TMA load uses multicast.  Every mbarrier wait is bounded; a wait that
// runs out records a fault code and the CTA winds down.
#pragma once
#include <cuda.h>
#include <cstdint>

#include "tac_gemm_tc.cuh"
#include "tac_sm100.cuh"

namespace tac {

struct Tc2Cfg {
  static constexpr int kBM = 128;                       // rows per CTA (256 per pair)
  static constexpr int kBN = 256;                       // columns per pair tile (128 staged per CTA)
  static constexpr int kBK = 128;                       // bytes of K per stage
  static constexpr int kABytes = kBM * kBK;             // 16 KB
  static constexpr int kBBytes = (kBN / 2) * kBK;       // 16 KB
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 6;
  static constexpr int kTmemCols = 2 * kBN;             // two accumulators
  static constexpr int kSmem = kStages * kStageBytes + 1024;
  static constexpr int kThreads = 192;
  static constexpr uint32_t kIdesc = sm100::idesc_i8(2 * kBM, kBN, 1);
  static constexpr uint32_t kIdescK = sm100::idesc_i8(2 * kBM, kBN, 0);
};

// p.m_tiles counts 256-row pair tiles, p.n_tiles 256-column tiles;
// p.total_units = m_tiles * n_tiles.  Launched with clusters of two CTAs.
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    TcGemmParams p) {
  using Cfg = Tc2Cfg;
  constexpr int S = Cfg::kStages;
  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) uint64_t full_bar[S], empty_bar[S], acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_ctarank();
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(&acc_full[b], 1);
      sm100::mbar_init(&acc_empty[b], 8);   // 4 epilogue warps x 2 CTAs
    }
    sm100::mbar_init(&drain_bar, 1);
    abort_flag = 0;
    sm100::mbar_fence_init();
  }
  if (warp == 1) sm100::tmem_alloc_pair(&tmem_base, Cfg::kTmemCols);
  sm100::tc_fence_before();
  sm100::cluster_sync();   // barriers and TMEM of both CTAs exist before any remote use
  sm100::tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int total = p.total_units;
  volatile int* abort_v = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs) ----
      uint32_t it = 0;
      for (int tile = cid; tile < total && !*abort_v; tile += ncl) {
        const int mb = tile % p.m_tiles, nb = tile / p.m_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!sm100::mbar_wait(&empty_bar[s], ph ^ 1, p.fault, TC_TIMEOUT_EMPTY) || *abort_v) {
            *abort_v = 1;
            break;
          }
          if (rank == 0) sm100::mbar_arrive_expect_tx(&full_bar[s], 2 * Cfg::kStageBytes);
          const uint32_t bar0 = sm100::mapa_shared(&full_bar[s], 0);
          uint8_t* st = smem + s * Cfg::kStageBytes;
          sm100::tma_load_2d_pair(st, &tm_a, kb * Cfg::kBK, mb * 2 * Cfg::kBM + int(rank) * Cfg::kBM, bar0);
          const int n0 = nb * Cfg::kBN + int(rank) * (Cfg::kBN / 2);
          sm100::tma_load_2d_pair(st + Cfg::kABytes, &tm_b, p.b_kmajor ? kb * Cfg::kBK : n0,
                                  p.b_kmajor ? n0 : kb * Cfg::kBK, bar0);
        }
        if (*abort_v) break;
      }
      if (rank == 0) {
        // both CTAs' copies of the stages still in flight land on these barriers
        const uint32_t first = it > uint32_t(S) ? it - S : 0;
        for (uint32_t j = first; j < it; ++j)
          sm100::mbar_wait(&full_bar[j % S], (j / S) & 1, p.fault, TC_TIMEOUT_DRAIN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      if (rank == 0) {
        // ---- MMA issuer (rank 0 only) ----
        uint32_t it = 0, local = 0;
        for (int tile = cid; tile < total && !*abort_v; tile += ncl, ++local) {
          const uint32_t b = local & 1, aph = (local >> 1) & 1;
          if (!sm100::mbar_wait(&acc_empty[b], aph ^ 1, p.fault, TC_TIMEOUT_ACC)) {
            *abort_v = 1;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t d = tmem + b * Cfg::kBN;
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
              // A: K-major 128-byte rows, 8-row groups 1024 B apart; B: MN-major
              // 128-byte rows (one per K), 8-K groups 1024 B apart; 32 K per MMA
              const uint64_t da = sm100::smem_desc_sw128(a_addr + k * 32, 16, 1024);
              const uint64_t db = p.b_kmajor ? sm100::smem_desc_sw128(b_addr + k * 32, 16, 1024)
                                             : sm100::smem_desc_sw128(b_addr + k * 32 * 128, 128 * Cfg::kBK, 1024);
              sm100::mma_i8_pair(d, da, db, p.b_kmajor ? Cfg::kIdescK : Cfg::kIdesc, (kb | k) != 0);
            }
            sm100::mma_commit_pair(&empty_bar[s], 0x3);
          }
          if (!ok) break;
          sm100::mma_commit_pair(&acc_full[b], 0x3);
        }
        // every MMA issued must finish before either CTA releases TMEM
        sm100::mma_commit_pair(&drain_bar, 0x3);
      }
      sm100::mbar_wait(&drain_bar, 0, p.fault, TC_TIMEOUT_DRAIN);
    }
  } else {
    // ---- epilogue: warps 2..5 own TMEM lane quadrants (warp % 4) ----
    const int q = warp & 3;
    const uint32_t acc_empty0_0 = sm100::mapa_shared(&acc_empty[0], 0), acc_empty0_1 = sm100::mapa_shared(&acc_empty[1], 0);
    uint32_t local = 0;
    for (int tile = cid; tile < total; tile += ncl, ++local) {
      const uint32_t b = local & 1, aph = (local >> 1) & 1;
      if (*abort_v) break;
      if (!sm100::mbar_wait(&acc_full[b], aph, p.fault, TC_TIMEOUT_ACC)) {
        *abort_v = 1;
        break;
      }
      __syncwarp();
      sm100::tc_fence_after();
      const int mb = tile % p.m_tiles, nb = tile / p.m_tiles;
      const int row = mb * 2 * Cfg::kBM + int(rank) * Cfg::kBM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < Cfg::kBN / 32; ++c) {
        uint32_t v[32];
        __syncwarp();   // tcgen05.ld is warp-aligned
        sm100::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + b * Cfg::kBN + c * 32, v);
        tc_store_chunk(p, row, nb * Cfg::kBN + c * 32, v);
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive_remote(b ? acc_empty0_1 : acc_empty0_0);
    }
  }

  sm100::tc_fence_before();
  sm100::cluster_sync();   // no CTA leaves while its peer may still touch its shared memory or TMEM
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem, Cfg::kTmemCols);
  }
}

}  // namespace tac
