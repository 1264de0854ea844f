// QuaRot W8A16 layer, second of its two launches: the W8A16 dynamic matmul
// (software/taccel/runtime/w8a16_simulator_reference.py:96-135) over the rows
// the first launch rotated, with the activation quantisation done while the
// GEMM's A operand is staged.
//
// One CTA per 128 x 256 output tile (a persistent loop when there are more
// tiles than SMs), 12 warps:
//   warp 0      one thread streams the tile's W stages by TMA (128 K rows x
//               256 columns, two 128-column boxes, 128-byte swizzle, no
//               multicast);
//   warp 1      one thread issues tcgen05.mma kind::i8 (M 128, N 256, K 32)
//               into one TMEM accumulator, each 128-byte K block once its A
//               block and W stage have arrived;
//   warps 2..11 quantise the tile's 128 rotated FP16 rows into shared memory,
//               K block by K block, in the 128-byte-swizzled K-major layout
//               the MMA reads (16-byte chunk c of row r at (r / 8) * 1024 +
//               (r % 8) * 128 + (c ^ r % 8) * 16 of each block): rint(x * inv)
//               clipped to int8, inv the FP16 scale 127 / max(max|x|, 2^-9)
//               from the first launch's per-CTA maxima.  The loads of the
//               next block are issued before the current block is converted.
//               Then warps 2..5 apply fp16((f32(acc) * f32(w_scale[n])) *
//               f32(fwd) + bias[n]) from their TMEM lane quadrants.
// Every mbarrier wait is bounded; a wait that runs out records a fault code
// and the CTA winds down.
#pragma once
#include <cuda.h>
#include <cstdint>

#include "tac_gemm_epi.h"
#include "tac_gemm_tc.cuh"
#include "tac_sm100.cuh"

namespace tac {

constexpr int kQrBM = 128;
constexpr int kQrBN = 256;
constexpr int kQrBK = 128;                        // K bytes per A block / W stage
constexpr int kQrABlock = kQrBM * kQrBK;          // 16 KB
constexpr int kQrBStage = kQrBK * kQrBN;          // 32 KB
constexpr int kQrMaxK = 1024;
constexpr int kQrMaxStages = 4;
constexpr int kQrThreads = 384;
constexpr int kQrProducers = kQrThreads - 64;   // warps 2..11
constexpr int kQrMaxKBlocks = 1024 / 128;
constexpr int kQrItems = (128 * 8 + kQrProducers - 1) / kQrProducers;   // 16-byte chunks per producer per block
constexpr int kQrSmemBudget = 192 * 1024;          // A blocks + W stages
constexpr uint32_t kQrIdesc = sm100::idesc_i8(kQrBM, kQrBN, 1);

struct QrParams {
  const uint16_t* xr;       // rotated FP16 rows, [M][K]
  const uint32_t* slots;    // float bits of each rotation CTA's max |x|
  int n_slots;
  const uint16_t* w_scale;  // FP16 per column
  const uint16_t* bias;     // FP16 per column or null
  uint16_t* y;              // FP16 [M][N]
  int M, N, K;
  int m_tiles, n_tiles, k_blocks, stages;
  int* fault;
};

// Stages of W that fit beside a K-resident A tile.
__host__ __device__ constexpr int qr_stages(int K) {
  const int a = ((K + kQrBK - 1) / kQrBK) * kQrABlock;
  const int s = (kQrSmemBudget - a) / kQrBStage;
  return s > kQrMaxStages ? kQrMaxStages : s;
}
__host__ __device__ constexpr int qr_smem_bytes(int K) {
  return ((K + kQrBK - 1) / kQrBK) * kQrABlock + qr_stages(K) * kQrBStage + 1024;
}

__global__ void __launch_bounds__(kQrThreads, 1)
    quarot_gemm_kernel(const __grid_constant__ CUtensorMap tm_w, QrParams p) {
  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) uint64_t full_bar[kQrMaxStages], empty_bar[kQrMaxStages], acc_bar, a_bar[kQrMaxKBlocks];
  __shared__ uint32_t tmem_base;
  __shared__ float red[kQrThreads / 32];
  __shared__ float inv_s;
  __shared__ uint16_t fwd_h;
  __shared__ int abort_flag;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tile = smem;
  uint8_t* w_stages = smem + p.k_blocks * kQrABlock;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&empty_bar[s], 1);
    }
    sm100::mbar_init(&acc_bar, 1);
    for (int kb = 0; kb < p.k_blocks; ++kb) sm100::mbar_init(&a_bar[kb], kQrProducers);
    abort_flag = 0;
    sm100::mbar_fence_init();
  }
  if (warp == 1) sm100::tmem_alloc(&tmem_base, kQrBN);
  // the activation scales: the largest of the rotation launch's maxima
  float m = 0.f;
  for (int i = threadIdx.x; i < p.n_slots; i += kQrThreads) m = fmaxf(m, __uint_as_float(p.slots[i]));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  if (threadIdx.x == 0) {
    float mx = red[0];
    for (int w = 1; w < kQrThreads / 32; ++w) mx = fmaxf(mx, red[w]);
    // max(max_abs, 2^-9); the scales are divided in float64 and rounded once to FP16
    const double me = (0.001953125 > double(mx)) ? 0.001953125 : double(mx);
    inv_s = h2f(d2h(127.0 / me));
    fwd_h = d2h(me / 127.0);
  }
  __syncthreads();
  const uint32_t tmem = tmem_base;
  const float inv = inv_s;
  volatile int* abort_v = &abort_flag;
  const int total = p.m_tiles * p.n_tiles;
  uint32_t it_load = 0, it_mma = 0;        // W stages loaded (thread 0) / consumed (the MMA thread)
  int local = 0;

  auto load_stage = [&](int nb, int kb) -> bool {
    const uint32_t s = it_load % S, ph = (it_load / S) & 1;
    if (!sm100::mbar_wait(&empty_bar[s], ph ^ 1, p.fault, TC_TIMEOUT_EMPTY) || *abort_v) {
      *abort_v = 1;
      return false;
    }
    uint8_t* st = w_stages + s * kQrBStage;
    sm100::mbar_arrive_expect_tx(&full_bar[s], kQrBStage);
    for (int h = 0; h < 2; ++h)
      sm100::tma_load_2d(st + h * 128 * kQrBK, &tm_w, nb * kQrBN + h * 128, kb * kQrBK, &full_bar[s]);
    ++it_load;
    return true;
  };

  for (int tile = blockIdx.x; tile < total && !*abort_v; tile += gridDim.x, ++local) {
    const int mb = tile % p.m_tiles, nb = tile / p.m_tiles;
    if (warp == 0) {
      if (lane == 0)
        for (int kb = 0; kb < p.k_blocks; ++kb)
          if (!load_stage(nb, kb)) break;
    } else if (warp == 1) {
      if (lane == 0) {
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it_mma) {
          const uint32_t s = it_mma % S, ph = (it_mma / S) & 1;
          if (!sm100::mbar_wait(&a_bar[kb], uint32_t(local) & 1, p.fault, TC_TIMEOUT_FULL) ||
              !sm100::mbar_wait(&full_bar[s], ph, p.fault, TC_TIMEOUT_FULL) || *abort_v) {
            *abort_v = 1;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_addr = sm100::smem_u32(a_tile + kb * kQrABlock);
          const uint32_t b_addr = sm100::smem_u32(w_stages + s * kQrBStage);
#pragma unroll
          for (int k = 0; k < kQrBK / 32; ++k) {
            const uint64_t da = sm100::smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t db = sm100::smem_desc_sw128(b_addr + k * 32 * 128, 128 * kQrBK, 1024);
            sm100::mma_i8(tmem, da, db, kQrIdesc, (kb | k) != 0);
          }
          sm100::mma_commit(&empty_bar[s]);
        }
        // arrives once every MMA of the tile has completed (also on a failed
        // tile, so nothing waits for MMAs still in flight)
        sm100::mma_commit(&acc_bar);
      }
    } else {
      // ---- A producers: block kb's 1024 chunks, the next block's loads in flight ----
      const int t = threadIdx.x - 64;
      uint4 cur[kQrItems][2], nxt[kQrItems][2];
      auto fetch = [&](int kb, uint4 (&buf)[kQrItems][2]) {
#pragma unroll
        for (int j = 0; j < kQrItems; ++j) {
          const int i = t + j * kQrProducers, r = i >> 3, cc = i & 7;
          const int row = mb * kQrBM + r;
          if (i < 128 * 8 && row < p.M) {
            const uint4* src =
                reinterpret_cast<const uint4*>(p.xr + uint64_t(row) * p.K + uint64_t(kb) * kQrBK + uint64_t(cc) * 16);
            buf[j][0] = __ldcg(src);
            buf[j][1] = __ldcg(src + 1);
          } else {
            buf[j][0] = buf[j][1] = make_uint4(0, 0, 0, 0);
          }
        }
      };
      fetch(0, cur);
      for (int kb = 0; kb < p.k_blocks; ++kb) {
        if (kb + 1 < p.k_blocks) fetch(kb + 1, nxt);
#pragma unroll
        for (int j = 0; j < kQrItems; ++j) {
          const int i = t + j * kQrProducers, r = i >> 3, cc = i & 7;
          if (i >= 128 * 8) continue;
          const uint32_t h[8] = {cur[j][0].x, cur[j][0].y, cur[j][0].z, cur[j][0].w,
                                 cur[j][1].x, cur[j][1].y, cur[j][1].z, cur[j][1].w};
          uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int8_t q = sat8(__fmul_rn(h2f(uint16_t(h[e / 2] >> (16 * (e & 1)))), inv));
            w[e / 4] |= uint32_t(uint8_t(q)) << (8 * (e & 3));
          }
          uint8_t* dst = a_tile + kb * kQrABlock + (r >> 3) * 1024 + (r & 7) * 128 + ((cc ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        sm100::fence_proxy_async();   // the generic-proxy A writes, before the MMAs read them
        sm100::mbar_arrive(&a_bar[kb]);
#pragma unroll
        for (int j = 0; j < kQrItems; ++j) {
          cur[j][0] = nxt[j][0];
          cur[j][1] = nxt[j][1];
        }
      }
      if (warp < 6) {
        const int q = warp & 3;
        if (sm100::mbar_wait(&acc_bar, uint32_t(local) & 1, p.fault, TC_TIMEOUT_ACC) && !*abort_v) {
          __syncwarp();
          sm100::tc_fence_after();
          TcGemmParams ep{};
          ep.out = p.y;
          ep.scale_f16 = p.w_scale;
          ep.act_scale = &fwd_h;
          ep.bias = p.bias;
          ep.M = p.M;
          ep.N = p.N;
          ep.epi = EPI_DEQUANT_SCALED;
          const int row = mb * kQrBM + q * 32 + lane;
#pragma unroll 1
          for (int c = 0; c < kQrBN / 32; ++c) {
            if (nb * kQrBN + c * 32 >= p.N) break;
            uint32_t v[32];
            __syncwarp();
            sm100::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + c * 32, v);
            tc_store_chunk(ep, row, nb * kQrBN + c * 32, v);
          }
        } else {
          *abort_v = 1;
        }
      }
    }
    sm100::tc_fence_before();
    __syncthreads();   // A blocks and the accumulator are free for the next tile
    sm100::tc_fence_after();
  }
  // the producer's last stages (the only ones that can still be in flight)
  // must land before the CTA exits
  if (threadIdx.x == 0)
    for (uint32_t j = it_load > uint32_t(S) ? it_load - S : 0; j < it_load; ++j)
      sm100::mbar_wait(&full_bar[j % S], (j / S) & 1, p.fault, TC_TIMEOUT_DRAIN);
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, kQrBN);
  }
}

}  // namespace tac
