// Weight-only INT8 GEMM on tcgen05: Y[M,N] float32 = X[M,K] FP16 x dequant(Q),
// dequant(Q)[k,n] = Q[k,n] * scale[n], plus an optional bias[n]: the W8A32
// weight-only path of the reference (INT8 weights with per-output-channel
// float32 scales, dequantised and multiplied in float32:
// software/taccel/runtime/fp32_reference.py:330-345 _weight_only_qdq_per_channel
// and its use in build_weight_only_int8_reference, :389).
//
// An INT8 weight is exact in FP16 and an FP16 x FP16 product is exact in
// float32, so Y = scale[n] * sum_k X[m,k] * Q[k,n] (+ bias) is computed as one
// kind::f16 MMA with float32 accumulation in TMEM and the per-column scale in
// the epilogue.  Against the reference's float32 products of X with the
// dequantised weight the result differs only by rounding order (float32
// accumulation), within the tolerance the tests state.
//
// One CTA per SM walks 128 x 256 output tiles; K blocks of 64 (128 bytes of
// FP16 A).  Per stage: A by TMA (128 rows x 128 bytes, 128-byte swizzle), the
// raw INT8 weights by TMA ([64 K rows][256 columns], no swizzle), and the
// converted FP16 weights, written by converter warps in the MN-major
// 128-byte-swizzled layout the MMA reads (four 64-column blocks of
// [64 K rows x 128 bytes], 16-byte chunk c of K row k at
// (k / 8) * 1024 + (k % 8) * 128 + (c ^ k % 8) * 16).  Warp roles:
//   warp 0      one thread issues the TMA loads,
//   warp 1      allocates TMEM; one thread issues tcgen05.mma kind::f16
//               (M 128, N 256, K 16) into one of two accumulators,
//   warps 2..5  epilogue: float32 accumulator * scale (+ bias) -> Y,
//   warps 6..9  convert each stage's INT8 weights to FP16.
// No load uses multicast.  Every mbarrier wait is bounded.
#pragma once
#include <cuda.h>
#include <cstdint>

#include "tac_gemm_tc.cuh"
#include "tac_sm100.cuh"

namespace tac {

constexpr int kWoBM = 128, kWoBN = 256, kWoBK = 64;          // K elements per stage
constexpr int kWoABytes = kWoBM * kWoBK * 2;                  // 16 KB FP16
constexpr int kWoRawBytes = kWoBK * kWoBN;                    // 16 KB INT8
constexpr int kWoBBytes = kWoBK * kWoBN * 2;                  // 32 KB FP16
constexpr int kWoStageBytes = kWoABytes + kWoRawBytes + kWoBBytes;
constexpr int kWoStages = 3;
constexpr int kWoSmem = kWoStages * kWoStageBytes + 1024;
constexpr int kWoThreads = 320;
constexpr int kWoConv = 128;                                  // converter threads (warps 6..9)
constexpr int kWoTmemCols = 2 * kWoBN;

// Instruction descriptor, kind::f16: FP16 A and B, float32 accumulate, A
// K-major, B MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t M, uint32_t N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (0u << 15) | (1u << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

struct WoParams {
  const float* scale;   // per column
  const float* bias;    // per column or null
  float* y;             // [M][N]
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
  int* fault;
};

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                        uint32_t accumulate) {
  const uint32_t no_mask = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}\n" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate), "r"(no_mask));
}

__global__ void __launch_bounds__(kWoThreads, 1)
    gemm_wo_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_q, WoParams p) {
  constexpr int S = kWoStages;
  extern __shared__ uint8_t dyn_smem[];
  __shared__ __align__(8) uint64_t full_bar[S], conv_bar[S], empty_bar[S], acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      sm100::mbar_init(&full_bar[s], 1);
      sm100::mbar_init(&conv_bar[s], kWoConv);
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
  if (warp == 1) sm100::tmem_alloc(&tmem_base, kWoTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = tmem_base;
  const int total = p.m_tiles * p.n_tiles;
  volatile int* abort_v = &abort_flag;
  auto stage_a = [&](uint32_t s) { return smem + s * kWoStageBytes; };
  auto stage_raw = [&](uint32_t s) { return smem + s * kWoStageBytes + kWoABytes; };
  auto stage_b = [&](uint32_t s) { return smem + s * kWoStageBytes + kWoABytes + kWoRawBytes; };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < total && !*abort_v; tile += gridDim.x) {
        const int mb = tile % p.m_tiles, nb = tile / p.m_tiles;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!sm100::mbar_wait(&empty_bar[s], ph ^ 1, p.fault, TC_TIMEOUT_EMPTY) || *abort_v) {
            *abort_v = 1;
            break;
          }
          sm100::mbar_arrive_expect_tx(&full_bar[s], kWoABytes + kWoRawBytes);
          sm100::tma_load_2d(stage_a(s), &tm_x, kb * kWoBK, mb * kWoBM, &full_bar[s]);
          sm100::tma_load_2d(stage_raw(s), &tm_q, nb * kWoBN, kb * kWoBK, &full_bar[s]);
        }
      }
      const uint32_t first = it > uint32_t(S) ? it - S : 0;
      for (uint32_t j = first; j < it; ++j)
        sm100::mbar_wait(&full_bar[j % S], (j / S) & 1, p.fault, TC_TIMEOUT_DRAIN);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t it = 0, local = 0;
      const uint32_t idesc = idesc_f16(kWoBM, kWoBN);
      for (int tile = blockIdx.x; tile < total && !*abort_v; tile += gridDim.x, ++local) {
        const uint32_t b = local & 1, aph = (local >> 1) & 1;
        if (!sm100::mbar_wait(&acc_empty[b], aph ^ 1, p.fault, TC_TIMEOUT_ACC)) {
          *abort_v = 1;
          break;
        }
        sm100::tc_fence_after();
        bool ok = true;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!sm100::mbar_wait(&conv_bar[s], ph, p.fault, TC_TIMEOUT_FULL) || *abort_v) {
            *abort_v = 1;
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t a_addr = sm100::smem_u32(stage_a(s)), b_addr = sm100::smem_u32(stage_b(s));
#pragma unroll
          for (int k = 0; k < kWoBK / 16; ++k) {
            // A: K-major 128-byte rows (64 FP16), 8-row groups 1024 B apart, 32 B per K step of 16;
            // B: MN-major 128-byte rows (64 FP16 columns) per K row, 8-row groups 1024 B apart,
            // 64-column blocks 8 KB apart, 16 K rows (2 KB) per step
            const uint64_t da = sm100::smem_desc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t db = sm100::smem_desc_sw128(b_addr + k * 16 * 128, kWoBK * 128, 1024);
            mma_f16(tmem + b * kWoBN, da, db, idesc, (kb | k) != 0);
          }
          sm100::mma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        sm100::mma_commit(&acc_full[b]);
      }
      sm100::mma_commit(&drain_bar);
      sm100::mbar_wait(&drain_bar, 0, p.fault, TC_TIMEOUT_DRAIN);
    }
  } else if (warp >= 6) {
    // ---- converters: INT8 [64][256] -> FP16 MN-major swizzled ----
    const int t = threadIdx.x - 192;
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < total && !*abort_v; tile += gridDim.x) {
      for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
        const uint32_t s = it % S, ph = (it / S) & 1;
        if (!sm100::mbar_wait(&full_bar[s], ph, p.fault, TC_TIMEOUT_FULL) || *abort_v) {
          *abort_v = 1;
          break;
        }
        const uint8_t* raw = stage_raw(s);
        uint8_t* dst = stage_b(s);
#pragma unroll 2
        for (int i = t; i < kWoRawBytes / 16; i += kWoConv) {
          const int k = i / (kWoBN / 16), n0 = (i % (kWoBN / 16)) * 16;   // 16 columns of K row k
          const uint4 v = *reinterpret_cast<const uint4*>(raw + k * kWoBN + n0);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
          uint32_t h[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int8_t lo = int8_t((w[j / 2] >> (16 * (j & 1))) & 0xFF);
            const int8_t hi = int8_t((w[j / 2] >> (16 * (j & 1) + 8)) & 0xFF);
            h[j] = uint32_t(__half_as_ushort(__short2half_rn(lo))) |
                   (uint32_t(__half_as_ushort(__short2half_rn(hi))) << 16);
          }
          const int blk = n0 >> 6, c = (n0 & 63) >> 3;   // 64-column block, 16-byte chunk in the 128-byte row
          uint8_t* row = dst + blk * (kWoBK * 128) + (k >> 3) * 1024 + (k & 7) * 128;
          *reinterpret_cast<uint4*>(row + ((c ^ (k & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
          *reinterpret_cast<uint4*>(row + (((c + 1) ^ (k & 7)) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
        }
        sm100::fence_proxy_async();   // generic writes of the FP16 weights before the MMA reads them
        sm100::mbar_arrive(&conv_bar[s]);
      }
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
      const int mb = tile % p.m_tiles, nb = tile / p.m_tiles;
      const int row = mb * kWoBM + q * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < kWoBN / 32; ++c) {
        const int col0 = nb * kWoBN + c * 32;
        uint32_t v[32];
        __syncwarp();
        sm100::tmem_ld32(tmem + (uint32_t(q * 32) << 16) + b * kWoBN + c * 32, v);
        if (col0 >= p.N) continue;
        const int cm = col0 + lane;
        const float sc_mine = cm < p.N ? p.scale[cm] : 0.f;
        const float b_mine = (p.bias && cm < p.N) ? p.bias[cm] : 0.f;
        float o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float sc = __shfl_sync(0xffffffffu, sc_mine, j);
          const float bb = __shfl_sync(0xffffffffu, b_mine, j);
          o[j] = __fadd_rn(__fmul_rn(__uint_as_float(v[j]), sc), bb);
        }
        if (row < p.M) {
          float* dst = p.y + uint64_t(row) * p.N + col0;
          if (col0 + 32 <= p.N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < p.N) dst[j] = o[j];
          }
        }
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
    sm100::tmem_dealloc(tmem, kWoTmemCols);
  }
}

}  // namespace tac
