// Portable INT8 GEMM tile (mma.sync m16n8k32) used for shapes the tcgen05
// kernel does not take (M, N or K not multiples of its tile).  C = A @ B with
// A [M,K] row-major int8, B [K,N] row-major int8, int32 accumulation, and the
// epilogues of tac_gemm.cu applied per element.
#pragma once
#include <cstdint>

#include "tac_gemm_epi.h"
#include "tac_numerics.cuh"

namespace tac {


struct GemmArgs {
  const int8_t* A;
  const int8_t* B;
  void* out;
  const uint16_t* scale_f16;   // EPI_REQUANT_PC
  const int32_t* mult;         // EPI_REQUANT_SHIFT
  const int32_t* shift;
  int M, N, K;
  int epi;
  const uint16_t* act_scale;   // EPI_DEQUANT_SCALED: one FP16 activation scale (device memory)
  const uint16_t* bias;        // EPI_DEQUANT_SCALED: per-column FP16 bias or null
};

// DEQUANT_ACCUM_FP32_SCALED arithmetic: fp16((f32(acc) * f32(pc)) * f32(act) [+ f32(bias)])
__device__ __forceinline__ uint16_t dequant_scaled(int32_t acc, float pc, float act, const uint16_t* bias, int col) {
  float y = __fmul_rn(__fmul_rn(__int2float_rn(acc), pc), act);
  if (bias) y = __fadd_rn(y, h2f(bias[col]));
  return f2h(y);
}

// clip((acc * mult + 2^(shift-1)) >> shift) in int64, floor shift; shift 0 = no rounding term.
__device__ __forceinline__ int8_t requant_shift(int32_t acc, int32_t mult, int32_t shift) {
  int64_t v = static_cast<int64_t>(acc) * mult;
  if (shift > 0) v = (v + (int64_t(1) << (shift - 1))) >> shift;
  v = v < -128 ? -128 : (v > 127 ? 127 : v);
  return static_cast<int8_t>(v);
}

__device__ __forceinline__ void gemm_store(const GemmArgs& g, int row, int col, int32_t acc) {
  if (row >= g.M || col >= g.N) return;
  const uint64_t idx = uint64_t(row) * g.N + col;
  switch (g.epi) {
    case EPI_I32:
      static_cast<int32_t*>(g.out)[idx] = acc;
      break;
    case EPI_REQUANT_PC:
      static_cast<int8_t*>(g.out)[idx] = sat8(__fmul_rn(__int2float_rn(acc), h2f(g.scale_f16[col])));
      break;
    case EPI_DEQUANT_SCALED:
      static_cast<uint16_t*>(g.out)[idx] = dequant_scaled(acc, h2f(g.scale_f16[col]), h2f(*g.act_scale), g.bias, col);
      break;
    default:
      static_cast<int8_t*>(g.out)[idx] = requant_shift(acc, g.mult[col], g.shift[col]);
      break;
  }
}

constexpr int kSgBM = 128, kSgBN = 128, kSgBK = 64;
constexpr int kSgStride = kSgBK + 16;

__global__ void __launch_bounds__(256) gemm_sync_kernel(GemmArgs g) {
  __shared__ __align__(16) uint8_t As[kSgBM * kSgStride];
  __shared__ __align__(16) uint8_t Bs[kSgBN * kSgStride];
  const int m0 = blockIdx.y * kSgBM, n0 = blockIdx.x * kSgBN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, q = lane & 3;
  int acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0;
  for (int k0 = 0; k0 < g.K; k0 += kSgBK) {
    __syncthreads();
    // A tile: 128 rows x 64 bytes, 4-byte granules (any K)
    for (int i = threadIdx.x; i < kSgBM * (kSgBK / 4); i += blockDim.x) {
      const int r = i / (kSgBK / 4), c = (i % (kSgBK / 4)) * 4;
      uint32_t v = 0;
      const int gr = m0 + r;
      if (gr < g.M) {
        const int8_t* src = g.A + uint64_t(gr) * g.K + k0 + c;
        if (k0 + c + 3 < g.K && ((reinterpret_cast<uintptr_t>(src) & 3) == 0)) {
          v = *reinterpret_cast<const uint32_t*>(src);
        } else {
          for (int b = 0; b < 4; ++b)
            if (k0 + c + b < g.K) v |= uint32_t(uint8_t(src[b])) << (8 * b);
        }
      }
      *reinterpret_cast<uint32_t*>(As + r * kSgStride + c) = v;
    }
    // B tile transposed: Bs[n][k]
    for (int i = threadIdx.x; i < kSgBK * kSgBN; i += blockDim.x) {
      const int kk = i / kSgBN, nn = i % kSgBN;
      int8_t v = 0;
      if (k0 + kk < g.K && n0 + nn < g.N) v = g.B[uint64_t(k0 + kk) * g.N + n0 + nn];
      Bs[nn * kSgStride + kk] = static_cast<uint8_t>(v);
    }
    __syncthreads();
    const uint8_t* ar0 = As + (warp * 16 + gq) * kSgStride;
    const uint8_t* ar8 = As + (warp * 16 + gq + 8) * kSgStride;
#pragma unroll
    for (int ks = 0; ks < kSgBK; ks += 32) {
      const uint32_t a0 = *reinterpret_cast<const uint32_t*>(ar0 + ks + q * 4);
      const uint32_t a1 = *reinterpret_cast<const uint32_t*>(ar8 + ks + q * 4);
      const uint32_t a2 = *reinterpret_cast<const uint32_t*>(ar0 + ks + 16 + q * 4);
      const uint32_t a3 = *reinterpret_cast<const uint32_t*>(ar8 + ks + 16 + q * 4);
#pragma unroll
      for (int ns = 0; ns < 16; ++ns) {
        const uint8_t* bc = Bs + (ns * 8 + gq) * kSgStride;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(bc + ks + q * 4);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(bc + ks + 16 + q * 4);
        asm volatile(
            "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
            : "+r"(acc[ns][0]), "+r"(acc[ns][1]), "+r"(acc[ns][2]), "+r"(acc[ns][3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
      }
    }
  }
#pragma unroll
  for (int ns = 0; ns < 16; ++ns) {
    const int col = n0 + ns * 8 + q * 2;
    const int row = m0 + warp * 16 + gq;
    gemm_store(g, row, col, acc[ns][0]);
    gemm_store(g, row, col + 1, acc[ns][1]);
    gemm_store(g, row + 8, col, acc[ns][2]);
    gemm_store(g, row + 8, col + 1, acc[ns][3]);
  }
}

}  // namespace tac
