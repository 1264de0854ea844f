// QuaRot W8A16 layer: online block Walsh-Hadamard rotation of FP16
// activations, then the W8A16 dynamic matmul of the reference's W8A16 path
// (software/taccel/runtime/w8a16_simulator_reference.py:96-135: per-tensor
// max|x| -> FP16 scales -> INT8 quantisation -> INT8 x INT8 GEMM -> FP16
// dequant with per-column weight scales and bias).
//
//   fwht_kernel      one warp per (row, block): the block's elements sit in
//                    registers, E = block / 32 per lane; butterflies of
//                    half-width < E run inside a lane, wider ones pair lanes
//                    with __shfl_xor.  float32 throughout, x 1/sqrt(block),
//                    one rounding to FP16; the max |x| of the rotated rows
//                    goes to an atomicMax on the float's bits.
//   quant_act_kernel FP16 scales from that max (float64 division, one FP16
//                    rounding), then rint(x * inv) clipped to int8.
//   GEMM             the tcgen05 INT8 kernel with the DEQUANT_SCALED epilogue.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/taccel_b200.h"
#include "tac_gemm_epi.h"
#include "tac_numerics.cuh"

namespace tac {
int gemm_launch(const int8_t* A, const int8_t* B, void* out, const uint16_t* scale, const int32_t* mult,
                const int32_t* shift, int M, int N, int K, int epi, void* stream, const uint16_t* act_scale,
                const uint16_t* bias);
// The QuaRot layer's GEMM over rotated rows, quantised while staged
// (tac_quarot_fused.cuh, launched from tac_gemm.cu).
bool quarot_gemm_ok(const int8_t* W, const uint16_t* Y, int M, int N, int K);
int quarot_gemm_launch(const uint16_t* xr, const uint32_t* slots, int n_slots, const int8_t* W,
                       const uint16_t* w_scale, const uint16_t* bias, uint16_t* Y, int M, int N, int K,
                       cudaStream_t st);
}

namespace {

using tac::d2h;
using tac::f2h;
using tac::h2f;
using tac::sat8;

constexpr int kFwhtWarps = 8;

// max_bits: null (no maximum), one word for an atomicMax over the float
// bits (per_cta 0), or one word per CTA that receives the CTA's maximum
// (per_cta 1; no atomics and no zeroing before the launch).
template <int E>
__global__ void __launch_bounds__(kFwhtWarps * 32)
    fwht_kernel(const uint16_t* __restrict__ X, uint16_t* __restrict__ Y, int M, int K, float norm,
                uint32_t* max_bits, int per_cta) {
  constexpr int kBlock = 32 * E;
  const int lane = threadIdx.x & 31;
  const int nb = K / kBlock;
  const long total = long(M) * nb;
  float mx = 0.f;
  for (long w = long(blockIdx.x) * kFwhtWarps + (threadIdx.x >> 5); w < total; w += long(gridDim.x) * kFwhtWarps) {
    const long row = w / nb;
    const int bi = int(w % nb);
    const uint64_t base = uint64_t(row) * K + uint64_t(bi) * kBlock + uint64_t(lane) * E;
    float v[E];
    if constexpr (E % 8 == 0) {
#pragma unroll
      for (int q = 0; q < E / 8; ++q) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(X + base) + q);
        const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) v[8 * q + j] = h2f(uint16_t(wd[j / 2] >> (16 * (j & 1))));
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) v[j] = h2f(X[base + j]);
    }
    // butterflies inside the lane: half-width 1 .. E/2
#pragma unroll
    for (int h = 1; h < E; h <<= 1) {
#pragma unroll
      for (int i = 0; i < E; ++i) {
        if (!(i & h)) {
          const float a = v[i], c = v[i + h];
          v[i] = __fadd_rn(a, c);
          v[i + h] = __fsub_rn(a, c);
        }
      }
    }
    // butterflies across lanes: half-width E * hl; the lower lane keeps a + c, the upper a - c
#pragma unroll
    for (int hl = 1; hl < 32; hl <<= 1) {
      const bool upper = lane & hl;
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const float other = __shfl_xor_sync(0xffffffffu, v[i], hl);
        v[i] = upper ? __fsub_rn(other, v[i]) : __fadd_rn(v[i], other);
      }
    }
    uint16_t h16[E];
#pragma unroll
    for (int i = 0; i < E; ++i) {
      h16[i] = f2h(__fmul_rn(v[i], norm));
      mx = fmaxf(mx, fabsf(h2f(h16[i])));
    }
    if constexpr (E % 8 == 0) {
#pragma unroll
      for (int q = 0; q < E / 8; ++q) {
        uint32_t wd[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) wd[j] = uint32_t(h16[8 * q + 2 * j]) | (uint32_t(h16[8 * q + 2 * j + 1]) << 16);
        reinterpret_cast<uint4*>(Y + base)[q] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < E; ++j) Y[base + j] = h16[j];
    }
  }
  if (max_bits) {
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (!per_cta) {
      if (lane == 0) atomicMax(max_bits, __float_as_uint(mx));
    } else {
      __shared__ float wmax[kFwhtWarps];
      if (lane == 0) wmax[threadIdx.x >> 5] = mx;
      __syncthreads();
      if (threadIdx.x == 0) {
        float m = wmax[0];
        for (int w = 1; w < kFwhtWarps; ++w) m = fmaxf(m, wmax[w]);
        max_bits[blockIdx.x] = __float_as_uint(m);
      }
    }
  }
}

// Dynamic activation quantiser: stat[0] = bits of max |x|, stat[1] low half <- forward scale.
__global__ void quant_act_kernel(const uint16_t* __restrict__ XR, int8_t* __restrict__ XQ, long n,
                                 uint32_t* stat) {
  const float m = __uint_as_float(stat[0]);
  // max(max_abs, 2^-9) with Python's rule: a NaN maximum stays NaN
  const double me = (0.001953125 > double(m)) ? 0.001953125 : double(m);
  const float inv = h2f(d2h(127.0 / me));
  if (blockIdx.x == 0 && threadIdx.x == 0) stat[1] = d2h(me / 127.0);
  for (long i = (long(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n; i += long(gridDim.x) * blockDim.x * 8) {
    if (i + 8 <= n) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(XR + i));
      const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int8_t q = sat8(__fmul_rn(h2f(uint16_t(wd[j / 2] >> (16 * (j & 1)))), inv));
        if (j < 4) lo |= uint32_t(uint8_t(q)) << (8 * j);
        else hi |= uint32_t(uint8_t(q)) << (8 * (j - 4));
      }
      *reinterpret_cast<uint2*>(XQ + i) = make_uint2(lo, hi);
    } else {
      for (long j = i; j < n; ++j) {
        XQ[j] = sat8(__fmul_rn(h2f(XR[j]), inv));
      }
    }
  }
}

bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }
uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

int fwht_grid(int M, int K, int block) {
  const long work = long(M) * (K / block);
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long want = (work + kFwhtWarps - 1) / kFwhtWarps;
  return int(want < long(sms) * 8 ? want : long(sms) * 8);
}

int launch_fwht(const uint16_t* X, uint16_t* Y, int M, int K, int block, uint32_t* max_bits, cudaStream_t st,
                int per_cta = 0) {
  if (!X || !Y || M <= 0 || K <= 0 || !pow2(block) || block < 32 || block > 1024 || K % block) return TAC_E_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(Y)) & 15) return TAC_E_ARGUMENT;
  const float norm = static_cast<float>(1.0 / std::sqrt(double(block)));
  const int grid = fwht_grid(M, K, block);
  switch (block / 32) {
    case 1: fwht_kernel<1><<<grid, kFwhtWarps * 32, 0, st>>>(X, Y, M, K, norm, max_bits, per_cta); break;
    case 2: fwht_kernel<2><<<grid, kFwhtWarps * 32, 0, st>>>(X, Y, M, K, norm, max_bits, per_cta); break;
    case 4: fwht_kernel<4><<<grid, kFwhtWarps * 32, 0, st>>>(X, Y, M, K, norm, max_bits, per_cta); break;
    case 8: fwht_kernel<8><<<grid, kFwhtWarps * 32, 0, st>>>(X, Y, M, K, norm, max_bits, per_cta); break;
    case 16: fwht_kernel<16><<<grid, kFwhtWarps * 32, 0, st>>>(X, Y, M, K, norm, max_bits, per_cta); break;
    default: fwht_kernel<32><<<grid, kFwhtWarps * 32, 0, st>>>(X, Y, M, K, norm, max_bits, per_cta); break;
  }
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

}  // namespace

extern "C" int tac_fwht_f16(const uint16_t* X, uint16_t* Y, int M, int K, int block, void* stream) {
  return launch_fwht(X, Y, M, K, block, nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" uint64_t tac_quarot_workspace_bytes(int M, int K) {
  if (M <= 0 || K <= 0) return 0;
  const uint64_t mk = uint64_t(M) * uint64_t(K);
  // rotated FP16 rows; then their INT8 quantisation (four-launch path) or the
  // rotation CTAs' maxima (two-launch path, at most 8 per SM); scale words
  return align256(mk * 2) + align256(mk > 8192 ? mk : 8192) + 256;
}

extern "C" int tac_quarot_w8a16(const uint16_t* X, const int8_t* W, const uint16_t* w_scale, const uint16_t* bias,
                                uint16_t* Y, void* workspace, uint64_t workspace_bytes, int M, int N, int K,
                                int block, void* stream) {
  if (!X || !W || !w_scale || !Y || !workspace || M <= 0 || N <= 0 || K <= 0) return TAC_E_ARGUMENT;
  if (workspace_bytes < tac_quarot_workspace_bytes(M, K) || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return TAC_E_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint64_t mk = uint64_t(M) * uint64_t(K);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint16_t* xr = reinterpret_cast<uint16_t*>(ws);
  int8_t* xq = reinterpret_cast<int8_t*>(ws + align256(mk * 2));
  uint32_t* stat = reinterpret_cast<uint32_t*>(ws + align256(mk * 2) + align256(mk > 8192 ? mk : 8192));
  if (tac::quarot_gemm_ok(W, Y, M, N, K)) {
    // two launches: rotation with per-CTA maxima, then the GEMM that quantises while staging A
    uint32_t* slots = reinterpret_cast<uint32_t*>(xq);
    if (int s = launch_fwht(X, xr, M, K, block, slots, st, 1)) return s;
    return tac::quarot_gemm_launch(xr, slots, fwht_grid(M, K, block), W, w_scale, bias, Y, M, N, K, st);
  }
  if (cudaMemsetAsync(stat, 0, 16, st) != cudaSuccess) return TAC_E_CUDA;
  if (int s = launch_fwht(X, xr, M, K, block, stat, st)) return s;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long groups = long((mk + 7) / 8);
  const int qgrid = int(std::min<long>((groups + 255) / 256, long(sms) * 8));
  quant_act_kernel<<<qgrid, 256, 0, st>>>(xr, xq, long(mk), stat);
  if (cudaGetLastError() != cudaSuccess) return TAC_E_CUDA;
  return tac::gemm_launch(xq, W, Y, w_scale, nullptr, nullptr, M, N, K, tac::EPI_DEQUANT_SCALED, stream,
                          reinterpret_cast<const uint16_t*>(stat + 1), bias);
}
