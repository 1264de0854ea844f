// Offline weight quantisation on the GPU: the per-channel (or per-tensor)
// symmetric INT8 quantiser of software/taccel/quantizer/quantize.py:6-33,
// fused with the pad-to-16 and [out, in] -> [K, N] transpose that
// software/taccel/runtime/tiny_fixture.py:149-159 (_quantize_linear_weight)
// applies before a weight enters a program image.
//
//   row_scale_kernel   one warp per output channel: max |W[n, :]| in float32,
//                      scale = max(m, float32(1e-8)) / 127 (IEEE float32
//                      division, as NumPy computes it on a float32 array).
//                      Per-tensor mode writes the row maxima first and
//                      tensor_scale_kernel turns their maximum into one scale.
//   quant_t_kernel     a 32-channel x 128-input tile: coalesced float32 row
//                      reads, q = clip(rint(w / scale), -128, 127) with the
//                      division correctly rounded, bytes staged in shared
//                      memory (XOR-swizzled words) and written as 16-byte
//                      rows of the transposed, zero-padded [K_pad, N_pad]
//                      image; FP16 scales (round to nearest even, padded with
//                      the last channel's scale).
//   quant_rows_kernel  per-channel weights with in_features <= 1600 (every
//                      GPT-2 weight but the c_proj of the MLP): 16 whole
//                      channels staged in shared memory, their scales taken
//                      from there and each thread writing the 16 channel
//                      bytes of one input row -- W is read from DRAM once.
//
// HBM-bound: the staged kernel reads W once; the two-pass path reads it
// twice (the second read from L2 for weights below its size).  The INT8
// image is written once.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/taccel_b200.h"
#include "tac_numerics.cuh"

namespace {

using tac::f2h;

constexpr int kTileN = 32;    // channels per tile (two 16-byte output halves)
constexpr int kTileK = 128;   // input features per tile

__device__ __forceinline__ float channel_scale(float m) {
  // np.maximum(max_vals, 1e-8) with the Python float cast to float32, then / 127.0 in float32
  return __fdiv_rn(fmaxf(m, 1e-8f), 127.0f);
}

__global__ void row_scale_kernel(const float* __restrict__ W, int O, int I, int per_channel,
                                 float* __restrict__ scale_f32) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= O) return;
  const float* row = W + uint64_t(warp) * I;
  float m = 0.f;
  for (int k = lane; k < I; k += 32) m = fmaxf(m, fabsf(__ldg(row + k)));
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) scale_f32[warp] = per_channel ? channel_scale(m) : m;
}

// Per-tensor: scale_f32[0..O) holds row maxima on entry, the common scale on exit.
__global__ void tensor_scale_kernel(float* __restrict__ scale_f32, int O) {
  __shared__ float red[32];
  float m = 0.f;
  for (int n = threadIdx.x; n < O; n += blockDim.x) m = fmaxf(m, scale_f32[n]);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) red[0] = channel_scale(m);
  }
  __syncthreads();
  const float s = red[0];
  for (int n = threadIdx.x; n < O; n += blockDim.x) scale_f32[n] = s;
}

// 256 threads.  Load phase: warp w quantises channels n0 + 4w .. n0 + 4w + 3
// at k = k0 + lane + 32 i (i < 4) and stores the four bytes as one 32-bit word
// of row k of the shared tile (8 words per row; word c sits at c ^ (k & 7)).
// Store phase: thread t writes 16 bytes (words 4h .. 4h + 3, h = t & 1) of
// row k = t >> 1.
__global__ void __launch_bounds__(256) quant_t_kernel(const float* __restrict__ W, int O, int I, int Np, int Kp,
                                                      const float* __restrict__ scale_f32, int8_t* __restrict__ Q,
                                                      uint16_t* __restrict__ scale_f16) {
  __shared__ uint32_t tile[kTileK * 8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTileN, k0 = blockIdx.y * kTileK;

  if (blockIdx.y == 0 && threadIdx.x < kTileN) {
    const int n = n0 + threadIdx.x;
    if (n < Np) scale_f16[n] = f2h(scale_f32[n < O ? n : O - 1]);
  }

  float inv[4];   // not a reciprocal: the scale itself, the division stays exact
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = n0 + warp * 4 + j;
    inv[j] = n < O ? scale_f32[n] : 1.f;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int kl = lane + 32 * i, k = k0 + kl;
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + warp * 4 + j;
      int q = 0;
      if (n < O && k < I) {
        const float v = __fdiv_rn(__ldg(W + uint64_t(n) * I + k), inv[j]);
        q = __float2int_rn(v);   // round half to even; saturating for |v| >= 2^31
        q = q < -128 ? -128 : (q > 127 ? 127 : q);
      }
      word |= uint32_t(uint8_t(int8_t(q))) << (8 * j);
    }
    tile[kl * 8 + (warp ^ (kl & 7))] = word;
  }
  __syncthreads();

  const int kl = threadIdx.x >> 1, h = threadIdx.x & 1;
  const int k = k0 + kl, n = n0 + 16 * h;
  if (k < Kp && n < Np) {
    uint32_t w[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) w[c] = tile[kl * 8 + ((4 * h + c) ^ (kl & 7))];
    *reinterpret_cast<uint4*>(Q + uint64_t(k) * Np + n) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

constexpr int kRowsCh = 16;            // channels per staged CTA
constexpr int kRowsMaxIn = 1600;       // in_features bound of the staged kernel (100 KB of shared memory)

// 256 threads, kRowsCh * I floats of dynamic shared memory.  Warp w loads
// channels 2w and 2w + 1 (coalesced), keeping their max |w|; then thread t
// quantises input rows k = t, t + 256, ... of all 16 channels.
__global__ void __launch_bounds__(256) quant_rows_kernel(const float* __restrict__ W, int O, int I, int Np, int Kp,
                                                         float* __restrict__ scale_f32, int8_t* __restrict__ Q,
                                                         uint16_t* __restrict__ scale_f16) {
  extern __shared__ float rows[];
  __shared__ float sc[kRowsCh];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kRowsCh;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int c = 2 * warp + j, n = n0 + c;
    float m = 0.f;
    float* dst = rows + c * I;
    if (n < O) {
      const float* src = W + uint64_t(n) * I;
#pragma unroll 4
      for (int k = lane; k < I; k += 32) {
        const float v = __ldg(src + k);
        dst[k] = v;
        m = fmaxf(m, fabsf(v));
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) {
      const float s = channel_scale(m);
      sc[c] = s;
      if (n < O) scale_f32[n] = s;
    }
  }
  __syncthreads();
  if (threadIdx.x < kRowsCh) {
    // padding channels repeat the last real channel's scale, whichever CTA computed it
    const int n = n0 + threadIdx.x;
    if (n < O) scale_f16[n] = f2h(sc[threadIdx.x]);
  }
  for (int k = threadIdx.x; k < Kp; k += blockDim.x) {
    uint32_t w[4] = {0, 0, 0, 0};
    if (k < I) {
#pragma unroll
      for (int c = 0; c < kRowsCh; ++c) {
        if (n0 + c < O) {
          int q = __float2int_rn(__fdiv_rn(rows[c * I + k], sc[c]));
          q = q < -128 ? -128 : (q > 127 ? 127 : q);
          w[c >> 2] |= uint32_t(uint8_t(int8_t(q))) << (8 * (c & 3));
        }
      }
    }
    *reinterpret_cast<uint4*>(Q + uint64_t(k) * Np + n0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// FP16 scales of the padding channels [O, Np): the last real channel's.
__global__ void pad_scales_kernel(const float* __restrict__ scale_f32, int O, int Np, uint16_t* __restrict__ scale_f16) {
  const int n = O + threadIdx.x;
  if (n < Np) scale_f16[n] = f2h(scale_f32[O - 1]);
}

}  // namespace

extern "C" int tac_quantize_weight_i8(const float* W, int out_ch, int in_features, int per_channel, int8_t* q_kn,
                                      uint16_t* scale_f16, float* scale_f32, void* stream) {
  if (!W || !q_kn || !scale_f16 || !scale_f32 || out_ch <= 0 || in_features <= 0) return TAC_E_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(q_kn) & 15) || (reinterpret_cast<uintptr_t>(W) & 3)) return TAC_E_ARGUMENT;
  const int Np = (out_ch + 15) & ~15, Kp = (in_features + 15) & ~15;
  if (Np < out_ch || Kp < in_features) return TAC_E_ARGUMENT;   // int overflow
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (per_channel && in_features <= kRowsMaxIn) {
    const int smem = kRowsCh * in_features * int(sizeof(float));
    static bool attr_set[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return TAC_E_CUDA;
    if (!attr_set[dev & 63]) {
      if (cudaFuncSetAttribute(quant_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               kRowsCh * kRowsMaxIn * int(sizeof(float))) != cudaSuccess)
        return TAC_E_CUDA;
      attr_set[dev & 63] = true;
    }
    quant_rows_kernel<<<Np / kRowsCh, 256, smem, st>>>(W, out_ch, in_features, Np, Kp, scale_f32, q_kn, scale_f16);
    if (cudaGetLastError() != cudaSuccess) return TAC_E_CUDA;
    if (Np > out_ch) {
      pad_scales_kernel<<<1, 16, 0, st>>>(scale_f32, out_ch, Np, scale_f16);
      if (cudaGetLastError() != cudaSuccess) return TAC_E_CUDA;
    }
    return TAC_OK;
  }
  const int warps_per_block = 8;
  row_scale_kernel<<<(out_ch + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, st>>>(
      W, out_ch, in_features, per_channel, scale_f32);
  if (cudaGetLastError() != cudaSuccess) return TAC_E_CUDA;
  if (!per_channel) {
    tensor_scale_kernel<<<1, 1024, 0, st>>>(scale_f32, out_ch);
    if (cudaGetLastError() != cudaSuccess) return TAC_E_CUDA;
  }
  const dim3 grid((Np + kTileN - 1) / kTileN, (Kp + kTileK - 1) / kTileK);
  if (grid.y > 65535u) return TAC_E_ARGUMENT;
  quant_t_kernel<<<grid, 256, 0, st>>>(W, out_ch, in_features, Np, Kp, scale_f32, q_kn, scale_f16);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}
