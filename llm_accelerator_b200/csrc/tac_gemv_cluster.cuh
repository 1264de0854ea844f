// Decode-sized MATMUL (M <= 16 rows) for the stand-alone GEMM entry points:
// split-K over a thread-block cluster, partial sums reduced through
// distributed shared memory, so the kernel needs no global scratch.
//
// Grid (ceil(N / 128) column blocks) x (splits), clusters of (1, splits, 1),
// splits <= 16 (<= 8 where the device cannot co-schedule 16).  CTA (cb, s) covers columns [128 cb, +128) and K rows
// [s * kper, +kper).  Lane l of warp w owns columns 128 cb + 4 l .. + 3 and
// walks groups of 4 K rows (w, w + 8, ...): four 4-byte loads per group
// (a warp reads 128 contiguous bytes of a row), a byte transpose into one
// 4-row word per column, dp4a with the 4 A bytes of each row m.  The 8
// warps add into a [M][128] int32 tile in shared memory; after a cluster
// barrier the CTAs sum the splits' tiles (distributed shared memory), each
// a share of the elements, apply the epilogue and store.  Integer sums wrap identically in any order, so
// the result equals the tensor-core GEMM bit for bit.
#pragma once
#include <cooperative_groups.h>
#include <cstdint>

#include "tac_gemm_epi.h"
#include "tac_gemm_sync.cuh"   // requant_shift
#include "tac_numerics.cuh"

namespace tac {

constexpr int kGcMaxM = 16;
constexpr int kGcCols = 128;
constexpr int kGcThreads = 256;
constexpr int kGcMaxSplits = 16;   // clusters above 8 CTAs need the non-portable size attribute

struct GcParams {
  const int8_t* A;
  const int8_t* B;
  void* out;
  const uint16_t* scale;       // REQUANT_PC, DEQUANT_SCALED
  const int32_t* mult;         // REQUANT_SHIFT
  const int32_t* shift;
  const uint16_t* act_scale;   // DEQUANT_SCALED
  const uint16_t* bias;
  int M, N, K, epi, kper;
};

__device__ __forceinline__ void gc_store(const GcParams& p, int m, int n, int32_t acc) {
  const uint64_t i = uint64_t(m) * p.N + n;
  if (p.epi == EPI_I32) {
    static_cast<int32_t*>(p.out)[i] = acc;
  } else if (p.epi == EPI_REQUANT_PC) {
    static_cast<int8_t*>(p.out)[i] = sat8(__fmul_rn(__int2float_rn(acc), h2f(p.scale[n])));
  } else if (p.epi == EPI_REQUANT_SHIFT) {
    static_cast<int8_t*>(p.out)[i] = int8_t(requant_shift(acc, p.mult[n], p.shift[n]));
  } else {   // EPI_DEQUANT_SCALED
    float y = __fmul_rn(__fmul_rn(__int2float_rn(acc), h2f(p.scale[n])), h2f(*p.act_scale));
    if (p.bias) y = __fadd_rn(y, h2f(p.bias[n]));
    static_cast<uint16_t*>(p.out)[i] = f2h(y);
  }
}

__global__ void __launch_bounds__(kGcThreads) gemv_cluster_kernel(GcParams p) {
  namespace cg = cooperative_groups;
  __shared__ int32_t red[kGcMaxM * kGcCols];   // 8 KB
  cg::cluster_group cl = cg::this_cluster();
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int M = p.M, N = p.N, K = p.K;
  const int col = blockIdx.x * kGcCols + lane * 4;   // this lane's first column
  const int k_begin = blockIdx.y * p.kper;
  const int k_end = min(K, k_begin + p.kper);        // a multiple of 4 (K and kper are)
  for (int i = t; i < M * kGcCols; i += kGcThreads) red[i] = 0;

  int32_t acc[kGcMaxM][4];
#pragma unroll
  for (int m = 0; m < kGcMaxM; ++m)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[m][c] = 0;

  const bool col_ok = col < N;   // N % 4 == 0: the lane's 4 columns are all in range or all out
#pragma unroll 4
  for (int k = k_begin + 4 * warp; k < k_end; k += 4 * (kGcThreads / 32)) {
    uint32_t b[4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
      b[r] = col_ok ? __ldg(reinterpret_cast<const uint32_t*>(p.B + uint64_t(k + r) * N + col)) : 0u;
    // byte c of b[r] is B[k + r][col + c]; bc[c] gathers B[k .. k + 3][col + c]
    const uint32_t lo01 = __byte_perm(b[0], b[1], 0x5140), hi01 = __byte_perm(b[0], b[1], 0x7362);
    const uint32_t lo23 = __byte_perm(b[2], b[3], 0x5140), hi23 = __byte_perm(b[2], b[3], 0x7362);
    const uint32_t bc[4] = {__byte_perm(lo01, lo23, 0x5410), __byte_perm(lo01, lo23, 0x7632),
                            __byte_perm(hi01, hi23, 0x5410), __byte_perm(hi01, hi23, 0x7632)};
#pragma unroll
    for (int m = 0; m < kGcMaxM; ++m) {
      if (m < M) {
        const int a4 = __ldg(reinterpret_cast<const int*>(p.A + uint64_t(m) * K + k));
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = __dp4a(a4, int(bc[c]), acc[m][c]);
      }
    }
  }
  __syncthreads();   // red cleared
#pragma unroll
  for (int m = 0; m < kGcMaxM; ++m)
    if (m < M)
#pragma unroll
      for (int c = 0; c < 4; ++c) atomicAdd(&red[m * kGcCols + lane * 4 + c], acc[m][c]);

  cl.sync();   // every split's tile is complete and visible to the cluster
  // the cluster's CTAs share the final sums: rank r takes 256-element chunks r, r + splits, ...
  const int splits = int(cl.num_blocks()), rank = int(cl.block_rank());
  for (int i = kGcThreads * rank + t; i < M * kGcCols; i += kGcThreads * splits) {
    const int m = i / kGcCols, n = blockIdx.x * kGcCols + i % kGcCols;
    if (n >= N) continue;
    uint32_t s = 0;
    for (int r = 0; r < splits; ++r) s += uint32_t(cl.map_shared_rank(red, r)[i]);
    gc_store(p, m, n, int32_t(s));
  }
  cl.sync();   // no CTA leaves while another may still read its tile
}

}  // namespace tac
