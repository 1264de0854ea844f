// Split-K GEMV for decode-sized MATMULs (M <= 16 rows) with the REQUANT_PC
// epilogue, whose partial sums and arrival counters live in file-scope device
// arrays, so the entry point allocates nothing.
//
// Grid: (ceil(N/64) column blocks) x (K splits).  Each CTA reduces its K range
// for 64 columns and all M rows into int32 partial sums (dp4a over 4 K bytes),
// writes them to the static workspace, and the last CTA of a column block
// (counted with an atomic) adds the splits and applies
// sat8(rint(f32(acc) * f32(scale[n]))).  Integer sums wrap identically in any
// order, so the result equals the tensor-core GEMM bit for bit.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/taccel_b200.h"
#include "tac_numerics.cuh"

namespace {

constexpr int kGvMaxRows = 16;                         // largest M
constexpr int kGvCols = 64;                            // output columns per CTA
constexpr int kGvKc = 128;                             // K bytes per chunk
constexpr int kGvThreads = 256;
constexpr size_t kGvPartialBytes = size_t(8) << 20;    // int32 partial sums: splits * M * N * 4 <= 8 MiB
constexpr int kGvMaxColBlocks = 1024;                  // N <= 65536

static __device__ __align__(256) int32_t g_gv_partial[kGvPartialBytes / 4];
static __device__ __align__(256) uint32_t g_gv_arrivals[kGvMaxColBlocks];

__global__ void __launch_bounds__(kGvThreads)
    gemv_splitk_requant_kernel(const int8_t* __restrict__ A, const int8_t* __restrict__ B,
                               const uint16_t* __restrict__ scale, int8_t* __restrict__ out, int M, int N, int K,
                               int splits, int kper, int32_t* partial, uint32_t* arrivals) {
  __shared__ __align__(16) int8_t Bs[kGvKc][kGvCols];          // 8 KB, [k][n]
  __shared__ __align__(16) int8_t As[kGvMaxRows][kGvKc];       // 2 KB, [m][k]
  __shared__ int32_t red[4][kGvMaxRows][kGvCols];              // 16 KB
  __shared__ int is_last;
  const int cb = blockIdx.x, sp = blockIdx.y;
  const int n0 = cb * kGvCols;
  const int k_begin = sp * kper;
  const int k_end = min(K, k_begin + kper);
  const int t = threadIdx.x, c = t & (kGvCols - 1), q = t >> 6;   // q: which 32-byte quarter of a chunk
  const bool vec_b = (N % 16) == 0 && (reinterpret_cast<uintptr_t>(B) & 15) == 0;

  int32_t acc[kGvMaxRows];
#pragma unroll
  for (int m = 0; m < kGvMaxRows; ++m) acc[m] = 0;

  for (int k0 = k_begin; k0 < k_end; k0 += kGvKc) {
    __syncthreads();
    for (int i = t; i < kGvKc * (kGvCols / 16); i += kGvThreads) {
      const int r = i >> 2, v = i & 3;
      const int k = k0 + r, col = n0 + v * 16;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (k < k_end) {
        const int8_t* src = B + size_t(k) * N + col;
        if (vec_b && col + 16 <= N) {
          val = __ldg(reinterpret_cast<const uint4*>(src));
        } else {
          uint32_t w[4] = {0, 0, 0, 0};
          for (int j = 0; j < 16; ++j)
            if (col + j < N) w[j >> 2] |= uint32_t(uint8_t(src[j])) << (8 * (j & 3));
          val = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      *reinterpret_cast<uint4*>(&Bs[r][v * 16]) = val;
    }
    for (int i = t; i < kGvMaxRows * kGvKc; i += kGvThreads) {
      const int m = i / kGvKc, kk = i % kGvKc, k = k0 + kk;
      As[m][kk] = (m < M && k < k_end) ? A[size_t(m) * K + k] : int8_t(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = q * 32; kk < q * 32 + 32; kk += 4) {
      const int b = int(uint8_t(Bs[kk][c])) | (int(uint8_t(Bs[kk + 1][c])) << 8) |
                    (int(uint8_t(Bs[kk + 2][c])) << 16) | (int(uint8_t(Bs[kk + 3][c])) << 24);
#pragma unroll
      for (int m = 0; m < kGvMaxRows; ++m)
        if (m < M) acc[m] = __dp4a(*reinterpret_cast<const int*>(&As[m][kk]), b, acc[m]);
    }
  }

  // combine the four K quarters, write this split's partial sums
#pragma unroll
  for (int m = 0; m < kGvMaxRows; ++m)
    if (m < M) red[q][m][c] = acc[m];
  __syncthreads();
  for (int i = t; i < M * kGvCols; i += kGvThreads) {
    const int m = i / kGvCols, cc = i % kGvCols, col = n0 + cc;
    if (col < N) {
      const uint32_t s = uint32_t(red[0][m][cc]) + uint32_t(red[1][m][cc]) + uint32_t(red[2][m][cc]) +
                         uint32_t(red[3][m][cc]);
      partial[(size_t(sp) * M + m) * N + col] = int32_t(s);
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) is_last = atomicAdd(&arrivals[cb], 1u) == uint32_t(splits - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int i = t; i < M * kGvCols; i += kGvThreads) {
    const int m = i / kGvCols, col = n0 + i % kGvCols;
    if (col >= N) continue;
    uint32_t s = 0;
    for (int j = 0; j < splits; ++j) s += uint32_t(__ldcg(&partial[(size_t(j) * M + m) * N + col]));
    out[size_t(m) * N + col] = tac::sat8(__fmul_rn(__int2float_rn(int32_t(s)), tac::h2f(scale[col])));
  }
  if (t == 0) arrivals[cb] = 0;   // leave the counter at zero for the next call
}

struct GvDevice {
  int32_t* partial = nullptr;
  uint32_t* arrivals = nullptr;
  int sms = 0;
  bool ready = false;
};

// Once per device (the device current at the call): symbol addresses of the
// static workspace, and the arrival counters cleared to zero by a memset on
// the caller's stream (ordered before the launch that follows; no device
// synchronisation).  Set-up is refused while the stream is capturing a graph:
// the symbol lookup may load the module, which a capture does not allow.
int gv_setup(cudaStream_t stream, GvDevice** out) {
  static GvDevice devs[64];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TAC_E_CUDA;
  std::lock_guard<std::mutex> lk(mu);
  GvDevice& d = devs[dev];
  if (!d.ready) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) return TAC_E_CUDA;
    if (cap != cudaStreamCaptureStatusNone) return TAC_E_UNSUPPORTED;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&d.partial), g_gv_partial) != cudaSuccess) return TAC_E_CUDA;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&d.arrivals), g_gv_arrivals) != cudaSuccess) return TAC_E_CUDA;
    if (cudaMemsetAsync(d.arrivals, 0, sizeof(uint32_t) * kGvMaxColBlocks, stream) != cudaSuccess) return TAC_E_CUDA;
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return TAC_E_CUDA;
    d.ready = true;
  }
  *out = &d;
  return TAC_OK;
}

}  // namespace

extern "C" int tac_gemv_i8_requant_pc_static(const int8_t* A, const int8_t* B, const uint16_t* scale_f16,
                                             int8_t* out, int M, int N, int K, void* stream) {
  if (!A || !B || !scale_f16 || !out || M < 1 || N < 1 || K < 1) return TAC_E_ARGUMENT;
  if (M > kGvMaxRows) return TAC_E_ARGUMENT;
  const int col_blocks = (N + kGvCols - 1) / kGvCols;
  if (col_blocks > kGvMaxColBlocks) return TAC_E_ARGUMENT;
  const size_t per_split = size_t(M) * size_t(N) * sizeof(int32_t);
  if (per_split > kGvPartialBytes) return TAC_E_ARGUMENT;
  GvDevice* d = nullptr;
  const int rc = gv_setup(static_cast<cudaStream_t>(stream), &d);
  if (rc != TAC_OK) return rc;
  // about two CTAs per SM, whole K chunks per split, bounded by the workspace
  const int chunks = (K + kGvKc - 1) / kGvKc;
  int splits = (2 * d->sms + col_blocks - 1) / col_blocks;
  splits = splits < 1 ? 1 : (splits > chunks ? chunks : splits);
  const int max_splits = int(kGvPartialBytes / per_split);
  if (splits > max_splits) splits = max_splits;
  const int kper = ((chunks + splits - 1) / splits) * kGvKc;
  splits = (K + kper - 1) / kper;
  dim3 grid(col_blocks, splits);
  gemv_splitk_requant_kernel<<<grid, kGvThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      A, B, scale_f16, out, M, N, K, splits, kper, d->partial, d->arrivals);
  if (cudaGetLastError() != cudaSuccess) {
    // a launch that did not run to its end may leave counters behind: the
    // next call repeats the set-up, which clears them
    d->ready = false;
    return TAC_E_CUDA;
  }
  return TAC_OK;
}
