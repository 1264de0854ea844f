// Stand-alone INT8 GEMM entry points (MATMUL + requant epilogues).
#include <cuda_runtime.h>

#include "../../include/taccel_b200.h"
#include "tac_gemm_sync.cuh"

namespace {

int launch_gemm(const int8_t* A, const int8_t* B, void* out, const uint16_t* scale, const int32_t* mult,
                const int32_t* shift, int M, int N, int K, int epi, void* stream) {
  if (!A || !B || !out || M <= 0 || N <= 0 || K <= 0) return TAC_E_ARGUMENT;
  if (epi == tac::EPI_REQUANT_PC && !scale) return TAC_E_ARGUMENT;
  if (epi == tac::EPI_REQUANT_SHIFT && (!mult || !shift)) return TAC_E_ARGUMENT;
  tac::GemmArgs g{A, B, out, scale, mult, shift, M, N, K, epi};
  dim3 grid((N + tac::kSgBN - 1) / tac::kSgBN, (M + tac::kSgBM - 1) / tac::kSgBM);
  tac::gemm_sync_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(g);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

}  // namespace

extern "C" int tac_gemm_i8_i32(const int8_t* A, const int8_t* B, int32_t* C, int M, int N, int K, void* stream) {
  return launch_gemm(A, B, C, nullptr, nullptr, nullptr, M, N, K, tac::EPI_I32, stream);
}

extern "C" int tac_gemm_i8_requant_pc(const int8_t* A, const int8_t* B, const uint16_t* scale_f16, int8_t* out,
                                      int M, int N, int K, void* stream) {
  return launch_gemm(A, B, out, scale_f16, nullptr, nullptr, M, N, K, tac::EPI_REQUANT_PC, stream);
}

extern "C" int tac_gemm_i8_requant_shift(const int8_t* A, const int8_t* B, const int32_t* mult,
                                         const int32_t* shift, int8_t* out, int M, int N, int K, void* stream) {
  return launch_gemm(A, B, out, nullptr, mult, shift, M, N, K, tac::EPI_REQUANT_SHIFT, stream);
}
