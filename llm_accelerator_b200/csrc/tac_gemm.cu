// Stand-alone INT8 GEMM entry points (MATMUL + requant epilogues).
//
// Shapes with K and N multiples of 16 and 16-byte aligned pointers run on the
// tcgen05 kernel (tac_gemm_tc.cuh); anything else on the mma.sync tile
// (tac_gemm_sync.cuh).  Both are exact integer GEMMs, so the choice never
// changes a result.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>

#include "../../include/taccel_b200.h"
#include "tac_gemm_sync.cuh"
#include "tac_gemm_tc.cuh"

namespace {

__device__ int g_tc_gemm_fault;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D int8 map over a row-major [outer, inner] matrix, 128 x 128 boxes, 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct DeviceInfo {
  int sms = 0;
  bool smem_set[2] = {false, false};
};

DeviceInfo& device_info(int dev) {
  static DeviceInfo infos[64];
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  DeviceInfo& d = infos[dev & 63];
  if (!d.sms) cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
  return d;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Output-tile width: 256 halves the shared-memory traffic per MMA, 128 gives
// finer waves; pick the one with fewer SM-tile-columns of work on the critical
// path (128-wide tiles are charged 15% for their shared-memory bound).
// TAC_GEMM_BN=128|256 overrides the choice.
int pick_bn(int M, int N, int sms) {
  static const int forced = [] {
    const char* s = std::getenv("TAC_GEMM_BN");
    return s ? std::atoi(s) : 0;
  }();
  if (forced == 128 || forced == 256) return forced;
  const long mt = (M + 127) / 128;
  const long t128 = mt * ((N + 127) / 128), t256 = mt * ((N + 255) / 256);
  const double c128 = double((t128 + sms - 1) / sms) * 128 * 1.15;
  const double c256 = double((t256 + sms - 1) / sms) * 256;
  return c256 <= c128 ? 256 : 128;
}

template <int BN>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, tac::TcGemmParams p, DeviceInfo& di,
              cudaStream_t stream) {
  using Cfg = tac::TcGemmCfg<BN>;
  auto kern = tac::gemm_tc_kernel<BN>;
  const int slot = BN == 256 ? 1 : 0;
  if (!di.smem_set[slot]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) != cudaSuccess)
      return TAC_E_CUDA;
    di.smem_set[slot] = true;
  }
  p.m_tiles = (p.M + Cfg::kBM - 1) / Cfg::kBM;
  p.n_tiles = (p.N + BN - 1) / BN;
  p.k_blocks = (p.K + Cfg::kBK - 1) / Cfg::kBK;
  const int tiles = p.m_tiles * p.n_tiles;
  const int grid = tiles < di.sms ? tiles : di.sms;
  kern<<<grid, Cfg::kThreads, Cfg::kSmem, stream>>>(ma, mb, p);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

}  // namespace

namespace tac {

// The stand-alone GEMM dispatcher (also used by the QuaRot layer).
int gemm_launch(const int8_t* A, const int8_t* B, void* out, const uint16_t* scale, const int32_t* mult,
                const int32_t* shift, int M, int N, int K, int epi, void* stream, const uint16_t* act_scale,
                const uint16_t* bias) {
  if (!A || !B || !out || M <= 0 || N <= 0 || K <= 0) return TAC_E_ARGUMENT;
  if ((epi == tac::EPI_REQUANT_PC || epi == tac::EPI_DEQUANT_SCALED) && !scale) return TAC_E_ARGUMENT;
  if (epi == tac::EPI_DEQUANT_SCALED && !act_scale) return TAC_E_ARGUMENT;
  if (epi == tac::EPI_REQUANT_SHIFT && (!mult || !shift)) return TAC_E_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K % 16 == 0 && N % 16 == 0 && aligned16(A) && aligned16(B) && aligned16(out)) {
    CUtensorMap ma, mb;
    if (make_map(&ma, A, uint64_t(K), uint64_t(M)) && make_map(&mb, B, uint64_t(N), uint64_t(K))) {
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess) return TAC_E_CUDA;
      DeviceInfo& di = device_info(dev);
      int* fault = nullptr;
      if (cudaGetSymbolAddress(reinterpret_cast<void**>(&fault), g_tc_gemm_fault) != cudaSuccess) return TAC_E_CUDA;
      tac::TcGemmParams p{out, scale, mult, shift, M, N, K, epi, 0, 0, 0, fault, act_scale, bias};
      return pick_bn(M, N, di.sms) == 256 ? launch_tc<256>(ma, mb, p, di, st) : launch_tc<128>(ma, mb, p, di, st);
    }
  }
  tac::GemmArgs g{A, B, out, scale, mult, shift, M, N, K, epi, act_scale, bias};
  dim3 grid((N + tac::kSgBN - 1) / tac::kSgBN, (M + tac::kSgBM - 1) / tac::kSgBM);
  tac::gemm_sync_kernel<<<grid, 256, 0, st>>>(g);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

}  // namespace tac

namespace {

int launch_gemm(const int8_t* A, const int8_t* B, void* out, const uint16_t* scale, const int32_t* mult,
                const int32_t* shift, int M, int N, int K, int epi, void* stream) {
  return tac::gemm_launch(A, B, out, scale, mult, shift, M, N, K, epi, stream, nullptr, nullptr);
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

extern "C" int tac_gemm_status(int* fault_code) {
  if (cudaDeviceSynchronize() != cudaSuccess) return TAC_E_CUDA;
  int code = 0;
  if (cudaMemcpyFromSymbol(&code, g_tc_gemm_fault, sizeof(int)) != cudaSuccess) return TAC_E_CUDA;
  if (fault_code) *fault_code = code;
  if (code) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_tc_gemm_fault, &zero, sizeof(int)) != cudaSuccess) return TAC_E_CUDA;
    return TAC_E_DEVICE;
  }
  return TAC_OK;
}
