// Stand-alone INT8 GEMM entry points (MATMUL + requant epilogues).
//
// Decode shapes (M <= 16, K and N multiples of 4, B row-major) run on the
// cluster split-K GEMV (tac_gemv_cluster.cuh).  Other shapes with K and N
// multiples of 16 and 16-byte aligned pointers run on the
// tcgen05 kernels (tac_gemm_tc.cuh; tac_gemm_tc2.cuh on CTA pairs when
// TAC_GEMM_2SM=1); anything else on the mma.sync tile
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
#include "tac_gemm_tc2.cuh"
#include "tac_gemv_cluster.cuh"
#include "tac_quarot_fused.cuh"
#include "tac_gemm_wo.cuh"

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
  int gemv_max_splits = 0;   // largest cluster the GEMV kernel may use (0: not yet queried)
  bool smem_set[3] = {false, false, false};
  int pair_clusters = -1;   // co-resident CTA pairs of gemm_tc2_kernel (0: none)
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

// 256-wide tiles of a last, partial wave run as two 128-wide units when that
// wave then still fits on the SMs (the units of one round run concurrently).
bool split_tail(long tiles, int sms) {
  const long rem = tiles % sms;
  return tiles > sms && rem > 0 && 2 * rem <= sms;
}

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
  const double c256 = split_tail(t256, sms) ? double(t256 / sms) * 256 + 128 * 1.15
                                            : double((t256 + sms - 1) / sms) * 256;
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
  p.full_units = p.total_units = tiles;
  if (BN == 256 && split_tail(tiles, di.sms)) {
    p.full_units = tiles - tiles % di.sms;
    p.total_units = p.full_units + 2 * (tiles % di.sms);
  }
  kern<<<grid, Cfg::kThreads, Cfg::kSmem, stream>>>(ma, mb, p);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

// 256 x 256 tiles on CTA pairs, opt-in (TAC_GEMM_2SM=1, read at every call),
// for shapes that fill at least one wave of 128 x 256 single-SM tiles.  At
// 4096^3 the pair kernel measured 72-76 us against 63-66 us for the
// single-SM kernel with half-width tail units: per SM both take the same
// time per 128 x 256 x K tile, and the pair kernel has no tail split.
bool use_pair(int M, int N, int sms) {
  const char* env = std::getenv("TAC_GEMM_2SM");
  if (!env || env[0] != '1' || pick_bn(M, N, sms) != 256) return false;
  return long((M + 127) / 128) * long((N + 255) / 256) >= sms;
}

int launch_tc2(const CUtensorMap& ma, const CUtensorMap& mb, tac::TcGemmParams p, DeviceInfo& di,
               cudaStream_t stream) {
  using Cfg = tac::Tc2Cfg;
  if (!di.smem_set[2]) {
    if (cudaFuncSetAttribute(tac::gemm_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) !=
        cudaSuccess)
      return TAC_E_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (di.sms / 2));
    cfg.blockDim = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tac::gemm_tc2_kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    di.pair_clusters = n < di.sms / 2 ? n : di.sms / 2;
    di.smem_set[2] = true;
  }
  if (di.pair_clusters <= 0) return -1;   // caller falls back to the single-SM kernel
  p.m_tiles = (p.M + 2 * Cfg::kBM - 1) / (2 * Cfg::kBM);
  p.n_tiles = (p.N + Cfg::kBN - 1) / Cfg::kBN;
  p.k_blocks = (p.K + Cfg::kBK - 1) / Cfg::kBK;
  p.full_units = p.total_units = p.m_tiles * p.n_tiles;
  const int clusters = p.total_units < di.pair_clusters ? p.total_units : di.pair_clusters;
  tac::gemm_tc2_kernel<<<2 * clusters, Cfg::kThreads, Cfg::kSmem, stream>>>(ma, mb, p);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

// Largest cluster of gemv_cluster_kernel the device can co-schedule: 16
// when the non-portable size is allowed and at least one such cluster fits,
// else the portable 8.  Queried once per device.
int gemv_max_splits(DeviceInfo& di) {
  if (di.gemv_max_splits) return di.gemv_max_splits;
  int best = 8;
  if (cudaFuncSetAttribute(tac::gemv_cluster_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, tac::kGcMaxSplits);
    cfg.blockDim = dim3(tac::kGcThreads);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = tac::kGcMaxSplits;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tac::gemv_cluster_kernel, &cfg) == cudaSuccess && n > 0)
      best = tac::kGcMaxSplits;
  }
  cudaGetLastError();
  di.gemv_max_splits = best;
  return best;
}

// M <= 16 rows (decode): split-K over a cluster of 8 CTAs (16 for narrow
// outputs), K rows per CTA a multiple of 32 (8 warps x 4 rows).
int launch_gemv_cluster(const tac::GcParams& base, DeviceInfo& di, cudaStream_t stream) {
  tac::GcParams p = base;
  const int col_blocks = (p.N + tac::kGcCols - 1) / tac::kGcCols;
  if (col_blocks > 65535) return -1;
  const int groups = (p.K + 31) / 32;
  const int max_splits = gemv_max_splits(di);
  // Measured on B200 (CUDA-graph replay, weights from HBM): portable 8-CTA
  // clusters are fastest once 8 splits give every SM a CTA (1 x 3072 x 768:
  // 5.8 us at 8, 7.1 at 6, 8.9 at 12 or 16); narrower outputs need 16
  // (1 x 768 x 3072: 8.5 us at 16, 14.0 at 8).
  int splits = col_blocks * 8 >= di.sms ? 8 : max_splits;
  if (splits > groups) splits = groups;
  // TAC_GEMV_SPLITS=n (1..16, read at every call) overrides the choice
  if (const char* env = std::getenv("TAC_GEMV_SPLITS")) {
    const int f = std::atoi(env);
    if (f >= 1 && f <= max_splits) splits = f < groups ? f : groups;
  }
  p.kper = ((groups + splits - 1) / splits) * 32;
  splits = (p.K + p.kper - 1) / p.kper;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(col_blocks, splits);
  cfg.blockDim = dim3(tac::kGcThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = splits;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, tac::gemv_cluster_kernel, p) == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }

}  // namespace

namespace tac {

// The stand-alone GEMM dispatcher (also used by the QuaRot layer).
// b_kmajor: B given transposed ([N, K] row-major); tcgen05 shapes only.
int gemm_launch_ex(const int8_t* A, const int8_t* B, void* out, const uint16_t* scale, const int32_t* mult,
                   const int32_t* shift, int M, int N, int K, int epi, void* stream, const uint16_t* act_scale,
                   const uint16_t* bias, int b_kmajor) {
  if (!A || !B || !out || M <= 0 || N <= 0 || K <= 0) return TAC_E_ARGUMENT;
  if ((epi == tac::EPI_REQUANT_PC || epi == tac::EPI_DEQUANT_SCALED) && !scale) return TAC_E_ARGUMENT;
  if (epi == tac::EPI_DEQUANT_SCALED && !act_scale) return TAC_E_ARGUMENT;
  if (epi == tac::EPI_REQUANT_SHIFT && (!mult || !shift)) return TAC_E_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!b_kmajor && M <= tac::kGcMaxM && K % 4 == 0 && N % 4 == 0 && aligned4(A) && aligned4(B)) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return TAC_E_CUDA;
    tac::GcParams g{A, B, out, scale, mult, shift, act_scale, bias, M, N, K, epi, 0};
    const int r = launch_gemv_cluster(g, device_info(dev), st);
    if (r >= 0) return r;
  }
  if (K % 16 == 0 && N % 16 == 0 && aligned16(A) && aligned16(B) && aligned16(out)) {
    CUtensorMap ma, mb;
    const bool mb_ok = b_kmajor ? make_map(&mb, B, uint64_t(K), uint64_t(N)) : make_map(&mb, B, uint64_t(N), uint64_t(K));
    if (make_map(&ma, A, uint64_t(K), uint64_t(M)) && mb_ok) {
      int dev = 0;
      if (cudaGetDevice(&dev) != cudaSuccess) return TAC_E_CUDA;
      DeviceInfo& di = device_info(dev);
      int* fault = nullptr;
      if (cudaGetSymbolAddress(reinterpret_cast<void**>(&fault), g_tc_gemm_fault) != cudaSuccess) return TAC_E_CUDA;
      tac::TcGemmParams p{out, scale, mult, shift, M, N, K, epi, 0, 0, 0, fault, act_scale, bias, 0, 0, b_kmajor};
      if (use_pair(M, N, di.sms)) {
        const int r = launch_tc2(ma, mb, p, di, st);
        if (r >= 0) return r;
      }
      return pick_bn(M, N, di.sms) == 256 ? launch_tc<256>(ma, mb, p, di, st) : launch_tc<128>(ma, mb, p, di, st);
    }
  }
  if (b_kmajor) return TAC_E_ARGUMENT;
  tac::GemmArgs g{A, B, out, scale, mult, shift, M, N, K, epi, act_scale, bias};
  dim3 grid((N + tac::kSgBN - 1) / tac::kSgBN, (M + tac::kSgBM - 1) / tac::kSgBM);
  tac::gemm_sync_kernel<<<grid, 256, 0, st>>>(g);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

// The QuaRot layer's GEMM (tac_quarot_fused.cuh): more than 16 rows (decode
// rows stream the weights faster on the cluster GEMV), K whole 128-byte
// blocks that fit in shared memory beside at least two W stages, N a
// multiple of 16, 16-byte aligned W and Y.
bool quarot_gemm_ok(const int8_t* W, const uint16_t* Y, int M, int N, int K) {
  return M > 16 && K > 0 && K % kQrBK == 0 && K <= kQrMaxK && qr_stages(K) >= 2 && N > 0 && N % 16 == 0 &&
         aligned16(W) && aligned16(Y);
}

int quarot_gemm_launch(const uint16_t* xr, const uint32_t* slots, int n_slots, const int8_t* W,
                       const uint16_t* w_scale, const uint16_t* bias, uint16_t* Y, int M, int N, int K,
                       cudaStream_t st) {
  static bool smem_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TAC_E_CUDA;
  DeviceInfo& di = device_info(dev);
  if (!smem_set[dev]) {
    // the largest dynamic shared memory any eligible K asks for
    if (cudaFuncSetAttribute(quarot_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kQrSmemBudget + 1024) !=
        cudaSuccess)
      return TAC_E_CUDA;
    smem_set[dev] = true;
  }
  CUtensorMap tm_w;
  if (!make_map(&tm_w, W, uint64_t(N), uint64_t(K))) return TAC_E_CUDA;
  QrParams p{};
  p.xr = xr;
  p.slots = slots;
  p.n_slots = n_slots;
  p.w_scale = w_scale;
  p.bias = bias;
  p.y = Y;
  p.M = M;
  p.N = N;
  p.K = K;
  p.m_tiles = (M + kQrBM - 1) / kQrBM;
  p.n_tiles = (N + kQrBN - 1) / kQrBN;
  p.k_blocks = K / kQrBK;
  p.stages = qr_stages(K);
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p.fault), g_tc_gemm_fault) != cudaSuccess) return TAC_E_CUDA;
  const int tiles = p.m_tiles * p.n_tiles;
  quarot_gemm_kernel<<<tiles < di.sms ? tiles : di.sms, kQrThreads, qr_smem_bytes(K), st>>>(tm_w, p);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

// Weight-only GEMM (tac_gemm_wo.cuh): X FP16 [M,K] (K a multiple of 8), Q INT8
// [K,N] (N a multiple of 16), both 16-byte aligned.
int gemm_wo_launch(const uint16_t* X, const int8_t* Q, const float* scale, const float* bias, float* Y, int M,
                   int N, int K, cudaStream_t st) {
  if (!X || !Q || !scale || !Y || M <= 0 || N <= 0 || K <= 0 || K % 8 || N % 16 || !aligned16(X) || !aligned16(Q) ||
      (reinterpret_cast<uintptr_t>(Y) & 3))
    return TAC_E_ARGUMENT;
  static bool smem_set[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TAC_E_CUDA;
  DeviceInfo& di = device_info(dev);
  if (!smem_set[dev]) {
    if (cudaFuncSetAttribute(gemm_wo_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kWoSmem) != cudaSuccess)
      return TAC_E_CUDA;
    smem_set[dev] = true;
  }
  auto fn = encode_fn();
  if (!fn) return TAC_E_CUDA;
  CUtensorMap tx, tq;
  const cuuint64_t xd[2] = {cuuint64_t(K), cuuint64_t(M)}, xs[1] = {cuuint64_t(K) * 2};
  const cuuint32_t xb[2] = {64, 128}, e1[2] = {1, 1};
  const cuuint64_t qd[2] = {cuuint64_t(N), cuuint64_t(K)}, qs[1] = {cuuint64_t(N)};
  const cuuint32_t qb[2] = {256, 64};
  if (fn(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<uint16_t*>(X), xd, xs, xb, e1,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
      fn(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(Q), qd, qs, qb, e1, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return TAC_E_CUDA;
  WoParams p{};
  p.scale = scale;
  p.bias = bias;
  p.y = Y;
  p.M = M;
  p.N = N;
  p.K = K;
  p.m_tiles = (M + kWoBM - 1) / kWoBM;
  p.n_tiles = (N + kWoBN - 1) / kWoBN;
  p.k_blocks = (K + kWoBK - 1) / kWoBK;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p.fault), g_tc_gemm_fault) != cudaSuccess) return TAC_E_CUDA;
  const int tiles = p.m_tiles * p.n_tiles;
  gemm_wo_kernel<<<tiles < di.sms ? tiles : di.sms, kWoThreads, kWoSmem, st>>>(tx, tq, p);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

// Device address of the fault word the tcgen05 GEMM kernels record timeouts
// in (read and cleared by tac_gemm_status); null on a CUDA error.
int* gemm_fault_word() {
  int* fault = nullptr;
  return cudaGetSymbolAddress(reinterpret_cast<void**>(&fault), g_tc_gemm_fault) == cudaSuccess ? fault : nullptr;
}

int gemm_launch(const int8_t* A, const int8_t* B, void* out, const uint16_t* scale, const int32_t* mult,
                const int32_t* shift, int M, int N, int K, int epi, void* stream, const uint16_t* act_scale,
                const uint16_t* bias) {
  return gemm_launch_ex(A, B, out, scale, mult, shift, M, N, K, epi, stream, act_scale, bias, 0);
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

extern "C" int tac_gemm_i8_requant_pc_bt(const int8_t* A, const int8_t* Bt, const uint16_t* scale_f16, int8_t* out,
                                         int M, int N, int K, void* stream) {
  return tac::gemm_launch_ex(A, Bt, out, scale_f16, nullptr, nullptr, M, N, K, tac::EPI_REQUANT_PC, stream, nullptr,
                             nullptr, 1);
}

extern "C" int tac_gemm_i8_i32_bt(const int8_t* A, const int8_t* Bt, int32_t* C, int M, int N, int K, void* stream) {
  return tac::gemm_launch_ex(A, Bt, C, nullptr, nullptr, nullptr, M, N, K, tac::EPI_I32, stream, nullptr, nullptr, 1);
}

extern "C" int tac_gemm_wo_f16_i8(const uint16_t* X, const int8_t* Q, const float* scale, const float* bias, float* Y,
                                  int M, int N, int K, void* stream) {
  return tac::gemm_wo_launch(X, Q, scale, bias, Y, M, N, K, static_cast<cudaStream_t>(stream));
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
