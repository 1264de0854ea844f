// Engine: device machine state for a batch of sequences and the C ABI that
// runs compiled plans on it (include/taccel_b200.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include "tac_exec.cuh"
#include "tac_tmap.h"
#include "tac_program.h"

struct tac_engine {
  int device = 0;
  int batch = 1;
  uint64_t dram_bytes = 0, shared_bytes = 0;
  uint64_t rw_bytes = 0;        // per-sequence writable DRAM image
  uint64_t arena_bytes = 0;     // per-sequence arena capacity
  uint64_t seq_stride = 0;      // bytes per sequence block
  uint8_t* d_seq = nullptr;
  uint8_t* d_shared = nullptr;
  uint16_t* d_sregs = nullptr;
  uint32_t sreg_stride = 16;
  uint64_t* d_params = nullptr;
  size_t params_cap = 0;
  uint32_t* d_status = nullptr;  // [0..3] fault info, [4..5] barrier
  int n_sms = 0;
  int grid = 0;
  std::vector<uint64_t> h_params;
  // pinned staging ring for parameter uploads: slot i is reusable once its
  // copy (event i) has completed, so several runs can be in flight
  static constexpr int kRing = 4;
  uint64_t* h_pinned = nullptr;
  size_t pinned_cap = 0;        // words per slot
  cudaEvent_t ring_ev[kRing] = {};
  uint64_t* d_prof = nullptr;     // per-level timestamps when profiling is on
  size_t prof_cap = 0;
  int profiling = 0;              // 0 off, 1 levels, 2 levels + task cycles
  uint32_t prof_levels = 0;
  uint32_t* d_task_prof = nullptr;   // per-task SM cycles (profiling mode 2)
  size_t task_prof_cap = 0;
  uint64_t prof_tasks = 0;
  bool ring_used[kRing] = {};
  int ring_next = 0;
};

namespace {

using namespace tac;

constexpr uint64_t kSramBytes = uint64_t(kSramUnits) * 16;

int cuda_fail(cudaError_t e, tac_fault* f, const char* what) {
  if (e == cudaSuccess) return TAC_OK;
  if (f) {
    std::memset(f, 0, sizeof(*f));
    f->status = TAC_E_CUDA;
    std::snprintf(f->message, sizeof(f->message), "%s: %s", what, cudaGetErrorString(e));
  }
  return TAC_E_CUDA;
}

#define CK(expr, f, what) do { cudaError_t _e = (expr); if (_e != cudaSuccess) return cuda_fail(_e, f, what); } while (0)

uint64_t round_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

int set_fault(tac_fault* f, int status, const char* msg, uint64_t pc = 0) {
  if (f) {
    std::memset(f, 0, sizeof(*f));
    f->status = status;
    f->pc = pc;
    std::snprintf(f->message, sizeof(f->message), "%s", msg);
  }
  return status;
}

// Grows the per-sequence arena, keeping SRAM and writable-DRAM contents.
int ensure_arena(tac_engine* e, uint64_t need_bytes, tac_fault* f) {
  if (need_bytes <= e->arena_bytes) return TAC_OK;
  uint64_t new_arena = std::max<uint64_t>(need_bytes, e->arena_bytes * 2);
  new_arena = round_up(new_arena, 1 << 20);
  const uint64_t new_stride = round_up(kSramBytes + e->rw_bytes + new_arena, 256);
  uint8_t* nb = nullptr;
  CK(cudaMalloc(&nb, new_stride * e->batch), f, "cudaMalloc arena");
  const uint64_t keep = kSramBytes + e->rw_bytes;
  CK(cudaDeviceSynchronize(), f, "sync");
  CK(cudaMemcpy2D(nb, new_stride, e->d_seq, e->seq_stride, keep, e->batch, cudaMemcpyDeviceToDevice), f,
     "copy state");
  CK(cudaFree(e->d_seq), f, "cudaFree");
  e->d_seq = nb;
  e->seq_stride = new_stride;
  e->arena_bytes = new_arena;
  return TAC_OK;
}

int ensure_sregs(tac_engine* e, uint32_t slots, tac_fault* f) {
  const uint32_t need = 16 + slots;
  if (need <= e->sreg_stride) return TAC_OK;
  const uint32_t ns = static_cast<uint32_t>(round_up(std::max<uint32_t>(need, e->sreg_stride * 2), 64));
  uint16_t* nb = nullptr;
  CK(cudaMalloc(&nb, size_t(ns) * 2 * e->batch), f, "cudaMalloc sregs");
  CK(cudaMemset(nb, 0, size_t(ns) * 2 * e->batch), f, "memset sregs");
  CK(cudaDeviceSynchronize(), f, "sync");
  CK(cudaMemcpy2D(nb, size_t(ns) * 2, e->d_sregs, size_t(e->sreg_stride) * 2, 32, e->batch,
                  cudaMemcpyDeviceToDevice), f, "copy sregs");
  CK(cudaFree(e->d_sregs), f, "cudaFree");
  e->d_sregs = nb;
  e->sreg_stride = ns;
  return TAC_OK;
}

int upload_program(tac_engine* e, tac_program* p, tac_fault* f) {
  if (p->d_blob && p->device == e->device) return TAC_OK;
  if (p->d_blob) {
    cudaFree(p->d_blob);
    p->d_blob = nullptr;
  }
  const uint64_t s_ops = p->ops.size() * sizeof(DevOp), s_segs = p->segs.size() * sizeof(Segment);
  const uint64_t s_tasks = p->tasks.size() * sizeof(Task), s_lv = p->level_off.size() * 4;
  p->off_ops = 0;
  p->off_segs = round_up(s_ops, 256);
  p->off_tasks = p->off_segs + round_up(s_segs, 256);
  p->off_levels = p->off_tasks + round_up(s_tasks, 256);
  const uint64_t total = p->off_levels + round_up(s_lv, 256) + 256;
  std::vector<uint8_t> blob(total, 0);
  if (s_ops) std::memcpy(blob.data() + p->off_ops, p->ops.data(), s_ops);
  if (s_segs) std::memcpy(blob.data() + p->off_segs, p->segs.data(), s_segs);
  if (s_tasks) std::memcpy(blob.data() + p->off_tasks, p->tasks.data(), s_tasks);
  std::memcpy(blob.data() + p->off_levels, p->level_off.data(), s_lv);
  CK(cudaMalloc(&p->d_blob, total), f, "cudaMalloc program");
  CK(cudaMemcpy(p->d_blob, blob.data(), total, cudaMemcpyHostToDevice), f, "upload program");
  p->device = e->device;
  return TAC_OK;
}

// TMA maps of the tcgen05 MATMULs for this engine's memory layout: A as
// [batch][M][K] over the sequences' blocks (128-byte swizzle, box 128 B x M rows
// x 128/M sequences), the shared weights B as [K][N] (64-byte swizzle, box 64 x
// 128).  Rebuilt when the layout changes (arena growth, another engine).
int ensure_maps(tac_engine* e, tac_program* p, tac_fault* f) {
  if (!p->n_tc) return TAC_OK;
  const uint64_t key[4] = {reinterpret_cast<uint64_t>(e->d_seq), e->seq_stride,
                           reinterpret_cast<uint64_t>(e->d_shared), uint64_t(e->batch)};
  if (p->d_maps && std::memcmp(key, p->maps_key, sizeof(key)) == 0) return TAC_OK;
  std::vector<CUtensorMap> maps(2 * size_t(p->n_tc));
  for (const DevOp& op : p->ops) {
    if (!(op.kind == K_MATMUL && (op.flags & F_TC))) continue;
    const uint8_t* a = static_cast<const uint8_t*>(e->d_seq) + (op.a << 4);
    const uint8_t* b = static_cast<const uint8_t*>(e->d_shared) + ((op.b & ~kSharedBit) << 4);
    const cuuint64_t adims[3] = {op.K, op.M, cuuint64_t(e->batch)};
    const cuuint64_t astr[2] = {op.K, e->seq_stride};
    // resident and split tasks load their sequences' rows only (q_rows, a multiple of 8)
    const cuuint32_t abox[3] = {128, op.M, op.q_rows ? op.q_rows / op.M : 128 / op.M};
    const bool wide = (op.flags & F_TC128) != 0;   // 128-column tiles: 128-byte swizzle, else 64
    const cuuint64_t bdims[2] = {op.N, op.K};
    const cuuint64_t bstr[1] = {op.N};
    const cuuint32_t bbox[2] = {wide ? 128u : 64u, 128};
    if (!tmap_encode_u8(&maps[2 * op.seg0], a, 3, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !tmap_encode_u8(&maps[2 * op.seg0 + 1], b, 2, bdims, bstr, bbox,
                        wide ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
      return set_fault(f, TAC_E_CUDA, "cuTensorMapEncodeTiled rejected a MATMUL operand map");
  }
  if (!p->d_maps) CK(cudaMalloc(&p->d_maps, maps.size() * sizeof(CUtensorMap)), f, "cudaMalloc tensor maps");
  else CK(cudaDeviceSynchronize(), f, "wait for runs using the old maps");
  CK(cudaMemcpy(p->d_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice), f,
     "upload tensor maps");
  std::memcpy(p->maps_key, key, sizeof(key));
  return TAC_OK;
}

uint32_t insn_bits(uint64_t w, int shift, int width) { return static_cast<uint32_t>((w >> shift) & ((1ull << width) - 1)); }

// Decodes one sequence's runtime words into parameters and checks them
// against the ranges the plan was compiled for.
int check_params(const tac_program* p, const uint64_t* params, tac_fault* f);

int decode_params(const tac_program* p, const uint64_t* words, uint64_t* params, tac_fault* f) {
  for (size_t i = 0; i < p->vars.size(); ++i) {
    const VarInfo& v = p->vars[i];
    if (v.kind == 0) {
      const uint64_t lo = words[v.word0], hi = words[v.word0 + 1];
      if (insn_bits(lo, 59, 5) != OP_SET_ADDR_LO || insn_bits(hi, 59, 5) != OP_SET_ADDR_HI ||
          insn_bits(lo, 57, 2) != v.addr_reg || insn_bits(hi, 57, 2) != v.addr_reg)
        return set_fault(f, TAC_E_RECOMPILE, "runtime SET_ADDR word changed its opcode or register", v.lo_pc);
      params[i] = (uint64_t(insn_bits(hi, 29, 28)) << 28) | insn_bits(lo, 29, 28);
    } else {
      const uint64_t w = words[v.word0];
      if (insn_bits(w, 59, 5) != OP_CONFIG_ATTN || (w & ((1ull << 33) - 1)))
        return set_fault(f, TAC_E_RECOMPILE, "runtime CONFIG_ATTN word changed its form", v.lo_pc);
      params[i] = uint64_t(insn_bits(w, 47, 12)) | (uint64_t(insn_bits(w, 35, 12)) << 16) |
                  (uint64_t(insn_bits(w, 33, 2)) << 32);
    }
  }
  return check_params(p, params, f);
}

// The parameters the runtime words of one sequence would decode to, from its
// token and position through the program's site formulas: the same values,
// and the same faults, as encoding the words (SET_ADDR_LO/HI carry 28 bits
// each; CONFIG_ATTN's fields are 12 bits, and a wider value reaches the
// opcode bits of the word).
int formula_params(const tac_program* p, int64_t token, int64_t position, uint64_t* params, tac_fault* f) {
  const uint64_t tok = static_cast<uint64_t>(token), pos = static_cast<uint64_t>(position);
  for (size_t i = 0; i < p->vars.size(); ++i) {
    const VarInfo& v = p->vars[i];
    const VarFormula& fm = p->formula[i];
    if (v.kind == 0) {
      params[i] = (fm.base + tok * fm.tok_mul + pos * fm.pos_mul) & ((1ull << 56) - 1);
    } else {
      if ((pos << 47) >> 59 || ((pos + 1) << 35) >> 59)
        return set_fault(f, TAC_E_RECOMPILE, "runtime CONFIG_ATTN word changed its form", v.lo_pc);
      params[i] = (pos & 0xFFF) | (((pos + 1) & 0xFFF) << 16) | (uint64_t(fm.mode & 3) << 32);
    }
  }
  return check_params(p, params, f);
}

int check_params(const tac_program* p, const uint64_t* params, tac_fault* f) {
  for (const RtCheck& c : p->checks) {
    const uint64_t v = params[c.param];
    bool ok = true;
    if (c.kind == CHK_ADDR) {
      const uint64_t a = v + static_cast<uint64_t>(c.dconst);
      ok = (a % 16 == 0 || c.nbytes == 0) && a >= c.lo && a + c.nbytes <= c.hi && a + c.nbytes <= p->dram_bytes;
    } else if (c.kind == CHK_SAME) {
      ok = c.lo < p->vars.size() && v == params[c.lo];
    } else {
      const uint32_t vkl = (v >> 16) & 0xFFFF, mode = (v >> 32) & 3;
      if (c.kind == CHK_ATTN_SET) ok = mode != 0 && vkl != 0;
      else {
        const uint32_t keys = static_cast<uint32_t>(c.lo);
        ok = mode != 0 && vkl != 0 && !((mode == 1 || mode == 3) && keys < vkl) && !(mode == 2 && keys != vkl);
      }
    }
    if (!ok) return set_fault(f, TAC_E_RECOMPILE, "runtime word outside the compiled range", c.pc);
  }
  return TAC_OK;
}

}  // namespace

extern "C" {

int tac_engine_create(int device, int batch, uint64_t dram_bytes, uint64_t shared_bytes, tac_engine** out) {
  if (!out || batch <= 0 || shared_bytes > dram_bytes || shared_bytes % 16) return TAC_E_ARGUMENT;
  *out = nullptr;
  if (cudaSetDevice(device) != cudaSuccess) return TAC_E_CUDA;
  tac_engine* e = new (std::nothrow) tac_engine();
  if (!e) return TAC_E_ARGUMENT;
  e->device = device;
  e->batch = batch;
  e->dram_bytes = dram_bytes;
  e->shared_bytes = shared_bytes;
  e->rw_bytes = round_up(dram_bytes - shared_bytes, 256);
  e->arena_bytes = 0;
  e->seq_stride = round_up(kSramBytes + e->rw_bytes, 256);
  bool ok = cudaMalloc(&e->d_seq, e->seq_stride * batch) == cudaSuccess &&
            cudaMemset(e->d_seq, 0, e->seq_stride * batch) == cudaSuccess &&
            cudaMalloc(&e->d_shared, std::max<uint64_t>(round_up(shared_bytes, 256), 256)) == cudaSuccess &&
            cudaMemset(e->d_shared, 0, std::max<uint64_t>(round_up(shared_bytes, 256), 256)) == cudaSuccess &&
            cudaMalloc(&e->d_sregs, size_t(e->sreg_stride) * 2 * batch) == cudaSuccess &&
            cudaMemset(e->d_sregs, 0, size_t(e->sreg_stride) * 2 * batch) == cudaSuccess &&
            cudaMalloc(&e->d_status, 64) == cudaSuccess && cudaMemset(e->d_status, 0, 64) == cudaSuccess;
  if (ok) {
    cudaDeviceGetAttribute(&e->n_sms, cudaDevAttrMultiProcessorCount, device);
    cudaFuncSetAttribute(exec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kExecSmem));
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, exec_kernel, kCtaThreads, kExecSmem);
    e->grid = e->n_sms * std::max(1, std::min(per_sm, 1));
    ok = cudaDeviceSynchronize() == cudaSuccess && per_sm >= 1;
  }
  if (!ok) {
    tac_engine_destroy(e);
    return TAC_E_CUDA;
  }
  *out = e;
  return TAC_OK;
}

int tac_engine_destroy(tac_engine* e) {
  if (!e) return TAC_E_ARGUMENT;
  cudaSetDevice(e->device);
  cudaDeviceSynchronize();
  cudaFree(e->d_seq);
  cudaFree(e->d_shared);
  cudaFree(e->d_sregs);
  cudaFree(e->d_params);
  cudaFree(e->d_status);
  cudaFree(e->d_prof);
  cudaFree(e->d_task_prof);
  if (e->h_pinned) cudaFreeHost(e->h_pinned);
  for (int i = 0; i < tac_engine::kRing; ++i)
    if (e->ring_ev[i]) cudaEventDestroy(e->ring_ev[i]);
  delete e;
  return TAC_OK;
}

int tac_engine_batch(const tac_engine* e) { return e ? e->batch : 0; }

int tac_engine_grid(const tac_engine* e) { return e ? e->grid : 0; }

int tac_engine_layout(const tac_engine* e, void** seq_base, uint64_t* seq_stride, void** shared_base) {
  if (!e) return TAC_E_ARGUMENT;
  if (seq_base) *seq_base = e->d_seq;
  if (seq_stride) *seq_stride = e->seq_stride;
  if (shared_base) *shared_base = e->d_shared;
  return TAC_OK;
}

static int dram_copy(tac_engine* e, int seq, uint64_t addr, void* host, uint64_t len, bool write) {
  if (!e || (len && !host) || seq < -1 || seq >= e->batch || addr + len > e->dram_bytes || addr + len < addr)
    return TAC_E_ARGUMENT;
  if (!write && seq < 0) return TAC_E_ARGUMENT;
  if (cudaSetDevice(e->device) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return TAC_E_CUDA;
  uint8_t* h = static_cast<uint8_t*>(host);
  // shared part
  if (addr < e->shared_bytes) {
    const uint64_t n = std::min(len, e->shared_bytes - addr);
    cudaError_t c = write ? cudaMemcpy(e->d_shared + addr, h, n, cudaMemcpyHostToDevice)
                          : cudaMemcpy(h, e->d_shared + addr, n, cudaMemcpyDeviceToHost);
    if (c != cudaSuccess) return TAC_E_CUDA;
    h += n;
    addr += n;
    len -= n;
  }
  if (!len) return TAC_OK;
  const uint64_t off = kSramBytes + (addr - e->shared_bytes);
  const int s0 = seq < 0 ? 0 : seq, s1 = seq < 0 ? e->batch : seq + 1;
  for (int s = s0; s < s1; ++s) {
    uint8_t* d = e->d_seq + uint64_t(s) * e->seq_stride + off;
    cudaError_t c = write ? cudaMemcpy(d, h, len, cudaMemcpyHostToDevice) : cudaMemcpy(h, d, len, cudaMemcpyDeviceToHost);
    if (c != cudaSuccess) return TAC_E_CUDA;
  }
  return TAC_OK;
}

int tac_dram_write(tac_engine* e, int seq, uint64_t addr, const void* src, uint64_t len) {
  return dram_copy(e, seq, addr, const_cast<void*>(src), len, true);
}
int tac_dram_read(tac_engine* e, int seq, uint64_t addr, void* dst, uint64_t len) {
  return dram_copy(e, seq, addr, dst, len, false);
}

static int sram_copy(tac_engine* e, int seq, int buf, uint64_t off, void* host, uint64_t len, bool write) {
  if (!e || buf < 0 || buf > 2 || seq < -1 || seq >= e->batch || (len && !host)) return TAC_E_ARGUMENT;
  if (off + len > uint64_t(kBufUnits[buf]) * 16 || (!write && seq < 0)) return TAC_E_ARGUMENT;
  if (cudaSetDevice(e->device) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return TAC_E_CUDA;
  const int s0 = seq < 0 ? 0 : seq, s1 = seq < 0 ? e->batch : seq + 1;
  for (int s = s0; s < s1; ++s) {
    uint8_t* d = e->d_seq + uint64_t(s) * e->seq_stride + uint64_t(kBufUnitBase[buf]) * 16 + off;
    cudaError_t c = write ? cudaMemcpy(d, host, len, cudaMemcpyHostToDevice) : cudaMemcpy(host, d, len, cudaMemcpyDeviceToHost);
    if (c != cudaSuccess) return TAC_E_CUDA;
  }
  return TAC_OK;
}

int tac_sram_write(tac_engine* e, int seq, int buf, uint64_t byte_off, const void* src, uint64_t len) {
  return sram_copy(e, seq, buf, byte_off, const_cast<void*>(src), len, true);
}
int tac_sram_read(tac_engine* e, int seq, int buf, uint64_t byte_off, void* dst, uint64_t len) {
  return sram_copy(e, seq, buf, byte_off, dst, len, false);
}

int tac_sregs_write(tac_engine* e, int seq, const uint16_t* regs16) {
  if (!e || !regs16 || seq < -1 || seq >= e->batch) return TAC_E_ARGUMENT;
  if (cudaSetDevice(e->device) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return TAC_E_CUDA;
  const int s0 = seq < 0 ? 0 : seq, s1 = seq < 0 ? e->batch : seq + 1;
  for (int s = s0; s < s1; ++s)
    if (cudaMemcpy(e->d_sregs + size_t(s) * e->sreg_stride, regs16, 32, cudaMemcpyHostToDevice) != cudaSuccess)
      return TAC_E_CUDA;
  return TAC_OK;
}

int tac_sregs_read(tac_engine* e, int seq, uint16_t* regs16) {
  if (!e || !regs16 || seq < 0 || seq >= e->batch) return TAC_E_ARGUMENT;
  if (cudaSetDevice(e->device) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return TAC_E_CUDA;
  if (cudaMemcpy(regs16, e->d_sregs + size_t(seq) * e->sreg_stride, 32, cudaMemcpyDeviceToHost) != cudaSuccess)
    return TAC_E_CUDA;
  return TAC_OK;
}

int tac_program_destroy(tac_program* p) {
  if (!p) return TAC_E_ARGUMENT;
  if (p->d_blob || p->d_maps) cudaSetDevice(p->device);
  if (p->d_maps) cudaFree(p->d_maps);
  if (p->d_blob) cudaFree(p->d_blob);
  delete p;
  return TAC_OK;
}

static int prepare(tac_engine* e, tac_program* p, tac_fault* f) {
  if (!e || !p || p->batch != e->batch || p->dram_bytes != e->dram_bytes || p->shared_bytes != e->shared_bytes)
    return set_fault(f, TAC_E_ARGUMENT, "program was compiled for a different engine layout");
  CK(cudaSetDevice(e->device), f, "cudaSetDevice");
  if (int s = upload_program(e, p, f)) return s;
  if (int s = ensure_arena(e, p->arena_units * 16, f)) return s;
  if (int s = ensure_sregs(e, p->n_slots, f)) return s;
  if (int s = ensure_maps(e, p, f)) return s;
  return TAC_OK;
}

static int launch(tac_engine* e, tac_program* p, const uint64_t* d_params, cudaStream_t st, tac_fault* f) {
  CK(cudaMemsetAsync(e->d_status, 0, 64, st), f, "reset status");
  const uint32_t n_levels = static_cast<uint32_t>(p->level_off.size() - 1);
  if (n_levels > 0 && !p->tasks.empty()) {
    ExecArgs A;
    const uint8_t* blob = static_cast<const uint8_t*>(p->d_blob);
    A.ops = reinterpret_cast<const DevOp*>(blob + p->off_ops);
    A.segs = reinterpret_cast<const Segment*>(blob + p->off_segs);
    A.tasks = reinterpret_cast<const Task*>(blob + p->off_tasks);
    A.level_off = reinterpret_cast<const uint32_t*>(blob + p->off_levels);
    A.n_levels = n_levels;
    A.n_params = std::max<uint32_t>(p->n_params, 1);
    A.seq_base = e->d_seq;
    A.seq_stride = e->seq_stride;
    A.shared_base = e->d_shared;
    A.sregs = e->d_sregs;
    A.sreg_stride = e->sreg_stride;
    A.params = d_params;
    A.status = e->d_status;
    A.barrier = e->d_status + 4;
    A.tmaps = static_cast<const CUtensorMap*>(p->d_maps);
    A.shared_bytes = e->shared_bytes;
    A.dram_bytes = e->dram_bytes;
    A.prof = nullptr;
    A.task_prof = nullptr;
    if (e->profiling) {
      if (e->prof_cap < n_levels + 1) {
        cudaFree(e->d_prof);
        e->prof_cap = n_levels + 1024;
        CK(cudaMalloc(&e->d_prof, e->prof_cap * 8), f, "cudaMalloc profile");
      }
      CK(cudaMemsetAsync(e->d_prof, 0, (n_levels + 1) * 8, st), f, "reset profile");
      A.prof = e->d_prof;
      e->prof_levels = n_levels;
      const uint64_t n_tasks = p->tasks.size();
      if (e->profiling == 2 && n_tasks) {
        if (e->task_prof_cap < n_tasks) {
          cudaFree(e->d_task_prof);
          e->task_prof_cap = n_tasks;
          CK(cudaMalloc(&e->d_task_prof, n_tasks * 4), f, "cudaMalloc task profile");
        }
        A.task_prof = e->d_task_prof;
        e->prof_tasks = n_tasks;
      }
    }
    void* args[] = {&A};
    CK(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(exec_kernel), dim3(e->grid), dim3(kCtaThreads), args,
                                   kExecSmem, st), f, "launch executor");
  }
  if (p->info.faulted) {
    if (f) *f = p->fault;
    return p->fault.status;
  }
  return TAC_OK;
}

uint64_t tac_program_param_count(const tac_program* p) { return p ? std::max<uint32_t>(p->n_params, 1) : 0; }

uint32_t tac_program_attn_key_cols(const tac_program* p) {
  if (!p) return 0;
  uint64_t keys = 0;
  for (const RtCheck& c : p->checks)
    if (c.kind == CHK_ATTN_KEYS && (keys == 0 || c.lo < keys)) keys = c.lo;
  return static_cast<uint32_t>(keys);
}

int tac_encode_params(const tac_program* p, int batch, const uint64_t* var_words, uint64_t* out, tac_fault* f) {
  if (!p || !out || batch <= 0 || (p->n_var_words && !var_words)) return set_fault(f, TAC_E_ARGUMENT, "bad arguments");
  const uint32_t np = std::max<uint32_t>(p->n_params, 1);
  std::memset(out, 0, sizeof(uint64_t) * np * batch);
  for (int s = 0; s < batch && p->n_params; ++s) {
    if (int r = decode_params(p, var_words + size_t(s) * p->n_var_words, out + size_t(s) * np, f)) {
      if (f) f->buf_id = s;
      return r;
    }
  }
  return TAC_OK;
}

int tac_program_set_var_formula(tac_program* p, uint32_t n_vars, const uint64_t* base, const uint64_t* tok_mul,
                                const uint64_t* pos_mul, const uint32_t* mode) {
  if (!p || n_vars != p->vars.size() || (n_vars && (!base || !tok_mul || !pos_mul || !mode))) return TAC_E_ARGUMENT;
  p->formula.resize(n_vars);
  for (uint32_t i = 0; i < n_vars; ++i) p->formula[i] = VarFormula{base[i], tok_mul[i], pos_mul[i], mode[i]};
  return TAC_OK;
}

int tac_encode_params_tp(const tac_program* p, int batch, const int64_t* tokens, const int64_t* positions,
                         uint64_t* out, tac_fault* f) {
  if (!p || !out || batch <= 0 || !tokens || !positions) return set_fault(f, TAC_E_ARGUMENT, "bad arguments");
  if (p->formula.size() != p->vars.size()) return set_fault(f, TAC_E_ARGUMENT, "no site formulas set");
  const uint32_t np = std::max<uint32_t>(p->n_params, 1);
  std::memset(out, 0, sizeof(uint64_t) * np * batch);
  for (int s = 0; s < batch && p->n_params; ++s) {
    if (int r = formula_params(p, tokens[s], positions[s], out + size_t(s) * np, f)) {
      if (f) f->buf_id = s;
      return r;
    }
  }
  return TAC_OK;
}

int tac_run_async_params(tac_engine* e, tac_program* p, const uint64_t* params_dev, void* stream, tac_fault* f) {
  if (int s = prepare(e, p, f)) return s;
  if (p->n_params && !params_dev) return set_fault(f, TAC_E_ARGUMENT, "missing parameters");
  return launch(e, p, p->n_params ? params_dev : reinterpret_cast<const uint64_t*>(e->d_status + 8), static_cast<cudaStream_t>(stream), f);
}

// Shared body of tac_run_async and tac_run_async_tp: the parameters are
// encoded into the next slot of the pinned staging ring (from runtime words,
// or from tokens and positions when `tokens` is set), uploaded on the stream
// and the step launched.
static int run_staged(tac_engine* e, tac_program* p, const uint64_t* var_words, const int64_t* tokens,
                      const int64_t* positions, void* stream, tac_fault* f) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint32_t np = std::max<uint32_t>(p->n_params, 1);
  const size_t n = size_t(np) * e->batch;
  if (e->pinned_cap < n || e->params_cap < n) {
    CK(cudaDeviceSynchronize(), f, "sync");
    if (e->h_pinned) cudaFreeHost(e->h_pinned);
    e->h_pinned = nullptr;
    e->pinned_cap = std::max<size_t>(n, 4096);
    CK(cudaMallocHost(&e->h_pinned, e->pinned_cap * 8 * tac_engine::kRing), f, "cudaMallocHost");
    cudaFree(e->d_params);
    e->params_cap = e->pinned_cap;
    CK(cudaMalloc(&e->d_params, e->params_cap * 8 * tac_engine::kRing), f, "cudaMalloc params");
    for (int i = 0; i < tac_engine::kRing; ++i) {
      if (!e->ring_ev[i]) CK(cudaEventCreateWithFlags(&e->ring_ev[i], cudaEventDisableTiming), f, "event");
      e->ring_used[i] = false;
    }
  }
  const int slot = e->ring_next;
  e->ring_next = (slot + 1) % tac_engine::kRing;
  if (e->ring_used[slot]) CK(cudaEventSynchronize(e->ring_ev[slot]), f, "staging slot");
  uint64_t* h = e->h_pinned + size_t(slot) * e->pinned_cap;
  uint64_t* d = e->d_params + size_t(slot) * e->params_cap;
  if (int r = tokens ? tac_encode_params_tp(p, e->batch, tokens, positions, h, f)
                     : tac_encode_params(p, e->batch, var_words, h, f))
    return r;
  CK(cudaMemcpyAsync(d, h, n * 8, cudaMemcpyHostToDevice, st), f, "upload params");
  CK(cudaEventRecord(e->ring_ev[slot], st), f, "record staging event");
  e->ring_used[slot] = true;
  return launch(e, p, d, st, f);
}

int tac_run_async(tac_engine* e, tac_program* p, const uint64_t* var_words, void* stream, tac_fault* f) {
  if (int s = prepare(e, p, f)) return s;
  if (p->n_var_words && !var_words) return set_fault(f, TAC_E_ARGUMENT, "missing runtime words");
  return run_staged(e, p, var_words, nullptr, nullptr, stream, f);
}

int tac_run_async_tp(tac_engine* e, tac_program* p, const int64_t* tokens, const int64_t* positions, void* stream,
                     tac_fault* f) {
  if (int s = prepare(e, p, f)) return s;
  if (!tokens || !positions) return set_fault(f, TAC_E_ARGUMENT, "missing tokens or positions");
  return run_staged(e, p, nullptr, tokens, positions, stream, f);
}

int tac_check_device_status(tac_engine* e, tac_fault* f) {
  if (!e) return TAC_E_ARGUMENT;
  uint32_t st[8];
  CK(cudaMemcpy(st, e->d_status, 32, cudaMemcpyDeviceToHost), f, "read status");
  switch (st[0]) {
    case DF_NONE: return TAC_OK;
    case DF_ZERO_DENOM:
      return set_fault(f, TAC_E_CONFIG, "CONFIG_ATTN produced zero softmax denominator");
    case DF_BARRIER_TIMEOUT:
      return set_fault(f, TAC_E_DEVICE, "executor grid barrier timed out");
    case DF_DYN_ADDRESS:
      return set_fault(f, TAC_E_DEVICE, "runtime address outside DRAM");
    case DF_MMA_TIMEOUT:
      return set_fault(f, TAC_E_DEVICE, "executor tensor-core MATMUL wait timed out");
    case DF_STAGE_TIMEOUT:
      return set_fault(f, TAC_E_DEVICE, "executor operand bulk copy wait timed out");
    default:
      return set_fault(f, TAC_E_DEVICE, "executor reported an invalid op");
  }
}

int tac_run(tac_engine* e, tac_program* p, const uint64_t* var_words, tac_fault* f) {
  int s = tac_run_async(e, p, var_words, nullptr, f);
  if (s != TAC_OK && !(p && p->info.faulted && s == p->fault.status)) return s;
  const int compiled_fault = s;
  CK(cudaStreamSynchronize(nullptr), f, "synchronize");
  CK(cudaGetLastError(), f, "executor");
  tac_fault df;
  std::memset(&df, 0, sizeof(df));
  int ds = tac_check_device_status(e, &df);
  if (ds != TAC_OK) {
    if (f) *f = df;
    return ds;
  }
  return compiled_fault;
}

int tac_set_profiling(tac_engine* e, int enable) {
  if (!e || enable < 0 || enable > 2) return TAC_E_ARGUMENT;
  e->profiling = enable;
  return TAC_OK;
}

int tac_read_task_profile(tac_engine* e, uint32_t* out_cycles, uint64_t max_entries, uint64_t* n_entries) {
  if (!e || !n_entries) return TAC_E_ARGUMENT;
  *n_entries = e->prof_tasks;
  if (!out_cycles || !e->d_task_prof || !e->prof_tasks) return TAC_OK;
  if (cudaSetDevice(e->device) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return TAC_E_CUDA;
  const uint64_t n = std::min<uint64_t>(max_entries, e->prof_tasks);
  if (cudaMemcpy(out_cycles, e->d_task_prof, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return TAC_E_CUDA;
  return TAC_OK;
}

int tac_read_profile(tac_engine* e, uint64_t* out_ns, uint32_t max_entries, uint32_t* n_entries) {
  if (!e || !n_entries) return TAC_E_ARGUMENT;
  *n_entries = e->prof_levels ? e->prof_levels + 1 : 0;
  if (!out_ns || !e->d_prof || !e->prof_levels) return TAC_OK;
  if (cudaSetDevice(e->device) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) return TAC_E_CUDA;
  const uint32_t n = std::min<uint32_t>(max_entries, e->prof_levels + 1);
  if (cudaMemcpy(out_ns, e->d_prof, n * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return TAC_E_CUDA;
  return TAC_OK;
}

int tac_argmax_f16(tac_engine* e, uint64_t addr, uint64_t count, int32_t* out_tokens_dev, void* stream) {
  if (!e || !out_tokens_dev || addr + 2 * count > e->dram_bytes) return TAC_E_ARGUMENT;
  if (cudaSetDevice(e->device) != cudaSuccess) return TAC_E_CUDA;
  argmax_f16_kernel<<<e->batch, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      e->d_seq, e->seq_stride, e->d_shared, e->shared_bytes, addr, count, out_tokens_dev);
  return cudaGetLastError() == cudaSuccess ? TAC_OK : TAC_E_CUDA;
}

}  // extern "C"
