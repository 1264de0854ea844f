// Host compiler: taccel instruction stream -> renamed dataflow plan.
//
// Semantics of each instruction (operands, bounds checks and their order,
// exceptions, cycle costs) follow the reference golden model:
//   fetch/run loop ........ golden_model/simulator.py:181-206,299-322
//   dispatch .............. golden_model/simulator.py:476-565
//   registers ............. golden_model/simulator.py:567-627
//   MATMUL ................ golden_model/systolic.py:31-71
//   LOAD/STORE/BUF_COPY ... golden_model/dma.py:27-97
//   SRAM bounds ........... golden_model/memory.py:29-366
//   INT8 / FP ops ......... golden_model/simulator.py:629-1140, golden_model/sfu.py:149-443
// The compiler does not compute data; it records, per instruction, which
// physical bytes hold each operand and emits a device op that the executor
// (tac_exec.cu) runs.  See tac_plan.h for the physical layout.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <unordered_map>
#include <new>
#include <string>
#include <tuple>

#include "tac_program.h"

namespace tac {
namespace {

constexpr uint64_t kNone = ~0ull;

enum PhysClass { PC_SHARED, PC_HOME_SRAM, PC_HOME_RW, PC_ARENA };

struct AddrReg {
  int kind = 0;          // 0 static, 1 runtime parameter, 2 partly known (unusable)
  uint64_t value = 0;    // static value (kind 0) or the known halves (kind 2)
  uint32_t known = 3;    // kind 2: bit 0 = bits [27:0] known, bit 1 = bits [55:28] known
  int param = -1;
  uint64_t lo = 0, hi = 0;  // runtime value range
};

struct Access {
  std::vector<std::pair<uint64_t, uint64_t>> reads;   // (phys, units)
  std::vector<std::pair<uint64_t, uint64_t>> writes;  // (phys, units)
  std::vector<uint32_t> slot_reads;
  std::vector<uint32_t> slot_writes;
  bool sreg_home_read = false;
  bool sreg_home_write = false;
  // a runtime-addressed DRAM access (the single writable-DRAM entry of reads,
  // or of writes when dyn_write): its parameter and its byte range relative
  // to the parameter's value
  int dyn_param = -1;
  bool dyn_write = false;
  int64_t dyn_c0 = 0, dyn_c1 = 0;
};

// A runtime-addressed store: kept out of the per-unit write levels so that two
// stores whose parameters hold one value and whose offsets do not overlap
// (the per-head KV-cache appends of a layer) stay unordered.
struct DynWrite {
  int param;
  int64_t c0, c1;       // bytes written, relative to the parameter's value
  uint64_t i0, i1;      // every writable-DRAM unit it may write
  int32_t level;
};

class Compiler {
 public:
  Compiler(tac_program* prog, const uint8_t* words, uint64_t n_insns, uint64_t entry_pc,
           uint64_t max_insns, const tac_regs* init, int sregs_reset, const tac_var_site* sites,
           int n_sites)
      : P(prog), words_(words), n_insns_(n_insns), entry_(entry_pc), max_insns_(max_insns),
        sites_(sites), n_sites_(n_sites) {
    dram_bytes_ = P->dram_bytes;
    shared_bytes_ = P->shared_bytes;
    ro_units_ = shared_bytes_ / kUnit;
    dram_units_ = (dram_bytes_ + kUnit - 1) / kUnit;
    rw_units_ = dram_units_ > ro_units_ ? dram_units_ - ro_units_ : 0;
    rw_base_ = kSramUnits;
    arena_base_ = rw_base_ + rw_units_;
    for (int r = 0; r < 4; ++r) areg_[r].value = init ? init->addr_regs[r] : 0;
    tile_valid_ = init && init->tile_valid;
    if (tile_valid_) for (int i = 0; i < 3; ++i) tile_[i] = init->tile[i];
    if (init && init->attn_valid) {
      attn_kind_ = 1;
      attn_qrb_ = init->attn_qrb;
      attn_vkl_ = init->attn_vkl;
      attn_mode_ = init->attn_mode;
    }
    for (int r = 0; r < 16; ++r) sreg_[r] = sregs_reset ? (kSregConst | 0u) : uint32_t(r);
    if (const char* path = std::getenv("TAC_LEVEL_TRACE")) trace_ = std::fopen(path, "a");
  }
  ~Compiler() {
    if (trace_) std::fclose(trace_);
  }
  Compiler(const Compiler&) = delete;
  Compiler& operator=(const Compiler&) = delete;

  int compile();
  void prefetch_hint(const DevOp& op, Task& t) const;
  void drop_dead_ops();
  void drop_dead_walk(std::vector<uint8_t>& keep, const std::vector<uint64_t>& chain_units);
  void merge_dyn_stores();
  void write_vadd_chains();
  int link_pv_pairs();
  void pack_arena();
  uint64_t arena_unpacked_ = 0;
  uint64_t dead_ops_ = 0;

 private:
  // ---- layout helpers ------------------------------------------------------
  PhysClass cls(uint64_t p) const {
    if (p & kSharedBit) return PC_SHARED;
    if (p < rw_base_) return PC_HOME_SRAM;
    if (p < arena_base_) return PC_HOME_RW;
    return PC_ARENA;
  }
  uint64_t rw_home(uint64_t rw_index) const { return rw_base_ + rw_index; }

  uint64_t alloc(uint64_t units) {
    uint64_t rounded = (units + 15) & ~15ull;  // 256-byte aligned extents
    uint64_t p = arena_base_ + arena_top_;
    arena_top_ += rounded;
    arena_lvl_.resize(arena_top_, 0);
    return p;
  }

  // ---- faults ----------------------------------------------------------------
  int fault(int status, const std::string& msg) {
    tac_fault& f = P->fault;
    f.status = status;
    f.pc = pc_;
    f.raw_word = word_;
    std::snprintf(f.message, sizeof(f.message), "%s", msg.c_str());
    return status;
  }
  int sram_fault(int buf, uint64_t off) {
    P->fault.buf_id = buf;
    P->fault.offset = static_cast<int64_t>(off);
    P->fault.limit = static_cast<int64_t>(kBufUnits[buf < 3 ? buf : 0]) - 1;
    return fault(TAC_E_SRAM_ACCESS, "SRAM access out of bounds");
  }
  int dram_fault(uint64_t addr) {
    P->fault.addr = addr;
    return fault(TAC_E_DRAM_ACCESS, "DRAM access out of bounds");
  }
  int ibuf_fault(int buf) {
    P->fault.buf_id = buf;
    return fault(TAC_E_ILLEGAL_BUFFER, "Illegal buffer ID: " + std::to_string(buf));
  }
  int config_fault(const std::string& msg) { return fault(TAC_E_CONFIG, msg); }
  int value_fault(const std::string& msg) { return fault(TAC_E_VALUE, msg); }
  int unsupported(const std::string& msg) { return fault(TAC_E_UNSUPPORTED, msg); }

  // End-of-range SRAM check shared by every tile / byte helper.
  bool sram_span_ok(int buf, uint64_t off, uint64_t nbytes) const {
    return off * kUnit + nbytes <= uint64_t(kBufUnits[buf]) * kUnit;
  }

  // ---- dependency levels ---------------------------------------------------------
  // Latest level of a runtime-addressed store that may touch writable-DRAM
  // units [i0, i1).  For a runtime-addressed access (param >= 0, bytes
  // [c0, c1) relative to the parameter's value), a store whose parameter is in
  // the same site group and whose relative bytes are disjoint cannot touch the
  // same bytes: it is skipped, and the equality of the two parameters becomes
  // a run-time check.
  int32_t dyn_level(uint64_t i0, uint64_t i1, int param, int64_t c0, int64_t c1) {
    int32_t L = 0;
    for (const DynWrite& d : dyn_w_) {
      if (d.i1 <= i0 || d.i0 >= i1 || d.level <= L) continue;
      if (param >= 0 && site_group_[d.param] == site_group_[param] && (d.c1 <= c0 || c1 <= d.c0)) {
        pending_same_.push_back(d.param);
        pending_same_.push_back(param);
        continue;
      }
      L = d.level;
    }
    return L;
  }

  int32_t level_for(const Access& a) {
    int32_t L = 0;
    why_ = "none";
    auto bump = [&](int32_t v, const char* tag) {
      if (v > L) {
        L = v;
        why_ = tag;
      }
    };
    for (auto& r : a.reads) {
      uint64_t p = r.first;
      switch (cls(p)) {
        case PC_ARENA:
          for (uint64_t i = 0; i < r.second; ++i) bump(arena_lvl_[p - arena_base_ + i], "arena-raw");
          break;
        case PC_HOME_RW:
          for (uint64_t i = 0; i < r.second; ++i) bump(rw_wl_[p - rw_base_ + i], "home-raw");
          if (!dyn_w_.empty()) {
            const bool dyn = a.dyn_param >= 0 && !a.dyn_write;
            bump(dyn_level(p - rw_base_, p - rw_base_ + r.second, dyn ? a.dyn_param : -1, a.dyn_c0, a.dyn_c1),
                 "home-dyn-raw");
          }
          break;
        default:
          break;  // shared: never written; SRAM home: written only by the final materialise
      }
    }
    for (auto& w : a.writes) {
      uint64_t p = w.first;
      switch (cls(p)) {
        case PC_HOME_RW:
          for (uint64_t i = 0; i < w.second; ++i) {
            bump(rw_wl_[p - rw_base_ + i], "home-waw");
            bump(rw_rl_[p - rw_base_ + i], "home-war");
          }
          if (!dyn_w_.empty()) {
            const bool dyn = a.dyn_param >= 0 && a.dyn_write;
            bump(dyn_level(p - rw_base_, p - rw_base_ + w.second, dyn ? a.dyn_param : -1, a.dyn_c0, a.dyn_c1),
                 "home-dyn-waw");
          }
          break;
        case PC_HOME_SRAM:
          for (uint64_t i = 0; i < w.second; ++i) bump(home_rl_[p + i], "sram-war");
          break;
        default:
          break;  // arena extents are fresh
      }
    }
    for (uint32_t s : a.slot_reads) bump(slot_lvl_[s], "slot-raw");
    if (a.sreg_home_write) bump(sreg_home_rl_, "sreg-war");
    return L + 1;
  }

  void commit(const Access& a, int32_t L) {
    for (auto& r : a.reads) {
      uint64_t p = r.first;
      PhysClass c = cls(p);
      if (c == PC_HOME_RW) {
        for (uint64_t i = 0; i < r.second; ++i) {
          int32_t& x = rw_rl_[p - rw_base_ + i];
          x = std::max(x, L);
          rw_home_read_[p - rw_base_ + i] = 1;
        }
      } else if (c == PC_HOME_SRAM) {
        for (uint64_t i = 0; i < r.second; ++i) home_rl_[p + i] = std::max(home_rl_[p + i], L);
        sram_home_read_ = true;
      }
    }
    for (auto& w : a.writes) {
      uint64_t p = w.first;
      PhysClass c = cls(p);
      if (c == PC_ARENA) {
        for (uint64_t i = 0; i < w.second; ++i) arena_lvl_[p - arena_base_ + i] = L;
      } else if (c == PC_HOME_RW) {
        if (a.dyn_param >= 0 && a.dyn_write) {
          dyn_w_.push_back(DynWrite{a.dyn_param, a.dyn_c0, a.dyn_c1, p - rw_base_, p - rw_base_ + w.second, L});
        } else {
          for (uint64_t i = 0; i < w.second; ++i) rw_wl_[p - rw_base_ + i] = L;
        }
      }
    }
    for (uint32_t s : a.slot_writes) slot_lvl_[s] = L;
    if (a.sreg_home_read) {
      sreg_home_rl_ = std::max(sreg_home_rl_, L);
      sreg_home_read_ = true;
    }
  }

  uint32_t emit(DevOp op, const Access& a) {
    std::vector<std::pair<uint64_t, uint64_t>> ar, aw;
    for (auto& r : a.reads)
      if (cls(r.first) == PC_ARENA) ar.push_back(r);
    bool pure = a.slot_writes.empty() && !a.sreg_home_write && op.kind != K_DYN_STORE && op.kind != K_SREG_FINAL;
    for (auto& w : a.writes) {
      pure = pure && cls(w.first) == PC_ARENA;
      if (cls(w.first) == PC_ARENA) aw.push_back(w);
    }
    pure = pure && !aw.empty();
    op_arena_reads_.push_back(std::move(ar));
    op_arena_writes_.push_back(std::move(aw));
    op_pure_.push_back(pure ? 1 : 0);
    for (auto& w : a.writes)
      if (cls(w.first) == PC_HOME_RW) {
        ++home_writes_;
        break;
      }
    pending_same_.clear();
    int32_t L = level_for(a);
    if (force_level_ >= 0) L = force_level_;   // a P.V MATMUL placed in its QK^T task's level
    commit(a, L);
    for (int prm : pending_same_) {   // equalities the level relied on
      const int g = site_group_[prm];
      if (prm == g || same_checked_[prm]) continue;
      same_checked_[prm] = 1;
      RtCheck c{};
      c.kind = CHK_SAME;
      c.param = static_cast<uint32_t>(prm);
      c.pc = pc_;
      c.lo = static_cast<uint64_t>(g);
      P->checks.push_back(c);
    }
    op.level = static_cast<uint32_t>(L);
    op.pc = static_cast<uint32_t>(pc_);
    if (trace_) {
      std::fprintf(trace_, "%llu %u %d %s", static_cast<unsigned long long>(pc_), op.kind, L, why_);
      for (auto& r : a.reads)
        if (cls(r.first) == PC_HOME_RW)
          std::fprintf(trace_, " r:%llu+%llu", static_cast<unsigned long long>(r.first - rw_base_),
                       static_cast<unsigned long long>(r.second));
      for (auto& w : a.writes)
        if (cls(w.first) == PC_HOME_RW)
          std::fprintf(trace_, " w:%llu+%llu", static_cast<unsigned long long>(w.first - rw_base_),
                       static_cast<unsigned long long>(w.second));
      if (op.kind == K_DYN_STORE || op.kind == K_DYN_LOAD)
        std::fprintf(trace_, " p:%d c:%lld n:%llu", op.param, static_cast<long long>(op.dconst),
                     static_cast<unsigned long long>(op.nbytes));
      std::fputc('\n', trace_);
    }
    P->ops.push_back(op);
    return static_cast<uint32_t>(P->ops.size() - 1);
  }

  static DevOp blank(uint16_t kind) {
    DevOp op;
    std::memset(&op, 0, sizeof(op));
    op.kind = kind;
    op.param = -1;
    return op;
  }

  // ---- register operands ------------------------------------------------------
  uint32_t new_slot() {
    uint32_t s = kSregSlotBase + n_slots_++;
    slot_lvl_.resize(s + 1, 0);
    return s;
  }
  void read_sreg(Access& a, uint32_t enc) {
    if (enc & kSregConst) return;
    if (enc < kSregSlotBase) a.sreg_home_read = true;
    else a.slot_reads.push_back(enc);
  }

  // ---- logical SRAM -> physical operand --------------------------------------------
  static uint32_t unit_of(int buf, uint64_t off) { return kBufUnitBase[buf] + uint32_t(off); }

  bool contiguous(const uint64_t* map, uint64_t n) const {
    PhysClass c0 = cls(map[0]);
    for (uint64_t i = 1; i < n; ++i)
      if (map[i] != map[0] + i || cls(map[i]) != c0) return false;
    return true;
  }

  // Appends a copy segment, split into pieces of at most kGatherChunkUnits.
  void push_seg(uint64_t src, uint64_t dst, uint64_t n) {
    while (n > kGatherChunkUnits) {
      P->segs.push_back(Segment{src, dst, kGatherChunkUnits});
      src += kGatherChunkUnits;
      dst += kGatherChunkUnits;
      n -= kGatherChunkUnits;
    }
    P->segs.push_back(Segment{src, dst, n});
  }

  // Gathers scattered physical units into one fresh arena extent.  Two gathers
  // of the same immutable sources share one extent.
  uint64_t gather(const uint64_t* map, uint64_t n) {
    std::vector<std::pair<uint64_t, uint64_t>> runs;
    bool mutable_src = false;
    uint64_t i = 0;
    while (i < n) {
      uint64_t j = i + 1;
      while (j < n && map[j] == map[i] + (j - i) && cls(map[j]) == cls(map[i])) ++j;
      runs.push_back({map[i], j - i});
      mutable_src |= cls(map[i]) == PC_HOME_RW;
      i = j;
    }
    std::string key;
    if (!mutable_src) {
      key.assign("G", 1);
      key.append(reinterpret_cast<const char*>(runs.data()), runs.size() * sizeof(runs[0]));
      auto it = cse_.find(key);
      if (it != cse_.end()) return P->ops[it->second].d;
    }
    uint64_t dst = alloc(n);
    DevOp op = blank(K_GATHER);
    op.seg0 = static_cast<uint32_t>(P->segs.size());
    Access acc;
    uint64_t off = 0;
    for (auto& r : runs) {
      push_seg(r.first, dst + off, r.second);
      acc.reads.push_back(r);
      off += r.second;
    }
    op.nseg = static_cast<uint32_t>(P->segs.size() - op.seg0);
    op.d = dst;
    op.N = static_cast<uint32_t>(n);
    acc.writes.push_back({dst, n});
    uint32_t idx = emit(op, acc);
    if (!mutable_src) cse_[key] = idx;
    return dst;
  }

  // Ops that may form a chain: per-sequence row ops whose whole tile one
  // task covers in a few steps.
  static bool chain_kind(const DevOp& op) {
    return (op.kind == K_VADD_F16 || op.kind == K_LAYERNORM_F16 || op.kind == K_MAX_ABS) &&
           uint64_t(op.M) * op.N <= 16384 && (op.flags2 & ~(FX_MAXQ | FX_CHAINED)) == 0;
  }

  // A chain-kind op that reads the result of the op emitted just before it
  // (itself of a chain kind), and whose other operands are ready by that op's
  // level, joins that op's level and runs right after it in the same task
  // (FX_CHAINED): one grid barrier and one task fewer per sequence.  Returns
  // the level to join, or -1.  A read that overlaps the previous op's
  // results without lying inside them refuses the chain.
  int32_t chain_level(const DevOp& op, const Access& acc) {
    if (!chain_kind(op) || P->ops.empty() || op_arena_writes_.size() != P->ops.size()) return -1;
    const size_t pi = P->ops.size() - 1;
    const DevOp& prev = P->ops[pi];
    if (!chain_kind(prev)) return -1;
    Access probe = acc;
    probe.reads.clear();
    bool reads_prev = false;
    for (auto& r : acc.reads) {
      bool inside = false, overlap = false;
      for (auto& w : op_arena_writes_[pi]) {
        if (r.first < w.first + w.second && w.first < r.first + r.second) overlap = true;
        if (r.first >= w.first && r.first + r.second <= w.first + w.second) inside = true;
      }
      if (overlap && !inside) return -1;
      if (inside) reads_prev = true;
      else probe.reads.push_back(r);
    }
    if (!reads_prev || level_for(probe) > int32_t(prev.level)) return -1;
    return static_cast<int32_t>(prev.level);
  }

  // Emits a compute op unless an identical op (same kind, shape and
  // immutable operands) already produced the value; then the destination
  // logical units (and scale-register slots) alias that op's output.
  void emit_compute(DevOp& op, Access& acc, uint32_t dst_u0, int sreg_idx) {
    bool mutable_src = false;
    for (auto& r : acc.reads) mutable_src |= cls(r.first) == PC_HOME_RW;
    std::string key;
    if (!mutable_src && op.kind != K_DYN_LOAD && op.kind != K_DYN_STORE && op.kind != K_SREG_FINAL) {
      DevOp k = op;
      k.d = 0;
      k.out_slot = 0;
      k.pc = 0;
      k.level = 0;
      if (op.flags & F_SEGA) k.seg0 = 0;   // a segment list is keyed by its contents
      key.assign(reinterpret_cast<const char*>(&k), sizeof(k));
      if (op.flags & F_SEGA)
        key.append(reinterpret_cast<const char*>(&P->segs[op.seg0]), op.nseg * sizeof(Segment));
      auto it = cse_.find(key);
      if (it != cse_.end()) {
        const DevOp& prev = P->ops[it->second];
        if ((op.flags & F_SEGA) && op.seg0 + op.nseg == P->segs.size()) P->segs.resize(op.seg0);
        if (op.kind == K_MAX_ABS) {
          sreg_[sreg_idx] = prev.out_slot;
          sreg_[sreg_idx + 1] = prev.out_slot + 1;
          if (op.out_slot + 2 == kSregSlotBase + n_slots_) n_slots_ -= 2;
        } else if (op.kind == K_SREG_LOAD) {
          sreg_[sreg_idx] = prev.out_slot;
          if (op.out_slot + 1 == kSregSlotBase + n_slots_) n_slots_ -= 1;
        } else {
          for (uint64_t i = 0; i < last_dst_units_; ++i) sram_[dst_u0 + i] = prev.d + i;
          const uint64_t rounded = (last_dst_units_ + 15) & ~15ull;
          if (op.d + rounded == arena_base_ + arena_top_) {
            arena_top_ -= rounded;
            arena_lvl_.resize(arena_top_);
          }
        }
        ++cse_hits_;
        return;
      }
    }
    uint32_t idx = emit(op, acc);
    if (!key.empty()) cse_[key] = idx;
  }

  // Operand B of a small per-sequence MATMUL (the wide task shape).  When B
  // is the transpose of an immutable [N][K] extent, that extent is read
  // directly (F_BT); when B (or that extent) is the output of a QUANT whose
  // FP16 source still holds the same bytes, the MATMUL quantises the source
  // itself (F_QB, register in s[1]).  The TRANSPOSE and QUANT outputs then go
  // unread and their ops are dropped.  Returns false for an ordinary operand.
  bool mm_b_source(uint32_t u0, uint32_t M, uint32_t N, uint32_t K, Access& acc, DevOp& op) {
    if (!wide_mm_ok(M, N, K, true, false)) return false;
    const uint64_t n = uint64_t(K) * N / kUnit;
    const uint64_t* m = &sram_[u0];
    if (!contiguous(m, n)) return false;
    uint64_t key = m[0];
    bool bt = false;
    auto it = transposed_.find(key);
    if (it != transposed_.end() && it->second.rows == N && it->second.cols == K) {
      key = it->second.src;
      bt = true;
    }
    auto q = quantized_.find(key);
    if (q != quantized_.end() && q->second.rows * q->second.cols == uint64_t(K) * N &&
        (cls(q->second.src) != PC_HOME_RW || q->second.epoch == home_writes_) && wide_mm_ok(M, N, K, bt, true)) {
      op.b = q->second.src;
      op.s[1] = q->second.scale;
      read_sreg(acc, op.s[1]);
      op.flags |= F_QB | F_WIDE | (bt ? F_BT : 0);
      acc.reads.push_back({op.b, 2 * n});
      return true;
    }
    if (!bt) return false;
    op.b = key;
    op.flags |= F_BT | F_WIDE;   // only the wide MATMUL reads B^T
    acc.reads.push_back({op.b, n});
    return true;
  }

  // Operand A of a wide MATMUL that is the output of a QUANT whose FP16
  // source still holds the same bytes: the MATMUL quantises the source itself
  // (F_QA, register in s[0]) and the QUANT goes unread.
  bool mm_a_source(uint32_t u0, uint32_t M, uint32_t N, uint32_t K, Access& acc, DevOp& op) {
    if (op.b & kSharedBit) return false;   // shared weights: the tensor-core path
    const bool bt = (op.flags & F_BT) != 0, qb = (op.flags & F_QB) != 0;
    if (!wide_mm_ok(M, N, K, bt, qb, true)) return false;
    const uint64_t n = uint64_t(M) * K / kUnit;
    const uint64_t* m = &sram_[u0];
    if (!contiguous(m, n)) return false;
    auto q = quantized_.find(m[0]);
    if (q == quantized_.end() || q->second.rows * q->second.cols != uint64_t(M) * K) return false;
    if (cls(q->second.src) == PC_HOME_RW && q->second.epoch != home_writes_) return false;
    op.a = q->second.src;
    op.s[0] = q->second.scale;
    read_sreg(acc, op.s[0]);
    op.flags |= F_QA | F_WIDE;
    acc.reads.push_back({op.a, 2 * n});
    return true;
  }

  // DEQUANT_ACCUM of a wide MATMUL's whole int32 result: the MATMUL writes the
  // FP16 result itself (F_DQ), provided the scale row is ready by the
  // MATMUL's level.  The DEQUANT's output extent is committed at that level.
  bool fuse_dequant(uint32_t s1, uint32_t s2, uint32_t d, uint64_t M, uint64_t N) {
    if ((N * 2) % kUnit) return false;
    const uint64_t na = M * N * 4 / kUnit, nb = N * 2 / kUnit;
    const uint64_t* ma = &sram_[s1];
    const uint64_t* mb = &sram_[s2];
    if (!contiguous(ma, na) || !contiguous(mb, nb)) return false;
    auto it = mm_out_.find(ma[0]);
    if (it == mm_out_.end()) return false;
    const uint32_t idx = it->second;
    DevOp& mm = P->ops[idx];
    if ((mm.flags & F_DQ) || uint64_t(mm.M) != M || uint64_t(mm.N) != N) return false;
    Access probe;
    probe.reads.push_back({mb[0], nb});
    if (level_for(probe) > int32_t(mm.level)) return false;
    Access acc;
    acc.reads.push_back({mb[0], nb});
    const uint64_t out = dst(d, M * N * 2, acc);
    commit(acc, int32_t(mm.level));
    mm.flags |= F_DQ;
    mm.c = mb[0];
    mm.dconst = static_cast<int64_t>(out);
    dq_out_[out] = idx;
    for (auto& w : acc.writes)
      if (cls(w.first) == PC_ARENA) op_arena_writes_[idx].push_back(w);
    if (cls(mb[0]) == PC_ARENA) op_arena_reads_[idx].push_back({mb[0], nb});
    if (cls(mb[0]) != PC_ARENA && cls(mb[0]) != PC_SHARED) op_pure_[idx] = 0;   // conservative
    return true;
  }

  // VADD of the running sum of an earlier VADD (or chain) and a new operand
  // ready before that op's level: the op becomes (or grows as) a
  // K_VADD_CHAIN, which adds the operands in the program's order with an FP16
  // rounding after each add, exactly as the separate VADDs do.  The new sum
  // is committed at the chain's level.  The chain's segments are written out
  // after compilation (write_vadd_chains); op.param numbers the chain.  op.d
  // stays the first sum, the value a CSE hit on the original VADD stands for.
  bool extend_vadd_chain(uint32_t s1, uint32_t s2, uint32_t d, uint64_t M, uint64_t N) {
    const uint64_t n = M * N * 2 / kUnit;
    if ((M * N * 2) % kUnit || n == 0) return false;
    const uint64_t* ma = &sram_[s1];
    const uint64_t* mb = &sram_[s2];
    if (!contiguous(ma, n) || !contiguous(mb, n)) return false;
    uint64_t tail = ma[0], other = mb[0];
    auto it = vadd_tail_.find(tail);
    if (it == vadd_tail_.end()) {
      std::swap(tail, other);   // a + b == b + a exactly
      it = vadd_tail_.find(tail);
    }
    if (it == vadd_tail_.end() || other == tail) return false;
    const uint32_t idx = it->second;
    DevOp& op = P->ops[idx];
    if (uint64_t(op.M) * op.N != M * N) return false;
    if (op.kind == K_VADD_CHAIN && chains_[op.param].size() >= kVaddChainMax) return false;
    Access probe;
    probe.reads.push_back({other, n});
    if (level_for(probe) > int32_t(op.level)) return false;
    if (op.kind == K_VADD_F16) {   // becomes a chain: its own two operands first
      op.kind = K_VADD_CHAIN;
      op.param = static_cast<int32_t>(chains_.size());
      chains_.push_back({Segment{op.a, 0, n}, Segment{op.b, op.d, n}});
      op.a = op.b = 0;
    }
    Access acc;
    acc.reads.push_back({other, n});
    const uint64_t out = dst(d, M * N * 2, acc);
    commit(acc, int32_t(op.level));
    chains_[op.param].push_back(Segment{other, out, n});
    vadd_tail_.erase(it);
    vadd_tail_[out] = idx;
    for (auto& w : acc.writes)
      if (cls(w.first) == PC_ARENA) op_arena_writes_[idx].push_back(w);
    if (cls(other) == PC_ARENA) op_arena_reads_[idx].push_back({other, n});
    if (cls(other) != PC_ARENA && cls(other) != PC_SHARED) op_pure_[idx] = 0;   // conservative
    return true;
  }

  // A MAX_ABS (with or without a segment list) whose operand runs lie in the
  // output of a GELU op reads that GELU's input instead, through segments
  // flagged kSegGelu (FX_GELUSEG): the executor applies the GELU to each value
  // and rounds it to FP16, which is the value the GELU op stores.  The GELU's
  // input must be immutable (arena or shared); its output then has one reader
  // fewer and, in the decode streams, none, so the GELU op and its level go.
  // Refused when the segment list would outgrow kMaxSegRuns.
  void gelu_into_maxabs(DevOp& op, Access& acc, uint64_t units) {
    if (gelu_out_.empty() || units == 0) return;
    struct Run { uint64_t src, dst, n; bool gelu; };
    std::vector<Run> in;
    if (op.flags & F_SEGA)
      for (uint32_t k = 0; k < op.nseg; ++k) in.push_back({P->segs[op.seg0 + k].src, P->segs[op.seg0 + k].dst,
                                                            P->segs[op.seg0 + k].n, false});
    else
      in.push_back({op.a, 0, units, false});
    std::vector<Run> out;
    bool any = false;
    for (const Run& r : in) {
      auto it = gelu_out_.upper_bound(r.src);
      if (it == gelu_out_.begin() || cls(r.src) != PC_ARENA) { out.push_back(r); continue; }
      --it;
      const DevOp& g = P->ops[it->second];
      const uint64_t gu = uint64_t(g.M) * g.N * 2 / kUnit;
      if (r.src < g.d || r.src + r.n > g.d + gu) { out.push_back(r); continue; }
      // GELU output unit o is GELU operand unit o: map [o, o + n) through the GELU's input
      uint64_t o = r.src - g.d, left = r.n, dst = r.dst;
      bool ok = true;
      std::vector<Run> pieces;
      while (left && ok) {
        uint64_t src = 0, run = 0;
        if (g.flags & F_SEGA) {
          ok = false;
          for (uint32_t k = 0; k < g.nseg; ++k) {
            const Segment& gs = P->segs[g.seg0 + k];
            if (gs.dst <= o && o < gs.dst + gs.n) {
              src = gs.src + (o - gs.dst);
              run = std::min(left, gs.dst + gs.n - o);
              ok = true;
              break;
            }
          }
        } else {
          src = g.a + o;
          run = left;
        }
        if (!ok || (cls(src) != PC_ARENA && cls(src) != PC_SHARED)) { ok = false; break; }
        pieces.push_back({src, dst, run, true});
        o += run;
        dst += run;
        left -= run;
      }
      if (!ok) { out.push_back(r); continue; }
      out.insert(out.end(), pieces.begin(), pieces.end());
      any = true;
    }
    if (!any || out.size() > kMaxSegRuns) return;
    // the op's segments are the last ones written (src_segments) or none yet
    if (op.flags & F_SEGA) P->segs.resize(op.seg0);
    op.seg0 = static_cast<uint32_t>(P->segs.size());
    acc.reads.erase(std::remove_if(acc.reads.begin(), acc.reads.end(),
                                   [&](const std::pair<uint64_t, uint64_t>& rd) {
                                     for (const Run& r : in)
                                       if (rd.first == r.src) return true;
                                     return false;
                                   }),
                    acc.reads.end());
    for (const Run& r : out) {
      P->segs.push_back(Segment{r.src, r.dst | (r.gelu ? kSegGelu : 0ull), r.n});
      acc.reads.push_back({r.src, r.n});
    }
    op.nseg = static_cast<uint32_t>(out.size());
    op.a = 0;
    op.flags |= F_SEGA;
    op.flags2 |= FX_GELUSEG;
  }

  // A STORE through a runtime register of the first r rows of a tcgen05
  // MATMUL's FX_DQS FP16 result (a decode step's K / V append), whose other
  // hazards are all settled by that MATMUL's level: the MATMUL's epilogue
  // writes those rows to the runtime address as well (FX_DSTORE), at its own
  // level, and the store op is not emitted.  The write is committed at that
  // level with the store's runtime-address bookkeeping (equalities it relies
  // on become run-time checks, as for any op).
  bool absorb_store(const DevOp& st, const Access& acc) {
    if (st.param < 0 || st.dconst < 0 || st.dconst >= (int64_t(1) << 32)) return false;
    auto it = dqs_out_.find(st.a);
    if (it == dqs_out_.end()) return false;
    DevOp& mm = P->ops[it->second];
    const uint64_t row = uint64_t(mm.N) * 2;
    if ((mm.flags2 & FX_DSTORE) || !(mm.flags2 & FX_DQS) || row == 0 || st.nbytes % row || st.nbytes / row == 0 ||
        st.nbytes / row > mm.M || !tc_eligible(mm.a, mm.b, mm.M, mm.N, mm.K) || (mm.flags & F_ACCUMULATE))
      return false;
    Access probe = acc;
    probe.reads.clear();
    for (auto& r : acc.reads)
      if (!(r.first >= st.a && r.first + r.second <= st.a + st.nbytes / kUnit)) probe.reads.push_back(r);
    pending_same_.clear();
    if (level_for(probe) > int32_t(mm.level)) return false;
    commit(acc, int32_t(mm.level));
    for (int prm : pending_same_) {   // equalities the level relied on
      const int g = site_group_[prm];
      if (prm == g || same_checked_[prm]) continue;
      same_checked_[prm] = 1;
      RtCheck c{};
      c.kind = CHK_SAME;
      c.param = static_cast<uint32_t>(prm);
      c.pc = pc_;
      c.lo = static_cast<uint64_t>(g);
      P->checks.push_back(c);
    }
    ++home_writes_;
    mm.flags2 |= FX_DSTORE;
    mm.param = st.param;
    mm.attn_qrb = static_cast<uint32_t>(st.dconst);
    mm.attn_vkl = static_cast<uint32_t>(st.nbytes / row);
    pure_before_store_[it->second] = op_pure_[it->second];
    op_pure_[it->second] = 0;   // a DRAM write: kept whatever reads its arena results
    return true;
  }

  // QUANT of exactly the units a MAX_ABS just reduced, with that MAX_ABS's
  // inverse scale: the MAX_ABS op writes the int8 result as well (FX_MAXQ).
  // The input units must be immutable (arena or shared), so the values the
  // MAX_ABS reads are the ones the QUANT would read; the QUANT's output is
  // committed at the MAX_ABS's level.  The operand checks (span, buffer
  // faults) have already run.
  bool fuse_quant_into_maxabs(const DevOp& q, uint32_t s1, uint32_t d, uint64_t M, uint64_t N) {
    const uint32_t slot = q.s[0];
    if (slot & kSregConst || slot < kSregSlotBase) return false;
    auto it = maxabs_by_slot_.find(slot);
    if (it == maxabs_by_slot_.end() || it->second.elems != M * N || M * N > 16384) return false;
    DevOp& mx = P->ops[it->second.op];
    if (mx.out_slot != slot) return false;
    const uint64_t n = (M * N * 2 + kUnit - 1) / kUnit;
    if (it->second.units.size() != n) return false;
    for (uint64_t i = 0; i < n; ++i) {
      const uint64_t u = sram_[s1 + i];
      if (u != it->second.units[i] || (cls(u) != PC_ARENA && cls(u) != PC_SHARED)) return false;
    }
    if (mx.flags2 & FX_MAXQ) {   // the same QUANT again: its result is the fused one (as CSE would do)
      const uint64_t nq = (M * N + kUnit - 1) / kUnit;
      for (uint64_t i = 0; i < nq; ++i) sram_[d + i] = mx.d + i;
      cycles_ += M * N;
      return true;
    }
    Access acc;
    const uint64_t out = dst(d, M * N, acc);
    commit(acc, int32_t(mx.level));
    mx.flags2 |= FX_MAXQ;
    mx.d = out;
    for (auto& w : acc.writes)
      if (cls(w.first) == PC_ARENA) op_arena_writes_[it->second.op].push_back(w);
    cycles_ += M * N;
    return true;
  }

  // DEQUANT_ACCUM_FP32_SCALED of a tcgen05 MATMUL's whole int32 result: the
  // MATMUL's epilogue writes the FP16 result (FX_DQS), provided the
  // [scale | bias] rows and the activation-scale register are ready by its
  // level.  The DEQUANT's output extent is committed at that level.
  bool fuse_dequant_scaled(uint32_t s1, uint32_t s2, uint32_t d, uint64_t M, uint64_t N, uint32_t sreg) {
    if ((N * 2) % kUnit) return false;
    const uint64_t na = M * N * 4 / kUnit, nh = N * 2 / kUnit;
    const uint64_t* ma = &sram_[s1];
    const uint64_t* mb = &sram_[s2];
    if (!contiguous(ma, na) || !contiguous(mb, nh) || !contiguous(mb + nh, nh)) return false;
    auto it = tc_out_.find(ma[0]);
    if (it == tc_out_.end()) return false;
    const uint32_t idx = it->second;
    DevOp& mm = P->ops[idx];
    if ((mm.flags2 & FX_DQS) || uint64_t(mm.M) != M || uint64_t(mm.N) != N) return false;
    Access probe;
    probe.reads.push_back({mb[0], nh});
    probe.reads.push_back({mb[nh], nh});
    read_sreg(probe, sreg);
    if (level_for(probe) > int32_t(mm.level)) return false;
    Access acc;
    acc.reads = probe.reads;
    acc.slot_reads = probe.slot_reads;
    acc.sreg_home_read = probe.sreg_home_read;
    const uint64_t out = dst(d, M * N * 2, acc);
    commit(acc, int32_t(mm.level));
    mm.flags2 |= FX_DQS;
    mm.c = mb[0];
    mm.nbytes = mb[nh];
    mm.s[0] = sreg;
    mm.dconst = static_cast<int64_t>(out);
    dqs_out_[out] = idx;
    for (auto& w : acc.writes)
      if (cls(w.first) == PC_ARENA) op_arena_writes_[idx].push_back(w);
    for (auto& r : acc.reads)
      if (cls(r.first) == PC_ARENA) op_arena_reads_[idx].push_back(r);
    for (auto& r : acc.reads)
      if (cls(r.first) != PC_ARENA && cls(r.first) != PC_SHARED) op_pure_[idx] = 0;   // conservative
    return true;
  }

  // SOFTMAX / MASKED_SOFTMAX of a fused DEQUANT's whole FP16 result: the
  // MATMUL computes the rows as well (F_SM), from shared memory.  `sm` holds
  // the softmax's attention context (set by the masked variant's check).
  bool fuse_softmax(uint32_t s1, uint32_t d, uint64_t M, uint64_t N, const DevOp& sm) {
    if (N % 8 || M > 32) return false;
    const uint64_t na = M * N * 2 / kUnit;
    const uint64_t* ma = &sram_[s1];
    if (!contiguous(ma, na)) return false;
    auto it = dq_out_.find(ma[0]);
    if (it == dq_out_.end()) return false;
    const uint32_t idx = it->second;
    DevOp& mm = P->ops[idx];
    if (!(mm.flags & F_DQ) || (mm.flags & F_SM) || uint64_t(mm.M) != M || uint64_t(mm.N) != N) return false;
    Access acc;
    const uint64_t out = dst(d, M * N * 2, acc);
    commit(acc, int32_t(mm.level));
    mm.flags |= F_SM | (sm.kind == K_MASKED_SOFTMAX_F16 ? F_SMMASK : 0) | (sm.flags & F_ATTN_DYN);
    mm.attn_qrb = sm.attn_qrb;
    mm.attn_vkl = sm.attn_vkl;
    mm.attn_mode = sm.attn_mode;
    mm.param = sm.param;
    mm.nbytes = out;
    sm_out_[out] = idx;
    for (auto& w : acc.writes)
      if (cls(w.first) == PC_ARENA) op_arena_writes_[idx].push_back(w);
    return true;
  }

  // A wide MATMUL whose A is the softmax output of a wide QK^T + softmax op
  // (quantised on load, F_QA) and whose other operands are ready by that op's
  // level: it runs in the QK^T op's task (FX_PV / FX_PVY), the softmax rows
  // going straight into its A tile.  Returns the QK^T op's index, or -1.
  int32_t pv_partner(const DevOp& op, const Access& acc) {
    if (!(op.flags & F_QA) || !(op.flags & F_WIDE) || (op.flags & F_ACCUMULATE)) return -1;
    auto it = sm_out_.find(op.a);
    if (it == sm_out_.end() || pv_of_.count(it->second)) return -1;
    const DevOp& x = P->ops[it->second];
    if (!(x.flags & F_WIDE) || x.M != op.M || x.N != op.K || op.M % 16 || op.K % 16 || !pv_ok(x.M, x.N)) return -1;
    Access rest = acc;   // every read but the softmax rows
    rest.reads.erase(std::remove_if(rest.reads.begin(), rest.reads.end(),
                                    [&](const std::pair<uint64_t, uint64_t>& r) { return r.first == op.a; }),
                     rest.reads.end());
    if (level_for(rest) > int32_t(x.level)) return -1;
    return static_cast<int32_t>(it->second);
  }

  // Physical start of a contiguous copy of logical SRAM units [u0, u0+n).
  uint64_t src(uint32_t u0, uint64_t nbytes, Access& acc) {
    uint64_t n = (nbytes + kUnit - 1) / kUnit;
    if (n == 0) n = 1;
    uint64_t* m = &sram_[u0];
    if (!contiguous(m, n)) {
      uint64_t g = gather(m, n);
      for (uint64_t i = 0; i < n; ++i) m[i] = g + i;
    }
    acc.reads.push_back({m[0], n});
    return m[0];
  }

  // A [first half | second half] vector operand (2 x half_bytes): when the
  // halves are each contiguous but not adjacent (two LOADs from different
  // places), the op reads them through b and c (F_SPLIT) instead of a gather.
  void src_pair(uint32_t u0, uint64_t half_bytes, Access& acc, DevOp& op) {
    const uint64_t h = half_bytes / kUnit;
    uint64_t* m = &sram_[u0];
    if (half_bytes % kUnit == 0 && h > 0 && !contiguous(m, 2 * h) && contiguous(m, h) && contiguous(m + h, h)) {
      acc.reads.push_back({m[0], h});
      acc.reads.push_back({m[h], h});
      op.b = m[0];
      op.c = m[h];
      op.flags |= F_SPLIT;
      return;
    }
    op.b = src(u0, 2 * half_bytes, acc);
  }

  // Operand a of a MAX_ABS / QUANT / VADD_F16 / GELU read straight from scattered
  // units through a segment list (F_SEGA) rather than gathered first: the
  // gather would be a dependency level of its own.  Returns false (nothing
  // emitted) when the units are contiguous or form too many runs.
  bool src_segments(uint32_t u0, uint64_t nbytes, Access& acc, DevOp& op) {
    const uint64_t n = (nbytes + kUnit - 1) / kUnit;
    const uint64_t* m = &sram_[u0];
    if (n < 2 || contiguous(m, n)) return false;
    std::vector<std::pair<uint64_t, uint64_t>> runs;   // (first unit, length)
    for (uint64_t i = 0; i < n;) {
      uint64_t j = i + 1;
      while (j < n && m[j] == m[i] + (j - i) && cls(m[j]) == cls(m[i])) ++j;
      runs.push_back({i, j - i});
      i = j;
    }
    if (runs.size() > kMaxSegRuns) return false;
    op.seg0 = static_cast<uint32_t>(P->segs.size());
    for (auto& r : runs) {
      push_seg(m[r.first], r.first, r.second);
      acc.reads.push_back({m[r.first], r.second});
    }
    op.nseg = static_cast<uint32_t>(P->segs.size() - op.seg0);
    if (op.nseg > kMaxSegRuns) {   // long runs were split: fall back to a gather
      P->segs.resize(op.seg0);
      acc.reads.resize(acc.reads.size() - runs.size());
      op.seg0 = op.nseg = 0;
      return false;
    }
    op.a = 0;
    op.flags |= F_SEGA;
    return true;
  }

  // Fresh destination extent for logical SRAM units [u0, u0+n).
  uint64_t dst(uint32_t u0, uint64_t nbytes, Access& acc) {
    uint64_t n = (nbytes + kUnit - 1) / kUnit;
    last_dst_units_ = n;
    uint64_t p = alloc(n);
    for (uint64_t i = 0; i < n; ++i) sram_[u0 + i] = p + i;
    acc.writes.push_back({p, n});
    return p;
  }

  // ---- DRAM value tracking ------------------------------------------------------
  // Flushes arena-resident values of writable DRAM units [i0, i1) (rw indices)
  // to their home location so that a runtime-addressed access sees them.
  void flush_rw(uint64_t i0, uint64_t i1) {
    std::vector<uint64_t> idx;
    for (uint64_t i = i0; i < i1; ++i)
      if (shadow_[i] != rw_home(i)) idx.push_back(i);
    if (idx.empty()) return;
    break_aliases(idx.front(), idx.back() + 1);
    DevOp op = blank(K_GATHER);
    op.seg0 = static_cast<uint32_t>(P->segs.size());
    Access acc;
    size_t k = 0;
    while (k < idx.size()) {
      size_t j = k + 1;
      while (j < idx.size() && idx[j] == idx[k] + (j - k) &&
             shadow_[idx[j]] == shadow_[idx[k]] + (j - k) &&
             cls(shadow_[idx[j]]) == cls(shadow_[idx[k]]))
        ++j;
      uint64_t n = j - k;
      push_seg(shadow_[idx[k]], rw_home(idx[k]), n);
      acc.reads.push_back({shadow_[idx[k]], n});
      acc.writes.push_back({rw_home(idx[k]), n});
      k = j;
    }
    op.nseg = static_cast<uint32_t>(P->segs.size() - op.seg0);
    emit(op, acc);
    for (uint64_t i : idx) shadow_[i] = rw_home(i);
  }

  // Writable-DRAM units that SRAM may alias in place, as disjoint intervals
  // [first, end) of rw indices.
  void note_alias(uint64_t i) {
    auto it = alias_iv_.upper_bound(i);
    if (it != alias_iv_.begin()) {
      auto pv = std::prev(it);
      if (pv->second >= i) {   // inside, or extends the interval ending at i
        if (pv->second == i) {
          pv->second = i + 1;
          if (it != alias_iv_.end() && it->first == i + 1) {
            pv->second = it->second;
            alias_iv_.erase(it);
          }
        }
        return;
      }
    }
    if (it != alias_iv_.end() && it->first == i + 1) {
      const uint64_t end = it->second;
      alias_iv_.erase(it);
      alias_iv_[i] = end;
      return;
    }
    alias_iv_[i] = i + 1;
  }

  // Before writable-DRAM units [i0, i1) are written: SRAM units that still
  // alias any of them are given a copy of the old value first (one gather,
  // which the write then orders after as a read of those units).
  void break_aliases(uint64_t i0, uint64_t i1) {
    auto it = alias_iv_.upper_bound(i0);
    if (it != alias_iv_.begin() && std::prev(it)->second > i0) --it;
    if (it == alias_iv_.end() || it->first >= i1) return;
    std::vector<uint32_t> us;
    std::vector<uint64_t> src;
    const uint64_t p0 = rw_home(i0), p1 = rw_home(i1);
    for (uint32_t u = 0; u < kSramUnits; ++u)
      if (sram_[u] >= p0 && sram_[u] < p1 && cls(sram_[u]) == PC_HOME_RW) {
        us.push_back(u);
        src.push_back(sram_[u]);
      }
    if (!us.empty()) {
      std::vector<uint64_t> uniq = src;
      std::sort(uniq.begin(), uniq.end());
      uniq.erase(std::unique(uniq.begin(), uniq.end()), uniq.end());
      const uint64_t g = gather(uniq.data(), uniq.size());
      for (size_t k = 0; k < us.size(); ++k)
        sram_[us[k]] = g + (std::lower_bound(uniq.begin(), uniq.end(), src[k]) - uniq.begin());
    }
    // drop [i0, i1) from the alias intervals
    std::vector<std::pair<uint64_t, uint64_t>> keep;
    while (it != alias_iv_.end() && it->first < i1) {
      if (it->first < i0) keep.push_back({it->first, i0});
      if (it->second > i1) keep.push_back({i1, it->second});
      it = alias_iv_.erase(it);
    }
    for (auto& kv : keep) alias_iv_[kv.first] = kv.second;
  }

  // Flushes only the units of [i0, i1) that lie in the caller's live-out ranges.
  void flush_live(uint64_t i0, uint64_t i1) {
    if (!opts_ || opts_->n_live == 0) {
      flush_rw(i0, i1);
      return;
    }
    for (uint32_t r = 0; r < opts_->n_live; ++r) {
      uint64_t lo = opts_->live[2 * r], hi = opts_->live[2 * r + 1];
      if (hi <= shared_bytes_) continue;
      lo = lo < shared_bytes_ ? 0 : (lo - shared_bytes_) / kUnit;
      hi = std::min<uint64_t>(rw_units_, (hi - shared_bytes_ + kUnit - 1) / kUnit);
      if (lo < hi) flush_rw(std::max(lo, i0), std::min(hi, i1));
    }
  }

  // Physical location of the current value of DRAM unit u.
  uint64_t dram_phys(uint64_t u) const {
    return u < ro_units_ ? (kSharedBit | u) : shadow_[u - ro_units_];
  }

  // ---- instruction handlers ------------------------------------------------------
  int step(const Insn& x);
  int h_load(const Insn& x);
  int h_store(const Insn& x);
  int h_buf_copy(const Insn& x);
  int h_rtype(const Insn& x);
  int h_set_scale(const Insn& x);
  int h_config_attn(const Insn& x);
  int attn_keys_check(uint32_t key_cols, DevOp& op);
  int effective_address(const Insn& x, uint64_t nbytes, bool& dynamic, uint64_t& addr,
                        uint64_t& lo, uint64_t& hi, int& param);
  void finalize();
  void build_tasks();

  // ---- state ----------------------------------------------------------------------
  tac_program* P;
  const uint8_t* words_;
  uint64_t n_insns_, entry_, max_insns_;
  const tac_var_site* sites_;
  int n_sites_;
  uint64_t dram_bytes_ = 0, shared_bytes_ = 0, ro_units_ = 0, dram_units_ = 0, rw_units_ = 0;
  uint64_t rw_base_ = 0, arena_base_ = 0, arena_top_ = 0;
  std::vector<uint64_t> sram_, shadow_;
  std::vector<int32_t> arena_lvl_, rw_wl_, rw_rl_, home_rl_, slot_lvl_;
  std::vector<DynWrite> dyn_w_;
  std::map<uint64_t, uint64_t> alias_iv_;   // see note_alias
  // arena extents written by TRANSPOSE ops -> their immutable [rows][cols] source
  struct TransposeOf {
    uint64_t src;
    uint64_t rows, cols;
  };
  std::unordered_map<uint64_t, TransposeOf> transposed_;
  // arena extents written by (non-segmented) QUANT ops -> FP16 source, register, shape,
  // and the count of writable-DRAM writes emitted before it (a source there must be unchanged)
  struct QuantOf {
    uint64_t src;
    uint32_t scale;
    uint64_t rows, cols;
    uint64_t epoch;
  };
  std::unordered_map<uint64_t, QuantOf> quantized_;
  // int32 result extent of each emitted wide MATMUL (no accumulate) -> op index,
  // and the FP16 result extent of each fused DEQUANT -> op index
  std::unordered_map<uint64_t, uint32_t> mm_out_, dq_out_;
  // int32 result extent of each emitted tcgen05 MATMUL (no accumulate) -> op index
  std::unordered_map<uint64_t, uint32_t> tc_out_;
  // inverse-scale slot of each emitted MAX_ABS -> the op and the physical units it reduced
  struct MaxAbsOf {
    uint32_t op = 0;
    std::vector<uint64_t> units;
    uint64_t elems = 0;
  };
  std::unordered_map<uint32_t, MaxAbsOf> maxabs_by_slot_;
  std::map<uint64_t, uint32_t> gelu_out_;   // GELU op output extent start -> op index
  std::unordered_map<uint64_t, uint32_t> dqs_out_;   // FX_DQS FP16 result extent -> tcgen05 MATMUL index
  std::unordered_map<uint32_t, uint8_t> pure_before_store_;   // FX_DSTORE MATMUL -> op_pure_ before the store
  // output extent of the latest VADD of each open chain -> op index; operand lists of the chains
  std::unordered_map<uint64_t, uint32_t> vadd_tail_;
  // softmax output extent of a wide QK^T + softmax op -> op index; QK^T op -> its P.V op
  std::unordered_map<uint64_t, uint32_t> sm_out_;
  std::unordered_map<uint32_t, uint32_t> pv_of_;
  int32_t force_level_ = -1;
  std::vector<std::vector<Segment>> chains_;
  std::vector<uint64_t> maxabs_pending_;
  uint64_t home_writes_ = 0;
  // per emitted op: its arena reads and writes, and whether arena writes are its only effect
  std::vector<std::vector<std::pair<uint64_t, uint64_t>>> op_arena_reads_, op_arena_writes_;
  std::vector<uint8_t> op_pure_;
  uint64_t narrowed_ops_ = 0;   // ops drop_dead_ops narrowed to the rows read
  std::unordered_map<uint32_t, uint32_t> pv_rows_;   // P.V op -> rows of its results read (drop_dead_walk)

  // Rows [0, m) of an op's outputs (first unit, units per row) hold every unit
  // a later op reads: the smallest such m, at least 1.
  template <class AnyRead>
  static uint32_t rows_read(uint32_t M, const std::vector<std::pair<uint64_t, uint64_t>>& outs, AnyRead&& any_read) {
    uint32_t m = M;
    auto read = [&](uint32_t r) {
      for (auto& o : outs)
        if (any_read(o.first + r * o.second, o.second)) return true;
      return false;
    };
    while (m > 1 && !read(m - 1)) --m;
    return m;
  }

  // Whether `reads(M, cb)` names exactly the arena units of `recorded`.
  template <class Reads>
  bool same_units(Reads&& reads, uint32_t M, const std::vector<std::pair<uint64_t, uint64_t>>& recorded) const {
    std::vector<uint64_t> want, got;
    auto units = [&](std::vector<uint64_t>& v, uint64_t p, uint64_t n) {
      if (cls(p) != PC_ARENA) return;
      for (uint64_t u = 0; u < n; ++u) v.push_back(p + u);
    };
    reads(M, [&](uint64_t p, uint64_t n) { units(want, p, n); });
    for (auto& r : recorded) units(got, r.first, r.second);
    std::sort(want.begin(), want.end());
    want.erase(std::unique(want.begin(), want.end()), want.end());
    std::sort(got.begin(), got.end());
    got.erase(std::unique(got.begin(), got.end()), got.end());
    return want == got;
  }
  // site i's group: the first address site with the same value range; sites of
  // one group are assumed (and checked at run time) to carry one value
  std::vector<int> site_group_;
  std::vector<int> pending_same_;          // parameters a disambiguation relied on
  std::vector<uint8_t> same_checked_;      // per parameter: CHK_SAME emitted
  int32_t sreg_home_rl_ = 0;
  uint32_t sreg_[16];
  uint32_t n_slots_ = 0;
  AddrReg areg_[4];
  bool tile_valid_ = false;
  uint32_t tile_[3] = {0, 0, 0};
  int attn_kind_ = 0;  // 0 unset, 1 static, 2 runtime parameter
  uint32_t attn_qrb_ = 0, attn_vkl_ = 0, attn_mode_ = 0;
  int attn_param_ = -1;
  uint64_t pc_ = 0, word_ = 0;
  // TAC_LEVEL_TRACE=<file>: one line per emitted op, "pc kind level cause", the
  // cause naming the access class that set the level (a diagnostic of the plan).
  FILE* trace_ = nullptr;
  const char* why_ = "none";
  uint64_t insn_region_bytes_ = 0;
  uint64_t cycles_ = 0;
  bool halted_ = false;
  // var-site lookup: pc -> (site index, role 0 = lo / attn, 1 = hi)
  std::map<uint64_t, std::pair<int, int>> var_pc_;
  // common-subexpression table: op signature -> op index
  std::unordered_map<std::string, uint32_t> cse_;
  uint64_t cse_hits_ = 0;
  uint64_t last_dst_units_ = 0;
  // what the run reads that it did not produce
  std::vector<uint8_t> rw_home_read_;
  bool sram_home_read_ = false, sreg_home_read_ = false;
 public:
  const tac_compile_opts* opts_ = nullptr;
};

// ---------------------------------------------------------------------------------
int Compiler::effective_address(const Insn& x, uint64_t nbytes, bool& dynamic, uint64_t& addr,
                                uint64_t& lo, uint64_t& hi, int& param) {
  const AddrReg& r = areg_[x.addr_reg];
  uint64_t off = uint64_t(x.dram_off) * kUnit;
  if (r.kind == 2) return unsupported("LOAD/STORE through a half-patched SET_ADDR pair");
  if (r.kind == 0) {
    dynamic = false;
    addr = r.value + off;
    if (addr + nbytes > dram_bytes_) return dram_fault(addr + nbytes);
    if (nbytes && (addr % kUnit)) return unsupported("DRAM address not 16-byte aligned");
    return 0;
  }
  dynamic = true;
  param = r.param;
  // [lo, hi): the bytes the access may touch.  The site's value lies in its
  // symbol's extent [range_lo, range_hi) and the whole access must stay in
  // that extent shifted by the instruction's offset; the run-time check
  // enforces it (a value outside asks for a recompile).  Runtime addresses
  // that overflow DRAM fail the same check and are recompiled statically to
  // raise the exact fault.
  lo = r.lo + off;
  hi = std::max(r.hi + off, lo + nbytes);
  if (hi > dram_bytes_) hi = std::max<uint64_t>(dram_bytes_, lo + nbytes);
  RtCheck c{};
  c.kind = CHK_ADDR;
  c.param = static_cast<uint32_t>(param);
  c.pc = pc_;
  c.dconst = static_cast<int64_t>(off);
  c.lo = lo;
  c.hi = hi;
  c.nbytes = nbytes;
  P->checks.push_back(c);
  return 0;
}

int Compiler::h_load(const Insn& x) {                       // dma.py:27-44
  uint64_t n = uint64_t(x.xfer_len) * kUnit;
  bool dyn = false;
  uint64_t addr = 0, lo = 0, hi = 0;
  int param = -1;
  if (int s = effective_address(x, n, dyn, addr, lo, hi, param)) return s;
  // write_bytes: the start offset is valid by decode; the end must fit.
  if (!sram_span_ok(x.buf_id, x.sram_off, n)) {
    if (x.buf_id == BUF_ACCUM)
      return value_fault("could not broadcast input array from shape (" + std::to_string(n) +
                         ",) into shape (" +
                         std::to_string(uint64_t(kBufUnits[BUF_ACCUM]) * kUnit - x.sram_off * kUnit) +
                         ",)");
    return sram_fault(x.buf_id, x.sram_off);
  }
  cycles_ += x.xfer_len;
  if (n == 0) return 0;
  uint32_t u0 = unit_of(x.buf_id, x.sram_off);
  uint64_t nu = n / kUnit;
  if (!dyn) {
    // The SRAM units alias the value's physical location, no device work.  A
    // unit that aliases writable DRAM in place is copied out only if a later
    // write reaches that DRAM unit while the alias lives (break_aliases).
    uint64_t a0 = addr / kUnit;
    for (uint64_t i = 0; i < nu; ++i) {
      sram_[u0 + i] = dram_phys(a0 + i);
      if (cls(sram_[u0 + i]) == PC_HOME_RW) note_alias(sram_[u0 + i] - rw_base_);
    }
    return 0;
  }
  // Runtime address: copy into a fresh extent.
  bool in_shared = hi <= shared_bytes_;
  bool in_rw = lo >= shared_bytes_;
  if (!in_shared && !in_rw) return unsupported("runtime-addressed LOAD straddles the shared DRAM region");
  Access acc;
  if (in_rw) {
    uint64_t i0 = (lo - shared_bytes_) / kUnit;
    uint64_t i1 = std::min<uint64_t>(rw_units_, (hi - shared_bytes_ + kUnit - 1) / kUnit);
    flush_rw(i0, i1);
    acc.reads.push_back({rw_home(i0), i1 - i0});
    acc.dyn_param = param;
    acc.dyn_c0 = int64_t(x.dram_off) * kUnit;
    acc.dyn_c1 = acc.dyn_c0 + int64_t(n);
  }
  DevOp op = blank(K_DYN_LOAD);
  op.param = param;
  op.dconst = int64_t(x.dram_off) * kUnit;
  op.nbytes = n;
  op.d = dst(u0, n, acc);
  emit(op, acc);
  return 0;
}

int Compiler::h_store(const Insn& x) {                      // dma.py:47-64
  uint64_t n = uint64_t(x.xfer_len) * kUnit;
  if (!sram_span_ok(x.buf_id, x.sram_off, n)) return sram_fault(x.buf_id, x.sram_off);
  bool dyn = false;
  uint64_t addr = 0, lo = 0, hi = 0;
  int param = -1;
  if (int s = effective_address(x, n, dyn, addr, lo, hi, param)) return s;
  uint64_t first = dyn ? lo : addr;
  if (n > 0 && first < insn_region_bytes_)
    return unsupported("STORE into the instruction region (self-modifying program)");
  if (n > 0 && first < shared_bytes_)
    return fault(TAC_E_SHARED_WRITE, "STORE may write the shared read-only DRAM region");
  cycles_ += x.xfer_len;
  if (n == 0) return 0;
  uint32_t u0 = unit_of(x.buf_id, x.sram_off);
  uint64_t nu = n / kUnit;
  if (!dyn) {
    uint64_t i0 = addr / kUnit - ro_units_;
    for (uint64_t i = 0; i < nu; ++i) shadow_[i0 + i] = sram_[u0 + i];  // lazy: flushed at the end
    return 0;
  }
  uint64_t i0 = (lo - shared_bytes_) / kUnit;
  uint64_t i1 = std::min<uint64_t>(rw_units_, (hi - shared_bytes_ + kUnit - 1) / kUnit);
  flush_rw(i0, i1);
  break_aliases(i0, i1);
  Access acc;
  DevOp op = blank(K_DYN_STORE);
  op.a = src(u0, n, acc);
  op.param = param;
  op.dconst = int64_t(x.dram_off) * kUnit;
  op.nbytes = n;
  acc.writes.push_back({rw_home(i0), i1 - i0});
  acc.dyn_param = param;
  acc.dyn_write = true;
  acc.dyn_c0 = op.dconst;
  acc.dyn_c1 = op.dconst + int64_t(n);
  if (absorb_store(op, acc)) return 0;
  emit(op, acc);
  return 0;
}

int Compiler::h_buf_copy(const Insn& x) {                   // dma.py:67-97
  uint64_t n = uint64_t(x.length) * kUnit;
  uint32_t su = unit_of(x.src_buf, x.src_off), du = unit_of(x.dst_buf_b, x.dst_off_b);
  auto dst_fits = [&]() -> int {
    if (sram_span_ok(x.dst_buf_b, x.dst_off_b, n)) return 0;
    if (x.dst_buf_b == BUF_ACCUM)
      return value_fault("could not broadcast input array from shape (" + std::to_string(n) +
                         ",) into shape (" +
                         std::to_string(uint64_t(kBufUnits[BUF_ACCUM]) * kUnit - x.dst_off_b * kUnit) +
                         ",)");
    return sram_fault(x.dst_buf_b, x.dst_off_b);
  };
  if (!x.transpose) {
    if (!sram_span_ok(x.src_buf, x.src_off, n)) return sram_fault(x.src_buf, x.src_off);
    if (int s = dst_fits()) return s;
    std::vector<uint64_t> tmp(sram_.begin() + su, sram_.begin() + su + n / kUnit);
    for (uint64_t i = 0; i < tmp.size(); ++i) sram_[du + i] = tmp[i];  // alias
    cycles_ += x.length;
    return 0;
  }
  uint64_t rows = uint64_t(x.src_rows) * 16;
  if (rows == 0) return 0;
  uint64_t cols = n / rows;
  if (cols == 0) return 0;
  if (!sram_span_ok(x.src_buf, x.src_off, n)) return sram_fault(x.src_buf, x.src_off);
  if (rows * cols != n)
    return value_fault("cannot reshape array of size " + std::to_string(n) + " into shape (" +
                       std::to_string(rows) + "," + std::to_string(cols) + ")");
  if (int s = dst_fits()) return s;
  Access acc;
  DevOp op = blank(K_TRANSPOSE);
  op.M = static_cast<uint32_t>(rows);
  op.N = static_cast<uint32_t>(cols);
  op.a = src(su, n, acc);
  op.d = dst(du, n, acc);
  emit_compute(op, acc, du, -1);
  // a MATMUL may later read the source with F_BT instead (immutable sources only)
  const uint64_t out = sram_[du];
  if (cls(op.a) == PC_ARENA && cls(out) == PC_ARENA) transposed_[out] = TransposeOf{op.a, rows, cols};
  cycles_ += x.length;
  return 0;
}

int Compiler::h_set_scale(const Insn& x) {                  // simulator.py:605-617
  if (x.src_mode == 0) {
    sreg_[x.sreg] = kSregConst | x.imm16;
    return 0;
  }
  int buf = x.src_mode == 1 ? BUF_ABUF : (x.src_mode == 2 ? BUF_WBUF : BUF_ACCUM);
  if (x.imm16 >= kBufUnits[buf] || !sram_span_ok(buf, x.imm16, 2)) return sram_fault(buf, x.imm16);
  Access acc;
  DevOp op = blank(K_SREG_LOAD);
  op.a = src(unit_of(buf, x.imm16), 2, acc);
  op.out_slot = new_slot();
  acc.slot_writes.push_back(op.out_slot);
  sreg_[x.sreg] = op.out_slot;
  emit_compute(op, acc, 0, x.sreg);
  return 0;
}

int Compiler::h_config_attn(const Insn& x) {                // simulator.py:567-580
  if (!tile_valid_) return config_fault("CONFIG_TILE not set");
  auto it = var_pc_.find(pc_);
  if (it != var_pc_.end()) {
    int site = it->second.first;
    RtCheck c{};
    c.kind = CHK_ATTN_SET;
    c.param = static_cast<uint32_t>(site);
    c.pc = pc_;
    P->checks.push_back(c);
    attn_kind_ = 2;
    attn_param_ = site;
    return 0;
  }
  if (x.mode == 0) return config_fault("CONFIG_ATTN mode 0b00 is reserved");
  if (x.vkl == 0) return config_fault("CONFIG_ATTN valid_kv_len must be > 0");
  attn_kind_ = 1;
  attn_qrb_ = x.qrb;
  attn_vkl_ = x.vkl;
  attn_mode_ = x.mode;
  return 0;
}

// simulator.py:582-603 (_validate_attn_context_for_key_cols).
int Compiler::attn_keys_check(uint32_t key_cols, DevOp& op) {
  if (!tile_valid_) return config_fault("CONFIG_TILE not set");
  if (attn_kind_ == 0) return config_fault("CONFIG_ATTN not set");
  if (attn_kind_ == 2) {
    RtCheck c{};
    c.kind = CHK_ATTN_KEYS;
    c.param = static_cast<uint32_t>(attn_param_);
    c.pc = pc_;
    c.lo = key_cols;
    P->checks.push_back(c);
    op.flags |= F_ATTN_DYN;
    op.param = attn_param_;
    return 0;
  }
  if (attn_mode_ == 0) return config_fault("CONFIG_ATTN mode 0b00 is reserved");
  if (attn_vkl_ == 0) return config_fault("CONFIG_ATTN valid_kv_len must be > 0");
  if ((attn_mode_ == 1 || attn_mode_ == 3) && key_cols < attn_vkl_)
    return config_fault("CONFIG_ATTN valid_kv_len=" + std::to_string(attn_vkl_) +
                        " exceeds softmax key columns " + std::to_string(key_cols));
  if (attn_mode_ == 2 && key_cols != attn_vkl_)
    return config_fault("CONFIG_ATTN pure-causal mode requires softmax key columns " +
                        std::to_string(key_cols) + " to equal valid_kv_len=" +
                        std::to_string(attn_vkl_));
  op.attn_qrb = attn_qrb_;
  op.attn_vkl = attn_vkl_;
  op.attn_mode = attn_mode_;
  return 0;
}

int Compiler::h_rtype(const Insn& x) {
  const uint8_t o = x.op;
  // Masked variants validate the attention context before their handler runs
  // (simulator.py:521-525, 534-542, 556-560).
  DevOp op = blank(0);
  if (o == OP_MASKED_SOFTMAX || o == OP_MASKED_SOFTMAX_FP32 || o == OP_MASKED_SOFTMAX_ATTNV) {
    if (!tile_valid_) return config_fault("CONFIG_TILE not set");
    uint32_t keys = (o == OP_MASKED_SOFTMAX_ATTNV ? tile_[2] + 1 : tile_[1] + 1) * 16;
    if (int s = attn_keys_check(keys, op)) return s;
  }
  if (!tile_valid_) return config_fault("CONFIG_TILE not set");
  const uint64_t M = (tile_[0] + 1) * 16ull, N = (tile_[1] + 1) * 16ull, K = (tile_[2] + 1) * 16ull;
  op.M = static_cast<uint32_t>(M);
  op.N = static_cast<uint32_t>(N);
  op.K = static_cast<uint32_t>(K);
  const uint32_t s1 = unit_of(x.src1_buf, x.src1_off), s2 = unit_of(x.src2_buf, x.src2_off),
                 d = unit_of(x.dst_buf, x.dst_off);
  Access acc;

  // Helpers mirroring memory.py read/write tile functions (ACCUM rules + end checks).
  auto rd_i8 = [&](int buf, uint64_t off, uint64_t nbytes) -> int {
    if (buf == BUF_ACCUM) return value_fault("Use read_int32_tile for ACCUM buffer");
    if (!sram_span_ok(buf, off, nbytes)) return sram_fault(buf, off);
    return 0;
  };
  auto wr_i8 = [&](int buf, uint64_t off, uint64_t nbytes) -> int {
    if (buf == BUF_ACCUM) return value_fault("Use write_int32_tile for ACCUM buffer");
    if (!sram_span_ok(buf, off, nbytes)) return sram_fault(buf, off);
    return 0;
  };
  auto span = [&](int buf, uint64_t off, uint64_t nbytes) -> int {
    if (!sram_span_ok(buf, off, nbytes)) return sram_fault(buf, off);
    return 0;
  };
  auto need_accum_src1 = [&]() -> int {
    if (x.src1_buf != BUF_ACCUM) return ibuf_fault(x.src1_buf);
    if (x.src2_buf == BUF_ACCUM) return ibuf_fault(x.src2_buf);
    if (x.dst_buf == BUF_ACCUM) return ibuf_fault(x.dst_buf);
    return 0;
  };
#define TRY(e) do { if (int _s = (e)) return _s; } while (0)

  switch (o) {
    case OP_MATMUL: {                                        // systolic.py:31-71
      TRY(rd_i8(x.src1_buf, x.src1_off, M * K));
      TRY(rd_i8(x.src2_buf, x.src2_off, K * N));
      if (x.flags & 1) TRY(span(x.dst_buf, x.dst_off, M * N * 4));
      TRY(span(x.dst_buf, x.dst_off, M * N * 4));
      op.kind = K_MATMUL;
      if (!mm_b_source(s2, M, N, K, acc, op)) op.b = src(s2, K * N, acc);
      if (!mm_a_source(s1, M, N, K, acc, op)) op.a = src(s1, M * K, acc);
      if (x.flags & 1) {
        op.flags |= F_ACCUMULATE;
        op.c = src(d, M * N * 4, acc);
      }
      op.d = dst(d, M * N * 4, acc);
      cycles_ += (M / 16) * (N / 16) * (K / 16) * 16;
      break;
    }
    case OP_REQUANT: {                                       // simulator.py:629-659
      TRY(span(x.src1_buf, x.src1_off, M * N * 4));
      TRY(wr_i8(x.dst_buf, x.dst_off, M * N));
      op.kind = K_REQUANT;
      op.s[0] = sreg_[x.sreg];
      read_sreg(acc, op.s[0]);
      op.a = src(s1, M * N * 4, acc);
      op.d = dst(d, M * N, acc);
      cycles_ += M * N;
      break;
    }
    case OP_REQUANT_PC: {                                    // simulator.py:661-688
      TRY(need_accum_src1());
      TRY(span(x.src1_buf, x.src1_off, M * N * 4));
      TRY(span(x.src2_buf, x.src2_off, N * 2));
      TRY(wr_i8(x.dst_buf, x.dst_off, M * N));
      op.kind = K_REQUANT_PC;
      op.a = src(s1, M * N * 4, acc);
      op.b = src(s2, N * 2, acc);
      op.d = dst(d, M * N, acc);
      cycles_ += M * N;
      break;
    }
    case OP_SCALE_MUL: {                                     // simulator.py:690-722
      op.s[0] = sreg_[x.sreg];
      if (x.src1_buf == BUF_ACCUM) {
        TRY(span(x.src1_buf, x.src1_off, M * N * 4));
        TRY(span(x.dst_buf, x.dst_off, M * N * 4));
        op.kind = K_SCALE_MUL_I32;
        read_sreg(acc, op.s[0]);
        op.a = src(s1, M * N * 4, acc);
        op.d = dst(d, M * N * 4, acc);
      } else {
        TRY(rd_i8(x.src1_buf, x.src1_off, M * N));
        TRY(wr_i8(x.dst_buf, x.dst_off, M * N));
        op.kind = K_SCALE_MUL_I8;
        read_sreg(acc, op.s[0]);
        op.a = src(s1, M * N, acc);
        op.d = dst(d, M * N, acc);
      }
      cycles_ += M * N;
      break;
    }
    case OP_VADD: {                                          // simulator.py:724-760
      if (x.src1_buf == BUF_ABUF) {
        TRY(rd_i8(x.src1_buf, x.src1_off, M * N));
        TRY(rd_i8(x.src2_buf, x.src2_off, M * N));
        TRY(wr_i8(x.dst_buf, x.dst_off, M * N));
        op.kind = K_VADD_I8;
        op.a = src(s1, M * N, acc);
        op.b = src(s2, M * N, acc);
        op.d = dst(d, M * N, acc);
      } else if (x.src1_buf == BUF_ACCUM) {
        TRY(span(x.src1_buf, x.src1_off, M * N * 4));
        TRY(span(x.src2_buf, x.src2_off, N * 4));
        TRY(span(x.dst_buf, x.dst_off, M * N * 4));
        op.kind = K_VADD_I32;
        op.a = src(s1, M * N * 4, acc);
        op.b = src(s2, N * 4, acc);
        op.d = dst(d, M * N * 4, acc);
      } else {
        return ibuf_fault(x.src1_buf);
      }
      cycles_ += M * N;
      break;
    }
    case OP_DEQUANT_ADD: {                                   // simulator.py:762-788
      TRY(need_accum_src1());
      if (x.sreg >= 15) return config_fault("DEQUANT_ADD sreg+1 out of range");
      TRY(span(x.src1_buf, x.src1_off, M * N * 4));
      TRY(rd_i8(x.src2_buf, x.src2_off, M * N));
      TRY(wr_i8(x.dst_buf, x.dst_off, M * N));
      op.kind = K_DEQUANT_ADD;
      op.s[0] = sreg_[x.sreg];
      op.s[1] = sreg_[x.sreg + 1];
      read_sreg(acc, op.s[0]);
      read_sreg(acc, op.s[1]);
      op.a = src(s1, M * N * 4, acc);
      op.b = src(s2, M * N, acc);
      op.d = dst(d, M * N, acc);
      cycles_ += M * N;
      break;
    }
    case OP_DEQUANT_ACCUM_FP32:                              // simulator.py:808-833
    case OP_DEQUANT_ACCUM_FP32_SCALED: {                     // simulator.py:1043-1086
      TRY(need_accum_src1());
      const uint64_t vec = (o == OP_DEQUANT_ACCUM_FP32 ? N : 2 * N) * 2;
      TRY(span(x.src1_buf, x.src1_off, M * N * 4));
      TRY(span(x.src2_buf, x.src2_off, vec));
      TRY(span(x.dst_buf, x.dst_off, M * N * 2));
      if (o == OP_DEQUANT_ACCUM_FP32 && fuse_dequant(s1, s2, d, M, N)) {
        cycles_ += M * N;
        return 0;
      }
      if (o == OP_DEQUANT_ACCUM_FP32_SCALED && fuse_dequant_scaled(s1, s2, d, M, N, sreg_[x.sreg])) {
        cycles_ += M * N;
        return 0;
      }
      op.kind = o == OP_DEQUANT_ACCUM_FP32 ? K_DEQUANT_ACCUM : K_DEQUANT_SCALED;
      if (o == OP_DEQUANT_ACCUM_FP32_SCALED) {
        op.s[0] = sreg_[x.sreg];
        read_sreg(acc, op.s[0]);
      }
      op.a = src(s1, M * N * 4, acc);
      if (o == OP_DEQUANT_ACCUM_FP32_SCALED) src_pair(s2, N * 2, acc, op);
      else op.b = src(s2, vec, acc);
      op.d = dst(d, M * N * 2, acc);
      cycles_ += M * N;
      break;
    }
    case OP_QUANT_FP32_INT8: {                               // simulator.py:835-867
      if (x.src1_buf == BUF_ACCUM) return ibuf_fault(x.src1_buf);
      if (x.dst_buf == BUF_ACCUM) return ibuf_fault(x.dst_buf);
      TRY(span(x.src1_buf, x.src1_off, M * N * 2));
      TRY(span(x.dst_buf, x.dst_off, M * N));
      op.kind = K_QUANT;
      op.s[0] = sreg_[x.sreg];
      if (fuse_quant_into_maxabs(op, s1, d, M, N)) return 0;
      read_sreg(acc, op.s[0]);
      if (!src_segments(s1, M * N * 2, acc, op)) op.a = src(s1, M * N * 2, acc);
      op.d = dst(d, M * N, acc);
      cycles_ += M * N;
      break;
    }
    case OP_VADD_FP32:                                       // simulator.py:869-891
    case OP_LAYERNORM_FP32: {                                // simulator.py:893-934
      if (x.src1_buf == BUF_ACCUM || x.src2_buf == BUF_ACCUM) return ibuf_fault(BUF_ACCUM);
      if (x.dst_buf == BUF_ACCUM) return ibuf_fault(x.dst_buf);
      const uint64_t b_bytes = o == OP_VADD_FP32 ? M * N * 2 : 2 * N * 2;
      TRY(span(x.src1_buf, x.src1_off, M * N * 2));
      TRY(span(x.src2_buf, x.src2_off, b_bytes));
      TRY(span(x.dst_buf, x.dst_off, M * N * 2));
      op.kind = o == OP_VADD_FP32 ? K_VADD_F16 : K_LAYERNORM_F16;
      if (o == OP_VADD_FP32 && extend_vadd_chain(s1, s2, d, M, N)) {
        cycles_ += M * N;
        return 0;
      }
      if (o == OP_LAYERNORM_FP32) {
        op.a = src(s1, M * N * 2, acc);
        src_pair(s2, N * 2, acc, op);
      } else if (src_segments(s1, M * N * 2, acc, op)) {
        op.b = src(s2, b_bytes, acc);
      } else if (src_segments(s2, b_bytes, acc, op)) {   // a + b == b + a exactly: read b as the list
        op.b = src(s1, M * N * 2, acc);
      } else {
        op.a = src(s1, M * N * 2, acc);
        op.b = src(s2, b_bytes, acc);
      }
      op.d = dst(d, M * N * 2, acc);
      cycles_ += M * N;
      break;
    }
    case OP_GELU_FP32:                                       // simulator.py:936-962
    case OP_SOFTMAX_FP32:                                    // simulator.py:964-988
    case OP_MASKED_SOFTMAX_FP32: {                           // simulator.py:990-1037
      if (x.src1_buf == BUF_ACCUM) return ibuf_fault(x.src1_buf);
      if (x.dst_buf == BUF_ACCUM) return ibuf_fault(x.dst_buf);
      TRY(span(x.src1_buf, x.src1_off, M * N * 2));
      TRY(span(x.dst_buf, x.dst_off, M * N * 2));
      op.kind = o == OP_GELU_FP32 ? K_GELU_F16
                                  : (o == OP_SOFTMAX_FP32 ? K_SOFTMAX_F16 : K_MASKED_SOFTMAX_F16);
      if (op.kind != K_GELU_F16 && fuse_softmax(s1, d, M, N, op)) {
        cycles_ += M * N;
        return 0;
      }
      if (op.kind != K_GELU_F16 || !src_segments(s1, M * N * 2, acc, op)) op.a = src(s1, M * N * 2, acc);
      op.d = dst(d, M * N * 2, acc);
      cycles_ += M * N;
      break;
    }
    case OP_MAX_ABS_REDUCE_FP32: {                           // simulator.py:1088-1140
      if (x.src1_buf == BUF_ACCUM) return ibuf_fault(x.src1_buf);
      if (x.sreg >= 15) return config_fault("MAX_ABS_REDUCE_FP32 sreg+1 out of range (must be 0..14)");
      TRY(span(x.src1_buf, x.src1_off, M * N * 2));
      op.kind = K_MAX_ABS;
      if (!src_segments(s1, M * N * 2, acc, op)) op.a = src(s1, M * N * 2, acc);
      gelu_into_maxabs(op, acc, M * N * 2 / kUnit);
      op.out_slot = new_slot();
      new_slot();
      acc.slot_writes.push_back(op.out_slot);
      acc.slot_writes.push_back(op.out_slot + 1);
      sreg_[x.sreg] = op.out_slot;
      sreg_[x.sreg + 1] = op.out_slot + 1;
      maxabs_pending_ = std::vector<uint64_t>(&sram_[s1], &sram_[s1] + (M * N * 2 + kUnit - 1) / kUnit);
      cycles_ += M * N;
      break;
    }
    case OP_LAYERNORM: {                                     // sfu.py:149-190
      if (x.sreg >= 15) return config_fault("SFU sreg+1 out of range");
      TRY(rd_i8(x.src1_buf, x.src1_off, M * N));
      TRY(span(x.src2_buf, x.src2_off, N * 4));
      TRY(wr_i8(x.dst_buf, x.dst_off, M * N));
      op.kind = K_LN_I8;
      op.s[0] = sreg_[x.sreg];
      op.s[1] = sreg_[x.sreg + 1];
      read_sreg(acc, op.s[0]);
      read_sreg(acc, op.s[1]);
      op.a = src(s1, M * N, acc);
      op.b = src(s2, N * 4, acc);
      op.d = dst(d, M * N, acc);
      cycles_ += M * N * 2;
      break;
    }
    case OP_SOFTMAX:                                         // sfu.py:193-235
    case OP_MASKED_SOFTMAX:                                  // sfu.py:238-272
    case OP_GELU: {                                          // sfu.py:275-320
      if (x.sreg >= 15) return config_fault("SFU sreg+1 out of range");
      uint64_t in_bytes = M * N;
      if (x.src1_buf == BUF_ACCUM) {
        op.flags |= F_SRC_I32;
        in_bytes = M * N * 4;
        TRY(span(BUF_ACCUM, x.src1_off, in_bytes));
      } else {
        TRY(rd_i8(x.src1_buf, x.src1_off, in_bytes));
      }
      TRY(wr_i8(x.dst_buf, x.dst_off, M * N));
      op.kind = o == OP_SOFTMAX ? K_SOFTMAX_I8 : (o == OP_GELU ? K_GELU_I8 : K_MASKED_SOFTMAX_I8);
      op.s[0] = sreg_[x.sreg];
      op.s[1] = sreg_[x.sreg + 1];
      read_sreg(acc, op.s[0]);
      read_sreg(acc, op.s[1]);
      op.a = src(s1, in_bytes, acc);
      op.d = dst(d, M * N, acc);
      cycles_ += M * N * 2;
      break;
    }
    case OP_SOFTMAX_ATTNV:                                   // sfu.py:323-381
    case OP_MASKED_SOFTMAX_ATTNV: {                          // sfu.py:384-443
      TRY(need_accum_src1());
      if (x.sreg >= 13) return config_fault("SFU sreg+3 out of range");
      TRY(span(BUF_ACCUM, x.src1_off, M * K * 4));
      TRY(rd_i8(x.src2_buf, x.src2_off, K * N));
      TRY(wr_i8(x.dst_buf, x.dst_off, M * N));
      op.kind = o == OP_SOFTMAX_ATTNV ? K_SOFTMAX_ATTNV : K_MASKED_SOFTMAX_ATTNV;
      for (int i = 0; i < 4; ++i) {
        op.s[i] = sreg_[x.sreg + i];
        read_sreg(acc, op.s[i]);
      }
      op.a = src(s1, M * K * 4, acc);
      op.b = src(s2, K * N, acc);
      op.d = dst(d, M * N, acc);
      cycles_ += M * K * 2 + (M / 16) * (N / 16) * (K / 16) * 16 + M * N;
      break;
    }
    default:
      return unsupported("unhandled opcode");
  }
#undef TRY
  if (op.kind == K_MATMUL && !(op.b & kSharedBit) &&
      wide_mm_ok(uint32_t(M), uint32_t(N), uint32_t(K), op.flags & F_BT, op.flags & F_QB, op.flags & F_QA))
    op.flags |= F_WIDE;
  const int32_t pv_x = op.kind == K_MATMUL ? pv_partner(op, acc) : -1;
  const size_t n_before = P->ops.size();
  const int32_t chain_lv = pv_x < 0 ? chain_level(op, acc) : -1;
  if (pv_x >= 0) force_level_ = static_cast<int32_t>(P->ops[pv_x].level);
  if (chain_lv >= 0) force_level_ = chain_lv;
  emit_compute(op, acc, d, x.sreg);
  force_level_ = -1;
  if (chain_lv >= 0 && P->ops.size() == n_before + 1) P->ops.back().flags2 |= FX_CHAINED;
  if (pv_x >= 0 && P->ops.size() == n_before + 1) {
    const uint32_t y = static_cast<uint32_t>(n_before);
    pv_of_[static_cast<uint32_t>(pv_x)] = y;
    DevOp& xo = P->ops[pv_x];
    xo.flags2 |= FX_PV;
    if ((op.flags & F_QB) && pvpf_ok(xo.M, xo.N, xo.K, op.N, op.flags & F_BT)) xo.flags2 |= FX_PVPF;
    P->ops[y].flags2 |= FX_PVY;
    auto& rd = op_arena_reads_[y];   // read inside the QK^T task: keeps nothing else live
    rd.erase(std::remove_if(rd.begin(), rd.end(),
                            [&](const std::pair<uint64_t, uint64_t>& r) { return r.first == op.a; }),
             rd.end());
  }
  if (op.kind == K_VADD_F16 && !(op.flags & F_SEGA) && !P->ops.empty() && P->ops.back().kind == K_VADD_F16 &&
      P->ops.back().d == op.d && cls(op.d) == PC_ARENA)
    vadd_tail_[op.d] = static_cast<uint32_t>(P->ops.size() - 1);
  if (op.kind == K_GELU_F16 && P->ops.size() == n_before + 1 && (op.flags & ~F_SEGA) == 0 &&
      cls(P->ops.back().d) == PC_ARENA)
    gelu_out_[P->ops.back().d] = static_cast<uint32_t>(n_before);
  if (op.kind == K_MAX_ABS) {   // remember the input of the MAX_ABS just emitted
    if (!P->ops.empty() && P->ops.back().kind == K_MAX_ABS && P->ops.back().out_slot == op.out_slot) {
      MaxAbsOf& m = maxabs_by_slot_[op.out_slot];
      m.op = static_cast<uint32_t>(P->ops.size() - 1);
      m.units = std::move(maxabs_pending_);
      m.elems = M * N;
    }
    maxabs_pending_.clear();
  }
  if (op.kind == K_QUANT && !(op.flags & F_SEGA) && cls(sram_[d]) == PC_ARENA)
    quantized_[sram_[d]] = QuantOf{op.a, op.s[0], M, N, home_writes_};
  if (op.kind == K_MATMUL && (op.flags & F_WIDE) && !(op.flags & F_ACCUMULATE) && !P->ops.empty() &&
      P->ops.back().kind == K_MATMUL && P->ops.back().d == op.d)
    mm_out_[op.d] = static_cast<uint32_t>(P->ops.size() - 1);
  if (op.kind == K_MATMUL && tc_eligible(op.a, op.b, op.M, op.N, op.K) && !(op.flags & F_ACCUMULATE) &&
      !P->ops.empty() && P->ops.back().kind == K_MATMUL && P->ops.back().d == op.d)
    tc_out_[op.d] = static_cast<uint32_t>(P->ops.size() - 1);
  return 0;
}

int Compiler::step(const Insn& x) {
  switch (x.op) {
    case OP_NOP:
    case OP_SYNC:
      cycles_ += 1;
      return 0;
    case OP_HALT:
      halted_ = true;
      return 0;
    case OP_CONFIG_TILE:
      tile_valid_ = true;
      tile_[0] = x.tm;
      tile_[1] = x.tn;
      tile_[2] = x.tk;
      return 0;
    case OP_CONFIG_ATTN:
      return h_config_attn(x);
    case OP_SET_SCALE:
      return h_set_scale(x);
    case OP_SET_ADDR_LO:
    case OP_SET_ADDR_HI: {                                   // simulator.py:619-627
      AddrReg& r = areg_[x.addr_reg];
      auto it = var_pc_.find(pc_);
      if (it != var_pc_.end()) {
        const tac_var_site& s = sites_[it->second.first];
        if (s.kind != 0 || s.addr_reg != x.addr_reg)
          return unsupported("runtime SET_ADDR site does not match its instruction");
        if (it->second.second == 0) {
          r.kind = 2;  // LO written, HI pending
          r.known = 0;
        } else {
          r.kind = 1;
          r.param = it->second.first;
          r.lo = s.range_lo;
          r.hi = s.range_hi;
        }
        return 0;
      }
      if (r.kind == 1) {  // a static half over a runtime value
        r.kind = 2;
        r.known = 0;
        r.value = 0;
      }
      if (x.op == OP_SET_ADDR_LO) {
        r.value = (r.value & ~0xFFFFFFFull) | x.imm28;
        r.known |= 1;
      } else {
        r.value = (r.value & 0xFFFFFFFull) | (uint64_t(x.imm28) << 28);
        r.known |= 2;
      }
      if (r.kind == 2 && r.known == 3) r.kind = 0;
      return 0;
    }
    case OP_LOAD:
      return h_load(x);
    case OP_STORE:
      return h_store(x);
    case OP_BUF_COPY:
      return h_buf_copy(x);
    default:
      return h_rtype(x);
  }
}

// Materialises the architectural state at the end of the run: writable DRAM,
// SRAM home images and scale registers.
void Compiler::finalize() {
  // 1. writable DRAM units whose value lives elsewhere
  flush_live(0, rw_units_);
  // 2. SRAM units whose value is not in place
  std::vector<uint32_t> moved;
  const bool sram_live = !opts_ || opts_->sram_live;
  for (uint32_t u = 0; sram_live && u < kSramUnits; ++u)
    if (sram_[u] != u) moved.push_back(u);
  if (!moved.empty()) {
    // Values still held in SRAM home locations are first copied out, so the
    // final copy never reads a unit it also writes.
    std::vector<uint64_t> from_home;
    for (uint32_t u : moved)
      if (cls(sram_[u]) == PC_HOME_SRAM) from_home.push_back(sram_[u]);
    if (!from_home.empty()) {
      std::vector<uint64_t> uniq = from_home;
      std::sort(uniq.begin(), uniq.end());
      uniq.erase(std::unique(uniq.begin(), uniq.end()), uniq.end());
      // gather them (in sorted order) into one extent and remap
      uint64_t g = gather(uniq.data(), uniq.size());
      for (uint32_t u : moved) {
        if (cls(sram_[u]) == PC_HOME_SRAM) {
          uint64_t k = std::lower_bound(uniq.begin(), uniq.end(), sram_[u]) - uniq.begin();
          sram_[u] = g + k;
        }
      }
    }
    DevOp op = blank(K_GATHER);
    op.seg0 = static_cast<uint32_t>(P->segs.size());
    Access acc;
    size_t k = 0;
    while (k < moved.size()) {
      size_t j = k + 1;
      while (j < moved.size() && moved[j] == moved[k] + (j - k) &&
             sram_[moved[j]] == sram_[moved[k]] + (j - k) &&
             cls(sram_[moved[j]]) == cls(sram_[moved[k]]))
        ++j;
      uint64_t n = j - k;
      push_seg(sram_[moved[k]], uint64_t(moved[k]), n);
      acc.reads.push_back({sram_[moved[k]], n});
      acc.writes.push_back({uint64_t(moved[k]), n});
      k = j;
    }
    op.nseg = static_cast<uint32_t>(P->segs.size() - op.seg0);
    emit(op, acc);
    for (uint32_t u : moved) sram_[u] = u;
  }
  // 3. scale registers
  if (opts_ && !opts_->sregs_live) return;
  bool any = false;
  for (int r = 0; r < 16; ++r) any |= sreg_[r] != uint32_t(r);
  if (any) {
    DevOp op = blank(K_SREG_FINAL);
    op.seg0 = static_cast<uint32_t>(P->segs.size());
    Access acc;
    for (int r = 0; r < 16; ++r) {
      if (sreg_[r] == uint32_t(r)) continue;
      P->segs.push_back(Segment{sreg_[r], uint64_t(r), 0});
      read_sreg(acc, sreg_[r]);
    }
    op.nseg = static_cast<uint32_t>(P->segs.size() - op.seg0);
    acc.sreg_home_write = true;
    emit(op, acc);
  }
}

// Row structure of a row-wise op: output row r depends only on row r of its
// row operands (plus vectors, weights and registers every row shares), so rows
// that no later op reads need not be computed.  Gives the element bytes of the
// row operands; a tcgen05 MATMUL (shared weights, no accumulate, at most the
// DEQUANT_SCALED epilogue) counts, its A rows being K int8 bytes.
static bool row_wise(const DevOp& op0, uint32_t& in_es) {
  DevOp op = op0;
  op.flags2 &= ~FX_CHAINED;   // chained or not, the op's rows are its own
  switch (op.kind) {
    case K_VADD_F16: case K_GELU_F16: in_es = 2; return op.flags2 == 0 && (op.flags & ~F_SEGA) == 0;
    case K_QUANT: in_es = 2; return op.flags2 == 0 && (op.flags & ~F_SEGA) == 0;
    case K_LAYERNORM_F16: in_es = 2; return op.flags2 == 0 && (op.flags & ~F_SPLIT) == 0;
    case K_SOFTMAX_F16: in_es = 2; return op.flags2 == 0 && op.flags == 0;
    case K_MASKED_SOFTMAX_F16: in_es = 2; return op.flags2 == 0 && (op.flags & ~F_ATTN_DYN) == 0;
    case K_DEQUANT_ACCUM: in_es = 4; return op.flags2 == 0 && op.flags == 0;
    case K_DEQUANT_SCALED: in_es = 4; return op.flags2 == 0 && (op.flags & ~F_SPLIT) == 0;
    case K_VADD_CHAIN: in_es = 2; return op.flags2 == 0 && op.flags == 0;
    case K_MATMUL:
      in_es = 1;
      return tc_eligible(op.a, op.b, op.M, op.N, op.K) && (op.flags & ~F_NOI32) == 0 &&
             (op.flags2 & ~(FX_DQS | FX_DSTORE)) == 0 && (!(op.flags & F_NOI32) || (op.flags2 & FX_DQS));
    default: return false;
  }
}

// The outputs of a row-wise op as (first unit, units per row): its
// destination, a chain's stored sums, a MATMUL's int32 and FP16 results.
static std::vector<std::pair<uint64_t, uint64_t>> row_outputs(const DevOp& op, const std::vector<Segment>* chain) {
  std::vector<std::pair<uint64_t, uint64_t>> o;
  const uint64_t n = op.N;
  switch (op.kind) {
    case K_VADD_CHAIN:
      for (size_t k = 1; k < chain->size(); ++k)
        if ((*chain)[k].dst) o.push_back({(*chain)[k].dst, n * 2 / kUnit});
      break;
    case K_QUANT: o.push_back({op.d, n / kUnit}); break;
    case K_MATMUL:
      if (!(op.flags & F_NOI32)) o.push_back({op.d, n * 4 / kUnit});
      if (op.flags2 & FX_DQS) o.push_back({static_cast<uint64_t>(op.dconst), n * 2 / kUnit});
      break;
    default: o.push_back({op.d, n * 2 / kUnit}); break;
  }
  return o;
}

// The ranges a row-wise op reads when it computes rows [0, m): the first m
// rows of each row operand (for a segment list, the runs' parts below m rows)
// and every vector operand whole.  `chain` holds a K_VADD_CHAIN's operands.
template <class F>
static void row_reads(const DevOp& op, uint32_t m, uint32_t in_es, const std::vector<Segment>& segs,
                      const std::vector<Segment>* chain, F&& cb) {
  const uint64_t ri = uint64_t(op.kind == K_MATMUL ? op.K : op.N) * in_es / kUnit, lim = m * ri;
  auto rows = [&](uint64_t p) { cb(p, lim); };
  auto vec = [&](uint64_t p, uint64_t bytes) { cb(p, (bytes + kUnit - 1) / kUnit); };
  auto seglist = [&]() {
    for (uint32_t k = op.seg0; k < op.seg0 + op.nseg; ++k)
      if (segs[k].dst < lim) cb(segs[k].src, std::min<uint64_t>(segs[k].n, lim - segs[k].dst));
  };
  const uint64_t vn = uint64_t(op.N) * 2;
  switch (op.kind) {
    case K_VADD_F16: (op.flags & F_SEGA) ? seglist() : rows(op.a); rows(op.b); break;
    case K_GELU_F16: case K_QUANT: (op.flags & F_SEGA) ? seglist() : rows(op.a); break;
    case K_SOFTMAX_F16: case K_MASKED_SOFTMAX_F16: rows(op.a); break;
    case K_LAYERNORM_F16: case K_DEQUANT_SCALED:
      rows(op.a);
      if (op.flags & F_SPLIT) { vec(op.b, vn); vec(op.c, vn); } else vec(op.b, 2 * vn);
      break;
    case K_DEQUANT_ACCUM: rows(op.a); vec(op.b, vn); break;
    case K_VADD_CHAIN:
      for (const Segment& c : *chain) rows(c.src);
      break;
    case K_MATMUL:
      rows(op.a);
      vec(op.b, uint64_t(op.K) * op.N);
      if (op.flags2 & FX_DQS) { vec(op.c, vn); vec(op.nbytes, vn); }
      break;
    default: break;
  }
}

// Removes ops whose only effect is arena extents no kept op reads (a
// TRANSPOSE whose MATMUL reads its source instead, a value overwritten before
// use).  Walks the ops backwards, keeping an op when it has another effect or
// a kept op reads any unit it writes.
//
// A kept row-wise op whose later rows no kept op reads is narrowed to the
// rows that are read (M becomes that count, m_decl keeps the tile's rows),
// and only those rows of its row operands count as read; an FX_MAXQ MAX_ABS
// stores only the QUANT rows that are read (q_rows).  The decode streams
// reload their padding rows from a constant region before every MAX_ABS, so
// most row-wise work on them is dead.  A row-wise op is narrowed only when
// the reads it recorded while compiling are exactly the ranges row_reads
// gives for all of its rows.
void Compiler::drop_dead_ops() {
  const size_t n = P->ops.size();
  if (op_arena_reads_.size() != n || op_arena_writes_.size() != n || op_pure_.size() != n) return;
  // A K_VADD_CHAIN op sits at the index of its first VADD but reads operands
  // that ops emitted after it produce, so the walk meets those producers
  // first: the chain's reads of them are marked up front.  A first walk marks
  // them whole and finds the rows each chain computes; a second walk, from
  // the ops as they were, marks only those rows (the chains' readers all come
  // after their operands' producers, so the rows found do not change).
  const std::vector<DevOp> ops0 = P->ops;
  const auto chains0 = chains_;
  std::vector<uint64_t> chain_units(chains_.size(), ~0ull);   // units of each operand a chain reads
  std::vector<uint8_t> keep;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass) {
      P->ops = ops0;
      chains_ = chains0;
      narrowed_ops_ = 0;
    }
    drop_dead_walk(keep, chain_units);
    if (chains_.empty()) break;
    for (size_t i = 0; i < n; ++i)
      if (keep[i] && P->ops[i].kind == K_VADD_CHAIN) chain_units[ops0[i].param] = chains_[ops0[i].param][0].n;
  }
  size_t j = 0;
  for (size_t i = 0; i < n; ++i)
    if (keep[i]) P->ops[j++] = P->ops[i];
  dead_ops_ = n - j;
  P->ops.resize(j);
}

// One backward walk of drop_dead_ops: sets keep[] and narrows the kept ops;
// chain_units bounds the up-front marks of each chain's later operands.
void Compiler::drop_dead_walk(std::vector<uint8_t>& keep, const std::vector<uint64_t>& chain_units) {
  const size_t n = P->ops.size();
  std::vector<uint8_t> read(arena_top_, 0);
  keep.assign(n, 0);
  pv_rows_.clear();
  auto mark = [&](uint64_t phys, uint64_t units) {
    for (uint64_t u = 0; u < units; ++u) {
      const uint64_t k = phys - arena_base_ + u;
      if (k < read.size()) read[k] = 1;
    }
  };
  auto any_read = [&](uint64_t phys, uint64_t units) {
    for (uint64_t u = 0; u < units; ++u) {
      const uint64_t k = phys - arena_base_ + u;
      if (k >= read.size() || read[k]) return true;
    }
    return false;
  };
  // a chain's later operands, marked up front (a chain whose sum nobody reads
  // would keep its operands' producers, which the decode streams never have)
  for (size_t c = 0; c < chains_.size(); ++c)
    for (size_t k = 2; k < chains_[c].size(); ++k) mark(chains_[c][k].src, std::min(chains_[c][k].n, chain_units[c]));
  for (size_t i = n; i-- > 0;) {
    bool live = !op_pure_[i];
    for (auto& w : op_arena_writes_[i]) live = live || any_read(w.first, w.second);
    auto pv = pv_of_.find(static_cast<uint32_t>(i));
    const bool pv_kept = pv != pv_of_.end() && keep[pv->second];
    live = live || pv_kept;   // the task that runs a kept P.V op
    if (!live) continue;
    keep[i] = 1;
    DevOp& op = P->ops[i];
    if (op.flags2 & FX_PV) {
      if (!pv_kept) op.flags2 &= ~FX_PV;
      else if (!any_read(op.nbytes, uint64_t(op.M) * op.N * 2 / kUnit)) op.flags2 |= FX_SMSKIP;
    }
    if (((op.flags & F_DQ) || (op.flags2 & FX_DQS)) && cls(op.d) == PC_ARENA &&
        !any_read(op.d, uint64_t(op.M) * op.N * 4 / kUnit))
      op.flags |= F_NOI32;   // only the FP16 result is read
    if ((op.flags & F_SM) && !any_read(static_cast<uint64_t>(op.dconst), uint64_t(op.M) * op.N * 2 / kUnit))
      op.flags |= F_NODQ;    // only the softmax rows are read
    if (op.kind == K_VADD_CHAIN) {   // intermediate sums nobody reads are not stored (the last always is)
      auto& ch = chains_[op.param];
      for (size_t k = 1; k + 1 < ch.size(); ++k)
        if (ch[k].dst && !any_read(ch[k].dst, ch[k].n)) ch[k].dst = 0;
    }
    if (op.kind == K_MAX_ABS && (op.flags2 & FX_MAXQ) && op.N % kUnit == 0) {
      const uint64_t ro = op.N / kUnit;   // int8 QUANT rows
      uint32_t m = op.M;
      while (m > 0 && !any_read(op.d + (m - 1) * ro, ro)) --m;
      if (m < op.M) {
        op.q_rows = m > 0 ? m : 1;
        ++narrowed_ops_;
      }
    }
    // An attention pair (FX_PV QK^T + softmax, its P.V op run in the same
    // task): both are row-wise in the query rows.  The P.V op, met first,
    // records the rows of its results that are read; the QK^T op narrows the
    // pair to the rows either op's results need.  Only the QK^T op reads a row
    // operand (the FP16 Q rows); the P.V op reads the softmax rows in shared
    // memory, V and a scale row.
    if (op.kind == K_MATMUL && (op.flags2 & FX_PVY)) {
      std::vector<std::pair<uint64_t, uint64_t>> outs;
      if (!(op.flags & F_NOI32)) outs.push_back({op.d, uint64_t(op.N) * 4 / kUnit});
      if ((op.flags & F_DQ) && !(op.flags & F_NODQ)) outs.push_back({static_cast<uint64_t>(op.dconst), uint64_t(op.N) * 2 / kUnit});
      pv_rows_[i] = rows_read(op.M, outs, any_read);
    }
    if (op.kind == K_MATMUL && (op.flags2 & FX_PV) && op_pure_[i] && op.N % 8 == 0 && op.K % 8 == 0 &&
        (op.flags & (F_ACCUMULATE | F_WIDE | F_QA | F_SM)) == (F_WIDE | F_QA | F_SM) && (op.flags & F_DQ)) {
      const uint32_t y = pv_of_.at(static_cast<uint32_t>(i));
      std::vector<std::pair<uint64_t, uint64_t>> outs;
      if (!(op.flags & F_NOI32)) outs.push_back({op.d, uint64_t(op.N) * 4 / kUnit});
      if (!(op.flags & F_NODQ)) outs.push_back({static_cast<uint64_t>(op.dconst), uint64_t(op.N) * 2 / kUnit});
      if (!(op.flags2 & FX_SMSKIP)) outs.push_back({op.nbytes, uint64_t(op.N) * 2 / kUnit});
      const uint32_t m = std::max(rows_read(op.M, outs, any_read), pv_rows_.count(y) ? pv_rows_[y] : P->ops[y].M);
      const uint64_t ra = uint64_t(op.K) * 2 / kUnit;   // FP16 Q row
      auto reads = [&](uint32_t rows, auto&& cb) {
        cb(op.a, rows * ra);
        cb(op.b, uint64_t(op.K) * op.N * 2 / kUnit);
        cb(op.c, uint64_t(op.N) * 2 / kUnit);
      };
      if (m < op.M && P->ops[y].M == op.M && same_units(reads, op.M, op_arena_reads_[i])) {
        op.m_decl = op.M;
        op.M = m;
        P->ops[y].m_decl = P->ops[y].M;
        P->ops[y].M = m;
        reads(m, mark);
        narrowed_ops_ += 2;
        continue;
      }
    }
    uint32_t in_es = 0;
    // an absorbed store is the only effect of an FX_DSTORE MATMUL besides its arena results
    const bool store_only = (op.flags2 & FX_DSTORE) && pure_before_store_.count(static_cast<uint32_t>(i)) &&
                            pure_before_store_[static_cast<uint32_t>(i)];
    if ((op_pure_[i] || store_only) && row_wise(op, in_es) && (uint64_t(op.K) * in_es) % kUnit == 0 &&
        (uint64_t(op.N) * in_es) % kUnit == 0 && op.N % kUnit == 0) {
      const std::vector<Segment>* chain = op.kind == K_VADD_CHAIN ? &chains_[op.param] : nullptr;
      const auto outs = row_outputs(op, chain);
      auto row_read = [&](uint32_t r) {
        for (auto& o : outs)
          if (any_read(o.first + r * o.second, o.second)) return true;
        return false;
      };
      uint32_t m = op.M;
      while (m > 1 && !row_read(m - 1)) --m;
      if (op.flags2 & FX_DSTORE) m = std::max(m, op.attn_vkl);   // the rows the store writes out
      if (op.kind == K_MATMUL)   // 128 / m sequences share one tensor-core tile
        while (!tc_rows_ok(m) && m < op.M) ++m;
      if (m < op.M) {
        // the recorded reads must be exactly row_reads over every row
        auto reads = [&](uint32_t rows, auto&& cb) { row_reads(op, rows, in_es, P->segs, chain, cb); };
        if (same_units(reads, op.M, op_arena_reads_[i])) {
          op.m_decl = op.M;
          op.M = m;
          if (chain)
            for (Segment& c : chains_[op.param]) c.n = uint64_t(m) * op.N * 2 / kUnit;
          row_reads(op, m, in_es, P->segs, chain, mark);
          ++narrowed_ops_;
          continue;
        }
      }
    }
    for (auto& r : op_arena_reads_[i]) mark(r.first, r.second);
  }
}

// Each FX_PV op names its P.V op (seg0) by index in the final op list: the
// P.V op is the FX_PVY op whose A is this op's softmax output.
int Compiler::link_pv_pairs() {
  std::unordered_map<uint64_t, uint32_t> ys;
  for (uint32_t i = 0; i < P->ops.size(); ++i)
    if (P->ops[i].flags2 & FX_PVY) ys[P->ops[i].a] = i;
  for (DevOp& op : P->ops) {
    if (!(op.flags2 & FX_PV)) continue;
    auto it = ys.find(op.nbytes);
    if (it == ys.end()) return unsupported("internal: a QK^T task lost its P.V op");
    op.seg0 = it->second;
    op.nseg = 0;
    ys.erase(it);
  }
  if (!ys.empty()) return unsupported("internal: a P.V op lost its QK^T task");
  return 0;
}

// Each K_VADD_CHAIN's operand list goes to the segment table, contiguously.
void Compiler::write_vadd_chains() {
  for (DevOp& op : P->ops) {
    if (op.kind != K_VADD_CHAIN) continue;
    const auto& ch = chains_[op.param];
    op.seg0 = static_cast<uint32_t>(P->segs.size());
    op.nseg = static_cast<uint32_t>(ch.size());
    P->segs.insert(P->segs.end(), ch.begin(), ch.end());
    op.param = -1;
  }
}

// The runtime-addressed stores of one level (the K and V appends of every
// head) become one K_DYN_STORE_MULTI op, so each sequence takes one task for
// all of them.  Ops of one level are independent, so their order within the
// merged op does not matter.
void Compiler::merge_dyn_stores() {
  std::map<uint32_t, std::vector<uint32_t>> by_level;
  for (uint32_t i = 0; i < P->ops.size(); ++i) {
    const DevOp& op = P->ops[i];
    if (op.kind == K_DYN_STORE && op.param >= 0 && op.dconst >= 0 && op.dconst < (int64_t(1) << 32))
      by_level[op.level].push_back(i);
  }
  std::vector<uint8_t> drop(P->ops.size(), 0);
  std::vector<DevOp> merged;
  for (auto& kv : by_level) {
    if (kv.second.size() < 2) continue;
    DevOp m = blank(K_DYN_STORE_MULTI);
    m.level = kv.first;
    m.pc = P->ops[kv.second.front()].pc;
    m.seg0 = static_cast<uint32_t>(P->segs.size());
    for (uint32_t i : kv.second) {
      const DevOp& op = P->ops[i];
      P->segs.push_back(Segment{op.a, (uint64_t(uint32_t(op.param)) << 32) | uint64_t(op.dconst), op.nbytes});
      drop[i] = 1;
    }
    m.nseg = static_cast<uint32_t>(kv.second.size());
    merged.push_back(m);
  }
  if (merged.empty()) return;
  size_t j = 0;
  for (size_t i = 0; i < P->ops.size(); ++i)
    if (!drop[i]) P->ops[j++] = P->ops[i];
  P->ops.resize(j);
  P->ops.insert(P->ops.end(), merged.begin(), merged.end());
}

// Reassigns arena addresses by liveness.  While the stream is compiled every
// compute op writes a fresh arena extent, so one decode step would touch tens
// of MB per sequence once each and its intermediates would leave L2 as
// write-backs.  Here the accesses of the final ops (per kind, the operand
// ranges the executor reads and writes) are unioned into groups of
// overlapping ranges; a group lives from the lowest to the highest level that
// touches it and may take the memory of a group whose last level is strictly
// lower than its first (the ops of one level run concurrently, and levels are
// separated by the executor's grid barrier).  A group keeps its offset modulo
// 256 bytes.  An op kind or flag combination this pass does not model leaves
// the arena as it is.
void Compiler::pack_arena() {
  struct Rng {
    uint64_t lo, hi;
    uint32_t level;
  };
  std::vector<Rng> rs;
  bool ok = true;
  const uint64_t a0 = arena_base_, a1 = arena_base_ + arena_top_;
  auto in_arena = [&](uint64_t x) { return !(x & kSharedBit) && x >= a0 && x < a1; };
  auto add = [&](uint64_t x, uint64_t bytes, uint32_t L) {
    if (bytes && in_arena(x)) rs.push_back(Rng{x, x + (bytes + kUnit - 1) / kUnit, L});
  };
  // per segment: bit 0 = src is an address, bit 1 = dst is an address, bit 2 = seen
  std::vector<uint8_t> role(P->segs.size(), 0);
  auto segs = [&](const DevOp& op, uint8_t r, uint64_t bytes_each, bool n_is_bytes) {
    for (uint32_t k = 0; k < op.nseg; ++k) {
      const uint32_t i = op.seg0 + k;
      if (i >= P->segs.size() || ((role[i] & 4) && (role[i] & 3) != r)) {
        ok = false;
        return;
      }
      role[i] = r | 4;
      const Segment& sg = P->segs[i];
      const uint64_t b = bytes_each ? bytes_each : (n_is_bytes ? sg.n : sg.n * kUnit);
      if (r & 1) add(sg.src, b, op.level);
      if ((r & 2) && sg.dst) add(sg.dst, b, op.level);
    }
  };
  for (const DevOp& op : P->ops) {
    const uint32_t L = op.level;
    const uint64_t M = op.M, N = op.N, K = op.K, MN = M * N;
    const bool sega = (op.flags & F_SEGA) != 0;
    auto src_a = [&](uint64_t bytes) {
      if (sega) segs(op, 1, 0, false);
      else add(op.a, bytes, L);
    };
    switch (op.kind) {
      case K_GATHER: segs(op, 3, 0, false); break;
      case K_DYN_LOAD: add(op.d, op.nbytes, L); break;
      case K_DYN_STORE: add(op.a, op.nbytes, L); break;
      case K_DYN_STORE_MULTI: segs(op, 1, 0, true); break;
      case K_SREG_LOAD: add(op.a, 2, L); break;
      case K_SREG_FINAL: break;
      case K_VADD_CHAIN: segs(op, 3, MN * 2, false); break;
      case K_MATMUL: {
        const bool dq = (op.flags & F_DQ) || (op.flags2 & FX_DQS);
        if ((op.flags & F_ACCUMULATE) && dq) ok = false;
        add(op.a, M * K * ((op.flags & F_QA) ? 2 : 1), L);
        add(op.b, K * N * ((op.flags & F_QB) ? 2 : 1), L);
        if (op.flags & F_ACCUMULATE) add(op.c, MN * 4, L);
        else if (dq) add(op.c, N * 2, L);
        if (!(op.flags & F_NOI32)) add(op.d, MN * 4, L);
        if (dq) add(static_cast<uint64_t>(op.dconst), MN * 2, L);
        if (op.flags2 & FX_DQS) add(op.nbytes, N * 2, L);
        if (op.flags & F_SM) add(op.nbytes, MN * 2, L);
        break;
      }
      case K_TRANSPOSE: add(op.a, MN, L); add(op.d, MN, L); break;
      case K_MAX_ABS:
        src_a(MN * 2);
        if (op.flags2 & FX_MAXQ) add(op.d, MN, L);
        break;
      case K_QUANT: src_a(MN * 2); add(op.d, MN, L); break;
      case K_GELU_F16: src_a(MN * 2); add(op.d, MN * 2, L); break;
      case K_VADD_F16: src_a(MN * 2); add(op.b, MN * 2, L); add(op.d, MN * 2, L); break;
      case K_REQUANT: add(op.a, MN * 4, L); add(op.d, MN, L); break;
      case K_REQUANT_PC: add(op.a, MN * 4, L); add(op.b, N * 2, L); add(op.d, MN, L); break;
      case K_SCALE_MUL_I32: add(op.a, MN * 4, L); add(op.d, MN * 4, L); break;
      case K_SCALE_MUL_I8: add(op.a, MN, L); add(op.d, MN, L); break;
      case K_VADD_I8: add(op.a, MN, L); add(op.b, MN, L); add(op.d, MN, L); break;
      case K_VADD_I32: add(op.a, MN * 4, L); add(op.b, N * 4, L); add(op.d, MN * 4, L); break;
      case K_DEQUANT_ADD: add(op.a, MN * 4, L); add(op.b, MN, L); add(op.d, MN, L); break;
      case K_DEQUANT_ACCUM: add(op.a, MN * 4, L); add(op.b, N * 2, L); add(op.d, MN * 2, L); break;
      case K_DEQUANT_SCALED: case K_LAYERNORM_F16:
        add(op.a, MN * (op.kind == K_DEQUANT_SCALED ? 4 : 2), L);
        if (op.flags & F_SPLIT) {
          add(op.b, N * 2, L);
          add(op.c, N * 2, L);
        } else {
          add(op.b, N * 4, L);
        }
        add(op.d, MN * 2, L);
        break;
      case K_SOFTMAX_F16: case K_MASKED_SOFTMAX_F16: add(op.a, MN * 2, L); add(op.d, MN * 2, L); break;
      default: ok = false; break;
    }
    if (sega && op.kind != K_MAX_ABS && op.kind != K_QUANT && op.kind != K_GELU_F16 && op.kind != K_VADD_F16)
      ok = false;
    if (!ok) return;
  }
  if (rs.empty()) return;
  // groups of overlapping ranges: [lo, hi), levels [first, last]
  std::sort(rs.begin(), rs.end(), [](const Rng& x, const Rng& y) { return x.lo < y.lo; });
  struct Grp {
    uint64_t lo, hi;
    uint32_t first, last;
    uint64_t nlo;
  };
  std::vector<Grp> gs;
  for (const Rng& r : rs) {
    if (!gs.empty() && r.lo < gs.back().hi) {
      Grp& g = gs.back();
      g.hi = std::max(g.hi, r.hi);
      g.first = std::min(g.first, r.level);
      g.last = std::max(g.last, r.level);
    } else {
      gs.push_back(Grp{r.lo, r.hi, r.level, r.level, 0});
    }
  }
  // first-fit over blocks of 16 units, in order of first level
  std::vector<uint32_t> order(gs.size());
  for (uint32_t i = 0; i < gs.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](uint32_t x, uint32_t y) {
    return gs[x].first != gs[y].first ? gs[x].first < gs[y].first : gs[x].lo < gs[y].lo;
  });
  std::map<uint64_t, uint64_t> free_blocks;   // start -> units (relative to arena_base_)
  auto release = [&](uint64_t at, uint64_t n) {
    auto it = free_blocks.emplace(at, n).first;
    auto nx = std::next(it);
    if (nx != free_blocks.end() && it->first + it->second == nx->first) {
      it->second += nx->second;
      free_blocks.erase(nx);
    }
    if (it != free_blocks.begin()) {
      auto pv = std::prev(it);
      if (pv->first + pv->second == it->first) {
        pv->second += it->second;
        free_blocks.erase(it);
      }
    }
  };
  using Live = std::pair<uint32_t, uint32_t>;   // (last level, group)
  std::vector<Live> live;                      // min-heap on the last level
  auto cmp = [](const Live& x, const Live& y) { return x.first > y.first; };
  std::vector<uint64_t> block_at(gs.size(), 0), block_n(gs.size(), 0);
  uint64_t top = 0;
  for (uint32_t gi : order) {
    Grp& g = gs[gi];
    while (!live.empty() && live.front().first < g.first) {
      const uint32_t done = live.front().second;
      std::pop_heap(live.begin(), live.end(), cmp);
      live.pop_back();
      release(block_at[done], block_n[done]);
    }
    const uint64_t mis = (g.lo - a0) & 15;
    const uint64_t n = (mis + (g.hi - g.lo) + 15) & ~15ull;
    uint64_t at = kNone;
    for (auto it = free_blocks.begin(); it != free_blocks.end(); ++it) {
      if (it->second < n) continue;
      at = it->first;
      const uint64_t rest = it->second - n;
      free_blocks.erase(it);
      if (rest) free_blocks.emplace(at + n, rest);
      break;
    }
    if (at == kNone) {
      at = top;
      top += n;
    }
    block_at[gi] = at;
    block_n[gi] = n;
    g.nlo = a0 + at + mis;
    live.emplace_back(g.last, gi);
    std::push_heap(live.begin(), live.end(), cmp);
  }
  // relocate every address field; an arena address no modelled access covers
  // (a result the op does not store) goes to the arena's first unit
  auto reloc = [&](uint64_t x) -> uint64_t {
    if (!in_arena(x)) return x;
    size_t lo = 0, hi = gs.size();
    while (lo < hi) {
      const size_t mid = (lo + hi) / 2;
      if (gs[mid].hi <= x) lo = mid + 1;
      else hi = mid;
    }
    if (lo < gs.size() && gs[lo].lo <= x && x < gs[lo].hi) return gs[lo].nlo + (x - gs[lo].lo);
    return a0;
  };
  for (DevOp& op : P->ops) {
    op.a = reloc(op.a);
    op.b = reloc(op.b);
    op.c = reloc(op.c);
    op.d = reloc(op.d);
    if (op.kind == K_MATMUL && ((op.flags & F_DQ) || (op.flags2 & FX_DQS)))
      op.dconst = static_cast<int64_t>(reloc(static_cast<uint64_t>(op.dconst)));
    if (op.kind == K_MATMUL && ((op.flags & F_SM) || (op.flags2 & FX_DQS))) op.nbytes = reloc(op.nbytes);
  }
  for (size_t i = 0; i < P->segs.size(); ++i) {
    if (role[i] & 1) P->segs[i].src = reloc(P->segs[i].src);
    if ((role[i] & 2) && P->segs[i].dst) P->segs[i].dst = reloc(P->segs[i].dst);
  }
  arena_unpacked_ = arena_top_;
  arena_top_ = std::max<uint64_t>(top, 16);
}

// Splits each op into tasks (tile x sequence group) and orders them by level.
void Compiler::build_tasks() {
  const uint32_t B = static_cast<uint32_t>(P->batch);
  // compress levels
  std::vector<uint32_t> lv;
  for (auto& op : P->ops) lv.push_back(op.level);
  std::sort(lv.begin(), lv.end());
  lv.erase(std::unique(lv.begin(), lv.end()), lv.end());
  for (auto& op : P->ops) op.level = static_cast<uint32_t>(std::lower_bound(lv.begin(), lv.end(), op.level) - lv.begin());
  std::vector<std::vector<Task>> per_level(lv.size());
  // MATMULs whose weights (B) are shared and whose A rows of up to 128/M
  // sequences fill one 128-row tensor-core tile run on tcgen05, fed by TMA;
  // seg0 numbers their pair of tensor maps.
  P->n_tc = 0;
  for (auto& op : P->ops) {
    if (op.kind == K_MATMUL && tc_eligible(op.a, op.b, op.M, op.N, op.K)) {
      op.flags |= F_TC;
      // a task's A rows (its sequences' rows) rounded up to 8: when every K
      // chunk fits in shared memory at once, 64-column tasks load them all
      const uint32_t rows = (std::min<uint32_t>(128 / op.M, B) * op.M + 7) & ~7u;
      if (!(op.flags & F_ACCUMULATE) && tc_resident_fits(rows, op.K)) {
        op.flags2 |= FX_TCRES;
        op.q_rows = rows;
      } else {
        if (op.N >= 128) op.flags |= F_TC128;
        // a K loop through the stage ring is latency-bound: past kTcSplitRows
        // rows a task takes kTcSplitRows of them (q_rows), twice the tasks
        if (rows > kTcSplitRows && op.M <= kTcSplitRows && kTcSplitRows % op.M == 0) op.q_rows = kTcSplitRows;
      }
      op.seg0 = P->n_tc++;
      op.nseg = 0;
    }
  }
  auto per_seq = [&](uint32_t opi, uint32_t tiles) {
    for (uint32_t s = 0; s < B; ++s)
      for (uint32_t t = 0; t < tiles; ++t) per_level[P->ops[opi].level].push_back(Task{opi, s, 1, t, 0});
  };
  // aux of a segment-list element-wise task of tile t: the segments holding
  // its units, first | count << 16 (segments are in operand order)
  auto seg_aux = [&](const DevOp& op, uint32_t t) {
    const uint64_t units = uint64_t(op.M) * op.N / 8;
    const uint64_t u0 = uint64_t(t) * kSegTaskUnits, u1 = std::min<uint64_t>(units, u0 + kSegTaskUnits);
    uint32_t first = 0, last = 0;
    for (uint32_t k = 0; k < op.nseg; ++k) {
      const Segment& sg = P->segs[op.seg0 + k];
      if (sg.dst + sg.n <= u0) first = k + 1;
      if (sg.dst < u1) last = k;
    }
    return first | ((last - first + 1) << 16);
  };
  // One sequence's tasks of a chain op, as templates (tile, aux; seq0 unset).
  auto chain_tiles = [&](uint32_t opi, std::vector<Task>& out) {
    const DevOp& op = P->ops[opi];
    const uint64_t MN = uint64_t(op.M) * op.N;
    uint32_t tiles = 1;
    if (op.kind == K_LAYERNORM_F16) tiles = (op.M + row_task_rows(op.kind, op.N) - 1) / row_task_rows(op.kind, op.N);
    else if (op.kind == K_VADD_CHAIN) tiles = static_cast<uint32_t>((MN + kVaddChainTask - 1) / kVaddChainTask);
    else if (op.kind != K_MAX_ABS && (op.flags & F_SEGA))
      tiles = static_cast<uint32_t>(std::max<uint64_t>(1, (MN / 8 + kSegTaskUnits - 1) / kSegTaskUnits));
    else if (op.kind != K_MAX_ABS)
      tiles = static_cast<uint32_t>(std::max<uint64_t>(1, (MN + ew_task_elems(op.kind) - 1) / ew_task_elems(op.kind)));
    for (uint32_t t = 0; t < tiles; ++t)
      out.push_back(Task{opi, 0, 1, t, (op.kind != K_MAX_ABS && (op.flags & F_SEGA)) ? seg_aux(op, t) : 0u});
  };
  std::vector<Task> templates;
  std::vector<std::pair<size_t, uint32_t>> heads;   // (level, index in per_level) of chain / group head tasks
  std::map<uint32_t, std::vector<uint32_t>> attn_pairs;   // level -> its row-attention QK^T ops
  std::map<uint32_t, std::vector<uint32_t>> max_ops;      // level -> its pairable MAX_ABS + QUANT ops
  auto attn_groupable = [&](const DevOp& x) {
    if (!(x.flags2 & FX_PV) || x.M != 1) return false;
    const DevOp& y = P->ops[x.seg0];
    return attn_row_shape_ok(x.M, x.K, x.N, x.flags, x.flags2, y.M, y.K, y.N, y.flags);
  };
  for (uint32_t i = 0; i < P->ops.size(); ++i) {
    const DevOp& op = P->ops[i];
    const uint64_t MN = uint64_t(op.M) * op.N;
    if (op.flags2 & FX_CHAINED) continue;   // runs in its chain head's task
    if (i + 1 < P->ops.size() && (P->ops[i + 1].flags2 & FX_CHAINED)) {
      // a chain: one task per sequence runs every tile of each op in order
      const uint32_t first = static_cast<uint32_t>(templates.size());
      chain_tiles(i, templates);
      for (uint32_t j = i + 1; j < P->ops.size() && (P->ops[j].flags2 & FX_CHAINED); ++j) chain_tiles(j, templates);
      P->ops[i].flags2 |= FX_CHAINHEAD;
      const uint32_t count = static_cast<uint32_t>(templates.size()) - first;
      for (uint32_t s = 0; s < B; ++s) {
        heads.push_back({op.level, static_cast<uint32_t>(per_level[op.level].size())});
        per_level[op.level].push_back(Task{i, s, 1, first, count});
      }
      continue;
    }
    switch (op.kind) {
      case K_GATHER: {
        // runs of whole segments of about kGatherChunkUnits units per task
        uint32_t first = 0;
        uint64_t acc_units = 0;
        for (uint32_t k = 0; k < op.nseg; ++k) {
          const uint64_t n = P->segs[op.seg0 + k].n;
          if (k > first && acc_units + n > kGatherChunkUnits) {
            for (uint32_t s = 0; s < B; ++s) per_level[op.level].push_back(Task{i, s, 1, first, k});
            first = k;
            acc_units = 0;
          }
          acc_units += n;
        }
        if (op.nseg > first)
          for (uint32_t s = 0; s < B; ++s) per_level[op.level].push_back(Task{i, s, 1, first, op.nseg});
        break;
      }
      case K_MATMUL: {
        if (op.flags2 & FX_PVY) break;   // runs in its QK^T op's task
        const uint32_t ntile = (op.N + 63) / 64;
        const bool shared_b = (op.b & kSharedBit) != 0;
        if ((op.flags & F_WIDE) || (!(op.flags & F_TC) && !shared_b && wide_mm_ok(op.M, op.N, op.K, false, false))) {
          P->ops[i].flags |= F_WIDE;   // one task per sequence, every column
          if (attn_groupable(P->ops[i])) {
            attn_pairs[op.level].push_back(i);   // tasks below, per pair or per head group
            break;
          }
          per_seq(i, 1);
          break;
        }
        if (op.M >= 128 || !shared_b) {
          const uint32_t mchunks = (op.M + 127) / 128;
          per_seq(i, ntile * mchunks);
        } else {
          const uint32_t spt = ((op.flags & F_TC) && op.q_rows) ? op.q_rows / op.M : std::max<uint32_t>(1, 128 / op.M);
          const uint32_t nt = (op.flags & F_TC128) ? (op.N + 127) / 128 : ntile;
          for (uint32_t s = 0; s < B; s += spt)
            for (uint32_t t = 0; t < nt; ++t)
              per_level[op.level].push_back(Task{i, s, std::min(spt, B - s), t,
                                                 (op.flags & F_TC) ? (kTaskTcMap | op.seg0) : 0u});
        }
        break;
      }
      case K_SREG_LOAD:
      case K_SREG_FINAL: {
        for (uint32_t s = 0; s < B; s += 256)
          per_level[op.level].push_back(Task{i, s, std::min<uint32_t>(256, B - s), 0, 0});
        break;
      }
      case K_MAX_ABS:
        if (max_pair_ok(op.M, op.N, op.nseg, op.flags, op.flags2)) {
          max_ops[op.level].push_back(i);   // tasks below, per op or per pair
          break;
        }
        per_seq(i, 1);
        break;
      case K_DYN_LOAD:
      case K_DYN_STORE:
      case K_DYN_STORE_MULTI:
        per_seq(i, 1);
        break;
      case K_VADD_CHAIN:
        per_seq(i, static_cast<uint32_t>((MN + kVaddChainTask - 1) / kVaddChainTask));
        break;
      case K_LAYERNORM_F16: case K_SOFTMAX_F16: case K_MASKED_SOFTMAX_F16:
      case K_LN_I8: case K_SOFTMAX_I8: case K_MASKED_SOFTMAX_I8:
      case K_SOFTMAX_ATTNV: case K_MASKED_SOFTMAX_ATTNV: {
        const uint32_t rpt = row_task_rows(op.kind, op.N);   // one warp per row, 8 or 16 rows per task
        per_seq(i, (op.M + rpt - 1) / rpt);
        break;
      }
      case K_TRANSPOSE:
        per_seq(i, static_cast<uint32_t>(std::max<uint64_t>(1, (MN + 16383) / 16384)));
        break;
      default: {  // element-wise ops: ew_task_elems(kind) elements per task
        if (op.flags & F_SEGA) {   // segment-list operand: kSegTaskUnits operand units per task
          const uint64_t units = MN / 8;
          const uint32_t tiles = static_cast<uint32_t>(std::max<uint64_t>(1, (units + kSegTaskUnits - 1) / kSegTaskUnits));
          for (uint32_t t = 0; t < tiles; ++t) {
            const uint32_t aux = seg_aux(op, t);
            for (uint32_t s = 0; s < B; ++s) per_level[op.level].push_back(Task{i, s, 1, t, aux});
          }
          break;
        }
        const uint64_t te = ew_task_elems(op.kind);
        if (B > 1 && MN > 0 && MN * 2 <= te) {
          // small ops: one task takes several whole sequences
          const uint32_t spt = static_cast<uint32_t>(te / MN);
          for (uint32_t s = 0; s < B; s += spt)
            per_level[op.level].push_back(Task{i, s, std::min(spt, B - s), 0, 0});
        } else {
          per_seq(i, static_cast<uint32_t>(std::max<uint64_t>(1, (MN + te - 1) / te)));
        }
        break;
      }
    }
  }
  // Row-attention pairs of a level: when a task per pair and sequence would
  // take more than one round over the executor's halves, pairs of one shape
  // go in head groups (FX_ATTNGRP) of g pairs of a sequence, the least g
  // that fits one round (at most kAttnGroupMax when none does): a group task
  // overlaps each pair's copies with the pair before it.
  for (auto& lp : attn_pairs) {
    std::map<std::tuple<uint32_t, uint32_t, uint32_t>, std::vector<uint32_t>> by_shape;
    for (uint32_t i : lp.second) {
      const DevOp& x = P->ops[i];
      by_shape[std::make_tuple(x.K, x.N, P->ops[x.seg0].N)].push_back(i);
    }
    for (auto& sh : by_shape) {
      const std::vector<uint32_t>& xs = sh.second;
      const uint32_t n = static_cast<uint32_t>(xs.size()), gmax = std::min(n, kAttnGroupMax);
      uint32_t g = 1;
      if (uint64_t(B) * n > kTargetHalves) {
        g = gmax;
        for (uint32_t c = 2; c <= gmax; ++c)
          if (uint64_t(B) * ((n + c - 1) / c) <= kTargetHalves) {
            g = c;
            break;
          }
      }
      for (uint32_t k0 = 0; k0 < n; k0 += g) {
        if (g == 1) {
          per_seq(xs[k0], 1);
          continue;
        }
        const uint32_t first = static_cast<uint32_t>(templates.size()), cnt = std::min(g, n - k0);
        for (uint32_t k = k0; k < k0 + cnt; ++k) templates.push_back(Task{xs[k], 0, 1, 0, 0});
        P->ops[xs[k0]].flags2 |= FX_ATTNGRP;
        for (uint32_t s = 0; s < B; ++s) {
          heads.push_back({lp.first, static_cast<uint32_t>(per_level[lp.first].size())});
          per_level[lp.first].push_back(Task{xs[k0], s, 1, first, cnt});
        }
      }
    }
  }
  // MAX_ABS + QUANT ops of a level: when a task per op and sequence would
  // take more than one round over the executor's halves, ops of one shape go
  // in pairs (FX_MAXGRP), one task per pair and sequence.
  for (auto& lm : max_ops) {
    std::map<std::pair<uint32_t, uint32_t>, std::vector<uint32_t>> by_shape;
    for (uint32_t i : lm.second) by_shape[{P->ops[i].M, P->ops[i].N}].push_back(i);
    for (auto& sh : by_shape) {
      const std::vector<uint32_t>& xs = sh.second;
      const bool pair = uint64_t(B) * xs.size() > kTargetHalves;
      for (size_t k0 = 0; k0 < xs.size(); k0 += pair ? 2 : 1) {
        if (!pair || k0 + 1 == xs.size()) {
          per_seq(xs[k0], 1);
          continue;
        }
        const uint32_t first = static_cast<uint32_t>(templates.size());
        templates.push_back(Task{xs[k0], 0, 1, 0, 0});
        templates.push_back(Task{xs[k0 + 1], 0, 1, 0, 0});
        P->ops[xs[k0]].flags2 |= FX_MAXGRP;
        for (uint32_t s = 0; s < B; ++s) {
          heads.push_back({lm.first, static_cast<uint32_t>(per_level[lm.first].size())});
          per_level[lm.first].push_back(Task{xs[k0], s, 1, first, 2});
        }
      }
    }
  }
  P->tasks.clear();
  P->level_off.assign(1, 0);
  for (auto& v : per_level) {
    for (Task& t : v) {
      const DevOp& op = P->ops[t.op];
      if (!(op.flags2 & FX_CHAINHEAD)) {
        prefetch_hint(op, t);
        continue;
      }
      // a chain head: the first LayerNorm's gamma (and beta, when they are
      // one vector) of its chain, read-only and ready before the level
      for (uint32_t j = t.op; j < P->ops.size() && (j == t.op || (P->ops[j].flags2 & FX_CHAINED)); ++j)
        if (P->ops[j].kind == K_LAYERNORM_F16) {
          const DevOp& l = P->ops[j];
          t.pf_phys = l.b;
          t.pf_units = static_cast<uint32_t>(uint64_t(l.N) * 2 * ((l.flags & F_SPLIT) ? 1 : 2) / kUnit);
          break;
        }
    }
    P->tasks.insert(P->tasks.end(), v.begin(), v.end());
    P->level_off.push_back(static_cast<uint32_t>(P->tasks.size()));
  }
  // chain templates after the last level; head tasks point at them
  const uint32_t base = static_cast<uint32_t>(P->tasks.size());
  P->tasks.insert(P->tasks.end(), templates.begin(), templates.end());
  for (auto& h : heads) P->tasks[P->level_off[h.first] + h.second].tile += base;
}

// The operand bytes a task reads first, for the executor to pull into L2
// while the task before it runs.  A hint never exceeds what the task itself
// reads; ops without a cheap contiguous estimate get none.
void Compiler::prefetch_hint(const DevOp& op, Task& t) const {
  constexpr uint64_t kMaxUnits = 4096;     // 64 KB
  constexpr uint64_t kMaxTcUnits = 16384;  // 256 KB of tcgen05 weights
  uint64_t phys = 0, units = 0;
  const uint64_t MN = uint64_t(op.M) * op.N;
  auto elem_bytes = [&](uint32_t kind) -> uint64_t {
    switch (kind) {
      case K_QUANT: case K_GELU_F16: case K_VADD_F16: case K_LAYERNORM_F16: case K_SOFTMAX_F16:
      case K_MASKED_SOFTMAX_F16: case K_MAX_ABS:
        return 2;
      case K_DEQUANT_SCALED: case K_DEQUANT_ACCUM: case K_REQUANT_PC: case K_REQUANT: case K_SCALE_MUL_I32:
      case K_VADD_I32: case K_DEQUANT_ADD:
        return 4;
      default:
        return 1;
    }
  };
  if (op.flags & F_SEGA) {   // the segment holding the task's first operand unit, from that unit on
    const uint64_t u0 = op.kind == K_MAX_ABS ? 0 : uint64_t(t.tile) * kSegTaskUnits;
    for (uint32_t k = 0; k < op.nseg; ++k) {
      const Segment& sg = P->segs[op.seg0 + k];
      const uint64_t sd = sg.dst & ~kSegGelu;
      if (sd <= u0 && u0 < sd + sg.n) {
        phys = sg.src + (u0 - sd);
        units = std::min<uint64_t>(sd + sg.n - u0, op.kind == K_MAX_ABS ? sg.n : kSegTaskUnits);
        break;
      }
    }
  } else {
    switch (op.kind) {
      case K_GATHER:
        if (t.tile < op.nseg) {
          phys = P->segs[op.seg0 + t.tile].src;
          units = P->segs[op.seg0 + t.tile].n;
        }
        break;
      case K_DYN_STORE:
        phys = op.a;
        units = op.nbytes / kUnit;
        break;
      case K_MATMUL:
        if (op.flags & F_TC) {
          // the first column tile's task hints the whole shared weight matrix
          // [K][N] (every tile's slice), up to kMaxTcUnits
          if (t.tile == 0 && (op.b & kSharedBit)) {
            t.pf_phys = op.b;
            t.pf_units = static_cast<uint32_t>(std::min<uint64_t>(uint64_t(op.K) * op.N / kUnit, kMaxTcUnits));
          }
          return;
        }
        if (!(op.b & kSharedBit)) {   // per-sequence B: the whole matrix (FP16 when quantised on load)
          phys = op.b;
          units = uint64_t(op.K) * op.N * ((op.flags & F_QB) ? 2 : 1) / kUnit;
        } else {
          phys = op.a;
          units = uint64_t(std::min<uint32_t>(op.M, 128)) * op.K / kUnit;
        }
        break;
      case K_TRANSPOSE:
      case K_MAX_ABS:
        phys = op.a;
        units = MN * elem_bytes(op.kind) / kUnit;
        break;
      case K_LAYERNORM_F16: case K_SOFTMAX_F16: case K_MASKED_SOFTMAX_F16: {
        const uint64_t row_units = uint64_t(op.N) * 2 / kUnit;
        const uint64_t rpt = row_task_rows(op.kind, op.N);
        const uint64_t r0 = uint64_t(t.tile) * rpt;
        if (r0 < op.M && op.N % 8 == 0) {
          phys = op.a + r0 * row_units;
          units = std::min<uint64_t>(rpt, op.M - r0) * row_units;
        }
        break;
      }
      case K_VADD_CHAIN: {   // the first operand's slice of this task
        const uint64_t e0 = uint64_t(t.tile) * kVaddChainTask;
        if (op.nseg && e0 < MN) {
          phys = P->segs[op.seg0].src + e0 * 2 / kUnit;
          units = std::min<uint64_t>(kVaddChainTask, MN - e0) * 2 / kUnit;
        }
        break;
      }
      case K_REQUANT: case K_REQUANT_PC: case K_SCALE_MUL_I32: case K_SCALE_MUL_I8: case K_VADD_I8:
      case K_VADD_I32: case K_DEQUANT_ADD: case K_DEQUANT_ACCUM: case K_DEQUANT_SCALED: case K_QUANT:
      case K_VADD_F16: case K_GELU_F16: {
        const uint64_t eb = elem_bytes(op.kind);
        if (t.nseq > 1) {
          units = MN * eb / kUnit;
          phys = op.a;
        } else {
          const uint64_t te = ew_task_elems(op.kind);
          const uint64_t e0 = uint64_t(t.tile) * te;
          if (e0 < MN && (e0 * eb) % kUnit == 0) {
            phys = op.a + e0 * eb / kUnit;
            units = std::min<uint64_t>(te, MN - e0) * eb / kUnit;
          }
        }
        break;
      }
      default:
        break;
    }
  }
  if (units == 0) return;
  t.pf_phys = phys;
  t.pf_units = static_cast<uint32_t>(std::min<uint64_t>(units, kMaxUnits));
}

int Compiler::compile() {
  sram_.resize(kSramUnits);
  for (uint32_t u = 0; u < kSramUnits; ++u) sram_[u] = u;
  shadow_.resize(rw_units_);
  for (uint64_t i = 0; i < rw_units_; ++i) shadow_[i] = rw_home(i);
  rw_wl_.assign(rw_units_, 0);
  rw_rl_.assign(rw_units_, 0);
  home_rl_.assign(kSramUnits, 0);
  slot_lvl_.assign(kSregSlotBase, 0);
  rw_home_read_.assign(rw_units_, 0);
  insn_region_bytes_ = n_insns_ * 8;

  // var sites
  uint32_t w = 0;
  for (int i = 0; i < n_sites_; ++i) {
    const tac_var_site& s = sites_[i];
    VarInfo v{};
    v.kind = s.kind;
    v.addr_reg = s.addr_reg;
    v.lo_pc = s.lo_pc;
    v.hi_pc = s.hi_pc;
    v.range_lo = s.range_lo;
    v.range_hi = s.range_hi;
    v.word0 = w;
    if (s.lo_pc >= n_insns_ || (s.kind == 0 && s.hi_pc >= n_insns_)) {
      pc_ = s.lo_pc;
      return unsupported("runtime site outside the instruction region");
    }
    v.base_lo = load_be64(words_ + s.lo_pc * 8);
    if (s.kind == 0) {
      v.base_hi = load_be64(words_ + s.hi_pc * 8);
      var_pc_[s.lo_pc] = {i, 0};
      var_pc_[s.hi_pc] = {i, 1};
      w += 2;
    } else {
      var_pc_[s.lo_pc] = {i, 0};
      w += 1;
    }
    P->vars.push_back(v);
  }
  P->n_var_words = w;
  P->n_params = static_cast<uint32_t>(n_sites_);
  site_group_.resize(n_sites_);
  same_checked_.assign(n_sites_, 0);
  for (int i = 0; i < n_sites_; ++i) {
    site_group_[i] = i;
    if (sites_[i].kind != 0) continue;
    for (int j = 0; j < i; ++j)
      if (sites_[j].kind == 0 && sites_[j].range_lo == sites_[i].range_lo && sites_[j].range_hi == sites_[i].range_hi) {
        site_group_[i] = j;
        break;
      }
  }

  uint64_t count = 0;
  pc_ = entry_;
  int status = 0;
  while (!halted_ && count < max_insns_) {
    if (pc_ >= n_insns_) {
      word_ = 0;
      status = fault(TAC_E_SIMULATOR, "PC=" + std::to_string(pc_) + " past end of program (" +
                                          std::to_string(n_insns_) + " insns)");
      break;
    }
    word_ = load_be64(words_ + pc_ * 8);
    Insn x;
    if (!decode(word_, x)) {
      status = fault(TAC_E_ILLEGAL_OPCODE, "Illegal opcode");
      break;
    }
    status = step(x);
    if (status) break;
    ++count;
    ++pc_;
  }
  if (status == TAC_E_UNSUPPORTED || status == TAC_E_SHARED_WRITE) return status;
  finalize();
  drop_dead_ops();
  merge_dyn_stores();
  write_vadd_chains();
  if (int s = link_pv_pairs()) return s;
  if (!opts_ || !(opts_->flags & TAC_COMPILE_NO_PACK)) pack_arena();
  build_tasks();

  tac_exec_info& I = P->info;
  I.executed = count;
  I.final_pc = pc_;
  I.halted = halted_ ? 1 : 0;
  I.faulted = status ? 1 : 0;
  I.cycles = cycles_;
  I.n_ops = P->ops.size();
  I.n_levels = P->level_off.size() - 1;
  I.n_tasks = P->tasks.size();
  I.n_segments = P->segs.size();
  I.arena_bytes = arena_top_ * kUnit;
  I.n_slots = n_slots_;
  I.n_var_words = P->n_var_words;
  for (int r = 0; r < 4; ++r) I.final_regs.addr_regs[r] = areg_[r].value;
  I.final_regs.tile_valid = tile_valid_;
  for (int i = 0; i < 3; ++i) I.final_regs.tile[i] = tile_[i];
  I.final_regs.attn_valid = attn_kind_ == 1;
  I.final_regs.attn_qrb = attn_qrb_;
  I.final_regs.attn_vkl = attn_vkl_;
  I.final_regs.attn_mode = attn_mode_;
  P->arena_units = arena_top_;
  P->n_slots = n_slots_;
  P->cse_hits = cse_hits_;
  P->sram_home_read = sram_home_read_;
  P->sreg_home_read = sreg_home_read_;
  P->home_read_ranges.clear();
  for (uint64_t i = 0; i < rw_units_;) {
    if (!rw_home_read_[i]) { ++i; continue; }
    uint64_t j = i;
    while (j < rw_units_ && rw_home_read_[j]) ++j;
    P->home_read_ranges.push_back({shared_bytes_ + i * kUnit, shared_bytes_ + j * kUnit});
    i = j;
  }
  return 0;
}

}  // namespace
}  // namespace tac

// ------------------------------------------------------------------------------------
extern "C" int tac_compile_ex(int batch, uint64_t dram_bytes, uint64_t shared_bytes,
                              const uint8_t* insn_bytes, uint64_t n_insns, uint64_t entry_pc,
                              uint64_t max_insns, const tac_regs* init_regs, int sregs_reset,
                              const tac_var_site* sites, int n_sites, const tac_compile_opts* opts,
                              tac_program** out, tac_exec_info* info, tac_fault* fault) {
  if (!out || !insn_bytes || batch <= 0 || shared_bytes > dram_bytes || (shared_bytes % 16) ||
      n_sites < 0 || (n_sites > 0 && !sites) || (opts && opts->n_live && !opts->live))
    return TAC_E_ARGUMENT;
  *out = nullptr;
  tac_program* p = new (std::nothrow) tac_program();
  if (!p) return TAC_E_ARGUMENT;
  p->batch = batch;
  p->dram_bytes = dram_bytes;
  p->shared_bytes = shared_bytes;
  tac::Compiler c(p, insn_bytes, n_insns, entry_pc, max_insns, init_regs, sregs_reset, sites, n_sites);
  c.opts_ = opts;
  int s = c.compile();
  if (fault) *fault = p->fault;
  if (s) {  // the stream cannot be planned at all
    delete p;
    return s;
  }
  if (info) *info = p->info;
  *out = p;
  return TAC_OK;
}

extern "C" int tac_compile(int batch, uint64_t dram_bytes, uint64_t shared_bytes,
                           const uint8_t* insn_bytes, uint64_t n_insns, uint64_t entry_pc,
                           uint64_t max_insns, const tac_regs* init_regs, int sregs_reset,
                           const tac_var_site* sites, int n_sites, tac_program** out,
                           tac_exec_info* info, tac_fault* fault) {
  return tac_compile_ex(batch, dram_bytes, shared_bytes, insn_bytes, n_insns, entry_pc, max_insns, init_regs,
                        sregs_reset, sites, n_sites, nullptr, out, info, fault);
}

extern "C" int tac_program_home_reads(const tac_program* p, uint64_t* ranges, uint32_t max_ranges,
                                      uint32_t* n_ranges, int32_t* sram_read, int32_t* sregs_read) {
  if (!p) return TAC_E_ARGUMENT;
  const uint32_t n = static_cast<uint32_t>(p->home_read_ranges.size());
  if (n_ranges) *n_ranges = n;
  for (uint32_t i = 0; ranges && i < n && i < max_ranges; ++i) {
    ranges[2 * i] = p->home_read_ranges[i].first;
    ranges[2 * i + 1] = p->home_read_ranges[i].second;
  }
  if (sram_read) *sram_read = p->sram_home_read ? 1 : 0;
  if (sregs_read) *sregs_read = p->sreg_home_read ? 1 : 0;
  return TAC_OK;
}

extern "C" int tac_program_info(const tac_program* p, tac_exec_info* info, tac_fault* fault) {
  if (!p) return TAC_E_ARGUMENT;
  if (info) *info = p->info;
  if (fault) *fault = p->fault;
  return TAC_OK;
}

extern "C" uint64_t tac_program_record_size(int which) {
  switch (which) {
    case 0: return sizeof(tac::DevOp);
    case 1: return sizeof(tac::Segment);
    case 2: return sizeof(tac::Task);
    default: return 0;
  }
}

extern "C" int tac_program_dump(const tac_program* p, void* ops, void* segments, void* tasks,
                                uint32_t* level_offsets) {
  if (!p) return TAC_E_ARGUMENT;
  if (ops && !p->ops.empty()) std::memcpy(ops, p->ops.data(), p->ops.size() * sizeof(tac::DevOp));
  if (segments && !p->segs.empty())
    std::memcpy(segments, p->segs.data(), p->segs.size() * sizeof(tac::Segment));
  if (tasks && !p->tasks.empty()) std::memcpy(tasks, p->tasks.data(), p->tasks.size() * sizeof(tac::Task));
  if (level_offsets) std::memcpy(level_offsets, p->level_off.data(), p->level_off.size() * sizeof(uint32_t));
  return TAC_OK;
}
