// Host-side representation of a compiled stream (shared by the compiler and
// the CUDA engine).
#pragma once
#include <cstdint>
#include <utility>
#include <vector>

#include "../../include/taccel_b200.h"
#include "tac_isa.h"
#include "tac_plan.h"

namespace tac {

// One runtime-patched site, in the order the caller listed them.
struct VarInfo {
  uint32_t kind;        // 0: SET_ADDR pair, 1: CONFIG_ATTN
  uint32_t addr_reg;
  uint64_t lo_pc, hi_pc;
  uint64_t range_lo, range_hi;
  uint32_t word0;       // index of the site's first word in a sequence's var-word row
  uint64_t base_lo, base_hi;  // compile-time words (opcode / register must not change)
};

// A runtime site's value as an affine function of a sequence's token and
// position (set by the runner; HostRunner's patches, host_runner.py:51-62):
// a SET_ADDR pair holds base + token * tok_mul + position * pos_mul; a
// CONFIG_ATTN word holds query_row_base = position, valid_kv_len =
// position + 1 and the site's mode.
struct VarFormula {
  uint64_t base = 0, tok_mul = 0, pos_mul = 0;
  uint32_t mode = 0;
};

// A condition on runtime parameters that the compiler could not decide.
enum CheckKind : uint32_t {
  CHK_ADDR = 1,        // param + dconst is 16-byte aligned; the nbytes there lie in [lo, hi)
  CHK_ATTN_SET = 2,    // CONFIG_ATTN: mode != 0 and valid_kv_len != 0
  CHK_ATTN_KEYS = 3,   // masked softmax: context fits `key_cols` columns
  CHK_SAME = 4,        // param equals param `lo` (sites over one symbol extent)
};

struct RtCheck {
  uint32_t kind;
  uint32_t param;
  uint64_t pc;
  int64_t dconst;
  uint64_t lo, hi;     // CHK_ADDR: allowed byte range; CHK_ATTN_KEYS: lo = key columns;
                       // CHK_SAME: lo = the other parameter
  uint64_t nbytes;
};

}  // namespace tac

struct tac_program {
  int batch = 1;
  uint64_t dram_bytes = 0, shared_bytes = 0;
  std::vector<tac::DevOp> ops;
  std::vector<tac::Segment> segs;
  std::vector<tac::Task> tasks;
  std::vector<uint32_t> level_off;
  std::vector<tac::VarInfo> vars;
  std::vector<tac::VarFormula> formula;  // per var, when the runner set one
  std::vector<tac::RtCheck> checks;
  uint32_t n_var_words = 0;
  uint32_t n_params = 0;
  uint64_t arena_units = 0;
  uint32_t n_slots = 0;
  tac_exec_info info{};
  tac_fault fault{};
  uint64_t cse_hits = 0;                 // ops removed as repeats of earlier ones
  bool sram_home_read = false;           // reads SRAM bytes an earlier run left
  bool sreg_home_read = false;           // reads scale registers an earlier run left
  std::vector<std::pair<uint64_t, uint64_t>> home_read_ranges;  // writable DRAM read before written
  // Device mirror (filled by the engine on first use).
  int device = -1;
  void* d_blob = nullptr;
  uint32_t n_tc = 0;                     // MATMULs flagged F_TC (two TMA maps each)
  void* d_maps = nullptr;                // their maps, encoded for one engine layout
  uint64_t maps_key[4] = {0, 0, 0, 0};   // seq_base, seq_stride, shared_base, batch
  uint64_t off_ops = 0, off_segs = 0, off_tasks = 0, off_levels = 0;
};

namespace tac {
// Layout constants of the per-sequence block, in 16-byte units.
inline uint64_t rw_base_units() { return kSramUnits; }
}  // namespace tac
