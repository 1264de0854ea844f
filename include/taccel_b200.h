/*
 * taccel_b200.h -- C ABI of the B200 execution engine for taccel programs.
 *
 * The engine replaces the NumPy execute loop of the taccel golden simulator
 * (SayatAbdikul/LLM_accelerator).  Every entry point takes plain pointers and
 * sizes; the Python class llm_accelerator_b200.B200Simulator binds them with
 * ctypes and keeps the reference simulator's interface.  Each declaration
 * names the reference interface it stands in for (paths are inside
 * software/taccel of the reference repository).
 *
 * Status codes: 0 is success; codes 1..7 mirror the reference simulator's
 * exception classes (golden_model/simulator.py:53-65, golden_model/memory.py:11-26)
 * and come with a filled tac_fault record.
 */
#ifndef TACCEL_B200_H
#define TACCEL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum tac_status {
  TAC_OK = 0,
  TAC_E_SIMULATOR = 1,       /* SimulatorError: PC past the end, DRAM capacity       */
  TAC_E_ILLEGAL_OPCODE = 2,  /* IllegalOpcodeError: word does not decode            */
  TAC_E_ILLEGAL_BUFFER = 3,  /* IllegalBufferError                                  */
  TAC_E_CONFIG = 4,          /* ConfigError                                         */
  TAC_E_SRAM_ACCESS = 5,     /* SRAMAccessError                                     */
  TAC_E_DRAM_ACCESS = 6,     /* DRAMAccessError                                     */
  TAC_E_VALUE = 7,           /* ValueError from the reference's SRAM helpers        */
  TAC_E_ARGUMENT = 16,       /* bad argument to this API                            */
  TAC_E_UNSUPPORTED = 17,    /* program form this engine rejects (self-modifying code,
                                unaligned DRAM address, split SET_ADDR pair)        */
  TAC_E_SHARED_WRITE = 18,   /* a STORE may write the shared read-only DRAM region  */
  TAC_E_CUDA = 19,           /* CUDA runtime error                                  */
  TAC_E_DEVICE = 20,         /* a device-side check failed (bounds, barrier timeout) */
  TAC_E_RECOMPILE = 21       /* runtime words fall outside the compiled ranges       */
};

/* Fault record: which instruction faulted and the fields the reference's
 * exception carries (pc/raw bytes, buffer id/offset/limit, DRAM address). */
typedef struct tac_fault {
  int32_t status;
  int32_t buf_id;
  uint64_t pc;
  uint64_t raw_word;
  uint64_t addr;
  int64_t offset;
  int64_t limit;
  char message[320];
} tac_fault;

/* Host-visible architectural registers that are fixed by the instruction
 * stream (golden_model/state.py:43-56): address registers, tile
 * configuration (0-based tile counts) and the attention context. */
typedef struct tac_regs {
  uint64_t addr_regs[4];
  int32_t tile_valid;
  uint32_t tile[3];
  int32_t attn_valid;
  uint32_t attn_qrb;
  uint32_t attn_vkl;
  uint32_t attn_mode;
} tac_regs;

/* A runtime-patched word.  kind 0: a SET_ADDR_LO/SET_ADDR_HI pair whose
 * register value lies in [range_lo, range_hi); kind 1: a CONFIG_ATTN word.
 * Mirrors RuntimePatchSite / RuntimeConfigAttnSite (assembler/assembler.py:127-160). */
typedef struct tac_var_site {
  uint32_t kind;
  uint32_t addr_reg;
  uint64_t lo_pc;
  uint64_t hi_pc;
  uint64_t range_lo;
  uint64_t range_hi;
} tac_var_site;

/* Static facts about a compiled stream. */
typedef struct tac_exec_info {
  uint64_t executed;     /* instructions retired (the value Simulator.run returns) */
  uint64_t final_pc;
  int32_t halted;
  int32_t faulted;       /* the stream faults after `executed` instructions */
  uint64_t cycles;       /* analytic cycle count added (golden_model cycle model) */
  uint64_t n_ops;
  uint64_t n_levels;
  uint64_t n_tasks;
  uint64_t n_segments;
  uint64_t arena_bytes;  /* per-sequence scratch the plan needs */
  uint64_t n_slots;      /* renamed scale-register slots */
  uint64_t n_var_words;  /* runtime words tac_run expects per sequence */
  tac_regs final_regs;
} tac_exec_info;

typedef struct tac_engine tac_engine;
typedef struct tac_program tac_program;

/* Machine state for `batch` independent sequences on one GPU
 * (golden_model/state.py:19-63 MachineState, one per sequence).  DRAM bytes
 * [0, shared_bytes) are one read-only copy shared by all sequences;
 * [shared_bytes, dram_bytes) are private to each sequence. */
int tac_engine_create(int device, int batch, uint64_t dram_bytes, uint64_t shared_bytes,
                      tac_engine** out);
int tac_engine_destroy(tac_engine* e);
int tac_engine_batch(const tac_engine* e);

/* DRAM image upload / read-back (Simulator.load_bundle simulator.py:162-179
 * and state.dram slicing as used by HostRunner._read_logits host_runner.py:66-76).
 * seq = -1 writes every sequence.  Shared-region writes go to the one shared copy. */
int tac_dram_write(tac_engine* e, int seq, uint64_t addr, const void* src, uint64_t len);
int tac_dram_read(tac_engine* e, int seq, uint64_t addr, void* dst, uint64_t len);
/* SRAM access (golden_model/memory.py:337-366 read_bytes / write_bytes). */
int tac_sram_write(tac_engine* e, int seq, int buf, uint64_t byte_off, const void* src, uint64_t len);
int tac_sram_read(tac_engine* e, int seq, int buf, uint64_t byte_off, void* dst, uint64_t len);
/* The 16 FP16 scale registers (state.scale_regs), as raw FP16 bits. */
int tac_sregs_write(tac_engine* e, int seq, const uint16_t* regs16);
int tac_sregs_read(tac_engine* e, int seq, uint16_t* regs16);

/* Decode and plan a stream (the work Simulator.step/_execute repeat for
 * every instruction, simulator.py:200-206,299-322,476-565, done once).
 * insn_bytes: the big-endian instruction region, n_insns words, fetched from
 * entry_pc on; at most max_insns retire.  init_regs: registers at entry;
 * sregs_reset != 0 means the scale registers start at zero (run_program's
 * volatile reset, simulator.py:147-160), else they keep their values.
 * sites: words that change between runs.  Needs no GPU.
 * A stream that faults still compiles: info->faulted is set, the plan
 * covers the instructions before the fault and *fault describes it. */
int tac_compile(int batch, uint64_t dram_bytes, uint64_t shared_bytes,
                const uint8_t* insn_bytes, uint64_t n_insns, uint64_t entry_pc,
                uint64_t max_insns, const tac_regs* init_regs, int sregs_reset,
                const tac_var_site* sites, int n_sites, tac_program** out,
                tac_exec_info* info, tac_fault* fault);
int tac_program_destroy(tac_program* p);
int tac_program_info(const tac_program* p, tac_exec_info* info, tac_fault* fault);

/* Compile options.  By default a run leaves the complete architectural state
 * behind (every SRAM byte, every DRAM byte, the scale registers), as the
 * golden simulator does.  A caller that only needs part of it (a batched
 * generation loop reads logits and keeps the KV cache) lists the DRAM byte
 * ranges that stay live after the run; values the run leaves in other
 * writable DRAM bytes, in SRAM (sram_live = 0) or in the scale registers
 * (sregs_live = 0) may then be dropped.  n_live = 0 keeps everything. */
typedef struct tac_compile_opts {
  uint32_t n_live;
  int32_t sram_live;
  int32_t sregs_live;
  int32_t flags;          /* TAC_COMPILE_* bits */
  const uint64_t* live;   /* [n_live][2] byte ranges [lo, hi) */
} tac_compile_opts;
/* Keep every intermediate in an arena extent of its own (no reuse by
 * liveness): plan checks that overwrite rows no op reads use it. */
#define TAC_COMPILE_NO_PACK 1

int tac_compile_ex(int batch, uint64_t dram_bytes, uint64_t shared_bytes,
                   const uint8_t* insn_bytes, uint64_t n_insns, uint64_t entry_pc,
                   uint64_t max_insns, const tac_regs* init_regs, int sregs_reset,
                   const tac_var_site* sites, int n_sites, const tac_compile_opts* opts,
                   tac_program** out, tac_exec_info* info, tac_fault* fault);

/* What a compiled run reads that an earlier run may have left behind:
 * writable-DRAM byte ranges (up to max_ranges, [lo, hi) pairs), and whether it
 * reads SRAM or scale registers it did not write itself. */
int tac_program_home_reads(const tac_program* p, uint64_t* ranges, uint32_t max_ranges, uint32_t* n_ranges,
                           int32_t* sram_read, int32_t* sregs_read);

/* Plan introspection (profiling and tests): copy out the device ops
 * (sizeof = tac_program_record_size(0)), gather segments (record size 1),
 * tasks (record size 2) and per-level task offsets (uint32, n_levels + 1). */
uint64_t tac_program_record_size(int which);
int tac_program_dump(const tac_program* p, void* ops, void* segments, void* tasks,
                     uint32_t* level_offsets);

/* Run a compiled stream on every sequence (Simulator.run_program
 * simulator.py:181-198; batched).  var_words: [batch][n_var_words] current
 * values of the runtime words in site order (a pair contributes its LO then
 * its HI word).  stream: a cudaStream_t or NULL.  tac_run_async returns
 * after enqueueing; tac_run waits and reports device-side faults. */
int tac_run_async(tac_engine* e, tac_program* p, const uint64_t* var_words, void* stream,
                  tac_fault* fault);
int tac_run(tac_engine* e, tac_program* p, const uint64_t* var_words, tac_fault* fault);
int tac_check_device_status(tac_engine* e, tac_fault* fault);

/* Split form of tac_run_async for callers that stage inputs ahead of time:
 * tac_encode_params decodes and range-checks one run's runtime words on the
 * host into params_out[batch][tac_program_param_count(p)] (no GPU needed);
 * tac_run_async_params runs with those parameters already in device memory. */
uint64_t tac_program_param_count(const tac_program* p);

/* The fewest softmax key columns any runtime-configured masked softmax of the
 * stream has (0 when none): a valid_kv_len, and so a decode position, must
 * fit them.  A runner uses it to bound the runtime KV-cache addresses it
 * declares (no reference counterpart; no GPU needed). */
uint32_t tac_program_attn_key_cols(const tac_program* p);
int tac_encode_params(const tac_program* p, int batch, const uint64_t* var_words, uint64_t* params_out,
                      tac_fault* fault);
int tac_run_async_params(tac_engine* e, tac_program* p, const uint64_t* params_dev, void* stream,
                         tac_fault* fault);

/* Runtime words as affine functions of a sequence's token and position, so a
 * runner need not build the words every step (the values HostRunner patches,
 * host_runner.py:51-62; no reference counterpart as an entry point).  One
 * entry per runtime site, in site order: a SET_ADDR pair holds
 * base + token * tok_mul + position * pos_mul; a CONFIG_ATTN word holds
 * query_row_base = position, valid_kv_len = position + 1 and mode (the other
 * arrays' entries are ignored).  tac_encode_params_tp gives exactly what
 * tac_encode_params gives for the words those formulas produce, faults
 * included (TAC_E_RECOMPILE outside the compiled ranges); tac_run_async_tp is
 * tac_run_async fed that way.  tokens, positions: int64[batch]. */
int tac_program_set_var_formula(tac_program* p, uint32_t n_sites, const uint64_t* base, const uint64_t* tok_mul,
                                const uint64_t* pos_mul, const uint32_t* mode);
int tac_encode_params_tp(const tac_program* p, int batch, const int64_t* tokens, const int64_t* positions,
                         uint64_t* params_out, tac_fault* fault);
int tac_run_async_tp(tac_engine* e, tac_program* p, const int64_t* tokens, const int64_t* positions, void* stream,
                     tac_fault* fault);

/* Greedy decode helpers for batched generation (HostRunner._greedy_token,
 * host_runner.py:97-101): argmax over `count` FP16 values at DRAM address
 * `addr` of every sequence, written to out_tokens (device int32[batch]).
 * Ties resolve to the lowest index, like numpy.argmax. */
int tac_argmax_f16(tac_engine* e, uint64_t addr, uint64_t count, int32_t* out_tokens_dev,
                   void* stream);

/* Profiling (the golden model's analytic cycle_count has no wall-clock
 * counterpart, golden_model/simulator.py:208-236 trace hooks): when enabled
 * (enable = 1), each run records the device time at the end of every plan
 * level; tac_read_profile copies the n_levels + 1 timestamps (ns) of the last
 * run.  enable = 2 also records each task's duration in SM cycles, read with
 * tac_read_task_profile (entry i = task i in level order; no reference
 * counterpart). */
int tac_set_profiling(tac_engine* e, int enable);
int tac_read_profile(tac_engine* e, uint64_t* out_ns, uint32_t max_entries, uint32_t* n_entries);
int tac_read_task_profile(tac_engine* e, uint32_t* out_cycles, uint64_t max_entries, uint64_t* n_entries);

/* CTAs of the persistent executor (SMs x resident CTAs per SM); no
 * reference counterpart. */
int tac_engine_grid(const tac_engine* e);

/* Per-sequence device pointer arithmetic for zero-copy callers. */
int tac_engine_layout(const tac_engine* e, void** seq_base, uint64_t* seq_stride,
                      void** shared_base);

/* ---- Stand-alone kernels ------------------------------------------------ */

/* INT8 GEMM with the REQUANT_PC epilogue: out[M,N] int8 =
 * clip(rint(float(A[M,K] @ B[K,N]) * float(scale[n]))), A K-major (row-major),
 * B row-major [K,N], scale FP16 bits.  The MATMUL + REQUANT_PC instruction
 * pair (golden_model/systolic.py:31-71, simulator.py:661-688) fused into one
 * tcgen05 kernel.  All pointers are device pointers. */
int tac_gemm_i8_requant_pc(const int8_t* A, const int8_t* B, const uint16_t* scale_f16,
                           int8_t* out, int M, int N, int K, void* stream);

/* INT8 GEMM with an integer requant epilogue: out = clip((acc * mult[n] +
 * 2^(shift[n]-1)) >> shift[n]) computed in int64, shift 8..15.  No reference
 * counterpart (the reference requant is FP16-scale based); parity unpinned. */
int tac_gemm_i8_requant_shift(const int8_t* A, const int8_t* B, const int32_t* mult,
                              const int32_t* shift, int8_t* out, int M, int N, int K,
                              void* stream);

/* Raw INT8 GEMM with int32 output C[M,N] = A @ B (MATMUL, systolic.py:31-71). */
int tac_gemm_i8_i32(const int8_t* A, const int8_t* B, int32_t* C, int M, int N, int K,
                    void* stream);

/* The same products with B supplied transposed, Bt[N,K] row-major (K-major,
 * as static weights can be stored once), the layout the INT8 tensor-core MMA
 * reads fastest.  tcgen05 shapes only: K and N multiples of 16, pointers
 * 16-byte aligned (TAC_E_ARGUMENT otherwise).  Results equal
 * tac_gemm_i8_requant_pc / tac_gemm_i8_i32 on B = Bt^T.  The MATMUL of
 * systolic.py:31-71 with a different operand layout. */
int tac_gemm_i8_requant_pc_bt(const int8_t* A, const int8_t* Bt, const uint16_t* scale_f16,
                              int8_t* out, int M, int N, int K, void* stream);
int tac_gemm_i8_i32_bt(const int8_t* A, const int8_t* Bt, int32_t* C, int M, int N, int K, void* stream);

/* Decode GEMV with the REQUANT_PC epilogue that allocates nothing: out[M,N]
 * int8 = the same result as tac_gemm_i8_requant_pc, for M <= 16 rows, computed
 * split-K over about two CTAs per SM.  Its int32 partial sums and per-column-
 * block arrival counters live in a static device workspace of 8 MiB
 * (requires M * N * 4 <= 8 MiB, N <= 65536; TAC_E_ARGUMENT otherwise).
 * The first call on each device does the set-up (looks up the workspace's
 * device address and clears the counters with a memset on `stream`; no device
 * synchronisation), so make it once before any stream capture: during a
 * capture that first call returns TAC_E_UNSUPPORTED and launches nothing.
 * Later calls only launch.  The counters return to zero at the end of every
 * call; after a failed launch (TAC_E_CUDA) the next call repeats the set-up,
 * and after cudaDeviceReset the caller must reload the library.  Calls that
 * overlap in time on one device share the workspace and race: issue them on
 * one stream.  No counterpart in the reference. */
int tac_gemv_i8_requant_pc_static(const int8_t* A, const int8_t* B, const uint16_t* scale_f16,
                                  int8_t* out, int M, int N, int K, void* stream);

/* Weight-only INT8 GEMM: Y[M,N] float32 = X[M,K] FP16 (bits) x (Q[K,N] * scale[n])
 * + bias[n] (bias may be null): the reference's W8A32 weight-only path, INT8
 * weights with per-output-channel float32 scales dequantised and multiplied in
 * float32 (runtime/fp32_reference.py:330-345 _weight_only_qdq_per_channel, used
 * by build_weight_only_int8_reference :389), with Q stored [K,N] as the ISA's
 * weights are.  tcgen05 kind::f16 with float32 accumulation (an INT8 weight and
 * an FP16 x FP16 product are exact), the scale and bias in the epilogue; the
 * result differs from the reference's float32 products only in summation
 * order.  K a multiple of 8, N of 16, X and Q 16-byte aligned (TAC_E_ARGUMENT
 * otherwise).  Device pointers; asynchronous on `stream`; timeouts are
 * reported by tac_gemm_status. */
int tac_gemm_wo_f16_i8(const uint16_t* X, const int8_t* Q, const float* scale, const float* bias, float* Y,
                       int M, int N, int K, void* stream);

/* ---- QuaRot W8A16 layer ----------------------------------------------------
 * The reference folds QuaRot's rotation into the weights offline
 * (quantizer/rotation.py:51-135) and has no runtime Hadamard; these entry
 * points add one.  All pointers are device pointers; FP16 values as bits. */

/* Y[M,K] = rows of X rotated by the normalised block Walsh-Hadamard
 * I (x) H_block / sqrt(block) (H the Sylvester matrix of rotation.py:108-114):
 * float32 butterflies, one rounding to FP16.  block: a power of two in
 * [32, 1024] dividing K; X and Y 16-byte aligned. */
int tac_fwht_f16(const uint16_t* X, uint16_t* Y, int M, int K, int block, void* stream);

/* Bytes of workspace tac_quarot_w8a16 needs (rotated FP16 rows, their INT8
 * quantisation, scale words). */
uint64_t tac_quarot_workspace_bytes(int M, int K);

/* Y[M,N] FP16 = the W8A16 dynamic matmul (runtime/w8a16_simulator_reference.py:96-135:
 * per-tensor max|x| floored at 2^-9, FP16 inverse / forward scales, INT8
 * round-half-even activations, INT8 x INT8 -> int32, then
 * fp16((f32(acc) * f32(w_scale[n])) * f32(fwd) + f32(bias[n]))) applied to the
 * block-Hadamard-rotated rows of X.  W int8 [K,N] row-major; bias may be null;
 * workspace >= tac_quarot_workspace_bytes(M, K), 256-byte aligned.  Four
 * stream-ordered launches: rotation (+ max|x|), activation quantisation,
 * tcgen05 GEMM with the dequant epilogue.  Calls sharing a workspace must not
 * overlap. */
int tac_quarot_w8a16(const uint16_t* X, const int8_t* W, const uint16_t* w_scale, const uint16_t* bias,
                     uint16_t* Y, void* workspace, uint64_t workspace_bytes, int M, int N, int K,
                     int block, void* stream);

/* ---- Offline weight quantisation ------------------------------------------
 * Per-channel (per_channel = 1) or per-tensor symmetric INT8 quantisation of
 * a float32 weight W[out_ch, in_features] (row-major, PyTorch layout), as
 * quantize_tensor (quantizer/quantize.py:6-33) computes it:
 * scale = max(max|W[n,:]|, 1e-8) / 127 in float32, q = clip(rint(W / scale),
 * -128, 127) with IEEE float32 division; then laid out as
 * _quantize_linear_weight (runtime/tiny_fixture.py:149-159) does: zero-padded
 * to multiples of 16 and transposed, q_kn[K_pad, N_pad] int8 (K = in_features,
 * N = out_ch), scale_f16[N_pad] FP16 bits (padding rows repeat the last
 * channel's scale), scale_f32[out_ch] scratch that ends holding the float32
 * scales of the out_ch channels.  Inputs must be finite.  All pointers are
 * device pointers; q_kn 16-byte aligned.  Stream-ordered, 2 or 3 launches. */
int tac_quantize_weight_i8(const float* W, int out_ch, int in_features, int per_channel, int8_t* q_kn,
                           uint16_t* scale_f16, float* scale_f32, void* stream);

/* ---- Bundle files ------------------------------------------------------------
 * A saved ProgramBundle (ProgramBundle.save: an uncompressed .npz of the
 * prefill and decode instruction streams, the shared data image and a JSON
 * metadata record, each a 1-D uint8 array) mapped read-only into memory.
 * The pointers stay valid until tac_bundle_close; nothing is copied.  Stands
 * in for loading the reference's ProgramBundle (assembler/assembler.py:163-548).
 * TAC_E_ARGUMENT for a missing, truncated or malformed file or entry,
 * TAC_E_UNSUPPORTED for a compressed entry.  Host only. */
typedef struct tac_bundle_view {
  const uint8_t* prefill;
  uint64_t prefill_len;
  const uint8_t* decode;
  uint64_t decode_len;
  const uint8_t* shared;
  uint64_t shared_len;
  const char* meta_json;   /* not NUL-terminated */
  uint64_t meta_len;
} tac_bundle_view;

int tac_bundle_open(const char* path, tac_bundle_view* view, void** handle);
int tac_bundle_close(void* handle);

/* The stand-alone GEMMs run on the tcgen05 kernel when K and N are
 * multiples of 16 and A, B and the output are 16-byte aligned, otherwise on
 * an mma.sync kernel; both are exact.  Every wait inside the tcgen05 kernel
 * is bounded: one that runs out sets a device fault code and the kernel
 * returns.  tac_gemm_status synchronizes the current device, returns
 * TAC_E_DEVICE (code in *fault_code, then cleared) if any launch since the
 * last call recorded one, else TAC_OK.  No reference counterpart. */
int tac_gemm_status(int* fault_code);

#ifdef __cplusplus
}
#endif

#endif /* TACCEL_B200_H */
