#!/usr/bin/env python
"""Benchmark: compiled GPT-2 decoder programs on the B200 engine.

Workload (default ``gpt2-medium``): GPT-2 medium (24 layers, d_model 1024,
16 heads, vocab 50257) compiled by the reference toolchain to a W8A16
ProgramBundle with a 256-position KV window; a fixed global batch of 64
independent sequences split over the N GPUs (strong scaling: each rank owns a
contiguous block of sequence ids, no collective on the data path; ``--weak``
gives every GPU 64 sequences of its own instead).  A step runs the decode
stream once for every sequence (one token each).  Every sequence first
consumes a 128-token random prompt (prefill + teacher-forced decode steps,
untimed; shorter when the KV window must also hold the warm-up, timed and e2e
steps), then runs W warm-up steps.  ``value`` times the next K teacher-forced
decode steps with their runtime parameters already in device memory; ``e2e``
times the K greedy steps after them through the public runner API with host
buffers (runtime words in, argmax token ids out, every step; the ranks
all-gather the token ids).  At N > 1 the same run also times 64 sequences per
GPU (``weak``).

Parity: after timing, the logits of the last timed step and the greedy tokens
of the e2e steps of the sequences the reference golden simulator ran
(tests/golden/run_gpt2_medium_late.npz) are compared with its results; the
line carries the outcome and the process exits 1 on a mismatch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gpt2-medium|gpt2-small] [--batch B] [--weak]

``--batch`` is the global batch (the per-GPU batch with ``--weak``).

``--impl reference`` times the CPU oracle port of the golden simulator on the
host cores (rank 0 only) with the same metric: whole decode steps, one
sequence per host process.
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import tempfile
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GPT-2 tokens/sec (1/2/4/8 B200) bit-exact vs golden sim; INT8 GEMM TOPS vs peak"
WORKLOADS = {
    "gpt2-medium": dict(recipe="tests/golden/recipe_gpt2_medium.npz", batch=64, n_layer=24, d_model=1024,
                        n_head=16, kv_len=256, prompt=128, new=128,
                        desc="GPT-2 medium (24 layers, d_model 1024, 16 heads, vocab 50257) W8A16 compiled "
                             "decode stream, KV cache 256 positions"),
    "gpt2-small": dict(recipe="tests/golden/recipe_gpt2_small.npz", batch=64, n_layer=12, d_model=768,
                       n_head=12, kv_len=48, prompt=16, new=32,
                       desc="GPT-2 small (12 layers, d_model 768, 12 heads, vocab 50257) W8A16 compiled "
                            "decode stream, KV cache 48 positions"),
}
VOCAB = 50257
SHARED = 1 << 63


# ----------------------------------------------------------------------------------------
# CPU oracle port of the golden simulator; workers fork before CUDA starts
# ----------------------------------------------------------------------------------------
_W = {}


def _worker_init():
    from oracle import golden as G
    sim = G.OracleSimulator()
    sim.state.dram = bytearray(_W["image"])
    sim.bundle = sim.program = _W["bundle"]
    _W["sim"] = sim


def _worker_step(_):
    """One whole decode step of this worker's sequence; its duration."""
    t = time.perf_counter()
    _W["sim"].run_program(_W["bundle"], "decode")
    return time.perf_counter() - t


def host_cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuSampler:
    """Whole decode steps on `workers` host processes, one sequence each (the
    golden simulator is single-threaded NumPy; its int32 matmul uses one
    core).  A sample is one step of every worker: `workers` tokens in the
    slowest worker's time."""

    def __init__(self, bundle, workers: int):
        _patch_decode(bundle, token=1, pos=1)
        self.bundle = bundle
        _W["bundle"] = bundle
        _W["image"] = bundle.materialize(reset_runtime=False)
        _patch_decode(bundle, token=1, pos=1)
        self.workers = workers
        self.pool = mp.get_context("fork").Pool(workers, initializer=_worker_init)

    def step(self):
        t = max(self.pool.map(_worker_step, range(self.workers)))
        return dict(tokens=float(self.workers), seconds=t)

    def close(self):
        self.pool.close()
        self.pool.join()

    def describe(self) -> str:
        return (f"{self.workers} host processes ({host_cpu_model()}), one sequence each; a step is one whole "
                f"decode step of every process (no extrapolation)")


def cpu_workers() -> int:
    """Host processes for the CPU arm: every core, at most 32 (each holds a
    private ~0.9 GB DRAM image)."""
    return max(1, min(os.cpu_count() or 1, 32))


def _patch_decode(b, token, pos):
    row = b.embedding_row_bytes
    for s in b.runtime_patch_sites:
        if s.stream == "decode":
            b.patch_runtime_site(s, {"token_embed": token * row, "pos_embed": pos * row,
                                     "kv_base": pos * b.kv_step_bytes}[s.kind])
    for s in b.runtime_config_attn_sites:
        if s.stream == "decode":
            b.patch_config_attn_site(s, query_row_base=pos, valid_kv_len=pos + 1)


# ----------------------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------------------
def load_workload(name):
    from llm_accelerator_b200.recipe import load_recipe
    w = WORKLOADS[name]
    return w, load_recipe(ROOT / w["recipe"])


def algorithmic_bytes(plan, batch, bundle, w, positions):
    """Bytes one decode step must move, averaged over the timed steps:
    the shared weights / tables it reads once (the union of the plan's shared
    operand ranges), plus per sequence
      - the KV cache it reads: n_layer x (K and V) x d_model x 2 B for each of
        the pos + 1 valid key positions of the step,
      - the KV rows it appends and the embedding rows it loads (the plan's
        runtime-addressed stores and loads),
      - the FP16 logits it writes.
    Returns (total, shared bytes, per-sequence bytes)."""
    ops, segs, _, _ = plan.dump()
    ranges = []
    per_seq = 0

    def add(p, nbytes):
        if int(p) & SHARED:
            u = int(p) & ~SHARED
            ranges.append((u, u + (int(nbytes) + 15) // 16))

    for op in ops:
        k, M, N, K = int(op["kind"]), int(op["M"]), int(op["N"]), int(op["K"])
        if k == 6:        # MATMUL
            add(op["a"], M * K)
            add(op["b"], K * N)
        elif k in (14, 15, 18):   # DEQUANT_ACCUM / DEQUANT_SCALED / LAYERNORM vectors
            add(op["b"], (2 * N if k == 14 else 4 * N))
        elif k in (2, 3):         # runtime-addressed loads (embedding rows) and stores (KV appends)
            per_seq += int(op["nbytes"])
        elif k == 30:             # merged runtime-addressed stores: one segment (n bytes) each
            per_seq += int(segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]["n"].sum())
        elif k == 1:      # gathers of shared data
            for sg in segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]:
                add(int(sg["src"]), int(sg["n"]) * 16)
    ranges.sort()
    total, cur_lo, cur_hi = 0, None, None
    for lo, hi in ranges:
        if cur_hi is None or lo > cur_hi:
            if cur_hi is not None:
                total += cur_hi - cur_lo
            cur_lo, cur_hi = lo, hi
        else:
            cur_hi = max(cur_hi, hi)
    if cur_hi is not None:
        total += cur_hi - cur_lo
    kv_read = w["n_layer"] * 2 * w["d_model"] * 2 * float(np.mean([p + 1 for p in positions]))
    per_seq += kv_read + int(bundle.logits_size)
    return total * 16 + batch * per_seq, total * 16, per_seq


class ClockSampler:
    def __init__(self, index):
        self.index = index
        self.p = None

    def __enter__(self):
        # samples go to $TAC_CLOCKS_DIR (kept) or a temporary directory
        d = os.environ.get("TAC_CLOCKS_DIR") or tempfile.mkdtemp(prefix="tac_clocks_")
        self.out = Path(d) / f"clocks_{os.getpid()}.csv"
        self.out.parent.mkdir(parents=True, exist_ok=True)
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.out, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()

    def summary(self):
        if not self.out.exists():
            return None
        rows = [r.split(", ") for r in self.out.read_text().strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


INT8_DENSE_PEAK_TOPS = 4500.0   # nominal dense INT8 tensor peak of one B200


def int8_gemm_line():
    """Second half of the metric: the stand-alone MATMUL + REQUANT_PC kernel at
    4096^3 against the dense INT8 tensor peak, with cuBLASLt INT8 timed beside it."""
    from llm_accelerator_b200.gemm import time_gemm
    r = time_gemm(4096, 4096, 4096, epilogue="requant_pc", iters=20, warmup=5)
    bf16 = None
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        bf16 = float(json.loads(p.read_text()).get("bf16_tflops", 0.0)) or None
    out = {"shape": r["shape"], "epilogue": "MATMUL + REQUANT_PC (int8 out)", "ms": round(r["ms"], 4),
           "ms_cold": round(r["ms_cold"], 4), "tops": round(r["tops"], 1), "peak_tops": INT8_DENSE_PEAK_TOPS,
           "peak_kind": "nominal dense INT8", "frac": round(r["tops"] / INT8_DENSE_PEAK_TOPS, 4),
           "timing": f"ms: steady state, {10 * r['operand_sets']} launches in one CUDA graph cycling through "
                     f"{r['operand_sets']} operand sets (256 MB, operands from HBM), CUDA events; ms_cold: one "
                     f"launch after an L2 flush (median of 20); cuBLASLt timed the same way"}
    if bf16:
        out["frac_of_2x_measured_bf16"] = round(r["tops"] / (2 * bf16), 4)
    if "cublas_tops" in r:
        out["cublas_int_mm_tops"] = round(r["cublas_tops"], 1)
        out["vs_cublas"] = round(r["tops"] / r["cublas_tops"], 3)
    return out


def quarot_line():
    """The QuaRot W8A16 layer workload (1024 x 768 activations = 8 x 128
    tokens, 768 x 3072 INT8 weights, block Hadamard 3 x 256): device time of
    rotation + quantisation + INT8 GEMM with the dequant epilogue."""
    from llm_accelerator_b200.quarot import time_layer
    r = time_layer(1024, 768, 3072, block=256)
    peak_gbs, _ = measured_peak()
    return {"shape": r["shape"], "block": r["block"], "ms": round(r["ms"], 4), "ms_cold": round(r["ms_cold"], 4),
            "tops": round(r["tflops"], 1),
            "frac_of_nominal_int8": round(r["tflops"] / INT8_DENSE_PEAK_TOPS, 4),
            "gbs": round(r["gbs"], 1), "frac_of_measured_hbm": round(r["gbs"] / peak_gbs, 4),
            "algorithmic_bytes": r["bytes"],
            "timing": f"2 stream-ordered launches per call (rotation with per-CTA maxima, then the GEMM that "
                      f"quantises the rotated rows while staging them); ms: steady state, {10 * r['input_sets']} "
                      f"calls in one CUDA graph cycling through {r['input_sets']} input sets (256 MB, so inputs "
                      f"come from HBM), CUDA events; ms_cold: one call after an L2 flush (median of 20)"}


def weight_only_line():
    """The weight-only INT8 GEMM at the W8A16 layer shape (1024 x 768 FP16
    activations, 768 x 3072 INT8 weights with float32 per-column scales,
    float32 out) against the measured HBM copy bandwidth and the measured
    bf16 tensor throughput (it runs kind::f16)."""
    from llm_accelerator_b200.gemm import time_gemm_wo
    r = time_gemm_wo(1024, 3072, 768)
    peak_gbs, _ = measured_peak()
    out = {"shape": r["shape"], "ms": round(r["ms"], 4), "ms_cold": round(r["ms_cold"], 4),
           "tflops": round(r["tflops"], 1), "gbs": round(r["gbs"], 1),
           "frac_of_measured_hbm": round(r["gbs"] / peak_gbs, 4), "algorithmic_bytes": r["bytes"],
           "timing": f"ms: steady state, {10 * r['input_sets']} calls in one CUDA graph cycling through "
                     f"{r['input_sets']} input sets (256 MB, inputs from HBM), CUDA events; ms_cold: one call "
                     f"after an L2 flush (median of 20)"}
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        bf16 = float(json.loads(p.read_text()).get("bf16_tflops", 0.0))
        if bf16:
            out["frac_of_measured_bf16"] = round(r["tflops"] / bf16, 4)
    return out


def gemv_line():
    """The decode GEMV of the MATMUL sweep (M 1, K 768, N 3072, MATMUL +
    REQUANT_PC): per-call device time with the weights cycling through 256 MB
    of distinct buffers, against the measured HBM copy bandwidth."""
    from llm_accelerator_b200.gemm import time_gemv
    r = time_gemv(1, 3072, 768)
    peak_gbs, _ = measured_peak()
    out = {"shape": r["shape"], "algorithmic_bytes": r["bytes"], "weight_buffers": r["weight_buffers"],
           "timing": "400 calls captured in one CUDA graph, replay timed with CUDA events (median of 3), "
                     "weights rotated over 256 MB"}
    for k in ("general", "splitk_static"):
        out[k] = {"us": round(r[k]["us"], 2), "gbs": round(r[k]["gbs"], 1),
                  "frac_of_measured_hbm": round(r[k]["gbs"] / peak_gbs, 4)}
    return out


def ptq_line():
    """Offline weight quantisation of GPT-2's lm_head (50257 x 768 float32 ->
    per-channel INT8 [768, 50272] image + FP16 scales): device time of
    tac_quantize_weight_i8 against the measured HBM copy bandwidth."""
    from llm_accelerator_b200.ptq import time_quantizer
    r = time_quantizer(50257, 768)
    peak_gbs, _ = measured_peak()
    return {"shape": r["shape"], "ms": round(r["ms"], 4), "gbs": round(r["gbs"], 1),
            "frac_of_measured_hbm": round(r["gbs"] / peak_gbs, 4), "algorithmic_bytes": r["bytes"],
            "timing": "median of 20 calls (2 stream-ordered launches), CUDA events, L2 flushed"}


def traffic_per_launch(workload, batch):
    """DRAM bytes per executor launch from the committed ncu summary (a
    capture of an earlier run of this bench command, not of this run): the
    line for this batch, else a least-squares line through the captured
    batches (None without a summary)."""
    f = ROOT / "profiles" / f"exec_kernel_{workload}.txt"
    if not f.exists():
        return None
    pts = {}
    for line in f.read_text().splitlines():
        if line.startswith("dram_bytes_batch_") and "=" in line:
            k, v = line.split("=", 1)
            pts[int(k.strip()[len("dram_bytes_batch_"):])] = float(v.strip())
    if not pts:
        return None
    if batch in pts:
        return pts[batch]
    if len(pts) == 1:
        (b0, v0), = pts.items()
        return v0 * batch / b0
    xs, ys = np.array(list(pts)), np.array(list(pts.values()))
    slope, icpt = np.polyfit(xs, ys, 1)
    return float(icpt + slope * batch)


# ----------------------------------------------------------------------------------------
# parity against the reference golden simulator's own runs
# ----------------------------------------------------------------------------------------
LATE_GOLDEN = {"gpt2-medium": "tests/golden/run_gpt2_medium_late.npz"}
# a logits vector that is not bit-exact may differ by at most this fraction of
# its largest |logit| (transcendental ops are evaluated in float64 and rounded
# once; NumPy's float32 exp / tanh are not correctly rounded, and a one-ulp
# difference can move an INT8 quantisation step further down the network)
LOGIT_TOL = 0.05


def sequence_tokens(seq: int, n: int) -> np.ndarray:
    """Token ids of sequence `seq`: the prompt and its teacher-forced
    continuation (prefix-consistent in n)."""
    return np.random.default_rng(int(seq)).integers(0, VOCAB, n)


class Parity:
    """The golden sequences this rank owns, checked against the reference's
    results: the logits after the last timed step (teacher-forced position q)
    and the greedy tokens of the e2e steps (when they continue the golden
    run, i.e. q is its last teacher-forced position)."""

    def __init__(self, workload, seqs):
        self.path = LATE_GOLDEN.get(workload)
        self.z = None
        if self.path and (ROOT / self.path).exists():
            z = np.load(ROOT / self.path)
            self.z = {k: z[k] for k in z.files}
        self.local = {}
        if self.z is not None:
            for s in self.z["seqs"].tolist():
                if s in seqs:
                    self.local[int(s)] = list(seqs).index(s)
        self.checks, self.failures = [], []

    def _fail(self, msg):
        self.failures.append(msg)

    def token_ok(self, s, pos, tok):
        """The reference's greedy token, or its runner-up when the two are
        within LOGIT_TOL of each other in the reference's own logits."""
        want = int(self.z[f"s{s}_token"][pos])
        if tok == want:
            return True
        top = self.z[f"s{s}_top_val"][pos].astype(np.float32)
        return (tok == int(self.z[f"s{s}_top_idx"][pos][1]) and
                float(top[0] - top[1]) <= LOGIT_TOL * float(self.z[f"s{s}_maxabs"][pos]))

    def check_logits(self, runner, q):
        if self.z is None or q > int(self.z["tf_last"][0]):
            return
        import hashlib
        for s, i in self.local.items():
            got = runner.logits("decode", i)
            dig = np.frombuffer(hashlib.sha256(got.tobytes()).digest(), np.uint8)
            exact = bool(np.array_equal(dig, self.z[f"s{s}_digest"][q]))
            v = got[:VOCAB].astype(np.float32)
            tok_ok = self.token_ok(s, q, int(np.argmax(v)))
            idx = np.concatenate([self.z["sample_idx"], self.z[f"s{s}_top_idx"][q]])
            want = np.concatenate([self.z[f"s{s}_sample"][q], self.z[f"s{s}_top_val"][q]]).astype(np.float32)
            fs = self.z["full_steps"].tolist()
            if q in fs:
                idx = np.arange(VOCAB)
                want = self.z[f"s{s}_full"][fs.index(q)][:VOCAB].astype(np.float32)
            err = float(np.max(np.abs(v[idx] - want)))
            tol = LOGIT_TOL * float(self.z[f"s{s}_maxabs"][q])
            self.checks.append(dict(seq=s, pos=q, exact=exact, token=tok_ok, max_abs_err=round(err, 5)))
            if not (exact or (tok_ok and err <= tol)):
                self._fail(f"seq {s} pos {q}: logits differ (max abs {err:.4g} > {tol:.4g} or token)")

    def check_tokens(self, seq_tokens, pos0, q):
        """seq_tokens[i]: the gathered greedy token of every sequence at position pos0 + i."""
        if self.z is None or q != int(self.z["tf_last"][0]):
            return
        last = int(self.z["tf_last"][0]) + int(self.z["greedy"][0])
        for s in self.z["seqs"].tolist():
            if s >= len(seq_tokens[0]):
                continue        # not in this run's batch
            want = self.z[f"s{s}_token"]
            n = ok = 0
            for i, toks in enumerate(seq_tokens):
                pos = pos0 + i
                if pos > last:
                    break
                n += 1
                if not self.token_ok(s, pos, int(toks[s])):
                    self._fail(f"seq {s} pos {pos}: greedy token {int(toks[s])} != reference {int(want[pos])}")
                    break
                if int(toks[s]) != int(want[pos]):
                    break       # a near tie went the other way: the runs part here
                ok += 1
            self.checks.append(dict(seq=int(s), greedy_steps=n, tokens_equal=ok))

    def summary(self):
        if self.z is None:
            return "unchecked: no reference run of this workload"
        if not self.checks:
            return "unchecked: timed positions outside the reference run"
        return "failed" if self.failures else "checked"


# ----------------------------------------------------------------------------------------
def run_reference(args, w, bundle, rank, world):
    if rank != 0:
        return
    sampler = CpuSampler(bundle, cpu_workers())
    W = args.warmup
    for _ in range(W):
        sampler.step()
    toks = secs = 0.0
    for _ in range(args.steps):
        r = sampler.step()
        toks += r["tokens"]
        secs += r["seconds"]
    sampler.close()
    v = toks / secs
    B_total = args.batch or w["batch"]
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": W, "ms_per_step": round(1000 * secs / args.steps, 1),
        "higher_is_better": True, "scaling": "weak" if args.weak else "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic: seeded random-init weights in the reference-compiled program",
        "config": {"workload": w["desc"], "global_batch": B_total * (max(args.gpus, world) if args.weak else 1)},
        "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": sampler.workers, "kind": "port",
                         "sample": sampler.describe(), "cpu": host_cpu_model()},
        "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def _time_decode(runner, prompts, p0, K, dev, stream, barrier):
    """K teacher-forced steps at positions p0.. with device-resident
    parameters; CUDA-event milliseconds on the launching stream."""
    import torch
    B = runner.batch
    params = np.stack([runner.params("decode", prompts[:, p], np.full(B, p)) for p in range(p0, p0 + K)])
    d_params = torch.from_numpy(params.view(np.int64)).to(dev)
    stride = params.shape[1] * params.shape[2] * 8
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    ev0.record(stream)
    for i in range(K):
        runner.step_params_async("decode", d_params.data_ptr() + i * stride, stream.cuda_stream)
    ev1.record(stream)
    barrier()
    runner.engine.check_device()
    return ev0.elapsed_time(ev1)


def _consume_prompt(runner, prompts, upto):
    B = runner.batch
    runner.step("prefill", prompts[:, 0], np.zeros(B, int))
    for pos in range(1, upto):
        runner.step("decode", prompts[:, pos], np.full(B, pos))


def _max_over_ranks(x, dev, world):
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args, w, bundle, rank, world, local_rank, cpu_baseline):
    import torch
    from llm_accelerator_b200.runner import BatchedRunner
    from llm_accelerator_b200.shard import gather_tokens, shard

    if args.weak:
        B_total = (args.batch or w["batch"]) * world
    else:
        B_total = args.batch or w["batch"]
        if B_total % world:
            raise SystemExit(f"batch {B_total} does not split over {world} GPUs")
    B = B_total // world
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize(dev)

    K, W = args.steps, args.warmup
    if 1 + W + 2 * K >= w["kv_len"]:
        raise SystemExit("steps + warmup exceed the KV length of the workload")
    # the prompt is consumed first (untimed), as far as the KV window leaves
    # room for the warm-up, timed and e2e steps after it
    P = max(1, min(w["prompt"], w["kv_len"] - 1 - W - 2 * K))
    p0 = P + W
    q = p0 + K - 1
    seqs = np.asarray(shard(B_total, world, rank))
    prompts = np.stack([sequence_tokens(s, P + W + K) for s in seqs])
    runner = BatchedRunner(bundle, B, device=local_rank)
    _consume_prompt(runner, prompts, P + W)

    with ClockSampler(local_rank) as clocks:
        ms = _time_decode(runner, prompts, p0, K, dev, stream, barrier)
    ms = _max_over_ranks(ms, dev, world)
    value = B_total * K / (ms / 1000.0)
    parity = Parity(args.workload, list(seqs))
    parity.check_logits(runner, q)

    # e2e: K greedy steps through the runner API with host buffers each step
    tok_dev = torch.zeros(B, dtype=torch.int32, device=dev)
    tok_host = torch.zeros(B, dtype=torch.int32).pin_memory()
    runner.argmax_async("decode", tok_dev.data_ptr(), VOCAB, stream.cuda_stream)
    tok_host.copy_(tok_dev)
    tokens = tok_host.numpy().astype(np.int64)
    first = gather_tokens(tok_dev, world).cpu().numpy()
    pos0 = p0 + K
    gathered = []
    all_host = torch.zeros(B_total, dtype=torch.int32).pin_memory()
    barrier()
    t0 = time.perf_counter()
    for i in range(K):
        runner.step_async("decode", tokens, np.full(B, pos0 + i), stream.cuda_stream)
        runner.argmax_async("decode", tok_dev.data_ptr(), VOCAB, stream.cuda_stream)
        all_dev = gather_tokens(tok_dev, world)   # every rank sees the whole batch's tokens (NCCL all-gather)
        all_host.copy_(all_dev, non_blocking=True)
        stream.synchronize()
        allt = all_host.numpy()
        gathered.append(allt.copy())
        tokens = allt[rank * B:(rank + 1) * B].astype(np.int64)
    barrier()
    e2e_s = _max_over_ranks(time.perf_counter() - t0, dev, world)
    e2e = B_total * K / e2e_s
    runner.engine.check_device()
    # the first greedy token (argmax at q) and the K e2e tokens, all sequences
    parity.check_tokens([first] + gathered, q, q)
    import hashlib
    tokens_sha = hashlib.sha256(np.stack([first] + gathered).astype(np.int32).tobytes()).hexdigest()[:16]

    plan = runner.plans["decode"]
    algo, shared_b, per_seq_b = algorithmic_bytes(plan, B, bundle, w, range(p0, p0 + K))
    from llm_accelerator_b200 import _lib as L
    n_params = int(L.lib.tac_program_param_count(plan.handle))   # 8-byte words staged per sequence and step
    del runner
    torch.cuda.empty_cache()

    # weak scaling beside the strong line: 64 sequences per GPU in the same run
    weak = None
    if world > 1 and not args.weak:
        Bw = args.batch or w["batch"]
        wseqs = np.asarray(shard(Bw * world, world, rank))
        wprompts = np.stack([sequence_tokens(s, P + W + K) for s in wseqs])
        wr = BatchedRunner(bundle, Bw, device=local_rank)
        _consume_prompt(wr, wprompts, P + W)
        wms = _max_over_ranks(_time_decode(wr, wprompts, p0, K, dev, stream, barrier), dev, world)
        weak = {"value": round(Bw * world * K / (wms / 1000.0), 2), "unit": "tokens/s",
                "global_batch": Bw * world, "per_gpu_batch": Bw, "ms_per_step": round(wms / K, 3)}
        del wr
        torch.cuda.empty_cache()

    gemm_line = quarot = ptq = gemv = wo = None
    if rank == 0 and not args.no_gemm:
        gemm_line = int8_gemm_line()
        gemv = gemv_line()
        quarot = quarot_line()
        wo = weight_only_line()
        ptq = ptq_line()
    barrier()

    n_fail = _max_over_ranks(len(parity.failures), dev, world)
    n_checks = _max_over_ranks(len(parity.checks), dev, world)
    if parity.failures:
        for f in parity.failures:
            print(f"rank {rank} parity: {f}", file=sys.stderr, flush=True)
    per_launch_s = ms / 1000.0 / K
    peak, peak_kind = measured_peak()
    achieved = algo / per_launch_s / 1e9
    clk = clocks.summary()
    status = "failed" if n_fail else parity.summary() if n_checks else "unchecked: no golden sequence in this run"
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms / K, 3), "higher_is_better": True,
            "scaling": "weak" if args.weak else "strong",
            "vs_baseline": None, "dtype": "int8",
            "data": "synthetic: seeded random-init weights in the reference-compiled program",
            "config": {"workload": w["desc"], "global_batch": B_total, "per_gpu_batch": B,
                       "parallelism": f"sequences sharded over {world} GPU(s)",
                       "timed": f"{K} teacher-forced decode steps (positions {p0}..{q}, after a "
                                f"{P}-token prompt and {W} warm-up steps); e2e: {K} greedy steps "
                                f"(positions {pos0}..{pos0 + K - 1})",
                       "l2": f"inputs larger than L2: {shared_b / 1e6:.0f} MB of weights read per step"},
            "parity": {"status": status, "reference": LATE_GOLDEN.get(args.workload),
                       "checks": parity.checks, "e2e_tokens_sha256_16": tokens_sha},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic_per_launch(args.workload, B),
                         "traffic_source": f"profiles/exec_kernel_{args.workload}.txt (ncu capture of an "
                                           f"earlier run at this batch), not measured in this run",
                         "peak_kind": peak_kind, "kernel": "tac::exec_kernel",
                         "algorithmic_bytes_per_launch": round(algo),
                         "algorithmic_split": {"shared_weights_tables": shared_b,
                                               "per_sequence_kv_logits_rows": round(per_seq_b)}},
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(B_total * n_params * 8),
                    "d2h_bytes_per_step": int(B_total * 4)},
            "gpu_launches": K,
            "clocks": clk,
        }
        if weak is not None:
            line["weak"] = weak
        if cpu_baseline is not None:
            line["cpu_baseline"] = cpu_baseline
        if gemm_line is not None:
            line["int8_gemm"] = gemm_line
        if quarot is not None:
            line["quarot_w8a16"] = quarot
        if wo is not None:
            line["weight_only_gemm"] = wo
        if gemv is not None:
            line["decode_gemv"] = gemv
        if ptq is not None:
            line["ptq_quantize"] = ptq
        print(json.dumps(line), flush=True)
    return 1 if n_fail else 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gpt2-medium", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=0, help="global batch (per-GPU batch with --weak)")
    ap.add_argument("--weak", action="store_true", help="every GPU runs a batch of its own")
    ap.add_argument("--strong", action="store_true", help="(default) split one global batch over the GPUs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true",
                    help="skip the stand-alone 4096^3 INT8 GEMM and QuaRot layer measurements")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference" and rank != 0:
        return 0
    w, bundle = load_workload(args.workload)
    if args.impl == "reference":
        run_reference(args, w, bundle, rank, world)
        return 0
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from llm_accelerator_b200.recipe import load_recipe
        sampler = CpuSampler(load_recipe(ROOT / w["recipe"]), cpu_workers())
        r = sampler.step()
        sampler.close()
        cpu_baseline = {"value": round(r["tokens"] / r["seconds"], 4), "unit": "tokens/s",
                        "cores": sampler.workers, "kind": "port", "sample": sampler.describe(),
                        "cpu": host_cpu_model()}
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        rc = run_ours(args, w, bundle, rank, world, local_rank, cpu_baseline)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
