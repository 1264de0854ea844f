#!/usr/bin/env python
"""Benchmark: compiled GPT-2 decoder programs on the B200 engine.

Workload (default ``gpt2-medium``): GPT-2 medium (24 layers, d_model 1024,
16 heads, vocab 50257) compiled by the reference toolchain to a W8A16
ProgramBundle with a 256-position KV cache; 64 independent sequences per GPU
(weak scaling: N GPUs run 64 x N sequences, each rank its own shard of the
sequence ids, no collective on the data path; ``--strong`` splits a fixed
global batch instead).  A step runs the decode stream once for every sequence
(one token each).  Every sequence first consumes a 128-token random prompt
(prefill + teacher-forced decode steps, untimed; shorter when the KV window
must also hold the warm-up, timed and e2e steps), then runs W warm-up steps.
``value`` times the next K teacher-forced decode steps with their runtime
parameters already in device memory; ``e2e`` times the K greedy steps after
them through the public runner API with host buffers (runtime words in,
argmax token ids out, every step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gpt2-medium|gpt2-small] [--batch B] [--strong]

``--batch`` is the per-GPU batch (the global batch with ``--strong``).

``--impl reference`` times the CPU oracle port of the golden simulator on the
host cores (rank 0 only) with the same metric.
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
# CPU oracle sample (golden-simulator port); runs in forked workers before CUDA starts
# ----------------------------------------------------------------------------------------
_W = {}


def _worker_init():
    from oracle import golden as G
    sim = G.OracleSimulator()
    sim.state.dram = bytearray(_W["image"])
    sim.bundle = sim.program = _W["bundle"]
    _W["sim"] = sim


def _worker_run(n_insns):
    t = time.perf_counter()
    _W["sim"].run_program(_W["bundle"], "decode", max_instructions=int(n_insns))
    return time.perf_counter() - t


def _mac_profile(bundle):
    """Cumulative padded MATMUL MACs along the decode stream."""
    from oracle import isa as OI
    raw = bundle.stream_bytes("decode")
    macs = np.zeros(len(raw) // 8, np.float64)
    tile = (0, 0, 0)
    for i in range(len(raw) // 8):
        x = OI.decode_bytes(raw[i * 8:i * 8 + 8])
        if x.opcode == OI.CONFIG_TILE:
            tile = (x.M, x.N, x.K)
        elif x.opcode == OI.MATMUL:
            macs[i] = (tile[0] + 1) * (tile[1] + 1) * (tile[2] + 1) * 4096.0
    return np.cumsum(macs)


class CpuSampler:
    """Times prefixes of one decode step on `workers` host processes (one
    sequence each) and extrapolates tokens/s by the prefix's share of the
    step's MATMUL work (MATMUL is ~83% of the golden simulator's time)."""

    def __init__(self, bundle, workers: int):
        _patch_decode(bundle, token=1, pos=1)
        self.bundle = bundle
        self.cum = _mac_profile(bundle)
        _W["bundle"] = bundle
        _W["image"] = bundle.materialize(reset_runtime=False)
        _patch_decode(bundle, token=1, pos=1)
        self.workers = workers
        self.pool = mp.get_context("fork").Pool(workers, initializer=_worker_init)
        # calibrate on the first ~2% of the step's work
        n_cal = int(np.searchsorted(self.cum, 0.02 * self.cum[-1])) + 1
        t = max(self.pool.map(_worker_run, [n_cal] * workers))
        self.rate = self.cum[n_cal - 1] / max(t, 1e-6)   # MAC/s per worker

    def sample(self, seconds: float):
        target = min(self.cum[-1], self.rate * seconds)
        n = int(np.searchsorted(self.cum, target)) + 1
        n = min(n, len(self.cum))
        t = max(self.pool.map(_worker_run, [n] * self.workers))
        frac = float(self.cum[n - 1] / self.cum[-1])
        return dict(tokens=self.workers * frac, seconds=t, insns=n, frac=frac)

    def close(self):
        self.pool.close()
        self.pool.join()


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


def algorithmic_bytes(plan, batch, bundle):
    """Bytes one decode step must move: the shared weights / tables it reads
    once (union of shared operand ranges) plus, per sequence, the KV-cache
    bytes it reads and appends and the embedding rows it loads."""
    ops, segs, _, _ = plan.dump()
    ranges = []
    per_seq = 0
    shared_bytes = bundle.temp_base // 16 * 16
    kv_lo = bundle.kv_cache_base - shared_bytes
    rw_base = 8192 + 16384 + 4096
    rw_end = rw_base + (max(16 << 20, bundle.required_dram_bytes) - shared_bytes + 15) // 16

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
        elif k == 2:      # runtime-addressed load (embedding rows)
            per_seq += int(op["nbytes"])
        elif k == 3:      # runtime-addressed store (KV append)
            per_seq += int(op["nbytes"])
        elif k == 1:      # gathers: KV-cache reads come from the writable home region
            for sg in segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]:
                src = int(sg["src"])
                if not (src & SHARED) and rw_base <= src < rw_end and (src - rw_base) * 16 >= kv_lo:
                    per_seq += int(sg["n"]) * 16
                add(src, int(sg["n"]) * 16)
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
           "tops": round(r["tops"], 1), "peak_tops": INT8_DENSE_PEAK_TOPS, "peak_kind": "nominal dense INT8",
           "frac": round(r["tops"] / INT8_DENSE_PEAK_TOPS, 4),
           "timing": "median of 20 launches, CUDA events, L2 flushed between launches"}
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
    return {"shape": r["shape"], "block": r["block"], "ms": round(r["ms"], 4), "tops": round(r["tflops"], 1),
            "frac_of_nominal_int8": round(r["tflops"] / INT8_DENSE_PEAK_TOPS, 4),
            "gbs": round(r["gbs"], 1), "frac_of_measured_hbm": round(r["gbs"] / peak_gbs, 4),
            "algorithmic_bytes": r["bytes"],
            "timing": "median of 20 calls (4 stream-ordered launches), CUDA events, L2 flushed"}


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
    """DRAM bytes per executor launch from the committed ncu summary: the
    measured line for this batch, else a least-squares line through the
    measured batches (None without a summary)."""
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
def run_reference(args, w, bundle, rank, world):
    if rank != 0:
        return
    workers = min(os.cpu_count() or 1, 16)
    sampler = CpuSampler(bundle, workers)
    budget = max(2.0, 150.0 / max(1, args.steps + min(args.warmup, 1)))
    for _ in range(min(args.warmup, 1)):
        sampler.sample(budget)
    toks = secs = 0.0
    last = None
    for _ in range(args.steps):
        s = sampler.sample(budget)
        toks += s["tokens"]
        secs += s["seconds"]
        last = s
    sampler.close()
    v = toks / secs
    sample = (f"{workers} host processes, one sequence each; per step each runs the first {last['insns']} "
              f"instructions of one decode step ({100 * last['frac']:.1f}% of its MATMUL work), "
              f"tokens credited by that MATMUL-work share")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": min(args.warmup, 1), "ms_per_step": round(1000 * secs / args.steps, 1),
        "higher_is_better": True, "scaling": "strong" if args.strong else "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": w["desc"],
                   "global_batch": (args.batch or w["batch"]) * (1 if args.strong else max(args.gpus, world))},
        "cpu_baseline": {"value": round(v, 4), "unit": "tokens/s", "cores": workers, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_ours(args, w, bundle, rank, world, local_rank, cpu_baseline):
    import torch
    import torch.distributed as dist
    from llm_accelerator_b200.runner import BatchedRunner

    from llm_accelerator_b200.shard import gather_tokens, shard
    if args.strong:
        B_total = args.batch or w["batch"]
        if B_total % world:
            raise SystemExit(f"batch {B_total} does not split over {world} GPUs")
    else:
        B_total = (args.batch or w["batch"]) * world
    B = B_total // world
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    stream = torch.cuda.current_stream(dev)
    runner = BatchedRunner(bundle, B, device=local_rank)
    seqs = np.asarray(shard(B_total, world, rank))
    K, W = args.steps, args.warmup
    if 1 + W + 2 * K >= w["kv_len"]:
        raise SystemExit("steps + warmup exceed the KV length of the workload")
    # the workload's prompt is consumed first (untimed), as far as the KV
    # window leaves room for the warm-up, timed and e2e steps after it
    P = max(1, min(w["prompt"], w["kv_len"] - 1 - W - 2 * K))
    # per-sequence tokens (seeded by sequence id): the prompt, then the
    # teacher-forced continuation of the warm-up and timed steps
    prompts = np.stack([np.random.default_rng(int(s)).integers(0, VOCAB, P + W + K) for s in seqs])

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # the prompt (prefill + P - 1 decode steps), then W warm-up steps, all teacher-forced
    runner.step("prefill", prompts[:, 0], np.zeros(B, int))
    for pos in range(1, P + W):
        runner.step("decode", prompts[:, pos], np.full(B, pos))
    # value: K teacher-forced steps, parameters staged on the device
    p0 = P + W
    params = np.stack([runner.params("decode", prompts[:, p], np.full(B, p)) for p in range(p0, p0 + K)])
    d_params = torch.from_numpy(params.view(np.int64)).to(dev)
    stride = params.shape[1] * params.shape[2] * 8
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local_rank) as clocks:
        ev0.record(stream)
        for i in range(K):
            runner.step_params_async("decode", d_params.data_ptr() + i * stride, stream.cuda_stream)
        ev1.record(stream)
        barrier()
    runner.engine.check_device()
    ms = ev0.elapsed_time(ev1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = B_total * K / (ms / 1000.0)

    # e2e: K greedy steps through the runner API with host buffers each step
    tok_dev = torch.zeros(B, dtype=torch.int32, device=dev)
    tok_host = torch.zeros(B, dtype=torch.int32).pin_memory()
    tokens = prompts[:, p0 + K - 1].copy()
    runner.argmax_async("decode", tok_dev.data_ptr(), VOCAB, stream.cuda_stream)
    tok_host.copy_(tok_dev)
    tokens = tok_host.numpy().astype(np.int64)
    pos0 = p0 + K
    barrier()
    t0 = time.perf_counter()
    for i in range(K):
        runner.step_async("decode", tokens, np.full(B, pos0 + i), stream.cuda_stream)
        runner.argmax_async("decode", tok_dev.data_ptr(), VOCAB, stream.cuda_stream)
        gather_tokens(tok_dev, world)   # every rank sees the whole batch's tokens (NCCL all-gather)
        tok_host.copy_(tok_dev, non_blocking=True)
        stream.synchronize()
        tokens = tok_host.numpy().astype(np.int64)
    barrier()
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e = B_total * K / float(t.item())
    runner.engine.check_device()

    gemm_line = quarot = ptq = gemv = None
    if rank == 0 and not args.no_gemm:
        gemm_line = int8_gemm_line()
        gemv = gemv_line()
        quarot = quarot_line()
        ptq = ptq_line()
    barrier()

    plan = runner.plans["decode"]
    algo, shared_b, per_seq_b = algorithmic_bytes(plan, B, bundle)
    per_launch_s = ms / 1000.0 / K
    peak, peak_kind = measured_peak()
    achieved = algo / per_launch_s / 1e9
    clk = clocks.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(ms / K, 3), "higher_is_better": True,
            "scaling": "strong" if args.strong else "weak",
            "vs_baseline": None, "dtype": "int8",
            "data": "synthetic: seeded random-init weights in the reference-compiled program",
            "config": {"workload": w["desc"], "global_batch": B_total, "per_gpu_batch": B,
                       "parallelism": f"sequences sharded over {world} GPU(s)",
                       "timed": f"{K} teacher-forced decode steps (positions {p0}..{p0 + K - 1}, after a "
                                f"{P}-token prompt and {W} warm-up steps); e2e: {K} greedy steps "
                                f"(positions {p0 + K}..{p0 + 2 * K - 1})",
                       "l2": f"inputs larger than L2: {shared_b / 1e6:.0f} MB of weights read per step"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic_per_launch(args.workload, B),
                         "peak_kind": peak_kind, "kernel": "tac::exec_kernel",
                         "algorithmic_bytes_per_launch": algo},
            "e2e": {"value": round(e2e, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(B_total * plan.n_var_words * 8),
                    "d2h_bytes_per_step": int(B_total * 4)},
            "gpu_launches": K,
            "clocks": clk,
        }
        if cpu_baseline is not None:
            line["cpu_baseline"] = cpu_baseline
        if gemm_line is not None:
            line["int8_gemm"] = gemm_line
        if quarot is not None:
            line["quarot_w8a16"] = quarot
        if gemv is not None:
            line["decode_gemv"] = gemv
        if ptq is not None:
            line["ptq_quantize"] = ptq
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gpt2-medium", choices=sorted(WORKLOADS))
    ap.add_argument("--batch", type=int, default=0, help="per-GPU batch (global batch with --strong)")
    ap.add_argument("--strong", action="store_true", help="split one global batch over the GPUs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true",
                    help="skip the stand-alone 4096^3 INT8 GEMM and QuaRot layer measurements")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference" and rank != 0:
        return
    w, bundle = load_workload(args.workload)
    if args.impl == "reference":
        run_reference(args, w, bundle, rank, world)
        return
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        workers = min(os.cpu_count() or 1, 16)
        from llm_accelerator_b200.recipe import load_recipe
        sampler = CpuSampler(load_recipe(ROOT / w["recipe"]), workers)
        s = sampler.sample(15.0)
        sampler.close()
        cpu_baseline = {"value": round(s["tokens"] / s["seconds"], 4), "unit": "tokens/s", "cores": workers,
                        "kind": "port",
                        "sample": f"{workers} host processes, one sequence each, first {s['insns']} "
                                  f"instructions of one decode step ({100 * s['frac']:.1f}% of its MATMUL work), "
                                  f"tokens credited by that share"}
    if world > 1:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, w, bundle, rank, world, local_rank, cpu_baseline)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
