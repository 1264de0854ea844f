"""Device-side profile of compiled decode steps (per level and per task).

    python -m llm_accelerator_b200.profile [--recipe tests/golden/recipe_gpt2_medium.npz]
                                           [--batch 64] [--steps 3] [--position 130] [--mhz 1965]
                                           [--levels LO:HI]

Runs a prefill and teacher-forced decode steps of a GPT-2 recipe through
BatchedRunner up to --position (the bench's timed steps follow a 128-token
prompt), then profiles --steps decode steps with the engine's profiling
mode 2: the device time at the end of every plan level (globaltimer) and the
SM cycles of every task.  Prints, per op kind and shape, the task count, the
median and 90th-percentile task time, and the task time summed over all
halves divided by the number of halves; then the step's level time, the sum
over levels of the busiest half's task time, and the rest (the grid-barrier
floor).  While profiling, the executor adds one clock read and one store per
task and nothing else.
"""
from __future__ import annotations

import argparse
import collections
from pathlib import Path

import numpy as np

KIND_NAMES = {1: "GATHER", 2: "DYN_LOAD", 3: "DYN_STORE", 4: "SREG_LOAD", 5: "SREG_FINAL", 6: "MATMUL",
              7: "REQUANT", 8: "REQUANT_PC", 9: "SCALE_MUL_I32", 10: "SCALE_MUL_I8", 11: "VADD_I8",
              12: "VADD_I32", 13: "DEQUANT_ADD", 14: "DEQUANT", 15: "DEQ_SCALED", 16: "QUANT", 17: "VADD_F16",
              18: "LN", 19: "GELU", 20: "SOFTMAX", 21: "MSOFTMAX", 22: "MAX_ABS", 23: "TRANSPOSE",
              24: "LN_I8", 25: "SOFTMAX_I8", 26: "MSOFTMAX_I8", 27: "GELU_I8", 28: "SOFTMAX_ATTNV",
              29: "MSOFTMAX_ATTNV", 30: "DYN_STORE_MULTI", 31: "VADD_CHAIN"}
SHARED = 1 << 63


def op_label(op) -> str:
    """Kind and shape of a plan op, with the fusions a MATMUL carries."""
    k = KIND_NAMES.get(int(op["kind"]), str(int(op["kind"])))
    f = int(op["flags"])
    if k == "MATMUL":
        tags = [t for bit, t in ((8, "tc"), (512, "qB"), (1024, "qA"), (128, "Bt"), (2048, "dq"), (8192, "softmax"))
                if f & bit]
        if int(op["flags2"]) & 1:
            tags.append("dqs")
        if int(op["flags2"]) & 4:
            tags.append("pv")
        k += (f"[{op['M']}x{op['K']}x{op['N']}{'s' if int(op['b']) & SHARED else 'p'}]" +
              ("+" + "+".join(tags) if tags else ""))
    elif int(op["flags2"]) & 128:
        k += f"[{op['M']}x{op['N']}]+chain"
    elif k not in ("GATHER", "DYN_STORE", "DYN_LOAD", "DYN_STORE_MULTI", "TRANSPOSE", "SREG_LOAD", "SREG_FINAL"):
        k += f"[{op['M']}x{op['N']}]" + ("seg" if f & 32 else "") + ("+quant" if int(op["flags2"]) & 2 else "")
        if k.startswith("VADD_CHAIN"):
            k += f"x{int(op['nseg'])}"
    if int(op["flags2"]) & (2048 | 4096):   # a head group / MAX_ABS pair: one task runs several ops
        k += "+group"
    return k


def profile_decode(recipe: str, batch: int, steps: int = 3, device: int = 0, position: int = 130):
    """(level_ns, task_cycles, ops, tasks, level_offsets, halves) of the decode
    plan, medians over `steps` profiled decode steps at positions
    position .. position + steps - 1 (earlier positions run unprofiled)."""
    from .recipe import load_recipe
    from .runner import BatchedRunner
    b = load_recipe(recipe)
    br = BatchedRunner(b, batch, device=device)
    toks = np.arange(batch) % 50257
    br.step("prefill", toks, np.zeros(batch, int))
    position = max(1, position)
    for pos in range(1, position):
        br.step("decode", toks, np.full(batch, pos))
    br.engine.set_profiling(True, tasks=True)
    durs, cycs = [], []
    for i in range(steps):
        br.step("decode", toks, np.full(batch, position + i))
        durs.append(np.diff(br.engine.read_profile().astype(np.int64)))
        cycs.append(br.engine.read_task_profile().astype(np.int64))
    br.engine.set_profiling(False)
    ops, _, tasks, lv = br.plans["decode"].dump()
    halves = 2 * br.engine.grid()
    return (np.median(np.stack(durs), axis=0), np.median(np.stack(cycs), axis=0), ops, tasks, lv, halves)


def summarize(level_ns, task_cycles, ops, tasks, lv, halves: int, mhz: float, top: int = 25) -> str:
    per = collections.defaultdict(list)
    for i, t in enumerate(tasks[:int(lv[-1])]):   # chain templates (after the last level) are not tasks
        per[op_label(ops[int(t["op"])])].append(task_cycles[i])
    lines = [f"{'op: kind[M x K x N] or [M x N], fusions':56s} {'tasks':>7s} {'median':>9s} {'p90':>9s} "
             f"{'sum/halves':>11s}"]
    for k, v in sorted(per.items(), key=lambda kv: -sum(kv[1]))[:top]:
        v = np.asarray(v, float) / mhz
        lines.append(f"{k:56s} {len(v):7d} {np.median(v):7.2f}us {np.percentile(v, 90):7.2f}us "
                     f"{v.sum() / halves:9.1f}us")
    busy = 0.0
    for L in range(len(level_ns)):
        c = task_cycles[lv[L]:lv[L + 1]]
        h = np.zeros(halves)
        np.add.at(h, np.arange(len(c)) % halves, c)
        busy += h.max() / mhz
    total = float(np.sum(level_ns)) / 1e3
    lines.append(f"levels {len(level_ns)}, tasks {len(tasks)}, level time {total:.0f} us, busiest-half task time "
                 f"{busy:.0f} us, barrier floor {total - busy:.0f} us (task times at {mhz:.0f} MHz)")
    return "\n".join(lines)


def level_table(level_ns, task_cycles, ops, tasks, lv, halves: int, mhz: float, lo: int, hi: int) -> str:
    """Levels lo..hi-1 one per line: the level's time (globaltimer), its task
    count, its busiest half's task time and its ops' labels."""
    lines = [f"{'level':>5s} {'time':>9s} {'tasks':>6s} {'busiest':>9s}  ops"]
    for L in range(max(0, lo), min(hi, len(level_ns))):
        c = task_cycles[lv[L]:lv[L + 1]]
        h = np.zeros(halves)
        np.add.at(h, np.arange(len(c)) % halves, c)
        labels = collections.Counter(op_label(ops[int(t["op"])]) for t in tasks[lv[L]:lv[L + 1]])
        lines.append(f"{L:5d} {level_ns[L] / 1e3:7.2f}us {len(c):6d} {h.max() / mhz:7.2f}us  "
                     + ", ".join(f"{k} x{n}" for k, n in labels.items()))
    return "\n".join(lines)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    root = Path(__file__).resolve().parent.parent
    ap.add_argument("--recipe", default=str(root / "tests" / "golden" / "recipe_gpt2_medium.npz"))
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--position", type=int, default=130, help="KV position of the first profiled step")
    ap.add_argument("--mhz", type=float, default=1965.0, help="SM clock that converts task cycles to time")
    ap.add_argument("--top", type=int, default=25)
    ap.add_argument("--levels", default="", help="LO:HI: also list levels LO..HI-1 one per line")
    a = ap.parse_args(argv)
    prof = profile_decode(a.recipe, a.batch, a.steps, position=a.position)
    print(summarize(*prof, mhz=a.mhz, top=a.top))
    if a.levels:
        lo, hi = (int(v) for v in a.levels.split(":"))
        print(level_table(*prof, mhz=a.mhz, lo=lo, hi=hi))


if __name__ == "__main__":
    main()
