"""Deterministic single-instruction cases shared by the fixture generator and
the tests.

Each case is rebuilt from its seed: random SRAM contents (FP16 activations or
int8 in ABUF, int8 weights and FP16 vectors in WBUF, int32 partial sums in
ACCUM), random scale registers, a tile configuration, an attention context
and one instruction word (or a short program).  The golden record stores only
what the reference changed, plus SHA-256 digests of the full post-state.
"""
from __future__ import annotations

import hashlib

import numpy as np

SEED = 20261201
ABUF, WBUF, ACCUM = 131072, 262144, 65536

R_OPS = {  # opcode: (src1 buffers, src2 buffers, dst buffers) on the op's normal path
    0x0A: ((0, 1), (1,), (2, 0)),    # MATMUL
    0x0B: ((2,), (0,), (0, 1)),      # REQUANT
    0x11: ((2,), (0, 1), (0,)),      # REQUANT_PC
    0x0C: ((2, 0), (0,), (0, 2)),    # SCALE_MUL
    0x0D: ((0, 2), (0, 2), (0, 2)),  # VADD
    0x13: ((2,), (0,), (0,)),        # DEQUANT_ADD
    0x17: ((2,), (1, 0), (0,)),      # DEQUANT_ACCUM_FP32
    0x18: ((0,), (0,), (0,)),        # QUANT_FP32_INT8
    0x19: ((0,), (0,), (0,)),        # VADD_FP32
    0x1A: ((0,), (1,), (0,)),        # LAYERNORM_FP32
    0x1B: ((0,), (0,), (0,)),        # GELU_FP32
    0x1C: ((0,), (0,), (0,)),        # SOFTMAX_FP32
    0x1D: ((0,), (0,), (0,)),        # MASKED_SOFTMAX_FP32
    0x1E: ((2,), (1,), (0,)),        # DEQUANT_ACCUM_FP32_SCALED
    0x1F: ((0,), (0,), (0,)),        # MAX_ABS_REDUCE_FP32
    0x0F: ((0,), (1,), (0,)),        # LAYERNORM (legacy INT8)
    0x0E: ((0, 2), (0,), (0,)),      # SOFTMAX (legacy)
    0x10: ((0, 2), (0,), (0,)),      # GELU (legacy)
    0x15: ((0, 2), (0,), (0,)),      # MASKED_SOFTMAX (legacy)
    0x12: ((2,), (1,), (0,)),        # SOFTMAX_ATTNV (legacy)
    0x16: ((2,), (1,), (0,)),        # MASKED_SOFTMAX_ATTNV (legacy)
}
FP16_INPUT_OPS = {0x17, 0x18, 0x19, 0x1A, 0x1B, 0x1C, 0x1D, 0x1E, 0x1F}
# ops whose results depend on exp / tanh / x**3 or a float32 matmul (tolerance, not bit-exact)
TRANSCENDENTAL_OPS = {0x1B, 0x1C, 0x1D, 0x0E, 0x10, 0x15, 0x12, 0x16}
N_PER_OP = 6
N_PROGRAMS = 10


def r_word(op, s1b, s1o, s2b, s2o, db, do, sreg, flags):
    return (op << 59) | (s1b << 57) | (s1o << 41) | (s2b << 39) | (s2o << 23) | (db << 21) | (do << 5) | (sreg << 1) | flags


def _fp16(rng, n, scale):
    return (rng.standard_normal(n).astype(np.float32) * np.float32(scale)).astype(np.float16)


def fill_state(rng, int8_abuf: bool):
    """(abuf, wbuf, accum, sregs) as uint8/uint8/uint8/uint16 arrays."""
    if int8_abuf:
        abuf = rng.integers(-128, 128, ABUF, dtype=np.int8).view(np.uint8)
    else:
        abuf = _fp16(rng, ABUF // 2, float(rng.choice([0.05, 1.0, 8.0]))).view(np.uint8)
    w8 = rng.integers(-128, 128, WBUF // 2, dtype=np.int8).view(np.uint8)
    w16 = (np.abs(_fp16(rng, WBUF // 4, 0.01)) + np.float16(1e-3)).astype(np.float16).view(np.uint8)
    wbuf = np.concatenate([w8, w16])
    accum = rng.integers(-60000, 60000, ACCUM // 4, dtype=np.int32).view(np.uint8)
    sregs = (np.abs(_fp16(rng, 16, 0.05)) + np.float16(0.01)).astype(np.float16).view(np.uint16)
    return abuf.copy(), wbuf.copy(), accum.copy(), sregs.copy()


def case_list():
    """All cases: dicts with kind ('insn' or 'program'), words, tile, attn, seed."""
    rng = np.random.default_rng(SEED)
    out = []
    for op, (b1s, b2s, dbs) in R_OPS.items():
        for k in range(N_PER_OP):
            m = int(rng.integers(0, 2))
            n = int(rng.integers(0, 4))
            kk = int(rng.integers(0, 4))
            if op in (0x1A, 0x1C, 0x1D, 0x0E, 0x15, 0x0F):
                n = int(rng.choice([0, 2, 3, 47]))       # rows of 16, 48, 64, 768
            attn = (0, 0, 0, 0)
            if op in (0x1D, 0x15, 0x16):
                keys = (kk if op == 0x16 else n) * 16 + 16
                attn = (1, int(rng.integers(0, 20)), int(rng.integers(1, keys + 1)), int(rng.choice([1, 3])))
            b1, b2, db = int(rng.choice(b1s)), int(rng.choice(b2s)), int(rng.choice(dbs))
            o1, o2, od = int(rng.integers(0, 64)), int(rng.integers(0, 64)), int(rng.integers(64, 128))
            if b2 == 1 and op in (0x17, 0x1E, 0x1A, 0x0F, 0x11):
                o2 = 8192 + int(rng.integers(0, 64))      # FP16 vectors: upper half of WBUF
            if b1 == 2:
                o1 = int(rng.integers(0, 16))
            if db == 2:
                od = int(rng.integers(1024, 2048))
            sreg = int(rng.integers(0, 12))
            flags = int(rng.integers(0, 2)) if op == 0x0A else 1
            out.append(dict(kind="insn", words=[r_word(op, b1, o1, b2, o2, db, od, sreg, flags)],
                            tile=(m, n, kk), attn=attn, seed=int(rng.integers(0, 2**31)),
                            int8_abuf=op not in FP16_INPUT_OPS, op=op))
    for k in range(N_PROGRAMS):
        base = int(rng.integers(0, 4096)) * 16
        n = int(rng.integers(1, 64))
        words = [
            (0x05 << 59) | (1 << 57) | (base << 29),
            (0x06 << 59) | (1 << 57),
            (0x07 << 59) | (int(rng.integers(0, 4000)) << 41) | (n << 25) | (1 << 23) | (int(rng.integers(0, 512)) << 7),
            (0x08 << 59) | (1 << 57) | (int(rng.integers(0, 4000)) << 41) | (n << 25) | (1 << 23) | (int(rng.integers(512, 1024)) << 7),
            (0x09 << 59) | (int(rng.integers(0, 64)) << 41) | (1 << 39) | (int(rng.integers(0, 64)) << 23) | (48 << 7) | (3 << 1) | 1,
            (0x09 << 59) | (1 << 57) | (int(rng.integers(0, 64)) << 41) | (int(rng.integers(4096, 5000)) << 23) | (n << 7),
            (0x04 << 59) | (3 << 55) | (2 << 53) | (int(rng.integers(0, 100)) << 37),
            (0x04 << 59) | (4 << 55) | (0x3C00 << 37),
            0x01 << 59,
        ]
        out.append(dict(kind="program", words=words, tile=None, attn=(0, 0, 0, 0),
                        seed=int(rng.integers(0, 2**31)), int8_abuf=True, op=-1))
    faults = [
        r_word(0x0A, 2, 0, 1, 0, 2, 0, 0, 0),     # MATMUL int8 read from ACCUM -> ValueError
        r_word(0x11, 0, 0, 0, 0, 0, 0, 0, 0),     # REQUANT_PC src1 not ACCUM -> IllegalBufferError
        r_word(0x1F, 0, 0, 0, 0, 0, 0, 15, 0),    # MAX_ABS sreg 15 -> ConfigError
        r_word(0x1F, 0, 8190, 0, 0, 0, 0, 0, 0),  # tile past ABUF end -> SRAMAccessError
        r_word(0x1D, 0, 0, 0, 0, 0, 0, 0, 0),     # masked softmax without CONFIG_ATTN -> ConfigError
        r_word(0x13, 2, 0, 0, 0, 0, 0, 15, 0),    # DEQUANT_ADD sreg 15 -> ConfigError
        r_word(0x19, 2, 0, 0, 0, 0, 0, 0, 0),     # VADD_FP32 ACCUM source -> IllegalBufferError
    ]
    for w in faults:
        out.append(dict(kind="insn", words=[w], tile=(0, 3, 3), attn=(0, 0, 0, 0),
                        seed=int(rng.integers(0, 2**31)), int8_abuf=False, op=w >> 59))
    return out


def pre_state(case):
    rng = np.random.default_rng(case["seed"])
    abuf, wbuf, accum, sregs = fill_state(rng, case["int8_abuf"])
    dram = rng.integers(0, 256, 1 << 20, dtype=np.uint8) if case["kind"] == "program" else None
    return abuf, wbuf, accum, sregs, dram


def sha(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def diff_ranges(pre: np.ndarray, post: np.ndarray):
    """[(offset, bytes)] for the changed spans (merged within 64 bytes)."""
    idx = np.flatnonzero(pre != post)
    if idx.size == 0:
        return []
    spans, s, e = [], int(idx[0]), int(idx[0])
    for i in idx[1:]:
        i = int(i)
        if i - e > 64:
            spans.append((s, e + 1))
            s = i
        e = i
    spans.append((s, e + 1))
    return [(a, bytes(post[a:b])) for a, b in spans]
