"""Test helper: executes a compiled device plan on the CPU with NumPy.

This checks the C++ compiler (renaming, aliasing, gathers, levels, final
materialisation) independently of the CUDA kernels: the plan is run level by
level with the oracle's NumPy arithmetic, and the resulting machine state is
compared with the oracle's.  It is test infrastructure only and is never used
by the engine.
"""
from __future__ import annotations

import numpy as np

from oracle import golden as G

SRAM_UNITS = 8192 + 16384 + 4096
SHARED = 1 << 63
CONST = 1 << 31
SEG_GELU = 1 << 62   # kSegGelu
K = dict(GATHER=1, DYN_LOAD=2, DYN_STORE=3, SREG_LOAD=4, SREG_FINAL=5, MATMUL=6, REQUANT=7, REQUANT_PC=8,
         SCALE_MUL_I32=9, SCALE_MUL_I8=10, VADD_I8=11, VADD_I32=12, DEQUANT_ADD=13, DEQUANT_ACCUM=14,
         DEQUANT_SCALED=15, QUANT=16, VADD_F16=17, LAYERNORM_F16=18, GELU_F16=19, SOFTMAX_F16=20,
         MASKED_SOFTMAX_F16=21, MAX_ABS=22, TRANSPOSE=23, DYN_STORE_MULTI=30, VADD_CHAIN=31)


class PlanMachine:
    """One sequence: shared image + per-sequence block + register file."""

    def __init__(self, dram: bytes, shared_bytes: int, arena_bytes: int, n_slots: int):
        self.shared_bytes = shared_bytes
        self.shared = np.frombuffer(bytes(dram[:shared_bytes]), np.uint8).copy()
        rw = np.frombuffer(bytes(dram[shared_bytes:]), np.uint8)
        self.rw_bytes = len(rw)
        self.block = np.zeros(SRAM_UNITS * 16 + len(rw) + arena_bytes, np.uint8)
        self.block[SRAM_UNITS * 16:SRAM_UNITS * 16 + len(rw)] = rw
        self.sregs = np.zeros(16 + n_slots, np.uint16)

    def load_sram(self, st: G.OracleState):
        self.block[0:131072] = np.frombuffer(bytes(st.abuf), np.uint8)
        self.block[131072:131072 + 262144] = np.frombuffer(bytes(st.wbuf), np.uint8)
        self.block[393216:458752] = st.accum.view(np.uint8)
        self.sregs[:16] = st.scale_regs.view(np.uint16)

    def mem(self, phys: int, nbytes: int) -> np.ndarray:
        if phys & SHARED:
            a = (phys & ~SHARED) * 16
            return self.shared[a:a + nbytes]
        a = phys * 16
        return self.block[a:a + nbytes]

    def dram_mem(self, addr: int, nbytes: int) -> np.ndarray:
        if addr < self.shared_bytes:
            return self.shared[addr:addr + nbytes]
        a = SRAM_UNITS * 16 + addr - self.shared_bytes
        return self.block[a:a + nbytes]

    def sreg(self, enc: int) -> np.float16:
        bits = enc & 0xFFFF if enc & CONST else int(self.sregs[enc])
        return np.array([bits], np.uint16).view(np.float16)[0]

    def dram_image(self) -> bytes:
        return bytes(self.shared) + bytes(self.block[SRAM_UNITS * 16:SRAM_UNITS * 16 + self.rw_bytes])


def _f16(m, p, n):
    return m.mem(p, n * 2).view(np.float16).astype(np.float32)


def _seg_read(m: PlanMachine, op, segs, nbytes: int) -> np.ndarray:
    """Operand a of an F_SEGA op: the runs of its segment list, in order."""
    out = np.zeros(nbytes, np.uint8)
    for sg in segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]:
        dst = int(sg["dst"])
        o, n = (dst & ~SEG_GELU) * 16, int(sg["n"]) * 16
        n = min(n, nbytes - o)   # an op narrowed to its first rows reads the runs below them
        if n > 0:
            v = m.mem(int(sg["src"]), n)
            if dst & SEG_GELU:   # a GELU's input: the value the GELU op stores (FX_GELUSEG MAX_ABS)
                x = v.view(np.float16).astype(np.float32)
                v = G._gelu_tanh(x).astype(np.float32).astype(np.float16).view(np.uint8)
            out[o:o + n] = v
    return out


def _attn_context(op, params):
    """(query_row_base, valid_kv_len) of a masked softmax: from its runtime
    parameter when the context is runtime-configured (flag 4), else the op."""
    if op["flags"] & 4:
        v = int(params[int(op["param"])])
        return v & 0xFFFF, (v >> 16) & 0xFFFF
    return int(op["attn_qrb"]), int(op["attn_vkl"])


def _softmax_rows(src, masked: bool, qrb: int, vkl: int):
    """FP32 rows of SOFTMAX_FP32 / MASKED_SOFTMAX_FP32 (simulator.py:964-1037)."""
    M, N = src.shape
    if not masked:
        e = np.exp((src - src.max(axis=-1, keepdims=True)).astype(np.float32))
        return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)
    out = np.zeros((M, N), np.float32)
    for i2 in range(M):
        last = min(i2 + qrb, vkl - 1)
        row = src[i2].copy()
        if last + 1 < N:
            row[last + 1:] = -np.inf
        e = np.exp((row - float(row.max())).astype(np.float32))
        if last + 1 < N:
            e[last + 1:] = 0.0
        den = float(e.sum())
        out[i2] = e / den if den > 0 else 0.0
    return out


def run_plan(m: PlanMachine, ops, segs, lv, params=None, reverse: bool = False, poison: bool = False):
    """Executes ops in level order, within a level in op order (reverse=True:
    the opposite order; ops of one level must not depend on one another, so
    both orders give the same state).  poison=True (plans compiled without
    arena reuse only) overwrites the rows a narrowed op leaves uncomputed."""
    if reverse:
        idx = np.arange(len(ops))
        order = np.lexsort((-idx, ops["level"]))
    else:
        order = np.argsort(ops["level"], kind="stable")
    for i in order:
        op = ops[i]
        if op["flags2"] & (8 | 64):   # FX_PVY: runs inside its QK^T op's task; FX_CHAINED: after its chain head
            continue
        _run_op(m, op, segs, params)
        if poison:
            _poison_dead_rows(m, op, segs)
        j = i + 1
        while j < len(ops) and ops[j]["flags2"] & 64:   # FX_CHAINED ops follow their head in op order
            _run_op(m, ops[j], segs, params)
            if poison:
                _poison_dead_rows(m, ops[j], segs)
            j += 1
        if op["flags2"] & 4:   # FX_PV: the P.V op right after the softmax rows
            _run_op(m, ops[int(op["seg0"])], segs, params)
            if op["flags2"] & 16:   # FX_SMSKIP: the rows are not stored; nothing else may read them
                m.mem(int(op["nbytes"]), int(op["M"]) * int(op["N"]) * 2)[:] = 0xFF


def _poison_dead_rows(m: PlanMachine, op, segs):
    """A row-wise op narrowed to the rows some later op reads (m_decl set)
    leaves its other rows as they were; they are overwritten with NaN / -127
    bytes here, so a plan that reads them anyway fails its comparison."""
    if int(op["kind"]) == K["MAX_ABS"] and int(op["q_rows"]):
        M, N = int(op["M"]), int(op["N"])
        m.mem(int(op["d"]), M * N)[int(op["q_rows"]) * N:] = 0x81
        return
    md = int(op["m_decl"])
    if not md:
        return
    k, M, N = int(op["kind"]), int(op["M"]), int(op["N"])
    outs = [(int(op["d"]), 1 if k == K["QUANT"] else 2)]
    if k == K["VADD_CHAIN"]:
        chain = segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]
        outs = [(int(sg["dst"]), 2) for sg in chain[1:] if int(sg["dst"])]
    elif k == K["MATMUL"]:
        # the int32 result unless F_NOI32; the FP16 result of FX_DQS, or of
        # F_DQ unless F_NODQ; the F_SM softmax rows unless FX_SMSKIP
        f, f2 = int(op["flags"]), int(op["flags2"])
        outs = ([] if f & 4096 else [(int(op["d"]), 4)]) + \
               ([(int(op["dconst"]), 2)] if (f2 & 1) or ((f & 2048) and not f & 32768) else []) + \
               ([(int(op["nbytes"]), 2)] if (f & 8192) and not f2 & 16 else [])
    for o, es in outs:
        m.mem(o, md * N * es)[M * N * es:] = 0x81 if es == 1 else 0xFF


def _run_op(m: PlanMachine, op, segs, params):
    """Executes one plan op on the machine."""
    k = int(op["kind"])
    M, N, Kd = int(op["M"]), int(op["N"]), int(op["K"])
    a, b, c, d = (int(op[x]) for x in "abcd")
    s = [int(v) for v in op["s"]]
    if k == K["GATHER"]:
        data = []
        for sg in segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]:
            data.append((int(sg["dst"]), m.mem(int(sg["src"]), int(sg["n"]) * 16).copy()))
        for dst, v in data:
            m.mem(dst, len(v))[:] = v
    elif k == K["DYN_STORE_MULTI"]:
        for sg in segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]:
            dstw, n = int(sg["dst"]), int(sg["n"])
            addr = int(params[dstw >> 32]) + (dstw & 0xFFFFFFFF)
            m.dram_mem(addr, n)[:] = m.mem(int(sg["src"]), n)
    elif k == K["VADD_CHAIN"]:
        # running FP16 sum of the segment operands, each add rounded (simulator.py:869-891)
        chain = segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]
        acc = m.mem(int(chain[0]["src"]), M * N * 2).view(np.float16).copy()
        for sg in chain[1:]:
            acc = (acc.astype(np.float32) + _f16(m, int(sg["src"]), M * N)).astype(np.float16)
            if int(sg["dst"]):
                m.mem(int(sg["dst"]), M * N * 2)[:] = acc.view(np.uint8)
    elif k in (K["DYN_LOAD"], K["DYN_STORE"]):
        addr = int(params[int(op["param"])]) + int(op["dconst"])
        n = int(op["nbytes"])
        if k == K["DYN_LOAD"]:
            m.mem(d, n)[:] = m.dram_mem(addr, n)
        else:
            m.dram_mem(addr, n)[:] = m.mem(a, n)
    elif k == K["SREG_LOAD"]:
        m.sregs[int(op["out_slot"])] = m.mem(a, 2).view(np.uint16)[0]
    elif k == K["SREG_FINAL"]:
        vals = [(int(sg["dst"]), m.sreg(int(sg["src"]))) for sg in segs[int(op["seg0"]):int(op["seg0"]) + int(op["nseg"])]]
        for r, v in vals:
            m.sregs[r] = np.array([v], np.float16).view(np.uint16)[0]
    elif k == K["MATMUL"]:
        if op["flags"] & 1024:   # F_QA: a is FP16, quantised like QUANT with register s[0]
            v = np.round(_f16(m, a, M * Kd) * np.float32(m.sreg(s[0])))
            A = np.where(np.isnan(v), np.float32(0), np.clip(v, -128, 127)).astype(np.int8).reshape(M, Kd)
            A = A.astype(np.int32)
        else:
            A = m.mem(a, M * Kd).view(np.int8).reshape(M, Kd).astype(np.int32)
        if op["flags"] & 512:   # F_QB: b is FP16, quantised like QUANT with register s[1]
            v = np.round(_f16(m, b, Kd * N) * np.float32(m.sreg(s[1])))
            raw = np.where(np.isnan(v), np.float32(0), np.clip(v, -128, 127)).astype(np.int8)
        else:
            raw = m.mem(b, Kd * N).view(np.int8)
        if op["flags"] & 128:   # F_BT: b holds B^T [N][K]
            B = raw.reshape(N, Kd).T.astype(np.int32)
        else:
            B = raw.reshape(Kd, N).astype(np.int32)
        acc = m.mem(c, M * N * 4).view(np.int32).reshape(M, N).copy() if op["flags"] & 1 else np.zeros((M, N), np.int32)
        acc += A @ B
        if not op["flags"] & 4096:   # F_NOI32: the int32 result is not stored
            m.mem(d, M * N * 4)[:] = acc.view(np.uint8).ravel()
        if op["flags2"] & 1:   # FX_DQS: DEQUANT_ACCUM_FP32_SCALED's FP16 result as well
            r = (acc.astype(np.float32) * _f16(m, c, N).reshape(1, N) * np.float32(m.sreg(s[0]))
                 + _f16(m, int(op["nbytes"]), N).reshape(1, N))
            out16 = r.astype(np.float32).astype(np.float16).view(np.uint8).ravel()
            m.mem(int(op["dconst"]), M * N * 2)[:] = out16
            if op["flags2"] & 1024:   # FX_DSTORE: the first attn_vkl rows to the runtime address too
                rows = int(op["attn_vkl"])
                addr = int(params[int(op["param"])]) + int(op["attn_qrb"])
                m.dram_mem(addr, rows * N * 2)[:] = out16[:rows * N * 2]
        if op["flags"] & 2048:   # F_DQ: DEQUANT_ACCUM's FP16 result as well
            out = (acc.astype(np.float32) * _f16(m, c, N).reshape(1, N)).astype(np.float16)
            if not op["flags"] & 32768:   # F_NODQ
                m.mem(int(op["dconst"]), M * N * 2)[:] = out.view(np.uint8).ravel()
            if op["flags"] & 8192:   # F_SM: the softmax rows of the dequantised result
                masked = bool(op["flags"] & 16384)
                qrb, vkl = _attn_context(op, params)
                sm = _softmax_rows(out.astype(np.float32), masked, qrb, vkl)
                m.mem(int(op["nbytes"]), M * N * 2)[:] = sm.astype(np.float16).view(np.uint8).ravel()
    elif k in (K["REQUANT"], K["REQUANT_PC"]):
        acc = m.mem(a, M * N * 4).view(np.int32).reshape(M, N).astype(np.float32)
        sc = np.float32(m.sreg(s[0])) if k == K["REQUANT"] else _f16(m, b, N).reshape(1, N)
        m.mem(d, M * N)[:] = G._sat8(acc * sc).view(np.uint8).ravel()
    elif k == K["SCALE_MUL_I32"]:
        v = np.round(m.mem(a, M * N * 4).view(np.int32).astype(np.float32) * np.float32(m.sreg(s[0])))
        with np.errstate(invalid="ignore"):
            r = np.clip(v, np.iinfo(np.int32).min, np.iinfo(np.int32).max).astype(np.int32)
        m.mem(d, M * N * 4)[:] = r.view(np.uint8)
    elif k == K["SCALE_MUL_I8"]:
        v = m.mem(a, M * N).view(np.int8).astype(np.float32) * np.float32(m.sreg(s[0]))
        m.mem(d, M * N)[:] = G._sat8(v).view(np.uint8)
    elif k == K["VADD_I8"]:
        v = m.mem(a, M * N).view(np.int8).astype(np.int16) + m.mem(b, M * N).view(np.int8).astype(np.int16)
        m.mem(d, M * N)[:] = np.clip(v, -128, 127).astype(np.int8).view(np.uint8)
    elif k == K["VADD_I32"]:
        v = m.mem(a, M * N * 4).view(np.int32).reshape(M, N) + m.mem(b, N * 4).view(np.int32).reshape(1, N)
        m.mem(d, M * N * 4)[:] = v.astype(np.int32).view(np.uint8).ravel()
    elif k == K["DEQUANT_ADD"]:
        acc = m.mem(a, M * N * 4).view(np.int32).astype(np.float32)
        skip = m.mem(b, M * N).view(np.int8).astype(np.float32)
        v = acc * np.float32(m.sreg(s[0])) + skip * np.float32(m.sreg(s[1]))
        m.mem(d, M * N)[:] = G._sat8(v).view(np.uint8)
    elif k == K["SOFTMAX_F16"]:
        r = _softmax_rows(_f16(m, a, M * N).reshape(M, N), False, 0, 0)
        m.mem(d, M * N * 2)[:] = r.astype(np.float16).view(np.uint8).ravel()
    elif k == K["QUANT"]:
        xa = _seg_read(m, op, segs, M * N * 2).view(np.float16).astype(np.float32) if op["flags"] & 32 \
            else _f16(m, a, M * N)
        x = xa * np.float32(m.sreg(s[0]))
        v = np.round(x)
        m.mem(d, M * N)[:] = np.where(np.isnan(v), np.float32(0), np.clip(v, -128, 127)).astype(np.int8).view(np.uint8)
    elif k == K["MAX_ABS"]:
        xa = _seg_read(m, op, segs, M * N * 2).view(np.float16).astype(np.float32) if op["flags"] & 32 \
            else _f16(m, a, M * N)
        inv, fwd = G.max_abs_scales(float(np.max(np.abs(xa))))
        m.sregs[int(op["out_slot"])] = np.array([inv], np.float16).view(np.uint16)[0]
        m.sregs[int(op["out_slot"]) + 1] = np.array([fwd], np.float16).view(np.uint16)[0]
        if op["flags2"] & 2:   # FX_MAXQ: QUANT's result with the inverse scale
            v = np.round(xa * np.float32(np.float16(inv)))
            q = np.where(np.isnan(v), np.float32(0), np.clip(v, -128, 127)).astype(np.int8)
            rows = int(op["q_rows"]) or M   # the rows of the result some op reads
            m.mem(d, rows * N)[:] = q.view(np.uint8)[:rows * N]
    elif k in (K["DEQUANT_SCALED"], K["DEQUANT_ACCUM"]):
        acc = m.mem(a, M * N * 4).view(np.int32).reshape(M, N).astype(np.float32)
        if op["flags"] & 16:   # F_SPLIT: second half of the vector at c
            vec = np.concatenate([_f16(m, b, N), _f16(m, c, N)])
        else:
            vec = _f16(m, b, 2 * N if k == K["DEQUANT_SCALED"] else N)
        if k == K["DEQUANT_SCALED"]:
            r = acc * vec[:N].reshape(1, N) * np.float32(m.sreg(s[0])) + vec[N:].reshape(1, N)
        else:
            r = acc * vec[:N].reshape(1, N)
        m.mem(d, M * N * 2)[:] = r.astype(np.float32).astype(np.float16).view(np.uint8).ravel()
    elif k == K["VADD_F16"]:
        xa = _seg_read(m, op, segs, M * N * 2).view(np.float16).astype(np.float32) if op["flags"] & 32 \
            else _f16(m, a, M * N)
        r = xa + _f16(m, b, M * N)
        m.mem(d, M * N * 2)[:] = r.astype(np.float16).view(np.uint8)
    elif k == K["LAYERNORM_F16"]:
        x = _f16(m, a, M * N).reshape(M, N)
        gb = np.concatenate([_f16(m, b, N), _f16(m, c, N)]) if op["flags"] & 16 else _f16(m, b, 2 * N)
        mean = x.mean(axis=-1, keepdims=True).astype(np.float32)
        var = x.var(axis=-1, keepdims=True).astype(np.float32)
        y = (x - mean) / np.sqrt(var + np.float32(1e-5))
        m.mem(d, M * N * 2)[:] = (y * gb[:N] + gb[N:]).astype(np.float32).astype(np.float16).view(np.uint8).ravel()
    elif k == K["GELU_F16"]:
        xa = _seg_read(m, op, segs, M * N * 2).view(np.float16).astype(np.float32) if op["flags"] & 32 \
            else _f16(m, a, M * N)
        m.mem(d, M * N * 2)[:] = G._gelu_tanh(xa).astype(np.float32).astype(np.float16).view(np.uint8)
    elif k == K["MASKED_SOFTMAX_F16"]:
        qrb, vkl = _attn_context(op, params)
        out = _softmax_rows(_f16(m, a, M * N).reshape(M, N), True, qrb, vkl)
        m.mem(d, M * N * 2)[:] = out.astype(np.float16).view(np.uint8).ravel()
    elif k == K["TRANSPOSE"]:
        src = m.mem(a, M * N).view(np.int8).reshape(M, N)
        m.mem(d, M * N)[:] = np.ascontiguousarray(src.T).view(np.uint8).ravel()
    else:
        raise NotImplementedError(f"plan executor: op kind {k}")


def final_state(m: PlanMachine):
    return dict(abuf=bytes(m.block[0:131072]), wbuf=bytes(m.block[131072:393216]),
                accum=bytes(m.block[393216:458752]), sregs=bytes(m.sregs[:16].tobytes()), dram=m.dram_image())
