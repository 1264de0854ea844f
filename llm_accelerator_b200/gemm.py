"""Stand-alone INT8 GEMM kernels on torch tensors (device memory plumbing).

``gemm_i8_i32``            C = A @ B (int32), the MATMUL instruction at any size
``gemm_i8_requant_pc``     int8 = clip(rint(f32(A @ B) * f32(scale[n]))), MATMUL + REQUANT_PC
                           (``golden_model/systolic.py:31-71``, ``golden_model/simulator.py:661-688``)
``gemm_i8_requant_shift``  int8 = clip((acc * mult[n] + 2^(shift[n]-1)) >> shift[n]) (int64),
                           an integer-multiplier epilogue with no reference counterpart
"""
from __future__ import annotations

from . import _lib as L


def _ptr(t):
    return t.data_ptr()


def _check(A, B):
    import torch
    if A.dtype != torch.int8 or B.dtype != torch.int8 or not A.is_cuda or not B.is_cuda:
        raise TypeError("A and B must be int8 CUDA tensors")
    if A.dim() != 2 or B.dim() != 2 or A.shape[1] != B.shape[0]:
        raise ValueError(f"shape mismatch {tuple(A.shape)} @ {tuple(B.shape)}")
    if not (A.is_contiguous() and B.is_contiguous()):
        raise ValueError("A and B must be contiguous (row-major)")
    return A.shape[0], B.shape[1], A.shape[1]


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def gemm_i8_i32(A, B, out=None):
    import torch
    M, N, K = _check(A, B)
    out = torch.empty((M, N), dtype=torch.int32, device=A.device) if out is None else out
    L.check(L.lib.tac_gemm_i8_i32(_ptr(A), _ptr(B), _ptr(out), M, N, K, _stream()), "tac_gemm_i8_i32")
    return out


def gemm_i8_requant_pc(A, B, scale_f16, out=None):
    import torch
    M, N, K = _check(A, B)
    if scale_f16.dtype != torch.float16 or scale_f16.numel() != N:
        raise ValueError("scale_f16 must be float16 with N elements")
    out = torch.empty((M, N), dtype=torch.int8, device=A.device) if out is None else out
    L.check(L.lib.tac_gemm_i8_requant_pc(_ptr(A), _ptr(B), _ptr(scale_f16.contiguous()), _ptr(out), M, N, K,
                                         _stream()), "tac_gemm_i8_requant_pc")
    return out


def _check_bt(A, Bt):
    import torch
    if A.dtype != torch.int8 or Bt.dtype != torch.int8 or not A.is_cuda or not Bt.is_cuda:
        raise TypeError("A and Bt must be int8 CUDA tensors")
    if A.dim() != 2 or Bt.dim() != 2 or A.shape[1] != Bt.shape[1]:
        raise ValueError(f"shape mismatch {tuple(A.shape)} @ {tuple(Bt.shape)}^T")
    if not (A.is_contiguous() and Bt.is_contiguous()):
        raise ValueError("A and Bt must be contiguous (row-major)")
    return A.shape[0], Bt.shape[0], A.shape[1]


def gemm_i8_i32_bt(A, Bt, out=None):
    """A @ Bt^T, int32; Bt is B transposed ([N, K] row-major)."""
    import torch
    M, N, K = _check_bt(A, Bt)
    out = torch.empty((M, N), dtype=torch.int32, device=A.device) if out is None else out
    L.check(L.lib.tac_gemm_i8_i32_bt(_ptr(A), _ptr(Bt), _ptr(out), M, N, K, _stream()), "tac_gemm_i8_i32_bt")
    return out


def gemm_i8_requant_pc_bt(A, Bt, scale_f16, out=None):
    """REQUANT_PC(A @ Bt^T); Bt is B transposed ([N, K] row-major)."""
    import torch
    M, N, K = _check_bt(A, Bt)
    if scale_f16.dtype != torch.float16 or scale_f16.numel() != N:
        raise ValueError("scale_f16 must be float16 with N elements")
    out = torch.empty((M, N), dtype=torch.int8, device=A.device) if out is None else out
    L.check(L.lib.tac_gemm_i8_requant_pc_bt(_ptr(A), _ptr(Bt), _ptr(scale_f16.contiguous()), _ptr(out), M, N, K,
                                            _stream()), "tac_gemm_i8_requant_pc_bt")
    return out


def gemm_i8_requant_shift(A, B, mult, shift, out=None):
    import torch
    M, N, K = _check(A, B)
    if mult.dtype != torch.int32 or shift.dtype != torch.int32 or mult.numel() != N or shift.numel() != N:
        raise ValueError("mult and shift must be int32 with N elements")
    out = torch.empty((M, N), dtype=torch.int8, device=A.device) if out is None else out
    L.check(L.lib.tac_gemm_i8_requant_shift(_ptr(A), _ptr(B), _ptr(mult.contiguous()), _ptr(shift.contiguous()),
                                            _ptr(out), M, N, K, _stream()), "tac_gemm_i8_requant_shift")
    return out


def gemm_wo_f16_i8(X, Q, scale, bias=None, out=None):
    """Y float32 [M, N] = X (float16 [M, K]) @ (Q int8 [K, N] * scale[N]) (+ bias[N]):
    the weight-only INT8 GEMM (tac_gemm_wo_f16_i8)."""
    import torch
    if X.dtype != torch.float16 or Q.dtype != torch.int8 or scale.dtype != torch.float32:
        raise TypeError("X float16, Q int8, scale float32 expected")
    M, K = X.shape
    if Q.shape[0] != K or scale.numel() != Q.shape[1]:
        raise ValueError(f"shape mismatch {tuple(X.shape)} x {tuple(Q.shape)}")
    N = Q.shape[1]
    out = torch.empty((M, N), dtype=torch.float32, device=X.device) if out is None else out
    L.check(L.lib.tac_gemm_wo_f16_i8(_ptr(X), _ptr(Q), _ptr(scale), None if bias is None else _ptr(bias), _ptr(out),
                                     M, N, K, _stream()), "tac_gemm_wo_f16_i8")
    return out


def time_gemm_wo(M: int = 1024, N: int = 3072, K: int = 768, iters: int = 20, warmup: int = 5, seed: int = 0,
                 rotate_bytes: int = 256 << 20) -> dict:
    """Device time of the weight-only GEMM: ms in steady state (calls back to
    back in a CUDA graph, each on its own input set of sets totalling
    rotate_bytes, so inputs come from HBM), ms_cold for one call after a
    256 MB write has flushed L2; algorithmic bytes X, Q, scales, bias, Y."""
    import numpy as np
    import torch
    from .quarot import _graph_time
    g = torch.Generator(device="cuda").manual_seed(seed)
    nbytes = M * K * 2 + K * N + 8 * N + M * N * 4
    n_sets = max(2, -(-rotate_bytes // nbytes))
    sets = [(torch.randn((M, K), generator=g, device="cuda").half(),
             torch.randint(-127, 128, (K, N), dtype=torch.int8, device="cuda", generator=g),
             torch.rand(N, generator=g, device="cuda") * 1e-3 + 1e-4,
             torch.randn(N, generator=g, device="cuda") * 0.02,
             torch.empty((M, N), dtype=torch.float32, device="cuda")) for _ in range(n_sets)]

    def call(i):
        X, Q, S, Bv, Y = sets[i]
        gemm_wo_f16_i8(X, Q, S, Bv, out=Y)

    ms = _graph_time(call, n_sets, 10 * n_sets)
    flush = torch.empty(256 << 20, dtype=torch.int8, device="cuda")
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        call(0)
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        call(0)
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return {"shape": [M, K, N], "ms": ms, "ms_cold": float(np.median(ts)), "tflops": 2.0 * M * N * K / ms / 1e9,
            "gbs": nbytes / ms / 1e6, "bytes": nbytes, "input_sets": n_sets}


def time_gemm(M: int, N: int, K: int, *, epilogue: str = "requant_pc", iters: int = 20, warmup: int = 5,
              seed: int = 0, compare_cublas: bool = True, b_transposed: bool = False) -> dict:
    """Device time of one stand-alone GEMM (median over `iters` launches, CUDA
    events on the launching stream, L2 flushed between launches by writing a
    256 MB buffer) and, for comparison, torch._int_mm (cuBLASLt INT8) on the
    same operands.  b_transposed: time the K-major-B entry points (B stored
    as [N, K])."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
    scale = torch.full((N,), 1e-3, dtype=torch.float16, device="cuda")
    Bt = B.t().contiguous() if b_transposed else None
    if b_transposed:
        out = torch.empty((M, N), dtype=torch.int32 if epilogue == "i32" else torch.int8, device="cuda")
        fn = ((lambda: gemm_i8_i32_bt(A, Bt, out)) if epilogue == "i32"  # noqa: E731
              else (lambda: gemm_i8_requant_pc_bt(A, Bt, scale, out)))
    elif epilogue == "i32":
        out = torch.empty((M, N), dtype=torch.int32, device="cuda")
        fn = lambda: gemm_i8_i32(A, B, out)  # noqa: E731
    else:
        out = torch.empty((M, N), dtype=torch.int8, device="cuda")
        fn = lambda: gemm_i8_requant_pc(A, B, scale, out)  # noqa: E731
    flush = torch.empty(256 << 20, dtype=torch.int8, device="cuda")
    stream = torch.cuda.current_stream()

    def med(f):
        for _ in range(warmup):
            f()
        torch.cuda.synchronize()
        ts = []
        for _ in range(iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            f()
            e1.record(stream)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    ms_cold = med(fn)
    st = L.lib.tac_gemm_status(None)
    if st != L.OK:
        raise RuntimeError(f"GEMM kernel reported device fault status {st}")
    ops = 2.0 * M * N * K
    # steady state: calls back to back in a CUDA graph, each on its own operand
    # set (A, B, out) of sets totalling 256 MB, so operands come from HBM
    from .quarot import _graph_time
    per_set = M * K + K * N + M * N * (4 if epilogue == "i32" else 1)
    n_sets = max(2, -(-(256 << 20) // per_set))
    sets = [(torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g),
             torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g),
             torch.empty_like(out)) for _ in range(n_sets)]
    if b_transposed:
        sets = [(a, b.t().contiguous(), o) for a, b, o in sets]
        one = ((lambda i: gemm_i8_i32_bt(sets[i][0], sets[i][1], sets[i][2])) if epilogue == "i32"  # noqa: E731
               else (lambda i: gemm_i8_requant_pc_bt(sets[i][0], sets[i][1], scale, sets[i][2])))
    elif epilogue == "i32":
        one = lambda i: gemm_i8_i32(sets[i][0], sets[i][1], sets[i][2])  # noqa: E731
    else:
        one = lambda i: gemm_i8_requant_pc(sets[i][0], sets[i][1], scale, sets[i][2])  # noqa: E731
    ms = _graph_time(one, n_sets, 10 * n_sets)
    res = {"shape": [M, N, K], "epilogue": epilogue, "b_layout": "[N,K]" if b_transposed else "[K,N]", "ms": ms,
           "ms_cold": ms_cold, "tops": ops / ms / 1e9, "operand_sets": n_sets}
    if compare_cublas and M > 16:
        Bc = B.t().contiguous().t()   # column-major operand for cuBLASLt
        cms_cold = med(lambda: torch._int_mm(A, Bc))
        csets = [(a, b.t().contiguous().t()) for a, b, _ in sets] if not b_transposed else \
            [(a, b.t()) for a, b, _ in sets]
        cms = _graph_time(lambda i: torch._int_mm(csets[i][0], csets[i][1]), n_sets, 10 * n_sets)
        res.update({"cublas_int_mm_ms": cms, "cublas_int_mm_ms_cold": cms_cold, "cublas_tops": ops / cms / 1e9})
    if L.lib.tac_gemm_status(None) != L.OK:
        raise RuntimeError("GEMM kernel reported a device fault")
    return res


if __name__ == "__main__":
    import argparse
    import json
    ap = argparse.ArgumentParser(description="time the stand-alone INT8 GEMM")
    ap.add_argument("M", type=int)
    ap.add_argument("N", type=int)
    ap.add_argument("K", type=int)
    ap.add_argument("--epilogue", default="requant_pc", choices=["requant_pc", "i32"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--bt", action="store_true", help="B stored transposed ([N, K], K-major)")
    a = ap.parse_args()
    print(json.dumps(time_gemm(a.M, a.N, a.K, epilogue=a.epilogue, iters=a.iters, warmup=a.warmup,
                               compare_cublas=not a.no_cublas, b_transposed=a.bt)))


def time_gemv(M: int = 1, N: int = 3072, K: int = 768, *, calls: int = 400, warmup: int = 20,
              rotate_bytes: int = 256 << 20, seed: int = 0) -> dict:
    """Decode GEMV (MATMUL + REQUANT_PC with M <= 16 rows): average device time
    per call over `calls` back-to-back calls whose weight operands cycle
    through distinct buffers totalling `rotate_bytes` (so every call reads its
    weights from HBM, not L2).  The calls are captured once in a CUDA graph
    and the graph replay is timed with CUDA events, so host issue time (a
    ctypes call costs more than the kernel) stays out of the figure.  Times
    the general entry point (the cluster split-K GEMV for these shapes) and
    the split-K kernel of tac_gemv_i8_requant_pc_static.  Algorithmic bytes
    per call: K*N weights + M*K activations + 2*N scale bytes + M*N output."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    nbuf = max(2, -(-rotate_bytes // (K * N)))
    Bs = [torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g) for _ in range(nbuf)]
    A = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    scale = torch.full((N,), 1e-3, dtype=torch.float16, device="cuda")
    out = torch.empty((M, N), dtype=torch.int8, device="cuda")
    stream = torch.cuda.current_stream()
    hbm = K * N + M * K + 2 * N + M * N
    res = {"shape": [M, N, K], "weight_buffers": nbuf, "bytes": hbm}

    def loop(fn):
        for i in range(warmup):   # first calls do the per-device set-up, outside the capture
            fn(Bs[i % nbuf])
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(calls):
                fn(Bs[i % nbuf])
        graph.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / calls)
        del graph
        return sorted(times)[1]

    def general(B):
        L.check(L.lib.tac_gemm_i8_requant_pc(_ptr(A), _ptr(B), _ptr(scale), _ptr(out), M, N, K, _stream()),
                "tac_gemm_i8_requant_pc")

    def splitk(B):
        L.check(L.lib.tac_gemv_i8_requant_pc_static(_ptr(A), _ptr(B), _ptr(scale), _ptr(out), M, N, K, _stream()),
                "tac_gemv_i8_requant_pc_static")

    for name, fn in (("general", general), ("splitk_static", splitk)):
        ms = loop(fn)
        res[name] = {"us": ms * 1e3, "gbs": hbm / ms / 1e6}
    if L.lib.tac_gemm_status(None) != L.OK:
        raise RuntimeError("GEMM kernel reported a device fault")
    return res
