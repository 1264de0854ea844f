"""QuaRot W8A16 layer on torch tensors (device memory plumbing).

``fwht_f16(X, block)``                rows of X rotated by I (x) H_block / sqrt(block)
``quarot_w8a16(X, W, scale, bias)``   the W8A16 dynamic matmul
                                      (software/taccel/runtime/w8a16_simulator_reference.py:96-135)
                                      of the rotated rows, FP16 out
"""
from __future__ import annotations

from . import _lib as L


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def fwht_f16(X, block: int = 256, out=None):
    import torch
    if X.dtype != torch.float16 or not X.is_cuda or X.dim() != 2 or not X.is_contiguous():
        raise TypeError("X must be a contiguous 2-D float16 CUDA tensor")
    out = torch.empty_like(X) if out is None else out
    L.check(L.lib.tac_fwht_f16(X.data_ptr(), out.data_ptr(), X.shape[0], X.shape[1], block, _stream()),
            "tac_fwht_f16")
    return out


def workspace(M: int, K: int, device="cuda"):
    """A workspace tensor for quarot_w8a16 (reuse it across calls on one stream)."""
    import torch
    n = int(L.lib.tac_quarot_workspace_bytes(M, K))
    return torch.empty(n + 256, dtype=torch.uint8, device=device)


def _aligned_ptr(ws):
    p = ws.data_ptr()
    return (p + 255) & ~255, ws.numel() - ((-p) & 255)


def quarot_w8a16(X, W, scale, bias=None, block: int = 256, out=None, ws=None):
    import torch
    if X.dtype != torch.float16 or W.dtype != torch.int8 or scale.dtype != torch.float16:
        raise TypeError("X float16, W int8, scale float16 expected")
    M, K = X.shape
    if W.shape[0] != K or scale.numel() != W.shape[1]:
        raise ValueError(f"shape mismatch {tuple(X.shape)} x {tuple(W.shape)}")
    N = W.shape[1]
    out = torch.empty((M, N), dtype=torch.float16, device=X.device) if out is None else out
    ws = workspace(M, K, X.device) if ws is None else ws
    wp, wn = _aligned_ptr(ws)
    bp = 0 if bias is None else bias.data_ptr()
    L.check(L.lib.tac_quarot_w8a16(X.data_ptr(), W.data_ptr(), scale.data_ptr(), bp or None, out.data_ptr(), wp, wn,
                                   M, N, K, block, _stream()), "tac_quarot_w8a16")
    return out


def _graph_time(call, n_sets: int, calls: int, warmup: int = 4) -> float:
    """Average ms per call of `calls` back-to-back calls captured in one CUDA
    graph, call i on input set i % n_sets; the replay is timed with CUDA
    events (median of 3), so host issue time stays out of the figure."""
    import torch
    for i in range(warmup):       # per-device set-up happens outside the capture
        call(i % n_sets)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(calls):
            call(i % n_sets)
    graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
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


def time_layer(M: int = 1024, K: int = 768, N: int = 3072, block: int = 256, iters: int = 20, warmup: int = 5,
               seed: int = 0, rotate_bytes: int = 256 << 20) -> dict:
    """Device time of one layer call on seeded inputs of the layer workload's
    distribution (N(0, 1) activations with 1% of channels x50, per-channel
    INT8 weights):
      ms       steady state: calls back to back in a CUDA graph, each on its own
               input set (X, W, scales, bias, Y) of sets totalling rotate_bytes,
               so every call reads its inputs from HBM (average per call);
      ms_cold  one call after a 256 MB write has flushed L2 (median of `iters`)."""
    import numpy as np
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    per_set = M * K * 2 + K * N + 4 * N + M * N * 2
    n_sets = max(2, -(-rotate_bytes // per_set))
    sets = []
    for _ in range(n_sets):
        X = torch.randn((M, K), generator=g, device="cuda", dtype=torch.float32)
        ch = torch.randperm(K, generator=g, device="cuda")[:max(1, K // 100)]
        X[:, ch] *= 50.0
        W = torch.randint(-127, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
        S = (torch.rand(N, generator=g, device="cuda") * 1e-3 + 1e-4).half()
        Bv = (torch.randn(N, generator=g, device="cuda") * 0.02).half()
        sets.append((X.half(), W, S, Bv, torch.empty((M, N), dtype=torch.float16, device="cuda")))
    ws = workspace(M, K)

    def call(i):
        X, W, S, Bv, Y = sets[i]
        quarot_w8a16(X, W, S, Bv, block, out=Y, ws=ws)

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
    ms_cold = float(np.median(ts))
    flops = 2.0 * M * N * K
    # algorithmic bytes: X in, W + scales + bias in, Y out (the rotated rows
    # pass through the workspace, and L2, between the two launches)
    hbm = per_set
    return {"shape": [M, K, N], "block": block, "ms": ms, "ms_cold": ms_cold, "tflops": flops / ms / 1e9,
            "gbs": hbm / ms / 1e6, "bytes": hbm, "input_sets": n_sets}
