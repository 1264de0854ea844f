"""The allocation-free decode GEMV (tac_gemv_i8_requant_pc_static), called
through the C ABI.

Some callers of this library cannot allocate device memory at the point where
they run a decode MATMUL: a decode loop that must not stall on cudaMalloc /
cudaFree (both may synchronise the device), or a service that holds a fixed
device-memory budget.  This entry point keeps its split-K partial sums in a
static device workspace instead.  Each case is checked, on two calls in a
row (the workspace keeps the last call's contents), against the MATMUL +
REQUANT_PC formula in NumPy (int64-exact products, then
clip(rint(f32(acc) * f32(scale)))) and against the existing
tac_gemm_i8_requant_pc entry point.

Kept in its own file, collected last, so it runs both alone and after every
other GPU test in the same process."""
from __future__ import annotations

import ctypes as C
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

from llm_accelerator_b200 import _lib as L

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _operands(M, N, K, seed):
    rng = np.random.default_rng(seed)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    scale = (rng.random(N) * 2e-4 + 1e-6).astype(np.float16)
    return A, B, scale


def _requant_pc_formula(A, B, scale):
    """MATMUL (systolic.py:31-71) + REQUANT_PC (simulator.py:661-688) in NumPy.
    The products are exact in float64 (|sum| < 2**53) and wrapped to int32."""
    acc = (A.astype(np.float64) @ B.astype(np.float64)).astype(np.int64)
    acc = ((acc + (1 << 31)) % (1 << 32) - (1 << 31)).astype(np.int32)
    v = acc.astype(np.float32) * scale.astype(np.float32)[None, :]
    return np.clip(np.round(v), -128, 127).astype(np.int8)


# (16, 65536, 2048): the largest N (1024 column blocks, one K split) with a
# 4 MiB partial-sum slice.  (With M <= 16 the split count from the SM count,
# ceil(2 * SMs * 64 / N), stays below the 8 MiB workspace's bound
# 2 MiB / (M * N) for every N, so that bound never binds.)
@pytest.mark.parametrize("M,N,K", [(1, 3072, 768), (16, 4096, 1024), (5, 200, 1000), (16, 64, 4096),
                                   (1, 50272, 1024), (16, 65536, 2048)])
def test_static_gemv_matches_formula_and_gemm_entry_point_twice(M, N, K):
    import torch
    A, B, scale = _operands(M, N, K, M * 131 + N + K)
    want = _requant_pc_formula(A, B, scale)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    dS = torch.from_numpy(scale.view(np.int16)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        got = torch.full((M, N), 99 + call, dtype=torch.int8, device="cuda")
        gemm = torch.full((M, N), -99, dtype=torch.int8, device="cuda")
        st = L.lib.tac_gemv_i8_requant_pc_static(dA.data_ptr(), dB.data_ptr(), dS.data_ptr(), got.data_ptr(),
                                                 M, N, K, stream)
        assert st == L.OK, f"call {call}: status {st}"
        st = L.lib.tac_gemm_i8_requant_pc(dA.data_ptr(), dB.data_ptr(), dS.data_ptr(), gemm.data_ptr(),
                                          M, N, K, stream)
        assert st == L.OK
        torch.cuda.synchronize()
        g = got.cpu().numpy()
        bad = np.argwhere(g != want)
        assert bad.size == 0, f"call {call}: {len(bad)} entries differ from the formula, first {bad[:3].tolist()}"
        assert np.array_equal(gemm.cpu().numpy(), g), f"call {call}: differs from tac_gemm_i8_requant_pc"
    assert L.lib.tac_gemm_status(None) == L.OK


def test_static_gemv_rejects_sizes_beyond_its_workspace():
    null = C.c_void_p(16)   # never dereferenced: the size checks come first
    assert L.lib.tac_gemv_i8_requant_pc_static(null, null, null, null, 17, 64, 64, None) == L.E_ARGUMENT
    assert L.lib.tac_gemv_i8_requant_pc_static(null, null, null, null, 16, 131072, 64, None) == L.E_ARGUMENT
    assert L.lib.tac_gemv_i8_requant_pc_static(null, null, null, null, 16, 65536 + 16, 64, None) == L.E_ARGUMENT
    assert L.lib.tac_gemv_i8_requant_pc_static(null, null, null, null, 0, 64, 64, None) == L.E_ARGUMENT


def test_static_gemv_first_call_during_capture_is_refused():
    """In a fresh process, a first call made while its stream captures a graph
    returns TAC_E_UNSUPPORTED without launching; after the capture the same
    call sets up and runs."""
    code = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(ROOT)!r})
        import numpy as np, torch
        from llm_accelerator_b200 import _lib as L
        M, N, K = 1, 256, 256
        A = torch.ones((M, K), dtype=torch.int8, device="cuda")
        B = torch.ones((K, N), dtype=torch.int8, device="cuda")
        S = torch.from_numpy(np.full(N, 0.25, np.float16).view(np.int16)).cuda()
        out = torch.zeros((M, N), dtype=torch.int8, device="cuda")
        args = (A.data_ptr(), B.data_ptr(), S.data_ptr(), out.data_ptr(), M, N, K)
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            g.capture_begin()
            st = L.lib.tac_gemv_i8_requant_pc_static(*args, s.cuda_stream)
            g.capture_end()
        assert st == L.E_UNSUPPORTED, st
        del g
        st = L.lib.tac_gemv_i8_requant_pc_static(*args, torch.cuda.current_stream().cuda_stream)
        assert st == L.OK, st
        torch.cuda.synchronize()
        assert int(out.min()) == int(out.max()) == 64    # rint(256 * 0.25)
        print("ok")
    """)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
