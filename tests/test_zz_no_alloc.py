"""The allocation-free decode GEMV (tac_gemv_i8_requant_pc_static), called
through the C ABI, against the existing MATMUL + REQUANT_PC entry point.

Kept in its own file, collected last, so it runs both alone and after every
other GPU test in the same process."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from llm_accelerator_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _operands(M, N, K, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    B = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
    rng = np.random.default_rng(seed)
    scale = torch.from_numpy((rng.random(N) * 2e-4 + 1e-6).astype(np.float16)).cuda()
    return A, B, scale


@pytest.mark.parametrize("M,N,K", [(1, 3072, 768), (16, 4096, 1024), (5, 200, 1000), (16, 64, 4096),
                                   (1, 50272, 1024)])
def test_static_gemv_matches_gemm_entry_point_twice(M, N, K):
    import torch
    A, B, scale = _operands(M, N, K, M * 131 + N + K)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        got = torch.full((M, N), 99, dtype=torch.int8, device="cuda")
        want = torch.full((M, N), -99, dtype=torch.int8, device="cuda")
        st = L.lib.tac_gemv_i8_requant_pc_static(A.data_ptr(), B.data_ptr(), scale.data_ptr(), got.data_ptr(),
                                                 M, N, K, stream)
        assert st == L.OK, f"call {call}: status {st}"
        st = L.lib.tac_gemm_i8_requant_pc(A.data_ptr(), B.data_ptr(), scale.data_ptr(), want.data_ptr(),
                                          M, N, K, stream)
        assert st == L.OK
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call}: {(got != want).sum().item()} entries differ"
    assert L.lib.tac_gemm_status(None) == L.OK


def test_static_gemv_rejects_sizes_beyond_its_workspace():
    null = C.c_void_p(16)   # never dereferenced: the size checks come first
    assert L.lib.tac_gemv_i8_requant_pc_static(null, null, null, null, 17, 64, 64, None) == L.E_ARGUMENT
    assert L.lib.tac_gemv_i8_requant_pc_static(null, null, null, null, 16, 131072 + 16, 64, None) == L.E_ARGUMENT
    assert L.lib.tac_gemv_i8_requant_pc_static(null, null, null, null, 0, 64, 64, None) == L.E_ARGUMENT
