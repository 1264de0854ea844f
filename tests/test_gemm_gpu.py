"""GPU parity of the stand-alone INT8 GEMM kernels (MATMUL sweep shapes).

Integer results are bit-exact.  Shapes the oracle computes in seconds are
checked in full against NumPy int64 matmul; at 4096^3 a sample of output
entries is recomputed exactly on the CPU (each entry is one int64 dot product).
"""
from __future__ import annotations

import numpy as np
import pytest

from llm_accelerator_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _requant_pc_ref(acc, scale):
    v = np.round(acc.astype(np.float32) * scale.astype(np.float32).reshape(1, -1))
    return np.where(np.isnan(v), 0, np.clip(v, -128, 127)).astype(np.int8)


def _requant_shift_ref(acc, mult, shift):
    v = acc.astype(np.int64) * mult.astype(np.int64).reshape(1, -1)
    sh = shift.astype(np.int64).reshape(1, -1)
    v = (v + (np.int64(1) << (sh - 1))) >> sh
    return np.clip(v, -128, 127).astype(np.int8)


# K and N multiples of 16 run on the tcgen05 kernel, the rest on the mma.sync
# tile.  Covered: partial 128-row / 128- and 256-column tiles, K not a multiple
# of the 128-byte K block, a single K block, the decode GEMV (M=1), and a
# 256-column-tile case with ragged M, N and K (1936 x 2064 x 784), and
# last partial waves run as half-width units (160 tiles on 148 SMs): whole,
# ragged in M, N and K, and with a half unit entirely past column N.  M <= 16
# with K and N multiples of 4 runs on the cluster split-K GEMV (clusters of
# 1 to 16 CTAs, odd sizes 7, 10 and 12 included; ragged column blocks).
SHAPES = [(64, 64, 64), (64, 768, 768), (768, 64, 3072), (1, 3072, 768), (16, 48, 64), (100, 200, 48),
          (768, 768, 768), (256, 4096, 512), (4096, 64, 768), (130, 272, 144), (1, 16, 16), (300, 208, 4096),
          (1936, 2064, 784), (3072, 3072, 64), (2560, 2048, 256), (2500, 2000, 400), (2560, 1920, 128),
          (5, 3072, 768), (16, 768, 3072), (7, 1000, 100), (3, 52, 36), (16, 50272, 1024), (2, 4, 4),
          (16, 256, 8192), (1, 256, 320), (4, 512, 224), (1, 768, 768)]


def _exact_matmul(A, B):
    # float64 BLAS is exact here: |A @ B| <= K * 2^14 < 2^53
    return (A.astype(np.float64) @ B.astype(np.float64)).astype(np.int64)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_exact(M, N, K):
    import torch
    from llm_accelerator_b200 import gemm
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    ref = _exact_matmul(A, B)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    got = gemm.gemm_i8_i32(dA, dB).cpu().numpy()
    np.testing.assert_array_equal(got, ref.astype(np.int32))
    scale = (rng.random(N).astype(np.float32) * 1e-4 + 1e-6).astype(np.float16)
    q = gemm.gemm_i8_requant_pc(dA, dB, torch.from_numpy(scale).cuda()).cpu().numpy()
    np.testing.assert_array_equal(q, _requant_pc_ref(ref.astype(np.int32), scale))
    mult = rng.integers(1, 1 << 12, N, dtype=np.int32)
    shift = rng.integers(8, 16, N, dtype=np.int32)
    q2 = gemm.gemm_i8_requant_shift(dA, dB, torch.from_numpy(mult).cuda(), torch.from_numpy(shift).cuda()).cpu().numpy()
    np.testing.assert_array_equal(q2, _requant_shift_ref(ref, mult, shift))
    assert L.lib.tac_gemm_status(None) == L.OK


def test_gemm_4096_cubed_sampled():
    import torch
    from llm_accelerator_b200 import gemm
    M = N = K = 4096
    g = torch.Generator(device="cuda").manual_seed(1)
    dA = torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda", generator=g)
    dB = torch.randint(-128, 128, (K, N), dtype=torch.int8, device="cuda", generator=g)
    C = gemm.gemm_i8_i32(dA, dB)
    A, B, Cn = dA.cpu().numpy().astype(np.int64), dB.cpu().numpy().astype(np.int64), C.cpu().numpy()
    rng = np.random.default_rng(0)
    rows, cols = rng.integers(0, M, 256), rng.integers(0, N, 256)
    for i, j in zip(rows, cols):
        assert Cn[i, j] == int(A[i] @ B[:, j])
    # full rows / columns too (catches tile-edge indexing)
    for i in (0, M - 1, 1234):
        np.testing.assert_array_equal(Cn[i], (A[i] @ B).astype(np.int32))
    # checksum of checksums: (1^T A) B == 1^T C
    np.testing.assert_array_equal(Cn.astype(np.int64).sum(axis=0), A.sum(axis=0) @ B)
    # fused requant epilogue at full size: equal to requantising the int32 result
    scale = torch.full((N,), 1.0 / 4096, dtype=torch.float16, device="cuda")
    scale[::7] = 3e-4
    q = gemm.gemm_i8_requant_pc(dA, dB, scale).cpu().numpy()
    np.testing.assert_array_equal(q, _requant_pc_ref(Cn, scale.cpu().numpy()))
    assert L.lib.tac_gemm_status(None) == L.OK



# B supplied transposed ([N, K], K-major): single-SM and CTA-pair kernels,
# whole and half-width tail units, ragged M, N and K.
BT_SHAPES = [(64, 768, 768), (130, 272, 144), (1936, 2064, 784), (2560, 2048, 256), (2500, 2000, 400),
             (2560, 1920, 128), (3072, 3072, 64)]


@pytest.mark.parametrize("M,N,K", BT_SHAPES)
def test_gemm_bt_exact(M, N, K):
    import torch
    from llm_accelerator_b200 import gemm
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int8)
    B = rng.integers(-128, 128, (K, N), dtype=np.int8)
    scale = (rng.random(N) * 2e-4 + 1e-5).astype(np.float16)
    acc = _exact_matmul(A, B)
    Ad, Btd = torch.from_numpy(A).cuda(), torch.from_numpy(np.ascontiguousarray(B.T)).cuda()
    got32 = gemm.gemm_i8_i32_bt(Ad, Btd).cpu().numpy()
    np.testing.assert_array_equal(got32, acc.astype(np.int32))
    got8 = gemm.gemm_i8_requant_pc_bt(Ad, Btd, torch.from_numpy(scale).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got8, _requant_pc_ref(acc, scale))
    assert L.lib.tac_gemm_status(None) == L.OK


def test_gemm_bt_rejects_non_tcgen05_shapes():
    import torch
    from llm_accelerator_b200 import gemm
    A = torch.zeros((8, 24), dtype=torch.int8, device="cuda")
    Bt = torch.zeros((40, 24), dtype=torch.int8, device="cuda")   # K = 24: not a multiple of 16
    with pytest.raises(Exception):
        gemm.gemm_i8_i32_bt(A, Bt)


@pytest.mark.parametrize("bt", [False, True])
def test_gemm_cta_pair_kernel_exact(bt, monkeypatch):
    """The opt-in CTA-pair (cta_group::2) kernel: 256 x 256 tiles, ragged M, N, K."""
    import torch
    from llm_accelerator_b200 import gemm
    monkeypatch.setenv("TAC_GEMM_2SM", "1")
    for M, N, K in [(2560, 2048, 256), (2500, 2000, 400), (2560, 1920, 128), (3072, 3072, 64)]:
        rng = np.random.default_rng(M + N + K + int(bt))
        A = rng.integers(-128, 128, (M, K), dtype=np.int8)
        B = rng.integers(-128, 128, (K, N), dtype=np.int8)
        scale = (rng.random(N) * 2e-4 + 1e-5).astype(np.float16)
        acc = _exact_matmul(A, B)
        Ad, sd = torch.from_numpy(A).cuda(), torch.from_numpy(scale).cuda()
        if bt:
            Btd = torch.from_numpy(np.ascontiguousarray(B.T)).cuda()
            got32, got8 = gemm.gemm_i8_i32_bt(Ad, Btd), gemm.gemm_i8_requant_pc_bt(Ad, Btd, sd)
        else:
            Bd = torch.from_numpy(B).cuda()
            got32, got8 = gemm.gemm_i8_i32(Ad, Bd), gemm.gemm_i8_requant_pc(Ad, Bd, sd)
        np.testing.assert_array_equal(got32.cpu().numpy(), acc.astype(np.int32))
        np.testing.assert_array_equal(got8.cpu().numpy(), _requant_pc_ref(acc, scale))
    assert L.lib.tac_gemm_status(None) == L.OK
