"""GPU parity of the QuaRot W8A16 layer against the oracle (bit-exact).

The rotation is float32 butterflies in the oracle's order with one FP16
rounding, the quantiser and the dequant epilogue are the reference's W8A16
arithmetic, so the CUDA results equal the oracle bit for bit."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from llm_accelerator_b200 import _lib as L
from oracle import quarot as Q

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,K,block", [(1024, 768, 256), (16, 2048, 32), (16, 2048, 64), (9, 2048, 128),
                                       (16, 2048, 512), (3, 2048, 1024)])
def test_fwht_bit_exact(M, K, block):
    import torch
    from llm_accelerator_b200.quarot import fwht_f16
    x, _, _, _ = Q.layer_inputs(M, K, 16, seed=block)
    got = fwht_f16(torch.from_numpy(x).cuda(), block).cpu().numpy()
    np.testing.assert_array_equal(got.view(np.uint16), Q.fwht_blocks(x, block).view(np.uint16))


def _fwht_grid(M, K, block, sms=148):
    """CTAs of the rotation launch (8 warps each, at most 8 per SM)."""
    return min(-(-M * (K // block) // 8), sms * 8)


@pytest.mark.parametrize("with_bias", [True, False])
def test_quarot_layer_bit_exact_at_workload_size(with_bias):
    """1024 x 768 activations (8 x 128 tokens, 1% outlier channels x50), 768 x 3072 weights:
    the two-launch path (rotation with per-CTA maxima, then the GEMM that
    quantises the rotated rows while staging them)."""
    import torch
    from llm_accelerator_b200.quarot import quarot_w8a16, workspace
    x, w, s, b = Q.layer_inputs(1024, 768, 3072, seed=0)
    bias = b if with_bias else None
    dX, dW, dS = (torch.from_numpy(a).cuda() for a in (x, w, s))
    dB = torch.from_numpy(b).cuda() if with_bias else None
    ws = workspace(1024, 768)
    want = Q.quarot_w8a16_layer(x, w, s, bias, block=256)
    for _ in range(2):   # the workspace is reused by the second call
        y = quarot_w8a16(dX, dW, dS, dB, block=256, ws=ws).cpu().numpy()
        np.testing.assert_array_equal(y.view(np.uint16), want.view(np.uint16))
    # intermediates: the rotated rows and the rotation CTAs' maxima of |x|
    base = (ws.data_ptr() + 255) & ~255
    host = ws.cpu().numpy()[base - ws.data_ptr():]
    mk = 1024 * 768
    xr = host[:mk * 2].view(np.float16).reshape(1024, 768)
    xr_want = Q.fwht_blocks(x, 256)
    np.testing.assert_array_equal(xr.view(np.uint16), xr_want.view(np.uint16))
    off = (mk * 2 + 255) // 256 * 256
    slots = host[off:off + 4 * _fwht_grid(1024, 768, 256)].view(np.float32)
    assert np.isfinite(slots).all()
    assert slots.max() == np.abs(xr_want.astype(np.float32)).max()
    assert L.lib.tac_gemm_status(None) == L.OK


@pytest.mark.parametrize("M,K,N,block", [(200, 512, 400, 128), (130, 1024, 16, 256), (17, 128, 272, 32)])
def test_quarot_two_launch_path_ragged_shapes(M, K, N, block):
    """Rows not a multiple of 128, a partial last column tile, K from one
    128-byte block to the 1024-byte limit: bit-exact against the oracle."""
    import torch
    from llm_accelerator_b200.quarot import quarot_w8a16
    x, w, s, b = Q.layer_inputs(M, K, N, seed=M + N)
    y = quarot_w8a16(*(torch.from_numpy(a).cuda() for a in (x, w, s, b)), block=block).cpu().numpy()
    np.testing.assert_array_equal(y.view(np.uint16), Q.quarot_w8a16_layer(x, w, s, b, block=block).view(np.uint16))
    assert L.lib.tac_gemm_status(None) == L.OK


def test_quarot_four_launch_path_above_the_shared_memory_limit():
    """K = 2048 does not fit the staged A tile: rotation, activation
    quantisation and the tcgen05 GEMM with the dequant epilogue run as
    separate launches; intermediates as the oracle computes them."""
    import torch
    from llm_accelerator_b200.quarot import quarot_w8a16, workspace
    M, K, N = 256, 2048, 1024
    x, w, s, b = Q.layer_inputs(M, K, N, seed=3)
    ws = workspace(M, K)
    y = quarot_w8a16(*(torch.from_numpy(a).cuda() for a in (x, w, s, b)), block=256, ws=ws).cpu().numpy()
    np.testing.assert_array_equal(y.view(np.uint16), Q.quarot_w8a16_layer(x, w, s, b, block=256).view(np.uint16))
    base = (ws.data_ptr() + 255) & ~255
    host = ws.cpu().numpy()[base - ws.data_ptr():]
    mk = M * K
    xr_want = Q.fwht_blocks(x, 256)
    _, inv, fwd = Q.act_scales(xr_want)
    off = (mk * 2 + 255) // 256 * 256
    np.testing.assert_array_equal(host[off:off + mk].view(np.int8).reshape(M, K), Q.quantize_act(xr_want, inv))
    stat = host[off + (max(mk, 8192) + 255) // 256 * 256:][:8].view(np.uint32)
    assert np.uint16(stat[1] & 0xFFFF) == np.float16(fwd).view(np.uint16)


def test_quarot_layer_unaligned_shape_takes_the_portable_gemm():
    """N not a multiple of 16: the INT8 GEMM runs on the mma.sync kernel."""
    import torch
    from llm_accelerator_b200.quarot import quarot_w8a16
    x, w, s, b = Q.layer_inputs(40, 512, 200, seed=5)
    y = quarot_w8a16(*(torch.from_numpy(a).cuda() for a in (x, w, s, b)), block=128).cpu().numpy()
    np.testing.assert_array_equal(y.view(np.uint16), Q.quarot_w8a16_layer(x, w, s, b, block=128).view(np.uint16))


@pytest.mark.parametrize("M,N,with_bias", [(1, 3072, True), (9, 200, False), (16, 768, True)])
def test_quarot_layer_decode_rows_take_the_cluster_gemv(M, N, with_bias):
    """M <= 16 rows: the dequant GEMM runs on the cluster split-K GEMV."""
    import torch
    from llm_accelerator_b200.quarot import quarot_w8a16
    x, w, s, b = Q.layer_inputs(M, 768, N, seed=M)
    bias = b if with_bias else None
    args = [torch.from_numpy(a).cuda() for a in (x, w, s)] + [torch.from_numpy(b).cuda() if with_bias else None]
    y = quarot_w8a16(*args, block=256).cpu().numpy()
    np.testing.assert_array_equal(y.view(np.uint16), Q.quarot_w8a16_layer(x, w, s, bias, block=256).view(np.uint16))


def test_quarot_rejects_bad_arguments_without_launching():
    p = C.c_void_p(256)
    assert L.lib.tac_fwht_f16(p, p, 4, 768, 48, None) == L.E_ARGUMENT        # block not a power of two
    assert L.lib.tac_fwht_f16(p, p, 4, 700, 256, None) == L.E_ARGUMENT       # block does not divide K
    need = int(L.lib.tac_quarot_workspace_bytes(64, 768))
    assert L.lib.tac_quarot_w8a16(p, p, p, None, p, p, need - 1, 64, 256, 768, 256, None) == L.E_ARGUMENT
