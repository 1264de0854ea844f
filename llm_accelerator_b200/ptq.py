"""Offline post-training quantisation steps on the GPU (torch tensors as
device-memory plumbing).

``quantize_linear_weight(W)``  tac_quantize_weight_i8: the per-channel INT8
                               quantisation of a PyTorch-layout [out, in]
                               float32 weight, padded and transposed to the
                               program image's [K, N] layout
                               (software/taccel/runtime/tiny_fixture.py:149-159)
``quantize_tensor(W)``         the same quantiser in quantize_tensor's
                               [out, in] layout (software/taccel/quantizer/quantize.py:6-33)
``rotate_residual_stream_state_dict(sd, model_args, R)``
                               QuaRot's offline weight rotation
                               (software/taccel/quantizer/rotation.py:158-321):
                               float32 matrix products with TF32 disabled,
                               plain cuBLAS GEMMs; the result matches NumPy's
                               float32 products to rounding, not bit for bit.
"""
from __future__ import annotations

from . import _lib as L


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def quantize_linear_weight(W, per_channel: bool = True):
    """(q_kn int8 [K_pad, N_pad], scales float16 [N_pad]) on W's device; W is
    a float32 CUDA tensor [out, in] (1-D means one channel)."""
    import torch
    if not W.is_cuda or W.dtype != torch.float32:
        raise TypeError("W must be a float32 CUDA tensor")
    if W.dim() == 1:
        W = W.reshape(1, -1)
    if W.dim() != 2:
        raise ValueError(f"W must be 1-D or 2-D, got shape {tuple(W.shape)}")
    W = W.contiguous()
    n, k = W.shape
    np_, kp = -(-n // 16) * 16, -(-k // 16) * 16
    q = torch.empty((kp, np_), dtype=torch.int8, device=W.device)
    s16 = torch.empty(np_, dtype=torch.float16, device=W.device)
    s32 = torch.empty(n, dtype=torch.float32, device=W.device)
    L.check(L.lib.tac_quantize_weight_i8(W.data_ptr(), n, k, int(bool(per_channel)), q.data_ptr(), s16.data_ptr(),
                                         s32.data_ptr(), _stream()), "tac_quantize_weight_i8")
    return q, s16


def quantize_tensor(W, per_channel: bool = True):
    """(q int8 [out, in], scales float16 [out]): quantize_tensor's result,
    read out of the [K_pad, N_pad] image."""
    n, k = (1, W.numel()) if W.dim() == 1 else W.shape
    q, s = quantize_linear_weight(W, per_channel)
    return q[:k, :n].t().contiguous(), s[:n].contiguous()


def rotate_residual_stream_state_dict(state_dict: dict, model_args: dict, R) -> list:
    """Rotates, in place, every weight and bias that touches the residual
    stream by the [d_model, d_model] orthogonal R, as
    rotation.py:158-321 does: embeddings, per-head c_attn and mlp.c_fc input
    columns and lm_head by W @ R^T; attn.c_proj and mlp.c_proj output rows and
    biases by R @ W.  Values may be torch tensors or NumPy arrays; products run
    in float32 on the current CUDA device and each value keeps its own dtype
    and device.  Returns the keys changed, in order."""
    import numpy as np
    import torch
    dev = torch.device("cuda", torch.cuda.current_device())
    Rt = torch.as_tensor(np.asarray(R, dtype=np.float32) if not torch.is_tensor(R) else R).to(dev, torch.float32)
    if Rt.dim() != 2 or Rt.shape[0] != Rt.shape[1]:
        raise ValueError(f"R must be square, got shape {tuple(Rt.shape)}")
    d = int(model_args["n_embd"])
    if Rt.shape[0] != d:
        raise ValueError(f"R shape {tuple(Rt.shape)} does not match n_embd={d}")
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    changed = []

    def apply(key, fn):
        if key not in state_dict:
            return
        old = state_dict[key]
        x = (old if torch.is_tensor(old) else torch.from_numpy(np.asarray(old))).to(dev, torch.float32)
        y = fn(x)
        if torch.is_tensor(old):
            state_dict[key] = y.to(old.device, old.dtype)
        else:
            state_dict[key] = y.cpu().numpy().astype(np.asarray(old).dtype, copy=False)
        changed.append(key)

    right = lambda w: w @ Rt.t()   # noqa: E731  input columns
    left = lambda w: Rt @ w        # noqa: E731  output rows / biases
    try:
        for key in ("transformer.wte.weight", "transformer.wpe.weight"):
            apply(key, right)
        for layer in range(int(model_args["n_layer"])):
            h = 0
            while f"transformer.h.{layer}.attn.c_attn.weight_h{h}_query" in state_dict:
                for kind in ("query", "key", "value"):
                    apply(f"transformer.h.{layer}.attn.c_attn.weight_h{h}_{kind}", right)
                h += 1
            apply(f"transformer.h.{layer}.mlp.c_fc.weight", right)
            for part in ("attn", "mlp"):
                apply(f"transformer.h.{layer}.{part}.c_proj.weight", left)
                apply(f"transformer.h.{layer}.{part}.c_proj.bias", left)
        apply("lm_head.weight", right)
        torch.cuda.current_stream().synchronize()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return changed


def time_quantizer(out_ch: int = 50257, in_features: int = 768, iters: int = 20, warmup: int = 5,
                   seed: int = 0) -> dict:
    """Device time of one tac_quantize_weight_i8 call (median, CUDA events on
    the launching stream, L2 flushed before each call by writing 256 MB) on a
    seeded N(0, 0.02) float32 weight; default shape: GPT-2's lm_head.
    Algorithmic bytes: W read once, the INT8 image and FP16 scales written."""
    import numpy as np
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = torch.randn((out_ch, in_features), generator=g, device="cuda", dtype=torch.float32) * 0.02
    flush = torch.empty(256 << 20, dtype=torch.int8, device="cuda")
    stream = torch.cuda.current_stream()
    for _ in range(warmup):
        quantize_linear_weight(W)
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        quantize_linear_weight(W)
        e1.record(stream)
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    ms = float(np.median(ts))
    np_, kp = -(-out_ch // 16) * 16, -(-in_features // 16) * 16
    hbm = 4 * out_ch * in_features + kp * np_ + 2 * np_
    return {"shape": [out_ch, in_features], "ms": ms, "gbs": hbm / ms / 1e6, "bytes": hbm}
