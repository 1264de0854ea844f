"""Oracle for offline weight quantisation: TEST INFRASTRUCTURE ONLY.

A NumPy restatement of
  quantize_tensor          software/taccel/quantizer/quantize.py:6-33
  _quantize_linear_weight  software/taccel/runtime/tiny_fixture.py:149-159
used to check tac_quantize_weight_i8.  It is pinned to the reference
functions by tests/golden/ptq_cases.npz (written by
tests/golden/make_ptq.py from the reference itself) and, when the reference
checkout is present, by calling them directly.
"""
from __future__ import annotations

import numpy as np


def quantize_tensor(tensor: np.ndarray, per_channel: bool = True):
    """(q int8 [out, in], scales FP16 [out]); float32 arithmetic throughout
    (quantize.py:19-33: max|row| floored at 1e-8, / 127, IEEE float32
    division, round half to even, clip to [-128, 127])."""
    t = np.asarray(tensor, dtype=np.float32)
    if t.ndim == 1:
        t = t.reshape(1, -1)
    m = np.max(np.abs(t), axis=1)
    if per_channel:
        s = np.maximum(m, np.float32(1e-8)) / np.float32(127.0)
    else:
        s = np.full(t.shape[0], np.maximum(np.max(m), np.float32(1e-8)) / np.float32(127.0), dtype=np.float32)
    q = np.clip(np.round(t / s.reshape(-1, 1)), -128, 127).astype(np.int8)
    return q, s.astype(np.float16)


def quantize_linear_weight(tensor: np.ndarray, per_channel: bool = True):
    """(q_kn int8 [K_pad, N_pad], scales FP16 [N_pad]): the per-channel
    quantisation of a PyTorch-layout [out, in] weight, zero-padded to
    multiples of 16 and transposed; padding channels repeat the last scale
    (tiny_fixture.py:151-159)."""
    q, s = quantize_tensor(tensor, per_channel)
    n, k = q.shape
    q = np.pad(q, ((0, (-n) % 16), (0, (-k) % 16)))
    if len(s) < q.shape[0]:
        s = np.pad(s, (0, q.shape[0] - len(s)), constant_values=s[-1])
    return np.ascontiguousarray(q.T), s.astype(np.float16)


def weight_case(out_ch: int, in_f: int, seed: int, std: float = 0.02, zero_rows=(), outlier=0.0):
    """Seeded float32 weight [out_ch, in_f] ~ N(0, std), optional all-zero
    rows and one outlier column scaled by `outlier`."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((out_ch, in_f)) * std).astype(np.float32)
    for r in zero_rows:
        w[r] = 0.0
    if outlier:
        w[:, rng.integers(0, in_f)] *= np.float32(outlier)
    return w


def rotation_case(d: int = 64, n_layer: int = 2, n_head: int = 2, vocab: int = 96, seed: int = 11):
    """A seeded float32 state dict with every key the QuaRot residual-stream
    rotation touches (per-head c_attn split as rotation.py:248-259 expects),
    and its model_args."""
    rng = np.random.default_rng(seed)
    g = lambda *shape: (rng.standard_normal(shape) * 0.02).astype(np.float32)  # noqa: E731
    dh = d // n_head
    sd = {"transformer.wte.weight": g(vocab, d), "transformer.wpe.weight": g(32, d), "lm_head.weight": g(vocab, d)}
    for layer in range(n_layer):
        for h in range(n_head):
            for kind in ("query", "key", "value"):
                sd[f"transformer.h.{layer}.attn.c_attn.weight_h{h}_{kind}"] = g(dh, d)
        sd[f"transformer.h.{layer}.mlp.c_fc.weight"] = g(4 * d, d)
        sd[f"transformer.h.{layer}.attn.c_proj.weight"] = g(d, d)
        sd[f"transformer.h.{layer}.attn.c_proj.bias"] = g(d)
        sd[f"transformer.h.{layer}.mlp.c_proj.weight"] = g(d, 4 * d)
        sd[f"transformer.h.{layer}.mlp.c_proj.bias"] = g(d)
    return sd, {"n_embd": d, "n_layer": n_layer, "n_head": n_head}
