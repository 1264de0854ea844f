"""Activation calibration on the GPU: per-node INT8 scales from FP32 forward
passes over calibration windows (an offline compile-time step; torch tensors
and cuBLAS float32 GEMMs with TF32 disabled, no hot-path kernel).

``build_calibration_seqs(payload, n_seqs, seq_len)``
    the calibration windows cut from the payload's text
    (software/taccel/runtime/calibration.py:60-80)
``build_calibration_seqs_from_token_ids(token_ids, n_seqs, seq_len)``
    the same windows from token ids (calibration.py:83-103)
``build_calibration_scales(payload, ...)``
    calibration.py:104-157: every window runs through the FP32 model at once
    (batched over windows), each node's percentile of |activation| is taken
    per window on the device, a node's scale is the largest over windows / 127
    (at least 1e-8 / 127); the token + position table scale is raised to cover
    |token| + |position| (calibration.py:1324-1361) and nodes no window
    produced get the compiler's defaults (calibration.py:1364-1402).

The node names and the forward follow _fp32_forward
(software/taccel/runtime/fake_quant_reference.py:1235-1322): LayerNorm with
float32 mean and variance, per-head query / key / value projections, causal
softmax attention scaled by d_head^-0.5, GELU (tanh form for gelu_new /
gelu_fast, else erf), residual adds, final LayerNorm and the last position's
logits.  Float32 GEMMs and reductions on the GPU sum in another order than
NumPy's, so scales agree with the reference to float32 rounding
(about 1e-5 relative), not bit for bit.
"""
from __future__ import annotations

from typing import Dict, List, Sequence

DEFAULT_SCALE = 6.0 / 127.0
SFU_DEFAULT_SCALE = 1.0 / 127.0


def _tokenize_text(text: str, stoi: Dict[str, int]) -> List[int]:
    return [stoi[ch] for ch in text if ch in stoi]


def _windows(tokens: List[int], n_seqs: int, seq_len: int) -> List[List[int]]:
    if len(tokens) < seq_len:
        tokens = tokens * ((seq_len // max(len(tokens), 1)) + 2)
    step = max(1, (len(tokens) - seq_len) // max(n_seqs, 1))
    out = []
    for i in range(n_seqs):
        start = (i * step) % (len(tokens) - seq_len + 1)
        out.append(tokens[start:start + seq_len])
    return out


def build_calibration_seqs(payload: dict, *, n_seqs: int = 8, seq_len: int = 16) -> List[List[int]]:
    """Windows of the payload's embedded text (calibration.py:60-80)."""
    text, stoi = str(payload.get("text", "")), payload.get("stoi", {})
    if not text or not stoi:
        return [[0] * seq_len]
    return _windows(_tokenize_text(text, stoi), n_seqs, seq_len)


def build_calibration_seqs_from_token_ids(token_ids: Sequence[int], *, n_seqs: int = 8,
                                          seq_len: int = 16) -> List[List[int]]:
    """Windows of already tokenised text (calibration.py:83-103)."""
    if seq_len <= 0:
        raise ValueError("seq_len must be positive")
    tokens = [int(t) for t in token_ids]
    if not tokens:
        return [[0] * seq_len]
    return _windows(tokens, n_seqs, seq_len)


def _t(x, device):
    import numpy as np
    import torch
    if hasattr(x, "detach"):
        return x.detach().to(device=device, dtype=torch.float32)
    return torch.as_tensor(np.asarray(x, dtype=np.float32), device=device)


def _per_window_stat(x, pct: float):
    """Per window (dim 0): the pct-th percentile of |x| (NumPy's linear
    interpolation), or the maximum at 100."""
    import torch
    a = x.abs().reshape(x.shape[0], -1)
    if pct >= 100.0:
        return a.amax(dim=1)
    return torch.quantile(a, pct / 100.0, dim=1, interpolation="linear")


def fp32_node_stats(state_dict: dict, model_args: dict, seqs: Sequence[Sequence[int]], *,
                    percentile: float = 99.9, overrides: Dict[str, float] | None = None,
                    ln_eps: float | None = None, device=None) -> Dict[str, List[float]]:
    """Per node, the per-window statistic of |activation| of the FP32
    forward (_fp32_forward's nodes), every window at once.  Windows must have
    one length."""
    import torch
    overrides = dict(overrides or {})
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    lens = {len(s) for s in seqs}
    if len(lens) != 1:
        raise ValueError("calibration windows must have one length")
    T = lens.pop()
    n_layer, n_head, d = int(model_args["n_layer"]), int(model_args["n_head"]), int(model_args["n_embd"])
    dh = d // n_head
    eps = ln_eps if ln_eps is not None else float(model_args.get("layer_norm_epsilon", 1e-5))
    act = str(model_args.get("activation_function",
                             "gelu_new" if bool(model_args.get("split_qkv_bias", False)) else "gelu"))
    sd = state_dict
    stats: Dict[str, List[float]] = {}

    def rec(name, x):
        if x.numel() == 0:
            return
        stats.setdefault(name, []).extend(_per_window_stat(x, float(overrides.get(name, percentile))).tolist())

    def ln(x, w, b):
        mean = x.mean(dim=-1, keepdim=True)
        var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
        return (x - mean) / torch.sqrt(var + torch.tensor(eps, dtype=torch.float32, device=device)) * w + b

    def gelu(x):
        if act in ("gelu_new", "gelu_fast"):
            c = torch.tensor(0.7978845608028654, dtype=torch.float32, device=device)   # f32(sqrt(2 / pi))
            return x * 0.5 * (1.0 + torch.tanh(c * (x + 0.044715 * x ** 3)))
        return x * 0.5 * (1.0 + torch.erf(x / torch.sqrt(torch.tensor(2.0, device=device))))

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        with torch.no_grad():
            tids = torch.as_tensor([list(map(int, s)) for s in seqs], device=device)
            S = tids.shape[0]
            wte, wpe = _t(sd["transformer.wte.weight"], device), _t(sd["transformer.wpe.weight"], device)
            tok = wte[tids]                                   # [S, T, d]
            pos = wpe[:T].unsqueeze(0).expand(S, T, d)
            rec("tok_embed", tok)
            rec("pos_embed", pos)
            x = tok + pos
            rec("tok_pos_add", x)
            causal = torch.ones(T, T, dtype=torch.bool, device=device).tril()
            zeros = torch.zeros(dh, dtype=torch.float32, device=device)
            for Lr in range(n_layer):
                p = f"transformer.h.{Lr}."
                h1 = ln(x, _t(sd[p + "ln_1.weight"], device), _t(sd[p + "ln_1.bias"], device))
                rec(f"block{Lr}_ln1", h1)
                heads = []
                for H in range(n_head):
                    qkv = {}
                    for role in ("query", "key", "value"):
                        w = _t(sd[f"{p}attn.c_attn.weight_h{H}_{role}"], device)
                        bk = f"{p}attn.c_attn.bias_h{H}_{role}"
                        b = _t(sd[bk], device) if bk in sd else zeros
                        qkv[role] = h1 @ w.T + b
                        rec(f"block{Lr}_head{H}_{role}", qkv[role])
                    if T == 1:
                        probs = torch.ones(S, 1, 1, dtype=torch.float32, device=device)
                    else:
                        att = (qkv["query"] @ qkv["key"].transpose(1, 2)) * (dh ** -0.5)
                        att = att.masked_fill(~causal, float("-inf"))
                        probs = torch.softmax(att, dim=-1)
                    rec(f"block{Lr}_head{H}_softmax", probs)
                    ho = probs @ qkv["value"]
                    rec(f"block{Lr}_head{H}_attn_v", ho)
                    heads.append(ho)
                cat = torch.cat(heads, dim=-1)
                rec(f"block{Lr}_concat", cat)
                o = cat @ _t(sd[p + "attn.c_proj.weight"], device).T + _t(sd[p + "attn.c_proj.bias"], device)
                rec(f"block{Lr}_out_proj", o)
                x = x + o
                rec(f"block{Lr}_residual1", x)
                h2 = ln(x, _t(sd[p + "ln_2.weight"], device), _t(sd[p + "ln_2.bias"], device))
                rec(f"block{Lr}_ln2", h2)
                f1 = h2 @ _t(sd[p + "mlp.c_fc.weight"], device).T + _t(sd[p + "mlp.c_fc.bias"], device)
                rec(f"block{Lr}_fc1", f1)
                g = gelu(f1)
                rec(f"block{Lr}_gelu", g)
                f2 = g @ _t(sd[p + "mlp.c_proj.weight"], device).T + _t(sd[p + "mlp.c_proj.bias"], device)
                rec(f"block{Lr}_fc2", f2)
                x = x + f2
                rec(f"block{Lr}_residual2", x)
            lf = ln(x, _t(sd["transformer.ln_f.weight"], device), _t(sd["transformer.ln_f.bias"], device))
            rec("ln_f", lf)
            logits = lf[:, -1:] @ _t(sd["lm_head.weight"], device).T
            if "lm_head.bias" in sd:
                logits = logits + _t(sd["lm_head.bias"], device)
            rec("lm_head", logits)
            # |token| + |position| over the same windows: the raw INT8 VADD of
            # the two tables must not clip (calibration.py:1324-1361)
            pct = float(overrides.get("tok_pos_add", percentile))
            stats["_tok_pos_bound"] = _per_window_stat(tok.abs() + pos.abs(), pct).tolist()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return stats


def fill_defaults(scales: Dict[str, float], model_args: dict) -> None:
    """Every compiler calibration key gets an entry (calibration.py:1364-1402)."""
    n_layer, n_head = int(model_args["n_layer"]), int(model_args["n_head"])
    d = scales.setdefault
    for k in ("tok_embed", "pos_embed", "tok_pos_add"):
        d(k, DEFAULT_SCALE)
    for Lr in range(n_layer):
        d(f"block{Lr}_ln1", DEFAULT_SCALE)
        for H in range(n_head):
            for role in ("query", "key", "value"):
                d(f"block{Lr}_head{H}_{role}", DEFAULT_SCALE)
            d(f"block{Lr}_head{H}_softmax", SFU_DEFAULT_SCALE)
            d(f"block{Lr}_head{H}_attn_v", DEFAULT_SCALE)
            # the decode graph's KV loads carry the key / value matmul outputs
            d(f"block{Lr}_head{H}_key_kv_load", scales.get(f"block{Lr}_head{H}_key", DEFAULT_SCALE))
            d(f"block{Lr}_head{H}_value_kv_load", scales.get(f"block{Lr}_head{H}_value", DEFAULT_SCALE))
        for k in ("concat", "out_proj", "residual1", "ln2", "fc1"):
            d(f"block{Lr}_{k}", DEFAULT_SCALE)
        d(f"block{Lr}_gelu", SFU_DEFAULT_SCALE)
        for k in ("fc2", "residual2"):
            d(f"block{Lr}_{k}", DEFAULT_SCALE)
    d("ln_f", DEFAULT_SCALE)
    d("lm_head", DEFAULT_SCALE)


def scales_from_stats(stats: Dict[str, List[float]], model_args: dict,
                      overrides: Dict[str, float] | None = None) -> Dict[str, float]:
    """Per-node scales from per-window statistics (calibration.py:140-157)."""
    overrides = dict(overrides or {})
    bound = stats.get("_tok_pos_bound", [])
    scales = {name: max(max(vals), 1e-8) / 127.0 for name, vals in stats.items() if not name.startswith("_") and vals}
    missing = sorted(set(overrides) - set(scales))
    if missing:
        raise ValueError(f"unknown activation percentile override nodes: {missing}")
    if bound:
        scales["tok_pos_add"] = max(float(scales.get("tok_pos_add", 0.0)), max(max(bound), 1e-8) / 127.0)
    fill_defaults(scales, model_args)
    return scales


def build_calibration_scales(payload: dict, *, n_seqs: int = 8, seq_len: int = 16, percentile: float = 99.9,
                             activation_percentile_overrides: Dict[str, float] | None = None,
                             device=None) -> Dict[str, float]:
    """Per-node INT8 scales of the payload's model from FP32 calibration runs
    on the GPU (calibration.py:104-157)."""
    seqs = build_calibration_seqs(payload, n_seqs=n_seqs, seq_len=seq_len)
    stats = fp32_node_stats(payload["state_dict"], payload["model_args"], seqs, percentile=percentile,
                            overrides=activation_percentile_overrides, device=device)
    return scales_from_stats(stats, payload["model_args"], activation_percentile_overrides)
