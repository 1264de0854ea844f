"""Compact, reproducible form of large decoder bundles.

A GPT-2-sized bundle is hundreds of MB, almost all of it INT8 weight matrices
(and the pre-tiled copies the compiler lays out for N-tiled matmuls) plus FP16
embedding tables.  A recipe keeps the compiled instruction streams, the
layout metadata and every small data symbol (scales, biases, LayerNorm
parameters, calibration tables) verbatim, and describes each large symbol by
how to regenerate it:

* ``zero``  all-zero bytes;
* ``i8``    seeded int8 weights: round(N(0, std)) clipped to [-127, 127];
* ``f16``   seeded FP16 values: N(0, std) rounded to float16;
* ``tile``  bytes [k0:k0+kn, n0:n0+nn] of another symbol's row-major [K, N]
            int8 matrix (the compiler's tiled copies).

Regeneration is deterministic (NumPy PCG64 seeded per symbol name) and is
checked against a stored SHA-256 of the shared data, so a bundle rebuilt on
any host is byte-identical to the one the golden runs used.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path
from typing import Union

import numpy as np

from .bundle import ProgramBundle, RelocationSite, RuntimeConfigAttnSite, RuntimePatchSite

RECIPE_VERSION = 1


def symbol_seed(global_seed: int, name: str) -> int:
    h = hashlib.sha256(f"{global_seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little")


def regenerate(kind: str, size: int, params: dict, name: str, global_seed: int, done: dict) -> np.ndarray:
    if kind == "zero":
        return np.zeros(size, np.uint8)
    rng = np.random.default_rng(symbol_seed(global_seed, name))
    if kind == "i8":
        v = np.rint(rng.standard_normal(size, dtype=np.float32) * np.float32(params["std"]))
        return np.clip(v, -127, 127).astype(np.int8).view(np.uint8)
    if kind == "f16":
        assert size % 2 == 0
        return (rng.standard_normal(size // 2, dtype=np.float32) * np.float32(params["std"])).astype(
            np.float16).view(np.uint8)
    if kind == "tile":
        base = done[params["base"]][:params["K"] * params["N"]].reshape(params["K"], params["N"])
        t = base[params["k0"]:params["k0"] + params["kn"], params["n0"]:params["n0"] + params["nn"]]
        out = np.zeros(size, np.uint8)
        flat = np.ascontiguousarray(t).ravel()
        out[:flat.size] = flat
        return out
    raise ValueError(f"unknown recipe kind {kind!r}")


def save_recipe(path: Union[str, Path], bundle: ProgramBundle, entries: list, verbatim: bytes,
                global_seed: int, shared_sha: str, extra: dict | None = None) -> None:
    meta = {
        "version": RECIPE_VERSION, "global_seed": global_seed, "shared_sha256": shared_sha,
        "shared_size": len(bundle.shared_data), "entries": entries, "extra": extra or {},
        "temp_size": bundle.temp_size, "logits_size": bundle.logits_size,
        "kv_cache_size": bundle.kv_cache_size, "input_offset": bundle.input_offset,
        "prefill_logits_offset": bundle.prefill_logits_offset,
        "decode_logits_offset": bundle.decode_logits_offset, "symbol_offsets": bundle.symbol_offsets,
        "symbol_regions": bundle.symbol_regions, "embedding_row_bytes": bundle.embedding_row_bytes,
        "kv_step_bytes": bundle.kv_step_bytes,
        "relocation_sites": [vars(s) for s in bundle.relocation_sites],
        "runtime_patch_sites": [vars(s) for s in bundle.runtime_patch_sites],
        "runtime_config_attn_sites": [vars(s) for s in bundle.runtime_config_attn_sites],
    }
    np.savez_compressed(path, prefill=np.frombuffer(bundle.prefill_instrs, np.uint8),
                        decode=np.frombuffer(bundle.decode_instrs, np.uint8),
                        verbatim=np.frombuffer(verbatim, np.uint8),
                        meta=np.frombuffer(json.dumps(meta).encode(), np.uint8))


def load_recipe(path: Union[str, Path], *, verify: bool = True) -> ProgramBundle:
    """Rebuilds the bundle a recipe describes."""
    z = np.load(path)
    meta = json.loads(bytes(z["meta"]).decode())
    if meta.get("version") != RECIPE_VERSION:
        raise ValueError(f"unsupported recipe version {meta.get('version')}")
    shared = np.zeros(meta["shared_size"], np.uint8)
    verbatim = z["verbatim"]
    done = {}
    entries = meta["entries"]
    # generated bases first, tiles after
    for e in sorted(entries, key=lambda e: e["kind"] == "tile"):
        off, size = e["off"], e["size"]
        if e["kind"] == "verbatim":
            shared[off:off + size] = verbatim[e["params"]["at"]:e["params"]["at"] + size]
        else:
            data = regenerate(e["kind"], size, e["params"], e["name"], meta["global_seed"], done)
            shared[off:off + size] = data
            if e["kind"] == "i8":
                done[e["name"]] = data
    if verify:
        got = hashlib.sha256(shared.tobytes()).hexdigest()
        if got != meta["shared_sha256"]:
            raise ValueError(f"recipe {path}: regenerated data digest {got} != {meta['shared_sha256']}")
    b = ProgramBundle(
        prefill_instrs=z["prefill"].tobytes(), decode_instrs=z["decode"].tobytes(), shared_data=shared.tobytes(),
        temp_size=meta["temp_size"], logits_size=meta["logits_size"], kv_cache_size=meta["kv_cache_size"],
        input_offset=meta["input_offset"], prefill_logits_offset=meta["prefill_logits_offset"],
        decode_logits_offset=meta["decode_logits_offset"], symbol_offsets=meta["symbol_offsets"],
        symbol_regions=meta["symbol_regions"],
        relocation_sites=[RelocationSite(**s) for s in meta["relocation_sites"]],
        runtime_patch_sites=[RuntimePatchSite(**s) for s in meta["runtime_patch_sites"]],
        runtime_config_attn_sites=[RuntimeConfigAttnSite(**s) for s in meta["runtime_config_attn_sites"]],
        embedding_row_bytes=meta["embedding_row_bytes"], kv_step_bytes=meta["kv_step_bytes"])
    b.recipe_extra = meta.get("extra", {})
    return b
