"""Compiles the GPT-2 benchmark bundles with the reference toolchain and
writes them as recipes (llm_accelerator_b200/recipe.py) plus golden runs.

    python tests/golden/make_bundles.py small     # GPT-2 small, 12 layers, key_len 48
    python tests/golden/make_bundles.py medium    # GPT-2 medium, 24 layers, key_len 256

Steps: random-init HF GPT-2 (torch seed 0, N(0, 0.02)) -> nanoGPT payload ->
``build_stage3_tiny_decoder_bundle(preset="weight_only_int8")`` (reference)
-> large weight / embedding symbols replaced by seeded regenerable values
(int8 weights keep the standard deviation of the reference's quantized
weights, FP16 embeddings N(0, 0.02)) -> recipe.  The reference golden
simulator then runs the rewritten bundle (GPT-2 small: prefill + 15
teacher-forced prompt tokens + 32 greedy tokens; medium: a few steps) and the
tokens and per-step logits are stored as the golden run.
"""
from __future__ import annotations

import hashlib
import os
import re
import sys
import time
from pathlib import Path

import numpy as np

REF = Path(os.environ.get("TACCEL_REFERENCE", "/root/reference"))
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(REF / "software"))
sys.path.insert(0, str(REF / "software" / "tools"))
sys.path.insert(0, str(HERE.parent.parent))
sys.dont_write_bytecode = True

from llm_accelerator_b200.bundle import ProgramBundle  # noqa: E402
from llm_accelerator_b200.recipe import load_recipe, regenerate, save_recipe  # noqa: E402

CONFIGS = {
    # name: (n_layer, d_model, n_head, vocab, n_positions, decode steps, golden prompt, golden new tokens)
    "small": (12, 768, 12, 50257, 1024, 47, 16, 32),
    "medium": (24, 1024, 16, 50257, 1024, 255, 4, 0),
}
GLOBAL_SEED = 0
TILE_RE = re.compile(r"^(?P<base>.+)__stage\d+_tile_k(?P<k0>\d+)_(?P<kn>\d+)_n(?P<n0>\d+)_(?P<nn>\d+)$")
W_RE = re.compile(r"\.weight(_h\d+_(query|key|value))?$")


def build_reference_bundle(cfg):
    import torch
    from transformers import GPT2Config, GPT2LMHeadModel
    from convert_hf_gpt2_to_nanogpt import convert_hf_state_dict_to_nanogpt
    from taccel.runtime.tiny_fixture import build_stage3_tiny_decoder_bundle
    n_layer, d, h, vocab, npos, steps = cfg[:6]
    torch.manual_seed(0)
    hf = GPT2Config(n_layer=n_layer, n_embd=d, n_head=h, n_positions=npos, vocab_size=vocab)
    payload = convert_hf_state_dict_to_nanogpt(GPT2LMHeadModel(hf).state_dict(), hf)
    return build_stage3_tiny_decoder_bundle(payload, smoke_decode_steps=steps, ptq_preset="weight_only_int8").build.bundle


def symbol_table(b: ProgramBundle):
    items = sorted((b.symbol_address(k), k) for k in b.symbol_offsets if b.symbol_regions.get(k, "data") == "data")
    out = []
    for i, (a, k) in enumerate(items):
        end = items[i + 1][0] if i + 1 < len(items) else b.temp_base
        out.append((k, a - b.data_base, end - a))
    return out


def make_recipe(rb, path: Path):
    b = ProgramBundle.from_any(rb)
    sd = np.frombuffer(b.shared_data, np.uint8)
    table = symbol_table(b)
    sizes = {k: n for k, _, n in table}
    offs = {k: o for k, o, _ in table}
    tiles = {}
    for k, _, _ in table:
        m = TILE_RE.match(k)
        if m:
            tiles.setdefault(m["base"], []).append((k, int(m["k0"]), int(m["kn"]), int(m["n0"]), int(m["nn"])))
    entries, verbatim = [], bytearray()
    covered = 0
    for k, off, n in table:
        data = sd[off:off + n]
        m = TILE_RE.match(k)
        if not data.any():
            entries.append(dict(name=k, off=off, size=n, kind="zero", params={}))
        elif m and m["base"] in sizes:
            base = m["base"]
            K = max(t[1] + t[2] for t in tiles[base])
            N = max(t[3] + t[4] for t in tiles[base])
            k0, kn, n0, nn = int(m["k0"]), int(m["kn"]), int(m["n0"]), int(m["nn"])
            bmat = sd[offs[base]:offs[base] + K * N].reshape(K, N)
            want = np.ascontiguousarray(bmat[k0:k0 + kn, n0:n0 + nn]).ravel()
            assert np.array_equal(data[:want.size], want) and not data[want.size:].any(), f"tile rule fails for {k}"
            entries.append(dict(name=k, off=off, size=n, kind="tile",
                                params=dict(base=base, K=K, N=N, k0=k0, kn=kn, n0=n0, nn=nn)))
        elif k in ("transformer.wte.weight", "transformer.wpe.weight"):
            entries.append(dict(name=k, off=off, size=n, kind="f16", params=dict(std=0.02)))
        elif W_RE.search(k) and ".ln_" not in k:
            std = float(data.view(np.int8).astype(np.float32).std())
            entries.append(dict(name=k, off=off, size=n, kind="i8", params=dict(std=round(std, 3))))
        else:
            entries.append(dict(name=k, off=off, size=n, kind="verbatim", params=dict(at=len(verbatim))))
            verbatim += data.tobytes()
        covered += n
    assert covered == len(sd) - table[0][1], "symbols do not tile the shared data"
    # rewrite the shared data with the regenerated values
    new = sd.copy()
    done = {}
    for e in sorted(entries, key=lambda e: e["kind"] == "tile"):
        if e["kind"] == "verbatim":
            continue
        v = regenerate(e["kind"], e["size"], e["params"], e["name"], GLOBAL_SEED, done)
        new[e["off"]:e["off"] + e["size"]] = v
        if e["kind"] == "i8":
            done[e["name"]] = v
    b.shared_data = new.tobytes()
    sha = hashlib.sha256(b.shared_data).hexdigest()
    save_recipe(path, b, entries, bytes(verbatim), GLOBAL_SEED, sha)
    kinds = {}
    for e in entries:
        kinds[e["kind"]] = kinds.get(e["kind"], 0) + e["size"]
    print("recipe", path.name, {k: f"{v / 1e6:.1f}MB" for k, v in kinds.items()})
    return b


def golden_run(b: ProgramBundle, cfg, path: Path):
    from taccel.assembler.assembler import ProgramBundle as RefBundle
    from taccel.assembler.assembler import RelocationSite as RS, RuntimeConfigAttnSite as RC, RuntimePatchSite as RP
    from taccel.golden_model.simulator import Simulator
    from taccel.runtime.host_runner import HostRunner
    rb = RefBundle(prefill_instrs=b.prefill_instrs, decode_instrs=b.decode_instrs, shared_data=b.shared_data,
                   temp_size=b.temp_size, logits_size=b.logits_size, kv_cache_size=b.kv_cache_size,
                   input_offset=b.input_offset, prefill_logits_offset=b.prefill_logits_offset,
                   decode_logits_offset=b.decode_logits_offset, symbol_offsets=b.symbol_offsets,
                   symbol_regions=b.symbol_regions, relocation_sites=[RS(**vars(x)) for x in b.relocation_sites],
                   runtime_patch_sites=[RP(**vars(x)) for x in b.runtime_patch_sites],
                   runtime_config_attn_sites=[RC(**vars(x)) for x in b.runtime_config_attn_sites],
                   embedding_row_bytes=b.embedding_row_bytes, kv_step_bytes=b.kv_step_bytes)
    vocab, prompt_len, new = cfg[3], cfg[6], cfg[7]
    r = HostRunner(rb, simulator=Simulator(), logits_dtype=np.float16)
    prompt = np.random.default_rng(0).integers(0, vocab, prompt_len).tolist()
    t = time.time()
    logits = [r.run_prefill([prompt[0]])]
    toks = list(prompt)
    for pos in range(1, prompt_len + new):
        tok = prompt[pos] if pos < prompt_len else int(np.argmax(logits[-1][:vocab]))
        if pos >= prompt_len:
            toks.append(tok)
        logits.append(r.run_decode_step(tok, pos))
    dt = time.time() - t
    print("golden tokens", toks, f"{dt:.1f}s for {len(logits)} runs")
    save_golden(path, prompt, toks, np.stack(logits), vocab, dt / len(logits))


KEEP_STEPS = (0, 1, 2)


def save_golden(path, prompt, toks, logits, vocab, sec_per_step):
    """Tokens, a SHA-256 per step of the FP16 logits, and full logits of a few steps."""
    keep = [i for i in KEEP_STEPS if i < len(logits)] + [len(logits) - 1]
    digests = np.stack([np.frombuffer(hashlib.sha256(x.tobytes()).digest(), np.uint8) for x in logits])
    np.savez_compressed(path, prompt=np.asarray(prompt), tokens=np.asarray(toks), logits_digest=digests,
                        kept_steps=np.asarray(keep), kept_logits=logits[keep], vocab=np.asarray([vocab]),
                        seconds_per_step=np.asarray([sec_per_step]), n_steps=np.asarray([len(logits)]))


def main(which):
    cfg = CONFIGS[which]
    t = time.time()
    rb = build_reference_bundle(cfg)
    print("reference compile", round(time.time() - t, 1), "s")
    rpath = HERE / f"recipe_gpt2_{which}.npz"
    b = make_recipe(rb, rpath)
    b2 = load_recipe(rpath)
    assert b2.shared_data == b.shared_data and b2.materialize() == b.materialize()
    golden_run(b, cfg, HERE / f"run_gpt2_{which}.npz")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "small")
