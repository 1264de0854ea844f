"""CPU test of the batched runner's runtime-word encoding (no GPU needed).

BatchedRunner.var_words builds, for every sequence, the SET_ADDR_LO/HI pair of
each runtime-patched address site and the CONFIG_ATTN word of each attention
site (the words the reference HostRunner patches into the instruction stream,
software/taccel/runtime/host_runner.py).  The vectorised encoder is compared
with a per-site restatement through the bundle's own patch helpers.
"""
from __future__ import annotations

import numpy as np
import pytest

from helpers import load_bundle
from llm_accelerator_b200 import isa
from llm_accelerator_b200.engine import Site
from llm_accelerator_b200.runner import BatchedRunner


class _Plan:
    def __init__(self, n):
        self.n_var_words = n


def _runner(bundle, name, batch):
    r = BatchedRunner.__new__(BatchedRunner)   # no engine: only the encoding is exercised
    r.bundle, r.batch = bundle, batch
    sites, meta = [], []
    for s in bundle.runtime_patch_sites:
        if s.stream == name:
            lo, hi = bundle.symbol_extent(s.base_symbol)
            sites.append(Site(0, s.addr_reg, s.absolute_lo_pc, s.absolute_hi_pc, lo, hi))
            meta.append(("addr", s))
    for s in bundle.runtime_config_attn_sites:
        if s.stream == name:
            sites.append(Site(1, 0, s.absolute_pc))
            meta.append(("attn", s))
    r._sites = {name: (sites, meta)}
    r.plans = {name: _Plan(sum(2 if s.kind == 0 else 1 for s in sites))}
    return r


@pytest.mark.parametrize("name", ["tiny_l1_d64", "tiny_l2_d128"])
@pytest.mark.parametrize("stream", ["prefill", "decode"])
def test_var_words_match_patched_instruction_words(name, stream):
    b = load_bundle(name)
    batch = 5
    r = _runner(b, stream, batch)
    rng = np.random.default_rng(3)
    tokens = rng.integers(0, 50257, batch)
    positions = rng.integers(0, 30, batch)
    got = r.var_words(stream, tokens, positions)
    sites, meta = r._sites[stream]
    row, kv = int(b.embedding_row_bytes), int(b.kv_step_bytes)
    for i in range(batch):
        for (kind, s) in meta:
            if kind == "addr":
                off = {"token_embed": int(tokens[i]) * row, "pos_embed": int(positions[i]) * row,
                       "kv_base": int(positions[i]) * kv}[s.kind]
                b.patch_runtime_site(s, off)
            else:
                b.patch_config_attn_site(s, query_row_base=int(positions[i]), valid_kv_len=int(positions[i]) + 1)
        region = bytes(b.instruction_region())
        want = []
        for site in sites:
            pcs = (site.lo_pc, site.hi_pc) if site.kind == 0 else (site.lo_pc,)
            want += [isa.word_of(region[pc * 8:pc * 8 + 8]) for pc in pcs]
        assert got[i].tolist() == want


@pytest.mark.parametrize("name", ["tiny_l1_d64", "tiny_l2_d128"])
@pytest.mark.parametrize("stream", ["prefill", "decode"])
def test_site_formulas_give_the_words_parameters(name, stream):
    """tac_encode_params_tp (the parameters from tokens and positions through
    the runner's site formulas) equals tac_encode_params of the runner's
    runtime words, values and faults alike: positions past the compiled KV
    window return TAC_E_RECOMPILE from both."""
    import ctypes as C
    from llm_accelerator_b200 import _lib as L
    from llm_accelerator_b200.engine import compile_program
    b = load_bundle(name)
    batch = 6
    r = _runner(b, stream, batch)
    sites = r._sites[stream][0]
    entry = b.prefill_pc if stream == "prefill" else b.decode_pc
    p = compile_program(batch, 16 << 20, b.temp_base // 16 * 16, bytes(b.instruction_region()), entry,
                        10_000_000, L.Regs(), True, sites)
    p.set_var_formula(*r.var_formula(stream))
    n = int(L.lib.tac_program_param_count(p.handle))
    rng = np.random.default_rng(5)
    keys = p.attn_key_cols() or 1
    seen = set()
    # position 0; positions inside the KV window (a prefill stream compiles for
    # position 0 only, so these recompile there); then tokens past the
    # embedding table and positions past the window and CONFIG_ATTN's fields
    for lo, hi, vocab in ((0, 1, 64), (0, keys, 64), (keys, 5000, 50257)):
        tokens = rng.integers(0, vocab, batch).astype(np.int64)   # the tiny bundles embed 128 tokens
        positions = rng.integers(lo, hi, batch).astype(np.int64)
        words = r.var_words(stream, tokens, positions)
        a, c = np.zeros((batch, max(n, 1)), np.uint64), np.zeros((batch, max(n, 1)), np.uint64)
        fa, fc = L.Fault(), L.Fault()
        sa = L.lib.tac_encode_params(p.handle, batch, words.ctypes.data, a.ctypes.data, C.byref(fa))
        sc = L.lib.tac_encode_params_tp(p.handle, batch, tokens.ctypes.data, positions.ctypes.data, c.ctypes.data,
                                        C.byref(fc))
        assert sa == sc
        assert fa.buf_id == fc.buf_id and fa.pc == fc.pc
        if sa == L.OK:
            assert np.array_equal(a, c)
        else:
            assert sa == L.E_RECOMPILE
        seen.add(sa)
    assert seen == {L.OK, L.E_RECOMPILE}
