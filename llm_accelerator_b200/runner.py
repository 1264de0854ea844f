"""Host runners for decoder ProgramBundles.

``HostRunner`` mirrors ``taccel.runtime.host_runner.HostRunner``
(``software/taccel/runtime/host_runner.py:12-123``): it patches the
runtime sites of a bundle (token / position embedding rows, KV-cache base,
attention context), runs the prefill or decode stream on a simulator and reads
the logits back.  It defaults to ``B200Simulator``.

``BatchedRunner`` is the B200-native form of the same loop: B independent
sequences share one compiled plan per stream and one read-only copy of the
weights; each sequence's patched words are passed as runtime parameters, the
greedy argmax runs on the GPU, and only token ids cross PCIe per step.
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Sequence

import numpy as np

from . import _lib as L
from . import isa
from .bundle import ProgramBundle, instruction_region, symbol_extent
from .engine import Engine, Site, compile_program, home_reads


class HostRunner:
    def __init__(self, bundle, simulator=None, *, logits_dtype=np.int32):
        if simulator is None:
            from .simulator import B200Simulator
            simulator = B200Simulator()
        self.bundle = bundle
        self.simulator = simulator
        self.logits_dtype = np.dtype(logits_dtype)
        self.simulator.load_bundle(bundle)

    def _sites(self, kind: str, stream: str):
        return [s for s in self.bundle.runtime_patch_sites if s.kind == kind and s.stream == stream]

    def _patch_sites(self, kind: str, stream: str, offsets: Sequence[int]) -> None:
        sites = self._sites(kind, stream)
        if not sites:
            return
        if len(sites) == 1 and len(offsets) != 1:
            raise ValueError(f"Runtime site kind={kind!r} stream={stream!r} supports one row, "
                             f"got {len(offsets)} offsets")
        if len(sites) != len(offsets):
            raise ValueError(f"Expected {len(sites)} offsets for kind={kind!r} stream={stream!r}, "
                             f"got {len(offsets)}")
        for site, off in zip(sites, offsets):
            self.bundle.patch_runtime_site(site, int(off))

    def _patch_embeddings(self, stream: str, token_ids, position_ids) -> None:
        row = int(self.bundle.embedding_row_bytes)
        self._patch_sites("token_embed", stream, [int(t) * row for t in token_ids])
        self._patch_sites("pos_embed", stream, [int(p) * row for p in position_ids])

    def _patch_kv_bases(self, position: int) -> None:
        off = int(position) * int(self.bundle.kv_step_bytes)
        for site in self._sites("kv_base", "decode"):
            self.bundle.patch_runtime_site(site, off)

    def _patch_decode_attention_context(self, position: int) -> None:
        for site in self.bundle.runtime_config_attn_sites:
            if site.stream == "decode":
                self.bundle.patch_config_attn_site(site, query_row_base=int(position),
                                                   valid_kv_len=int(position) + 1)

    def _read_logits(self, offset: int) -> np.ndarray:
        size = int(self.bundle.logits_size)
        if size <= 0:
            return np.asarray([], dtype=self.logits_dtype)
        if size % self.logits_dtype.itemsize:
            raise ValueError(f"logits_size={size} is not divisible by dtype size {self.logits_dtype.itemsize}")
        data = bytes(self.simulator.state.dram[int(offset):int(offset) + size])
        return np.frombuffer(data, dtype=self.logits_dtype).copy()

    def run_prefill(self, token_ids: Iterable[int], *, max_instructions: int = 10_000_000) -> np.ndarray:
        tokens = [int(t) for t in token_ids]
        if not tokens:
            raise ValueError("run_prefill requires at least one token")
        self._patch_embeddings("prefill", tokens, list(range(len(tokens))))
        self.simulator.run_program(self.bundle, "prefill", max_instructions=max_instructions)
        return self._read_logits(self.bundle.prefill_logits_offset)

    def run_decode_step(self, token_id: int, position: int, *, max_instructions: int = 10_000_000) -> np.ndarray:
        if position < 0:
            raise ValueError("position must be non-negative")
        self._patch_embeddings("decode", [int(token_id)], [int(position)])
        self._patch_kv_bases(int(position))
        self._patch_decode_attention_context(int(position))
        self.simulator.run_program(self.bundle, "decode", max_instructions=max_instructions)
        return self._read_logits(self.bundle.decode_logits_offset)

    @staticmethod
    def _greedy_token(logits: np.ndarray) -> int:
        return 0 if logits.size == 0 else int(np.argmax(logits))

    def generate(self, prompt_ids: Sequence[int], max_new_tokens: int, *, sampler: str = "greedy",
                 eos_token_id: Optional[int] = None) -> List[int]:
        if sampler != "greedy":
            raise ValueError("Stage 3 HostRunner only supports greedy sampling")
        if max_new_tokens < 0:
            raise ValueError("max_new_tokens must be non-negative")
        if not prompt_ids:
            raise ValueError("generate requires at least one prompt token")
        generated = [int(t) for t in prompt_ids]
        nxt = self._greedy_token(self.run_prefill(generated))
        for _ in range(max_new_tokens):
            generated.append(nxt)
            if eos_token_id is not None and nxt == eos_token_id:
                break
            nxt = self._greedy_token(self.run_decode_step(nxt, len(generated) - 1))
        return generated


class BatchedRunner:
    """Runs B independent sequences of one decoder bundle on one GPU.

    Sequence s keeps its own SRAM, temp, KV-cache and logits regions; the
    instruction streams and the shared data (weights, embeddings, tables) are
    held once.  Each step takes one token and one position per sequence."""

    def __init__(self, bundle, batch: int, *, device: int = 0):
        b = ProgramBundle.from_any(bundle)
        self.bundle, self.batch, self.device = b, int(batch), device
        self.dram_bytes = max(16 * 1024 * 1024, b.required_dram_bytes)
        self.shared_bytes = (b.temp_base // 16) * 16
        self.engine = Engine(self.batch, self.dram_bytes, self.shared_bytes, device)
        # the image without a materialised host copy: relocated streams, then
        # the shared data from the bundle's own buffer (a mapped file's view
        # stays a view); the writable tail starts zeroed in a new engine
        region = instruction_region(b, reset_runtime=True)
        self.engine.write_dram(-1, 0, region)
        self.engine.write_dram(-1, b.data_base, b.shared_data)
        self.region = bytes(region)
        self.logits_count = int(b.logits_size) // 2
        self.plans = {}
        self._sites = {}
        for name in ("prefill", "decode"):
            sites, meta = [], []
            for s in b.runtime_patch_sites:
                if s.stream == name:
                    lo, hi = symbol_extent(b, s.base_symbol)
                    sites.append(Site(0, s.addr_reg, s.absolute_lo_pc, s.absolute_hi_pc, lo, hi))
                    meta.append(("addr", s))
            for s in b.runtime_config_attn_sites:
                if s.stream == name:
                    sites.append(Site(1, 0, s.absolute_pc))
                    meta.append(("attn", s))
            self._sites[name] = (sites, meta)
            entry = b.prefill_pc if name == "prefill" else b.decode_pc
            masked = bytearray(self.region)
            for site in sites:
                for pc in ((site.lo_pc, site.hi_pc) if site.kind == 0 else (site.lo_pc,)):
                    w = isa.word_of(masked[pc * 8:pc * 8 + 8]) & (0x7F << 57)
                    masked[pc * 8:pc * 8 + 8] = isa.bytes_of(w)
            self._masked = getattr(self, "_masked", {})
            self._masked[name] = (bytes(masked), entry, sites)
        # State a step must leave behind: logits, the KV cache, and whatever a
        # later step reads before writing (found from the full-state plans).
        live = [(b.logits_base, b.kv_cache_base), (b.kv_cache_base, b.required_dram_bytes)]
        sram_live = sregs_live = False
        for name, (masked, entry, sites) in list(self._masked.items()):
            full = compile_program(self.batch, self.dram_bytes, self.shared_bytes, masked, entry, 10_000_000,
                                   L.Regs(), True, sites)
            if full.info.faulted:
                raise L.fault_to_exception(full.fault)
            ranges, sr, gr = home_reads(full)
            live += ranges
            sram_live |= sr
            sregs_live |= gr
            # A KV site's value is its bank's base + position * kv_step_bytes,
            # and a position must fit the stream's softmax key columns: declare
            # that narrower range (the run-time check still enforces it), so the
            # compiler sees each head's appends touch only its own window.
            keys = full.attn_key_cols()
            if keys:
                meta = self._sites[name][1]
                tight = []
                for site, (kind, s) in zip(sites, meta):
                    if kind == "addr" and s.kind == "kv_base":
                        hi = min(site.range_hi, site.range_lo + keys * int(b.kv_step_bytes))
                        site = Site(site.kind, site.addr_reg, site.lo_pc, site.hi_pc, site.range_lo, hi)
                    tight.append(site)
                self._masked[name] = (masked, entry, tight)
                self._sites[name] = (tight, meta)
        self.live = live
        for name, (masked, entry, sites) in self._masked.items():
            self.plans[name] = compile_program(self.batch, self.dram_bytes, self.shared_bytes, masked, entry,
                                               10_000_000, L.Regs(), True, sites, live=live,
                                               sram_live=sram_live, sregs_live=sregs_live)
            self.plans[name].set_var_formula(*self.var_formula(name))

    # ---- runtime words ------------------------------------------------------------------
    def _var_layout(self, name: str):
        """Per-stream coefficients of the runtime words, built once: address
        site i holds base_i + token * tok_mul_i + position * pos_mul_i."""
        cache = self.__dict__.setdefault("_var_layout_cache", {})
        if name in cache:
            return cache[name]
        b = self.bundle
        sites, meta = self._sites[name]
        row, kv = int(b.embedding_row_bytes), int(b.kv_step_bytes)
        a_col, a_base, a_tok, a_pos, a_reg, t_col, t_mode = [], [], [], [], [], [], []
        col = 0
        for (kind, s) in meta:
            if kind == "addr":
                a_col.append(col)
                a_base.append(b.symbol_address(s.base_symbol))
                a_tok.append(row if s.kind == "token_embed" else 0)
                a_pos.append(row if s.kind == "pos_embed" else (0 if s.kind == "token_embed" else kv))
                a_reg.append(s.addr_reg)
                col += 2
            else:
                t_col.append(col)
                t_mode.append(s.mode)
                col += 1
        u = lambda v: np.asarray(v, dtype=np.uint64)  # noqa: E731
        lay = dict(a_col=np.asarray(a_col, np.int64), a_base=u(a_base), a_tok=u(a_tok), a_pos=u(a_pos),
                   a_reg=u(a_reg) << np.uint64(57), t_col=np.asarray(t_col, np.int64),
                   t_mode=u(t_mode) << np.uint64(33), n=col)
        cache[name] = lay
        return lay

    def var_formula(self, name: str):
        """(base, tok_mul, pos_mul, mode) of every runtime site of a stream, in
        site order: the affine form var_words evaluates, for the engine's
        token / position path (Engine.run_async_tp)."""
        b = self.bundle
        row, kv = int(b.embedding_row_bytes), int(b.kv_step_bytes)
        out = ([], [], [], [])
        for (kind, s) in self._sites[name][1]:
            if kind == "addr":
                vals = (b.symbol_address(s.base_symbol), row if s.kind == "token_embed" else 0,
                        row if s.kind == "pos_embed" else (0 if s.kind == "token_embed" else kv), 0)
            else:
                vals = (0, 0, 0, s.mode)
            for lst, v in zip(out, vals):
                lst.append(v)
        return out

    def var_words(self, name: str, tokens: Sequence[int], positions: Sequence[int]) -> np.ndarray:
        """[batch, n_var_words] runtime words for one step of every sequence:
        SET_ADDR_LO/HI pairs of symbol + token * row, symbol + position * row
        or symbol + position * kv_step_bytes, and CONFIG_ATTN words with
        query_row_base = position, valid_kv_len = position + 1."""
        lay = self._var_layout(name)
        out = np.zeros((self.batch, self.plans[name].n_var_words), dtype=np.uint64)
        tok = np.asarray(tokens, dtype=np.int64).reshape(self.batch, 1).astype(np.uint64)
        pos = np.asarray(positions, dtype=np.int64).reshape(self.batch, 1).astype(np.uint64)
        if len(lay["a_col"]):
            v = lay["a_base"][None, :] + tok * lay["a_tok"][None, :] + pos * lay["a_pos"][None, :]
            m28 = np.uint64(isa.M28)
            out[:, lay["a_col"]] = (np.uint64(isa.SET_ADDR_LO << 59) | lay["a_reg"][None, :] |
                                    ((v & m28) << np.uint64(29)))
            out[:, lay["a_col"] + 1] = (np.uint64(isa.SET_ADDR_HI << 59) | lay["a_reg"][None, :] |
                                        (((v >> np.uint64(28)) & m28) << np.uint64(29)))
        if len(lay["t_col"]):
            out[:, lay["t_col"]] = (np.uint64(isa.CONFIG_ATTN << 59) | (pos << np.uint64(47)) |
                                    ((pos + np.uint64(1)) << np.uint64(35)) | lay["t_mode"][None, :])
        return out

    def params(self, name: str, tokens, positions) -> np.ndarray:
        """Host parameter block for one step (see Engine.encode_params)."""
        return self.engine.encode_params(self.plans[name], self.var_words(name, tokens, positions))

    def step_params_async(self, name: str, params_dev_ptr: int, stream=None) -> None:
        """One step with its parameter block already on the device."""
        self.engine.run_async_params(self.plans[name], params_dev_ptr, stream)

    def argmax_async(self, name: str, out_dev_ptr: int, vocab: int, stream=None) -> None:
        """Greedy token of every sequence (device int32[batch]) from this step's logits."""
        self.engine.argmax_f16(self.logits_offset(name), vocab, out_dev_ptr, stream)

    def step_async(self, name: str, tokens, positions, stream=None) -> None:
        """One step, its runtime parameters computed from tokens and positions
        on the host without building the instruction words (the same values
        and checks as var_words + Engine.run_async)."""
        self.engine.run_async_tp(self.plans[name], tokens, positions, stream)

    def step(self, name: str, tokens, positions) -> None:
        st = self.engine.run(self.plans[name], self.var_words(name, tokens, positions))
        if st != L.OK:
            raise L.fault_to_exception(self.engine._last_fault, st)

    def logits(self, name: str, seq: int) -> np.ndarray:
        off = self.bundle.prefill_logits_offset if name == "prefill" else self.bundle.decode_logits_offset
        return np.frombuffer(self.engine.read_dram(seq, off, self.logits_count * 2), dtype=np.float16).copy()

    def logits_offset(self, name: str) -> int:
        return self.bundle.prefill_logits_offset if name == "prefill" else self.bundle.decode_logits_offset
