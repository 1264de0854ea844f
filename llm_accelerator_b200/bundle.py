"""Program bundles: two instruction streams sharing one DRAM image.

``ProgramBundle`` has the fields, layout rules and patch helpers of the
reference's ``taccel.assembler.assembler.ProgramBundle``
(``software/taccel/assembler/assembler.py:113-372``) so that bundles compiled
by the reference toolchain can be converted one-to-one and run without it.
``save`` / ``load`` store a bundle as an uncompressed ``.npz`` (instruction
streams, shared data and a JSON metadata record).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field, replace
from pathlib import Path
from typing import Dict, List, Optional, Union

import numpy as np

from . import isa

VALID_RUNTIME_PATCH_KINDS = {"token_embed", "pos_embed", "kv_base"}
FORMAT_VERSION = 1


def _align(v: int, a: int) -> int:
    return (v + a - 1) & ~(a - 1)


def symbol_extent(bundle, symbol: str) -> tuple[int, int]:
    """[start, end) DRAM bytes a symbol may span: up to the next symbol of its
    region, or the end of the region.  Reads only fields and methods the
    reference's ProgramBundle has too (``symbol_address``, ``symbol_offsets``,
    ``symbol_regions`` and the region bases, ``assembler.py:163-300``), so it
    works on either class."""
    start = bundle.symbol_address(symbol)
    region = bundle.symbol_regions.get(symbol, "data")
    ends = {"data": bundle.temp_base, "shared_data": bundle.temp_base, "temp": bundle.logits_base,
            "logits": bundle.kv_cache_base, "kv_cache": bundle.required_dram_bytes}
    end = ends.get(region, bundle.required_dram_bytes)
    for name in bundle.symbol_offsets:
        if bundle.symbol_regions.get(name, "data") != region:
            continue
        a = bundle.symbol_address(name)
        if start < a < end:
            end = a
    return start, end


def instruction_region(bundle, *, reset_runtime: bool = False) -> bytearray:
    """Both runtime streams at their DRAM offsets (the image's first
    ``data_base`` bytes), from the public stream API of either ProgramBundle
    class; ``reset_runtime`` first re-applies the relocations, as
    ``materialize(reset_runtime=True)`` does."""
    if reset_runtime:
        bundle.reset_runtime_images()
    reg = bytearray(bundle.data_base)
    for name, off in (("prefill", bundle.prefill_instrs_offset), ("decode", bundle.decode_instrs_offset)):
        s = bundle.stream_bytes(name)
        reg[off:off + len(s)] = s
    return reg


@dataclass(frozen=True)
class RelocationSite:
    stream: str
    local_lo_pc: int
    local_hi_pc: int
    addr_reg: int
    symbol: str


@dataclass(frozen=True)
class RuntimePatchSite:
    stream: str
    kind: str
    local_lo_pc: int
    local_hi_pc: int
    absolute_lo_pc: int
    absolute_hi_pc: int
    addr_reg: int
    base_symbol: str


@dataclass(frozen=True)
class RuntimeConfigAttnSite:
    stream: str
    local_pc: int
    absolute_pc: int
    mode: int


def _read_pair(buf, lo_pc: int, hi_pc: int, addr_reg: int) -> int:
    lo = isa.word_of(buf[lo_pc * 8:lo_pc * 8 + 8])
    hi = isa.word_of(buf[hi_pc * 8:hi_pc * 8 + 8])
    if (lo >> 59) != isa.SET_ADDR_LO or (hi >> 59) != isa.SET_ADDR_HI:
        raise ValueError(f"PCs {lo_pc}/{hi_pc} are not a SET_ADDR_LO/HI pair")
    if ((lo >> 57) & 3) != addr_reg or ((hi >> 57) & 3) != addr_reg:
        raise ValueError(f"SET_ADDR pair at PCs {lo_pc}/{hi_pc} does not use R{addr_reg}")
    return (((hi >> 29) & isa.M28) << 28) | ((lo >> 29) & isa.M28)


def _write_pair(buf: bytearray, lo_pc: int, hi_pc: int, addr_reg: int, value: int) -> None:
    _read_pair(buf, lo_pc, hi_pc, addr_reg)  # validates the pair
    lo, hi = isa.set_addr_pair(addr_reg, value)
    buf[lo_pc * 8:lo_pc * 8 + 8] = isa.bytes_of(lo)
    buf[hi_pc * 8:hi_pc * 8 + 8] = isa.bytes_of(hi)


@dataclass
class ProgramBundle:
    prefill_instrs: bytes = b""
    decode_instrs: bytes = b""
    shared_data: bytes = b""
    temp_size: int = 0
    logits_size: int = 0
    kv_cache_size: int = 0
    input_offset: int = 0
    prefill_logits_offset: int = 0
    decode_logits_offset: int = 0
    symbol_offsets: Dict[str, int] = field(default_factory=dict)
    symbol_regions: Dict[str, str] = field(default_factory=dict)
    relocation_sites: List[RelocationSite] = field(default_factory=list)
    runtime_patch_sites: List[RuntimePatchSite] = field(default_factory=list)
    runtime_config_attn_sites: List[RuntimeConfigAttnSite] = field(default_factory=list)
    embedding_row_bytes: int = 16
    kv_step_bytes: int = 16

    def __post_init__(self):
        self.prefill_instrs = bytes(self.prefill_instrs)
        self.decode_instrs = bytes(self.decode_instrs)
        if not isinstance(self.shared_data, (bytes, np.ndarray)):
            self.shared_data = bytes(self.shared_data)
        if len(self.prefill_instrs) % 8 or len(self.decode_instrs) % 8:
            raise ValueError("ProgramBundle instruction streams must be 8-byte aligned")
        if min(self.temp_size, self.logits_size, self.kv_cache_size) < 0:
            raise ValueError("ProgramBundle region sizes must be non-negative")
        self.prefill_instrs_offset = 0
        self.decode_instrs_offset = _align(len(self.prefill_instrs), 8)
        decode_end = self.decode_instrs_offset + len(self.decode_instrs)
        self.data_base = _align(decode_end, 16)
        self.temp_base = _align(self.data_base + len(self.shared_data), 16)
        self.logits_base = _align(self.temp_base + self.temp_size, 16)
        self.kv_cache_base = _align(self.logits_base + self.logits_size, 16)
        self.kv_cache_size_bytes = self.kv_cache_size
        self.required_dram_bytes = self.kv_cache_base + self.kv_cache_size
        self.prefill_pc = 0
        self.decode_pc = self.decode_instrs_offset // 8
        self.insn_count = self.data_base // 8
        if self.input_offset == 0:
            self.input_offset = self.data_base
        if self.prefill_logits_offset == 0:
            self.prefill_logits_offset = self.logits_base
        if self.decode_logits_offset == 0:
            self.decode_logits_offset = self.logits_base
        base = {"prefill": self.prefill_pc, "decode": self.decode_pc}
        self.runtime_patch_sites = [
            replace(s, absolute_lo_pc=base[s.stream] + s.local_lo_pc, absolute_hi_pc=base[s.stream] + s.local_hi_pc)
            for s in self.runtime_patch_sites]
        self.runtime_config_attn_sites = [
            replace(s, absolute_pc=base[s.stream] + s.local_pc) for s in self.runtime_config_attn_sites]
        self._runtime: Optional[Dict[str, bytearray]] = None

    # ---- symbols -----------------------------------------------------------------
    def symbol_address(self, symbol: str) -> int:
        builtins = {"data_base": self.data_base, "shared_data": self.data_base, "temp_base": self.temp_base,
                    "logits_base": self.logits_base, "kv_cache_base": self.kv_cache_base,
                    "input_offset": self.input_offset, "prefill_logits_offset": self.prefill_logits_offset,
                    "decode_logits_offset": self.decode_logits_offset}
        if symbol in builtins:
            return builtins[symbol]
        if symbol in self.symbol_offsets:
            region = self.symbol_regions.get(symbol, "data")
            bases = {"data": self.data_base, "shared_data": self.data_base, "temp": self.temp_base,
                     "logits": self.logits_base, "kv_cache": self.kv_cache_base}
            if region not in bases:
                raise ValueError(f"Unknown ProgramBundle symbol region {region!r} for {symbol!r}")
            return bases[region] + int(self.symbol_offsets[symbol])
        raise KeyError(f"Unknown ProgramBundle symbol: {symbol}")

    def symbol_extent(self, symbol: str) -> tuple[int, int]:
        """[start, end) bytes a symbol may span (see the module function)."""
        return symbol_extent(self, symbol)

    # ---- runtime streams -------------------------------------------------------------
    def _stream(self, stream: str) -> bytearray:
        if self._runtime is None:
            self.reset_runtime_images()
        if stream not in self._runtime:
            raise ValueError("stream must be 'prefill' or 'decode'")
        return self._runtime[stream]

    def reset_runtime_images(self) -> None:
        streams = {"prefill": bytearray(self.prefill_instrs), "decode": bytearray(self.decode_instrs)}
        for s in self.relocation_sites:
            addend = _read_pair(streams[s.stream], s.local_lo_pc, s.local_hi_pc, s.addr_reg)
            _write_pair(streams[s.stream], s.local_lo_pc, s.local_hi_pc, s.addr_reg,
                        self.symbol_address(s.symbol) + addend)
        self._runtime = streams

    def patch_runtime_site(self, site_or_kind: Union[RuntimePatchSite, str], offset: int = 0, *,
                           stream: Optional[str] = None) -> RuntimePatchSite:
        if isinstance(site_or_kind, str):
            m = [s for s in self.runtime_patch_sites
                 if s.kind == site_or_kind and (stream is None or s.stream == stream)]
            if len(m) != 1:
                raise ValueError(f"Expected exactly one runtime patch site for kind={site_or_kind!r}, "
                                 f"stream={stream!r}; found {len(m)}")
            site = m[0]
        else:
            site = site_or_kind
        _write_pair(self._stream(site.stream), site.local_lo_pc, site.local_hi_pc, site.addr_reg,
                    self.symbol_address(site.base_symbol) + int(offset))
        return site

    def patch_config_attn_site(self, site: RuntimeConfigAttnSite, *, query_row_base: int,
                               valid_kv_len: int) -> RuntimeConfigAttnSite:
        buf = self._stream(site.stream)
        if (isa.word_of(buf[site.local_pc * 8:site.local_pc * 8 + 8]) >> 59) != isa.CONFIG_ATTN:
            raise ValueError(f"PC {site.local_pc} is not CONFIG_ATTN")
        buf[site.local_pc * 8:site.local_pc * 8 + 8] = isa.bytes_of(
            isa.config_attn_word(int(query_row_base), int(valid_kv_len), site.mode))
        return site

    def stream_bytes(self, stream: str) -> bytes:
        return bytes(self._stream(stream))

    def instruction_region(self) -> bytearray:
        """The instruction words of both runtime streams at their DRAM offsets."""
        reg = bytearray(self.data_base)
        p, d = self._stream("prefill"), self._stream("decode")
        reg[self.prefill_instrs_offset:self.prefill_instrs_offset + len(p)] = p
        reg[self.decode_instrs_offset:self.decode_instrs_offset + len(d)] = d
        return reg

    def materialize(self, *, reset_runtime: bool = True) -> bytes:
        if reset_runtime:
            self.reset_runtime_images()
        img = bytearray(self.required_dram_bytes)
        img[:self.data_base] = self.instruction_region()
        img[self.data_base:self.data_base + len(self.shared_data)] = bytes(self.shared_data)
        return bytes(img)

    # ---- persistence ---------------------------------------------------------------------
    def save(self, path: Union[str, Path]) -> None:
        meta = {
            "version": FORMAT_VERSION,
            "temp_size": self.temp_size, "logits_size": self.logits_size, "kv_cache_size": self.kv_cache_size,
            "input_offset": self.input_offset, "prefill_logits_offset": self.prefill_logits_offset,
            "decode_logits_offset": self.decode_logits_offset, "symbol_offsets": self.symbol_offsets,
            "symbol_regions": self.symbol_regions, "embedding_row_bytes": self.embedding_row_bytes,
            "kv_step_bytes": self.kv_step_bytes,
            "relocation_sites": [vars(s) for s in self.relocation_sites],
            "runtime_patch_sites": [vars(s) for s in self.runtime_patch_sites],
            "runtime_config_attn_sites": [vars(s) for s in self.runtime_config_attn_sites],
        }
        np.savez(path, prefill=np.frombuffer(self.prefill_instrs, np.uint8),
                 decode=np.frombuffer(self.decode_instrs, np.uint8),
                 shared=np.frombuffer(bytes(self.shared_data), np.uint8),
                 meta=np.frombuffer(json.dumps(meta).encode(), np.uint8))

    @classmethod
    def load(cls, path: Union[str, Path]) -> "ProgramBundle":
        z = np.load(path)
        meta = json.loads(bytes(z["meta"]).decode())
        if meta.get("version") != FORMAT_VERSION:
            raise ValueError(f"unsupported bundle format version {meta.get('version')}")
        return cls(
            prefill_instrs=z["prefill"].tobytes(), decode_instrs=z["decode"].tobytes(),
            shared_data=z["shared"].tobytes(), temp_size=meta["temp_size"], logits_size=meta["logits_size"],
            kv_cache_size=meta["kv_cache_size"], input_offset=meta["input_offset"],
            prefill_logits_offset=meta["prefill_logits_offset"],
            decode_logits_offset=meta["decode_logits_offset"], symbol_offsets=meta["symbol_offsets"],
            symbol_regions=meta["symbol_regions"],
            relocation_sites=[RelocationSite(**s) for s in meta["relocation_sites"]],
            runtime_patch_sites=[RuntimePatchSite(**s) for s in meta["runtime_patch_sites"]],
            runtime_config_attn_sites=[RuntimeConfigAttnSite(**s) for s in meta["runtime_config_attn_sites"]],
            embedding_row_bytes=meta["embedding_row_bytes"], kv_step_bytes=meta["kv_step_bytes"])

    @classmethod
    def load_mapped(cls, path: Union[str, Path]) -> "ProgramBundle":
        """load() through the native reader (tac_bundle_open): the file is
        mapped read-only and the shared image is a NumPy view of the mapping,
        not a copy.  The view owns a reference to the mapping, so the file
        stays mapped as long as the bundle or any array taken from it lives.
        Same result as load()."""
        import ctypes as C
        from . import _lib as L
        view, handle = L.BundleView(), C.c_void_p()
        st = L.lib.tac_bundle_open(str(path).encode(), C.byref(view), C.byref(handle))
        if st != L.OK:
            raise ValueError(f"cannot read bundle file {path} (status {st})")
        mapping = _BundleMapping(handle)

        def arr(ptr, n):
            if n == 0:
                return np.zeros(0, np.uint8)
            raw = (C.c_uint8 * int(n)).from_address(int(ptr))
            raw._mapping = mapping          # the array's buffer keeps the file mapped
            a = np.frombuffer(raw, np.uint8)
            a.flags.writeable = False
            return a

        meta = json.loads(C.string_at(view.meta_json, view.meta_len).decode())
        if meta.get("version") != FORMAT_VERSION:
            raise ValueError(f"unsupported bundle format version {meta.get('version')}")
        b = cls(
            prefill_instrs=arr(view.prefill, view.prefill_len).tobytes(),
            decode_instrs=arr(view.decode, view.decode_len).tobytes(),
            shared_data=arr(view.shared, view.shared_len), temp_size=meta["temp_size"],
            logits_size=meta["logits_size"], kv_cache_size=meta["kv_cache_size"], input_offset=meta["input_offset"],
            prefill_logits_offset=meta["prefill_logits_offset"],
            decode_logits_offset=meta["decode_logits_offset"], symbol_offsets=meta["symbol_offsets"],
            symbol_regions=meta["symbol_regions"],
            relocation_sites=[RelocationSite(**s) for s in meta["relocation_sites"]],
            runtime_patch_sites=[RuntimePatchSite(**s) for s in meta["runtime_patch_sites"]],
            runtime_config_attn_sites=[RuntimeConfigAttnSite(**s) for s in meta["runtime_config_attn_sites"]],
            embedding_row_bytes=meta["embedding_row_bytes"], kv_step_bytes=meta["kv_step_bytes"])
        b._mapping = mapping
        return b

    @classmethod
    def from_any(cls, b) -> "ProgramBundle":
        """Copies any object with ProgramBundle's fields (e.g. the reference's)."""
        if isinstance(b, cls):
            return b
        return cls(
            prefill_instrs=b.prefill_instrs, decode_instrs=b.decode_instrs, shared_data=b.shared_data,
            temp_size=b.temp_size, logits_size=b.logits_size, kv_cache_size=b.kv_cache_size,
            input_offset=b.input_offset, prefill_logits_offset=b.prefill_logits_offset,
            decode_logits_offset=b.decode_logits_offset, symbol_offsets=dict(b.symbol_offsets),
            symbol_regions=dict(b.symbol_regions),
            relocation_sites=[RelocationSite(s.stream, s.local_lo_pc, s.local_hi_pc, s.addr_reg, s.symbol)
                              for s in b.relocation_sites],
            runtime_patch_sites=[RuntimePatchSite(s.stream, s.kind, s.local_lo_pc, s.local_hi_pc,
                                                  s.absolute_lo_pc, s.absolute_hi_pc, s.addr_reg, s.base_symbol)
                                 for s in b.runtime_patch_sites],
            runtime_config_attn_sites=[RuntimeConfigAttnSite(s.stream, s.local_pc, s.absolute_pc, s.mode)
                                       for s in b.runtime_config_attn_sites],
            embedding_row_bytes=b.embedding_row_bytes, kv_step_bytes=b.kv_step_bytes)


class _BundleMapping:
    """Owns a tac_bundle_open handle; unmaps the file when collected."""

    def __init__(self, handle):
        self.handle = handle

    def __del__(self):
        if self.handle:
            from . import _lib as L
            L.lib.tac_bundle_close(self.handle)
            self.handle = None
