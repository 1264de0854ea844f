"""The native bundle-file reader (tac_bundle_open) against ProgramBundle.load (CPU)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from llm_accelerator_b200.bundle import ProgramBundle

GOLDEN = Path(__file__).parent / "golden"
BUNDLES = ["bundle_tiny_l1_d64.npz", "bundle_tiny_l2_d128.npz"]
FIELDS = ["prefill_instrs", "decode_instrs", "temp_size", "logits_size", "kv_cache_size", "input_offset",
          "prefill_logits_offset", "decode_logits_offset", "symbol_offsets", "symbol_regions", "relocation_sites",
          "runtime_patch_sites", "runtime_config_attn_sites", "embedding_row_bytes", "kv_step_bytes"]


def _same(a: ProgramBundle, b: ProgramBundle):
    for f in FIELDS:
        assert getattr(a, f) == getattr(b, f), f
    assert bytes(a.shared_data) == bytes(b.shared_data)
    assert a.materialize() == b.materialize()


@pytest.mark.parametrize("name", BUNDLES)
def test_mapped_load_equals_load(name):
    want = ProgramBundle.load(GOLDEN / name)
    got = ProgramBundle.load_mapped(GOLDEN / name)
    _same(got, want)
    assert isinstance(got.shared_data, np.ndarray) and not got.shared_data.flags.writeable   # a view, no copy


def test_save_then_map_round_trip(tmp_path):
    b = ProgramBundle.load(GOLDEN / BUNDLES[1])
    p = tmp_path / "b.npz"
    b.save(p)
    _same(ProgramBundle.load_mapped(p), b)


def _arrays(name):
    z = np.load(GOLDEN / name)
    return {k: z[k] for k in ("prefill", "decode", "shared", "meta")}


def test_compressed_entries_are_rejected(tmp_path):
    p = tmp_path / "c.npz"
    np.savez_compressed(p, **_arrays(BUNDLES[0]))
    with pytest.raises(ValueError, match="status 17"):
        ProgramBundle.load_mapped(p)


@pytest.mark.parametrize("case", ["truncated", "not_zip", "missing_meta", "wrong_dtype", "two_dims", "empty"])
def test_malformed_files_are_rejected(tmp_path, case):
    p = tmp_path / "bad.npz"
    arrs = _arrays(BUNDLES[0])
    if case == "truncated":
        good = tmp_path / "good.npz"
        np.savez(good, **arrs)
        p.write_bytes(good.read_bytes()[:-200])
    elif case == "not_zip":
        p.write_bytes(b"not a zip file at all" * 10)
    elif case == "missing_meta":
        del arrs["meta"]
        np.savez(p, **arrs)
    elif case == "wrong_dtype":
        arrs["shared"] = arrs["shared"][: len(arrs["shared"]) // 4 * 4].view(np.int32)
        np.savez(p, **arrs)
    elif case == "two_dims":
        arrs["prefill"] = arrs["prefill"][: len(arrs["prefill"]) // 8 * 8].reshape(-1, 8)
        np.savez(p, **arrs)
    else:
        p.write_bytes(b"")
    with pytest.raises(ValueError, match="status 16"):
        ProgramBundle.load_mapped(p)


def test_missing_file_is_rejected(tmp_path):
    with pytest.raises(ValueError, match="status 16"):
        ProgramBundle.load_mapped(tmp_path / "absent.npz")


def test_shared_data_outlives_the_bundle():
    """The mapped shared image keeps the file mapped after the bundle is gone."""
    import gc
    want = bytes(ProgramBundle.load(GOLDEN / BUNDLES[1]).shared_data)
    shared = ProgramBundle.load_mapped(GOLDEN / BUNDLES[1]).shared_data
    gc.collect()
    assert bytes(shared) == want
    view = shared[1000:2000]
    del shared
    gc.collect()
    assert bytes(view) == want[1000:2000]


@pytest.mark.parametrize("where", ["locator", "directory"])
def test_huge_zip64_offsets_are_rejected(tmp_path, where):
    """zip64 offsets near 2**64 must not wrap the reader's bounds checks."""
    import struct
    good = tmp_path / "good.npz"
    np.savez(good, **_arrays(BUNDLES[0]))
    data = good.read_bytes()
    eocd = data.rfind(b"PK\x05\x06")
    huge = (1 << 64) - 24
    if where == "locator":          # the locator points past the end of the file
        z64 = huge
        extra = b""
    else:                           # a valid zip64 record whose directory offset is huge
        z64 = eocd
        extra = struct.pack("<IQHHIIQQQQ", 0x06064b50, 44, 45, 45, 0, 0, 4, 4, 0, huge)
    locator = struct.pack("<IIQI", 0x07064b50, 0, z64, 1)
    p = tmp_path / "bad.npz"
    p.write_bytes(data[:eocd] + extra + locator + data[eocd:])
    with pytest.raises(ValueError, match="status 16"):
        ProgramBundle.load_mapped(p)
