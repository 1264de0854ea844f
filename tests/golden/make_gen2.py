"""Packs the reference's gen2 known-answer vectors (its RTL fixtures,
rtl/verilator/fixtures/gen2/<op>/<case>/: input tiles, scale registers before
and after, expected output, meta.json; 16 x 64 tiles, seed 20260516) into
tests/golden/gen2_kats.npz, so the tests replay them without the checkout.

    TACCEL_REFERENCE=<reference checkout> python tests/golden/make_gen2.py
"""
from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np

REF = Path(os.environ.get("TACCEL_REFERENCE", "/root/reference"))
HERE = Path(__file__).resolve().parent
FILES = ("input_src1.raw", "input_src2.raw", "scale_regs_pre.raw", "expected_out.raw", "scale_regs_post.raw")


def main():
    root = REF / "rtl" / "verilator" / "fixtures" / "gen2"
    out = {}
    names = []
    for d in sorted(root.glob("*/*")):
        name = f"{d.parent.name}/{d.name}"
        names.append(name)
        out[f"{name}/meta.json"] = np.frombuffer((d / "meta.json").read_bytes(), np.uint8)
        for f in FILES:
            if (d / f).exists():
                out[f"{name}/{f}"] = np.frombuffer((d / f).read_bytes(), np.uint8)
    out["cases"] = np.frombuffer(json.dumps(names).encode(), np.uint8)
    np.savez_compressed(HERE / "gen2_kats.npz", **out)
    print(f"wrote {len(names)} cases to {HERE / 'gen2_kats.npz'}")


if __name__ == "__main__":
    main()
