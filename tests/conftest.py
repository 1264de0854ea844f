import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (str(ROOT), str(ROOT / "tests"), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

REFERENCE = Path(os.environ.get("TACCEL_REFERENCE", "/root/reference"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")
    config.addinivalue_line("markers", "reference: reads the reference checkout (skipped when absent)")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def has_reference() -> bool:
    """The reference's taccel package: installed under baseline/_ref, or the
    checkout named by TACCEL_REFERENCE."""
    return (ROOT / "baseline" / "_ref" / "taccel").is_dir() or (REFERENCE / "software" / "taccel").is_dir()


def pytest_collection_modifyitems(config, items):
    gpu = has_gpu()
    skip_gpu = pytest.mark.skip(reason="no CUDA device")
    skip_ref = pytest.mark.skip(reason="reference checkout not present")
    for item in items:
        if "gpu" in item.keywords and not gpu:
            item.add_marker(skip_gpu)
        if "reference" in item.keywords and not has_reference():
            item.add_marker(skip_ref)
