import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
# the reference package, when it was installed next to the repo (pip --target baseline/_ref);
# only the tensorjit-integration tests import it, and they skip without it
_REF = ROOT / "baseline" / "_ref"
if _REF.exists() and str(_REF) not in sys.path:
    sys.path.append(str(_REF))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running (full-size configs)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="needs a CUDA GPU")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
