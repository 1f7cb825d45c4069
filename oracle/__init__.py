"""CPU oracle and golden-fixture access for parity tests (test infrastructure only)."""
from __future__ import annotations

import os
from pathlib import Path


def reference_checkout() -> Path:
    """Where the reference's sources are read from when fixtures or ``oracle/_ref`` are made:
    ``$TJ_REF`` if set, else a ``reference`` directory beside this checkout.  Only the fixture
    generator, the ``oracle/_ref`` recipe and ``build()`` read it; nothing that runs on a GPU
    machine does."""
    env = os.environ.get("TJ_REF")
    return Path(env) if env else Path(__file__).resolve().parents[2] / "reference"
