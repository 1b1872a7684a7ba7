"""Where the reference checkout is, for the scripts and tests that read it
(test infrastructure only).

The checkout is named by the environment variable PDB_REFERENCE_ROOT; without
it, a directory named ``reference`` beside this repository's directory is
used when it holds the reference's worker/llama.py. Nothing on the GPU side
needs the checkout: what it produced travels as tests/golden/*.pt fixtures
and as the prebuilt oracle/_ref/ module.
"""
from __future__ import annotations

import os
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def reference_root() -> Path | None:
    """The reference checkout, or None when there is none on this machine."""
    env = os.environ.get("PDB_REFERENCE_ROOT")
    if env:
        return Path(env)
    beside = REPO.parent / "reference"
    return beside if (beside / "worker" / "llama.py").exists() else None
