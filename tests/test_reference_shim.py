"""The Emmy interface shim reproduces the reference compiler's recorded PTX.

Runs the reference's own ``compile_file`` (unchanged) through
``oracle/ref_ptx.py`` and requires the SHA-256 of every emitted PTX to equal
the hash the reference recorded for that IR.  Needs the reference checkout
(``REFERENCE_CHECKOUT`` or a ``reference`` directory beside this repository);
skipped where it is absent (the GPU box has none).
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

from conftest import ROOT


def checkout():
    env = os.environ.get("REFERENCE_CHECKOUT")
    candidates = [Path(env)] if env else []
    candidates.append(ROOT.parent / "reference")
    for c in candidates:
        if (c / "ptx_backend.py").exists():
            return c
    return None


@pytest.mark.skipif(checkout() is None, reason="reference checkout not present")
def test_reference_compiler_reproduces_recorded_ptx():
    result = subprocess.run([sys.executable, str(ROOT / "oracle" / "ref_ptx.py"), str(checkout())],
                            capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stdout + result.stderr
    assert "25/25 recorded hashes reproduced" in result.stdout
