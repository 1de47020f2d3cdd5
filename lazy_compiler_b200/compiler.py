"""``compile_file``: the host-side mirror of ptx_backend.py:1821-1876.

It loads the package (:mod:`.ir`), recognises the operation class
(:mod:`.recognize`) and returns the launch plan as a JSON-ready dict.
"""
from __future__ import annotations

from pathlib import Path

from .ir import load_package
from .recognize import recognise


def compile_file(path: str | Path, meta_path: str | Path | None = None) -> dict:
    """Compile one ``*.ir.json`` package into a launch plan.

    Raises :class:`lazy_compiler_b200.ir.CompileError` (a ``ValueError``) for
    any IR this backend does not lower, before anything is printed.
    """
    package = load_package(path, meta_path)
    return recognise(package).to_json()
