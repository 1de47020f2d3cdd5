"""lazy_compiler_b200: a B200 (sm_100a) operator backend for Emmy Kernel IR packages.

Host side: :mod:`.ir` (IR loader), :mod:`.recognize` (operation classes),
:mod:`.compiler` (``compile_file``), :mod:`.runtime` (ctypes C-ABI launcher
over ``liblazyb200.so``), :mod:`.runner` (meta.json-driven package runner).
"""
from .ir import CompileError  # noqa: F401

__all__ = ["CompileError"]
