#!/usr/bin/env python3
"""Emmy Kernel IR -> B200 launch plan.  Stdout carries only the plan (JSON).

Drop-in for the reference CLI (compile.py:8-19 of Lazy-Compiler): same
invocation ``python compile.py kernel.ir.json``, the neighbouring
``meta.json`` read the same way, the same exit codes (2 for usage, 1 for a
compile error with ``compile.py: <message>`` on stderr), and nothing on
stdout unless the whole package compiled.  Where the reference prints PTX
text for ``ptxas``, this backend prints the plan that
``lazy_compiler_b200.runtime`` hands to the prebuilt sm_100a kernels of
``liblazyb200.so``.
"""
import json
import sys

from lazy_compiler_b200.ir import CompileError
from lazy_compiler_b200.compiler import compile_file


def main() -> int:
    if len(sys.argv) != 2:
        print("usage: python compile.py kernel.ir.json", file=sys.stderr)
        return 2
    try:
        plan = compile_file(sys.argv[1])
    except (CompileError, ValueError, OSError, KeyError, TypeError) as exc:
        print(f"compile.py: {exc}", file=sys.stderr)
        return 1
    sys.stdout.write(json.dumps(plan, indent=1, sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
