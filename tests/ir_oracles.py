"""The IR oracle of a package, chosen from the IR alone — TEST INFRASTRUCTURE.

Which oracle evaluates a package is decided by the structure of its Tile,
never by the plan the product's recogniser made: fragment programs go to
oracle/fragment_ir.py, block-cooperative Tiles (block_threads set) to the
lockstep simulation oracle/staged_ir.py, per-point bodies with loops to
oracle/serial_ir.py, straight-line bodies to oracle/pointwise_ir.py.  A
package the recogniser puts in the wrong fixed class is then checked
against what its IR says, not against the wrong class's formula.
"""
from lazy_compiler_b200.ir import load_package


COOPERATIVE = {"WarpShuffle", "TreeHalve", "Smem", "Sync", "CpAsyncCopy"}
FRAGMENT = ("Fragment", "RegFragment", "RegStore", "MmaSync", "Ldmatrix")


def _kinds(body) -> set:
    out = set()
    for s in body:
        if hasattr(s, "kind"):
            out.add(s.kind)
            out |= _kinds(s.get("body") or ()) | _kinds(s.get("else_body") or ())
    return out


def supported(ir) -> bool:
    """Whether an IR oracle exists for the package: one-warp fragment programs that stage
    operands through shared memory and multi-warp fragment programs have none (the golden
    vectors and the reference's own PTX pin them)."""
    pkg = load_package(ir)
    kinds = _kinds(pkg.body[0].body)
    if any(k.startswith(FRAGMENT) for k in kinds):
        warps = [a for a in pkg.body[0].axes if a.name.endswith(("_u", "_b")) and int(a.extent.value) > 1]
        return not (kinds & COOPERATIVE) and not warps
    return True


def ir_oracle(ir, arrays):
    pkg = load_package(ir)
    tile = pkg.body[0]
    kinds = _kinds(tile.body)
    if any(k.startswith(("Fragment", "RegFragment", "RegStore", "MmaSync", "Ldmatrix")) for k in kinds):
        from oracle import fragment_ir
        return fragment_ir.evaluate(ir, arrays)
    if tile.get("block_threads") or kinds & COOPERATIVE:
        from oracle import staged_ir
        return staged_ir.evaluate(ir, arrays)
    if kinds & {"Loop", "StridedLoop"}:
        from oracle import serial_ir
        return serial_ir.evaluate(ir, arrays)
    from oracle import pointwise_ir
    return pointwise_ir.evaluate(ir, arrays)
