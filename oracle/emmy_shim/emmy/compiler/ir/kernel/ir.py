"""Kernel-level IR nodes (tiles, cooperative statements, tensor and bulk nodes)."""
from __future__ import annotations

from ..base import IRNode, expressions, names
from ..expr import BinaryExpr, Expr, Literal, Var  # noqa: F401

# Fragment operand kinds and the environment names the tensor lowering binds.
FRAG, ROW, UNIFORM, COORD, GMEM = "frag", "row", "uniform", "coord", "gmem"
FRAG_ROW, FRAG_COL = "__frow", "__fcol"
ELEM_ROW, ELEM_COL = "__M__", "__N__"


class Dim(IRNode):
    _positional = ("value",)

    def as_static(self):
        return int(self.value)

    def __int__(self):
        return int(self.value)


class Window(IRNode):
    pass


class Axis(IRNode):
    _defaults = {"window": None}


class KernelOp(IRNode):
    _defaults = {"zero_delegated": (), "serial": ()}


class Tile(IRNode):
    _defaults = {"block_threads": None, "aux_threads": 0, "raster_axes": None,
                 "raster_group": None, "raster_orient": "m"}


class Smem(IRNode):
    pass


class Sync(IRNode):
    _defaults = {"barrier_id": 0, "count": None, "warp": False}


class WarpShuffle(IRNode):
    def deps(self):
        return names(self.state)


class TreeHalve(IRNode):
    def deps(self):
        return names(self.state)


class CpAsyncCopy(IRNode):
    _defaults = {"lane_index": None, "lane_rows": None, "swizzle": "NONE"}

    def exprs(self):
        return expressions((self.smem_index, self.src_index, self.lane_index))


class CpAsyncCommit(IRNode):
    pass


class CpAsyncWait(IRNode):
    _defaults = {"group": 0}


class MbarrierInit(IRNode):
    pass


class MbarrierArrive(IRNode):
    pass


class MbarrierArriveExpectTx(IRNode):
    pass


class MbarrierWait(IRNode):
    pass


class TmaDescriptor(IRNode):
    pass


class TmaLoad(IRNode):
    def exprs(self):
        return expressions(self.coords)


class RegFragment(IRNode):
    def defines(self):
        return (self.name,)


class LdmatrixLoad(IRNode):
    pass


class MmaSyncPtx(IRNode):
    pass


class RegStore(IRNode):
    pass


class FragLayout(IRNode):
    pass


class FragmentApply(IRNode):
    pass


class FragmentRepack(IRNode):
    pass


class FragmentRowReduce(IRNode):
    def defines(self):
        return names((self.top, self.bot))


def _m16n8_c_layout():
    """The m16n8k16 f32 C fragment: lane (g = lane/4, t = lane%4) holds rows g, g+8
    and columns 2t, 2t+1 — elements (g,2t), (g,2t+1), (g+8,2t), (g+8,2t+1)."""
    g, t = Var(name="_g"), Var(name="_t")
    col = lambda k: BinaryExpr(op="+", left=BinaryExpr(op="*", left=t, right=Literal(value=2, dtype="int")),  # noqa: E731
                               right=Literal(value=k, dtype="int"))
    return FragLayout(
        n_elems=4, elem_row=(0, 0, 1, 1), reduce_xors=(2, 1),
        lane_decl="const int _g = (threadIdx.x & 31) >> 2, _t = (threadIdx.x & 31) & 3;",
        lane_names=("_g", "_t"),
        row_off=(g, BinaryExpr(op="+", left=g, right=Literal(value=8, dtype="int"))),
        col_off=(col(0), col(1), col(0), col(1)))


M16N8 = _m16n8_c_layout()
