"""Element types as the IR spells them: DataType(name, np, nbytes)."""
from __future__ import annotations

import numpy as np

from .ir.base import IRNode


class DataType(IRNode):
    pass


F16 = DataType(name="f16", np=np.dtype("float16"), nbytes=2)
BF16 = DataType(name="bf16", np=np.dtype("float32"), nbytes=2)
F32 = DataType(name="f32", np=np.dtype("float32"), nbytes=4)
F64 = DataType(name="f64", np=np.dtype("float64"), nbytes=8)
I32 = DataType(name="i32", np=np.dtype("int32"), nbytes=4)
