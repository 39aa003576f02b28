"""Operation tags (src/ops.jl:45-138).

`SpMVOp(A_fmt, x_fmt, y_fmt)` builds an Op instance carrying the operand
formats, exactly like the reference's parametric singleton `Op{Tag, Formats}`.
Capability queries dispatch on (tag, formats) alone.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Op:
    tag: str
    formats: tuple

    def __repr__(self):
        return f"{self.tag}Op({', '.join(f.name for f in self.formats)})"


class OpType:
    """A named op (the reference's `const SpMVOp = Op{:SpMV}`)."""

    def __init__(self, tag: str, doc: str):
        self.tag = tag
        self.__doc__ = doc

    def __call__(self, *formats) -> Op:
        return Op(self.tag, tuple(formats))

    def __repr__(self):
        return f"{self.tag}Op"


SpVVOp = OpType("SpVV", "Sparse vector dot product.")
SpMVOp = OpType("SpMV", "y = alpha*A*x + beta*y (src/ops.jl:71-73).")
SpMMOp = OpType("SpMM", "C = alpha*A*B + beta*C (src/ops.jl:75-77).")
BatchedSpMMOp = OpType("BatchedSpMM", "Batched SpMM.")
SpGEMMOp = OpType("SpGEMM", "Sparse x sparse product.")
SpSVOp = OpType("SpSV", "Sparse triangular solve.")
SpSMOp = OpType("SpSM", "Sparse triangular solve, many right-hand sides.")
SDDMMOp = OpType("SDDMM", "C = alpha*(A*B) o spy(C) + beta*C (src/ops.jl:95-97).")
SparseToDenseOp = OpType("SparseToDense", "Sparse to dense.")
DenseToSparseOp = OpType("DenseToSparse", "Dense to sparse.")
BlockSpMVOp = OpType("BlockSpMV", "Block sparse matrix x vector (src/ops.jl:128-130).")
BlockSpMMOp = OpType("BlockSpMM", "Block sparse matrix x dense matrix (src/ops.jl:132-134).")
BBMSpMVOp = OpType("BBMSpMV", "Block-banded matrix x vector.")


def op_tag(op) -> str:
    return op.tag
