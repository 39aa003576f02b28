"""Tensor formats of the hot path, mirroring JLUST's format algebra.

A format is a list of level keys over the dimensions (i, j) plus one level
kind per key, as in src/formats.jl:177-185 and src/named_formats.jl.  Only the
formats the backend consumes or produces are defined: COO, CSR, CSC, DCSR,
DCSC (capability queries), BSRRight / BSRLeft (named_formats.jl:106-130) and
DensedRight (named_formats.jl:219-227).

dim2lvl / lvl2dim follow src/formats.jl:190-230,429-440: a key is a dimension,
`i // b` or `i % b`; with as_size=True a `%` key evaluates to its divisor (the
level extent) and a `//` key to the floor quotient.
"""
from __future__ import annotations

from dataclasses import dataclass

DENSE, COMPRESSED, COMPRESSED_NONUNIQUE, SINGLETON = "dense", "compressed", "compressed(nonunique)", "singleton"


@dataclass(frozen=True)
class Key:
    dim: str                  # "i" or "j" (or further letters for dense N-d)
    op: str | None = None     # None, "div" or "mod"
    arg: int = 0

    def __str__(self):
        if self.op == "div":
            return f"{self.dim}÷{self.arg}"
        if self.op == "mod":
            return f"{self.dim}%{self.arg}"
        return self.dim


@dataclass(frozen=True)
class TensorFormat:
    name: str
    family: str
    dimensions: tuple
    keys: tuple
    levels: tuple
    block: tuple | None = None   # (b1, b2) for block formats
    diag: tuple | None = None    # (shift, val) for ShiftedDiag

    def __eq__(self, other):
        return (isinstance(other, TensorFormat) and self.dimensions == other.dimensions
                and self.keys == other.keys and self.levels == other.levels)

    def __hash__(self):
        return hash((self.dimensions, self.keys, self.levels))

    def __repr__(self):
        body = ", ".join(f"{k} : {lv}" for k, lv in zip(self.keys, self.levels))
        return f"{self.name}({', '.join(self.dimensions)}) -> ({body})"

    @property
    def is_dense(self) -> bool:
        return all(lv == DENSE for lv in self.levels)

    def ndims(self) -> int:
        return len(self.dimensions)


def _eval(key: Key, dims, idx, as_size):
    v = idx[dims.index(key.dim)]
    if key.op == "div":
        return v // key.arg
    if key.op == "mod":
        return key.arg if as_size else v % key.arg
    return v


def dim2lvl(fmt: TensorFormat, dim_indices, as_size: bool = False):
    """Level coordinates (or level extents with as_size) of a dimension coordinate."""
    return [_eval(k, fmt.dimensions, list(dim_indices), as_size) for k in fmt.keys]


def lvl2dim(fmt: TensorFormat, lvl_indices):
    """Inverse of dim2lvl for dimension, div and mod keys (formats.jl:433-440)."""
    out = [0] * len(fmt.dimensions)
    for k, v in zip(fmt.keys, lvl_indices):
        d = fmt.dimensions.index(k.dim)
        if k.op == "div":
            out[d] = v * k.arg
        elif k.op == "mod":
            out[d] += v
        else:
            out[d] = v
    return out


def level_extents(fmt: TensorFormat, extents):
    """Level extents used to lay the format out.  For block formats the
    block-row level has ceil(m / b1) entries (cuSPARSE's BSR layout; equal to
    JLUST's dim2lvl(as_size=true) quotient when b1 divides m)."""
    out = []
    for k in fmt.keys:
        e = extents[fmt.dimensions.index(k.dim)]
        if k.op == "div":
            out.append(-(-e // k.arg))
        elif k.op == "mod":
            out.append(k.arg)
        else:
            out.append(e)
    return out


class Formats:
    """Named formats (src/named_formats.jl)."""

    COO = TensorFormat("COO", "COO", ("i", "j"), (Key("i"), Key("j")),
                       (COMPRESSED_NONUNIQUE, SINGLETON))
    CSR = TensorFormat("CSR", "CSR", ("i", "j"), (Key("i"), Key("j")), (DENSE, COMPRESSED))
    CSC = TensorFormat("CSC", "CSC", ("i", "j"), (Key("j"), Key("i")), (DENSE, COMPRESSED))
    DCSR = TensorFormat("DCSR", "DCSR", ("i", "j"), (Key("i"), Key("j")), (COMPRESSED, COMPRESSED))
    DCSC = TensorFormat("DCSC", "DCSC", ("i", "j"), (Key("j"), Key("i")), (COMPRESSED, COMPRESSED))

    @staticmethod
    def ShiftedDiag(shift: int = 0, val: float = 1.0) -> TensorFormat:
        """Shifted scaled identity (src/named_formats.jl:53-60): row r holds one
        entry, `val` at column r + shift, and the tensor stores no buffers."""
        return TensorFormat(f"ShiftedDiag(shift={int(shift)},val={float(val)})", "ShiftedDiag",
                            ("i", "j"), (Key("i"), Key("j")),
                            (DENSE, f"shifted_diag({int(shift)},{float(val)!r})"),
                            None, (int(shift), float(val)))

    @staticmethod
    def BSRRight(blocksize) -> TensorFormat:
        b1, b2 = blocksize
        return TensorFormat(f"BSRRight{b1}x{b2}", "BSR", ("i", "j"),
                            (Key("i", "div", b1), Key("j", "div", b2), Key("i", "mod", b1),
                             Key("j", "mod", b2)),
                            (DENSE, COMPRESSED, DENSE, DENSE), (b1, b2))

    @staticmethod
    def BSRLeft(blocksize) -> TensorFormat:
        b1, b2 = blocksize
        return TensorFormat(f"BSRLeft{b1}x{b2}", "BSR", ("i", "j"),
                            (Key("i", "div", b1), Key("j", "div", b2), Key("j", "mod", b2),
                             Key("i", "mod", b1)),
                            (DENSE, COMPRESSED, DENSE, DENSE), (b1, b2))

    @staticmethod
    def DensedRight(n: int) -> TensorFormat:
        ds = tuple(chr(ord("i") + d) for d in range(n))
        return TensorFormat(f"Dense{n}Right", "Dense", ds, tuple(Key(d) for d in ds),
                            tuple(DENSE for _ in ds))

    @staticmethod
    def DensedLeft(n: int) -> TensorFormat:
        ds = tuple(chr(ord("i") + d) for d in range(n))
        return TensorFormat(f"Dense{n}Left", "Dense", ds, tuple(Key(d) for d in reversed(ds)),
                            tuple(DENSE for _ in ds))


def format_family(fmt: TensorFormat) -> str:
    return fmt.family


def is_bsr_right(fmt: TensorFormat) -> bool:
    return fmt.family == "BSR" and fmt.keys[2] == Key("i", "mod", fmt.block[0])
