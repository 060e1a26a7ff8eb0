"""Source-level CKL types: scalars, named dimensions, buffer and constexpr annotations.

Mirrors the reference's public type surface (``python/ckl/types.py:8-90``): the same names,
the same validation and the same error class (``ValueError``) for malformed annotations.
"""
from __future__ import annotations

from dataclasses import dataclass

_MAX_EXTENT = 1 << 63


@dataclass(frozen=True)
class ScalarType:
    name: str

    @property
    def mlir(self) -> str:
        """The element spelling used in textual IR (``bool`` prints as ``i1``)."""
        return "i1" if self.name == "bool" else self.name

    @property
    def bytes(self) -> int:
        return {"f32": 4, "i32": 4, "f64": 8, "i64": 8, "index": 8, "bool": 1}[self.name]


f32 = ScalarType("f32")
f64 = ScalarType("f64")
i32 = ScalarType("i32")
i64 = ScalarType("i64")
index = ScalarType("index")
bool_ = ScalarType("bool")
NUMERIC_TYPES = (f32, f64, i32, i64)
SCALAR_TYPES = NUMERIC_TYPES + (index, bool_)


@dataclass(frozen=True)
class Dimension:
    """A named extent, bound to an integer when a program is specialized."""

    name: str

    def __post_init__(self) -> None:
        if not (isinstance(self.name, str) and self.name.isidentifier()):
            raise ValueError("dimension names must be Python identifiers")


def dim(name: str) -> Dimension:
    return Dimension(name)


def _valid_extent(value: object) -> bool:
    return isinstance(value, Dimension) or (type(value) is int and 0 < value < _MAX_EXTENT)


@dataclass(frozen=True)
class BufferType:
    dtype: ScalarType
    shape: tuple

    def __post_init__(self) -> None:
        if self.dtype not in NUMERIC_TYPES:
            raise ValueError("buffer elements must be f32, f64, i32, or i64")
        if not isinstance(self.shape, tuple) or not all(_valid_extent(d) for d in self.shape):
            raise ValueError(
                "buffer shapes must be tuples of positive extents within i64 or dimensions")


class Buffer:
    """``Buffer[element_type, shape_tuple]`` builds a :class:`BufferType` annotation."""

    def __class_getitem__(cls, arguments):
        if not (isinstance(arguments, tuple) and len(arguments) == 2):
            raise ValueError("use Buffer[element_type, shape_tuple]")
        return BufferType(arguments[0], arguments[1])


@dataclass(frozen=True)
class ConstexprType:
    dtype: ScalarType

    def __post_init__(self) -> None:
        if self.dtype not in SCALAR_TYPES:
            raise ValueError("constexpr requires a CKL scalar type")


class constexpr:
    """``constexpr[scalar_type]`` marks a parameter bound at specialization time."""

    def __class_getitem__(cls, dtype):
        return ConstexprType(dtype)


@dataclass(frozen=True)
class BufferSpec:
    """A concrete, contiguous buffer type used in signatures and allocations."""

    shape: tuple
    dtype: ScalarType
    layout: str = "identity"

    def __post_init__(self) -> None:
        BufferType(self.dtype, self.shape)
        if not all(type(d) is int for d in self.shape):
            raise ValueError("BufferSpec requires concrete integer extents")
        if self.layout != "identity":
            raise ValueError("only contiguous identity-layout buffers are supported")

    @property
    def mlir(self) -> str:
        return "memref<" + "".join(f"{d}x" for d in self.shape) + self.dtype.mlir + ">"

    @property
    def elements(self) -> int:
        count = 1
        for extent in self.shape:
            count *= extent
        return count

    @property
    def nbytes(self) -> int:
        return self.elements * self.dtype.bytes
