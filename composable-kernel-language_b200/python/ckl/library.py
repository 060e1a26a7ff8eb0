"""Catalogue of the sm_100a kernel library: which CKL kernels it implements and how to call them.

A dispatch is served by a library kernel when the dispatched kernel's canonical structure
(:func:`ckl.frontend.analysis.canonical_key`) equals that of one of the DSL definitions in
:mod:`ckl.workloads` and the launch covers the kernel's whole index space (so the library's
own launch geometry computes exactly the reference launch's effect).  Unknown kernels are
rejected at compile time; there is no fallback code path.

Each entry packs the dispatch into the native kernel's argument slots (its runtime operands
in order) followed by a specialization struct of int64 fields (``csrc/kernels/common.cuh``).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from functools import lru_cache
from typing import Callable

from .compiler import CompilationError
from .frontend.analysis import canonical_key
from .types import BufferSpec


def pack(*fields: int) -> bytes:
    return struct.pack(f"<{len(fields)}q", *(int(f) for f in fields))


@dataclass(frozen=True)
class Entry:
    """One library kernel implementing one CKL kernel body."""

    native: str
    source: str                                   # DSL definition the entry implements
    spec: Callable                                # (shapes, constants, extents) -> bytes
    covers: Callable                              # (shapes, extents) -> bool
    pointwise_op: int = -1                        # chain op code for pointwise fusion


def _extents(grid, block):
    return tuple(g * b for g, b in zip(grid, block))


def _gemm(M, K, N, layers, layer, A=0, D=0, T=0, tiles=0, config=0):
    return pack(M, K, N, layers, layer, A, D, T, tiles, config, M)


# Shapes are the runtime buffer operands' shapes in parameter order; constants are the
# constexpr values in parameter order; extents are the launch's global sizes per axis.
def _decoder_entries():
    E = []
    E.append(Entry("ckl.decoder.embedding", "embedding",
                   lambda s, k, e: pack(s[0][0], s[2][1], s[1][0]),
                   lambda s, e: e[0] >= s[2][1] and e[1] == s[2][0]))
    E.append(Entry("ckl.decoder.rms_stats", "rms_stats",
                   lambda s, k, e: pack(s[0][0], s[0][1]),
                   lambda s, e: e[0] >= s[0][0]))
    E.append(Entry("ckl.decoder.rms_apply", "rms_apply",
                   lambda s, k, e: pack(s[0][0], s[0][1], s[2][0], k[0]),
                   lambda s, e: e[0] >= s[0][1] and e[1] == s[0][0]))
    E.append(Entry("ckl.decoder.linear", "linear",
                   lambda s, k, e: _gemm(s[0][0], s[0][1], s[1][2], s[1][0], k[0]),
                   lambda s, e: e[0] >= s[1][2] and e[1] == s[0][0]))

    def rope_heads(s):
        c, r = s[0][1], s[1][1]
        return c // (2 * r) if c % (2 * r) == 0 else -1
    E.append(Entry("ckl.decoder.rope", "rope",
                   lambda s, k, e: pack(s[0][0], s[0][1], rope_heads(s), s[1][1], s[1][0]),
                   lambda s, e: rope_heads(s) > 0 and e[0] >= s[1][1] and e[1] == rope_heads(s)
                   and e[2] == s[0][0]))
    E.append(Entry("ckl.decoder.append_kv", "append_kv",
                   lambda s, k, e: pack(s[0][0], s[0][1], s[2][0], s[2][2], s[2][3], s[2][4], k[0]),
                   lambda s, e: e[0] >= s[2][4] and e[1] == s[2][2] and e[2] == s[2][1]
                   and s[2][1] == s[0][0]))
    E.append(Entry("ckl.decoder.attention_scores", "attention_scores",
                   lambda s, k, e: pack(s[0][0], s[0][1], s[1][0], s[1][2], s[1][3], s[1][4], k[0]),
                   lambda s, e: e[0] >= s[1][3] and e[1] == s[1][2] and e[2] == s[1][1]
                   and s[1][1] == s[0][0]))
    E.append(Entry("ckl.decoder.softmax", "softmax",
                   lambda s, k, e: pack(s[0][0], s[0][1], s[0][2]),
                   lambda s, e: e[0] >= s[0][0] and e[1] == s[0][1]))
    E.append(Entry("ckl.decoder.attention_values", "attention_values",
                   lambda s, k, e: pack(s[3][0], s[3][1], s[1][0], s[1][2], s[1][3], s[1][4], k[0]),
                   lambda s, e: e[0] >= s[1][4] and e[1] == s[1][2] and e[2] == s[1][1]
                   and s[1][1] == s[3][0]))
    for name in ("add", "multiply", "silu"):
        E.append(Entry(f"ckl.decoder.{name}", name,
                       lambda s, k, e: pack(s[0][0], s[0][1]),
                       lambda s, e: e[0] >= s[0][1] and e[1] == s[0][0]))
    E.append(Entry("ckl.decoder.greedy", "greedy",
                   lambda s, k, e: pack(s[0][0], s[0][1], s[2][0]),
                   lambda s, e: e[0] >= s[0][0]))
    E.append(Entry("ckl.decoder.advance", "advance",
                   lambda s, k, e: b"",
                   lambda s, e: e[0] * e[1] * e[2] == 1))
    return E


def _pointwise_entries():
    def spec(s, k, e):
        n = s[0][0]
        return pack(n, min(n, e[0]))
    return [Entry("ckl.pointwise.add_scalar", "update", spec, lambda s, e: True, pointwise_op=0),
            Entry("ckl.pointwise.mul_scalar", "scale", spec, lambda s, e: True, pointwise_op=1),
            Entry("ckl.pointwise.fill", "fill", spec, lambda s, e: True),
            Entry("ckl.pointwise.copy", "copy", spec, lambda s, e: True)]


@lru_cache(maxsize=1)
def catalogue() -> dict:
    """Canonical key -> Entry for every library kernel."""
    from .workloads import decoder, vector_pipeline

    sources = {**{name: getattr(decoder, name) for name in (
        "embedding", "rms_stats", "rms_apply", "linear", "rope", "append_kv",
        "attention_scores", "softmax", "attention_values", "add", "silu", "multiply",
        "greedy", "advance")},
        "update": vector_pipeline.update, "scale": vector_pipeline.scale,
        "fill": vector_pipeline.fill, "copy": vector_pipeline.copy}
    table = {}
    for entry in _decoder_entries() + _pointwise_entries():
        table[canonical_key(sources[entry.source])] = entry
    return table


@dataclass
class Selection:
    """A dispatch resolved to a library kernel."""

    entry: Entry
    spec: bytes


def select(dispatch) -> Selection:
    """Resolve one traced dispatch or raise :class:`CompilationError`."""
    spec_ = dispatch.specialization
    definition = spec_.definition
    key = _key(definition)
    entry = catalogue().get(key)
    if entry is None:
        raise CompilationError(("ckl-b200", "select"),
                               f"kernel '{definition.name}' ({dispatch.location}) has no sm_100a "
                               "library implementation")
    shapes = [p.dtype.shape for p in spec_.signature.parameters
              if not p.is_constant and isinstance(p.dtype, BufferSpec)]
    constants = [p.value for p in spec_.signature.parameters if p.is_constant]
    extents = _extents(dispatch.grid, dispatch.block)
    if not entry.covers(shapes, extents):
        raise CompilationError(("ckl-b200", "select"),
                               f"launch of '{definition.name}' ({dispatch.location}) with grid "
                               f"{dispatch.grid} block {dispatch.block} does not cover the kernel's "
                               "index space; the library implements whole-space launches only")
    return Selection(entry, entry.spec(shapes, constants, extents))


_KEYS: dict = {}


def _key(definition) -> str:
    key = _KEYS.get(definition.identity)
    if key is None:
        key = _KEYS[definition.identity] = canonical_key(definition)
    return key
