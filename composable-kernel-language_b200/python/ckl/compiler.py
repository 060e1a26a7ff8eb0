"""Compilation targets and errors.

``NVIDIATarget`` keeps the reference's fields (``python/ckl/compiler.py:19-50``).  The B200
build emits no MLIR and runs no external ``ckl-opt``: device code is the hand-written sm_100a
kernel library linked into the native runtime, so the target only validates the chip.
"""
from __future__ import annotations

import hashlib
from collections.abc import Sequence
from dataclasses import dataclass
from pathlib import Path

SUPPORTED_CHIPS = ("sm_100a", "sm_100")


class CompilationError(RuntimeError):
    def __init__(self, command: Sequence[str], stderr: str):
        self.command = tuple(command)
        self.stderr = stderr
        super().__init__(f"CKL compilation failed: {' '.join(command)}\n{stderr}")


@dataclass(frozen=True)
class NVIDIATarget:
    chip: str = "sm_100a"
    features: str = ""
    toolkit_root: Path | None = None
    binary_format: str = "bin"

    def pipeline(self) -> str:
        return f"ckl-b200 sm_100a library chip={self.chip} features={self.features}"

    def environment(self) -> dict[str, str]:
        return {}

    def cache_identity(self) -> str:
        toolkit = str(Path(self.toolkit_root).resolve()) if self.toolkit_root else "environment"
        return f"nvidia:{self.chip}:{self.features}:{self.binary_format}:{toolkit}"


@dataclass(frozen=True)
class CompilerOptions:
    ckl_opt: Path | None = None
    passes: tuple = ()
    target: NVIDIATarget | None = None

    def command(self) -> tuple:
        return ("ckl-b200", *self.passes)


@dataclass(frozen=True)
class GPUObject:
    data: bytes
    format: int
    target: str


@dataclass(frozen=True)
class CompiledModule:
    source: str
    mlir: str
    command: tuple
    cache_key: str
    gpu_objects: tuple = ()


def compilation_key(source: str, command: Sequence[str]) -> str:
    return hashlib.sha256(source.encode() + b"\0" + "\0".join(command).encode()).hexdigest()


def extract_gpu_objects(source: str) -> tuple:
    """The B200 build embeds no GPU objects in textual IR."""
    return ()


def compile_module(source: str, options: CompilerOptions) -> CompiledModule:
    raise CompilationError(options.command(), "the B200 build has no external MLIR optimizer; "
                                              "use LoweredProgram.compile")
