"""CKL on B200: the reference's kernel/program authoring API over an sm_100a runtime."""
from .compiler import (CompilationError, CompiledModule, CompilerOptions, GPUObject,
                       NVIDIATarget, extract_gpu_objects)
from .frontend import FrontendError, LoweredProgram, kernel, program
from .cuda import (CompiledProgram, Completion, Device, DeviceBuffer, Invocation,
                   PinnedHostBuffer)
from .frontend.source import INTRINSICS as _intrinsics
from .plan_io import load as load_program
from .types import Buffer, BufferSpec, constexpr, dim, f32, f64, i32, i64, index
from .types import bool_ as bool

globals().update(_intrinsics)

__all__ = [
    "CompilationError", "CompiledModule", "CompilerOptions", "GPUObject", "NVIDIATarget",
    "CompiledProgram", "Completion", "Device", "DeviceBuffer", "Invocation", "PinnedHostBuffer",
    "extract_gpu_objects", "load_program",
    "Buffer", "BufferSpec", "constexpr", "dim", "f32", "f64", "i32", "i64", "index", "bool",
    "FrontendError", "LoweredProgram", "kernel", "program", *_intrinsics,
]
