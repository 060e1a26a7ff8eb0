from .source import FrontendError, INTRINSICS, kernel, program
from .tracer import LoweredProgram

__all__ = ["FrontendError", "LoweredProgram", "kernel", "program"]
