"""Import location of the reference's emitter names (``ckl.frontend.emitter``).

Harness code imports ``identity`` and ``LoweredProgram`` from here
(``benchmarks/decoder/experiment.py:11``); the B200 build traces programs in
:mod:`ckl.frontend.tracer` instead of emitting MLIR.
"""
from .tracer import LoweredProgram, Specialization, identity, lower_program

__all__ = ["LoweredProgram", "Specialization", "identity", "lower_program"]
