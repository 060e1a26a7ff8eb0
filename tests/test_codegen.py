"""Generated kernels (CPU): typing rules and diagnostics of the reference's kernel emitter,
the emitted CUDA text, NVRTC compilation to an sm_100a CUBIN, and plans mixing library and
generated kernels.

The diagnostics restate ``python/ckl/frontend/emitter.py:181-726`` (explicit casts between
typed values, no integer division, branch results deferred, loop-carried scalars); the
arithmetic contract restates ``tests/Runtime/test_pointwise_fusion.py:105-118`` (no multiply-add
contraction) and ``tests/Runtime/test_kernel_loops.py`` (zero-trip and multi-carried loops).
"""
from __future__ import annotations

import pytest

import ckl
from ckl import _native, codegen
from ckl.compile import plan_program
from ckl.frontend import FrontendError
from ckl.workloads import decoder, vector_pipeline

update = vector_pipeline.update

N = ckl.dim("N")
Vector = ckl.Buffer[ckl.f32, (N,)]
Doubles = ckl.Buffer[ckl.f64, (4,)]
SPEC = ckl.BufferSpec((16,), ckl.f32)


def generated(kernel, signature, constants=None):
    """Lower a one-launch program around `kernel` and return its generated source."""
    spec = ckl.frontend.checker.bind(kernel, signature, constants or {})
    from ckl.frontend.tracer import identity
    return codegen.generate(kernel, spec, identity(kernel, spec)).source


@ckl.kernel
def fused_multiply_add(src: Vector, dst: Vector, factor: ckl.f32, bias: ckl.f32) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = src[i] * factor + bias


def test_float_arithmetic_rounds_every_operation():
    text = generated(fused_multiply_add, {"src": SPEC, "dst": SPEC, "factor": ckl.f32,
                                          "bias": ckl.f32})
    assert "__fmul_rn(" in text and "__fadd_rn(" in text
    assert "fmaf" not in text and "__fmaf" not in text


@ckl.kernel
def constants(dst: ckl.Buffer[ckl.f32, (2,)], wide: ckl.Buffer[ckl.i64, (1,)]) -> None:
    if ckl.global_id(0) == 0:
        dst[0] = dst[0] + 0.1
        dst[1] = dst[1] * -2.5
        wide[0] = wide[0] + -1099511627779


def test_constants_are_exact_bit_patterns():
    text = generated(constants, {"dst": ckl.BufferSpec((2,), ckl.f32),
                                 "wide": ckl.BufferSpec((1,), ckl.i64)})
    assert "__int_as_float(0x3dcccccd)" in text          # 0.1 rounded to f32
    assert "__int_as_float(0xc0200000)" in text          # -2.5
    assert "((long long)0xfffffefffffffffdull)" in text   # -(2**40 + 3) as i64


@ckl.kernel
def statistics(src: Doubles, dst: Doubles, count: ckl.i32) -> None:
    if ckl.global_id(0) == 0:
        total = src[0] * 0.0
        maximum = src[0]
        winner = count * 0
        for i in range(ckl.cast(count, ckl.index)):
            value = src[i]
            wins = value > maximum
            winner = ckl.select(wins, ckl.cast(i, ckl.i32), winner)
            maximum = ckl.select(wins, value, maximum)
            total = total + value
        dst[0] = total
        dst[1] = ckl.exp(maximum) * ckl.rsqrt(maximum * maximum + 1.0)
        dst[2] = ckl.cast(winner, ckl.f64)


def test_loop_carries_every_reassigned_outer_name():
    spec = ckl.BufferSpec((4,), ckl.f64)
    text = generated(statistics, {"src": spec, "dst": spec, "count": ckl.i32})
    # Three carried scalars (total, maximum, winner) declared before the loop.
    assert text.count("double c") == 2 and text.count("int c") == 1
    assert "exp(" in text and "rsqrt(" in text and "expf(" not in text


def _error(kernel, signature, constants=None):
    with pytest.raises(FrontendError) as info:
        generated(kernel, signature, constants)
    return str(info.value)


@ckl.kernel
def mixed_types(src: Vector, dst: Vector, count: ckl.i32) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = src[i] + count


@ckl.kernel
def integer_division(src: ckl.Buffer[ckl.i32, (4,)], dst: ckl.Buffer[ckl.i32, (4,)]) -> None:
    i = ckl.global_id(0)
    if i < 4:
        dst[i] = src[i] / 2


@ckl.kernel
def branch_result(src: Vector, dst: Vector) -> None:
    i = ckl.global_id(0)
    value = 0.0
    if i < N:
        value = src[i]
    dst[0] = value


@ckl.kernel
def branch_local_escapes(src: Vector, dst: Vector) -> None:
    i = ckl.global_id(0)
    if i < N:
        inner = src[i]
    dst[0] = inner


@ckl.kernel
def chained(src: Vector, dst: Vector) -> None:
    i = ckl.global_id(0)
    if 0 < i < N:
        dst[i] = src[i]


@ckl.kernel
def modulo(src: Vector, dst: Vector) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i % 4] = src[i]


@ckl.kernel
def integer_exp(src: ckl.Buffer[ckl.i32, (4,)], dst: ckl.Buffer[ckl.i32, (4,)]) -> None:
    i = ckl.global_id(0)
    if i < 4:
        dst[i] = ckl.exp(src[i])


@ckl.kernel
def index_to_float(dst: Vector) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = ckl.cast(i, ckl.f32)


@ckl.kernel
def static_select(dst: Vector) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = ckl.select(i < 4, 1.0, 2.0)


@ckl.kernel
def out_of_bounds(dst: Vector) -> None:
    dst[16] = 1.0


@ckl.kernel
def assigns_induction(dst: Vector) -> None:
    for i in range(4):
        i = i + 1
        dst[0] = 1.0


@ckl.kernel
def float_predicate(src: Vector, dst: Vector) -> None:
    i = ckl.global_id(0)
    if src[0]:
        dst[i] = 1.0


@ckl.kernel
def launches_inside(dst: Vector) -> None:
    ckl.launch(index_to_float, dst, grid=(1,), block=(1,))


@pytest.mark.parametrize("kernel,signature,message", [
    (mixed_types, {"src": SPEC, "dst": SPEC, "count": ckl.i32}, "expected f32, got i32"),
    (integer_division, {"src": ckl.BufferSpec((4,), ckl.i32), "dst": ckl.BufferSpec((4,), ckl.i32)},
     "division requires floating operands"),
    (branch_result, {"src": SPEC, "dst": SPEC}, "runtime branch results are deferred"),
    (branch_local_escapes, {"src": SPEC, "dst": SPEC}, "local 'inner' is not defined on this path"),
    (chained, {"src": SPEC, "dst": SPEC}, "chained comparisons are not supported"),
    (modulo, {"src": SPEC, "dst": SPEC}, "unsupported numeric operator: Mod"),
    (integer_exp, {"src": ckl.BufferSpec((4,), ckl.i32), "dst": ckl.BufferSpec((4,), ckl.i32)},
     "exp requires one typed floating-point scalar"),
    (index_to_float, {"dst": SPEC}, "cast through an integer type"),
    (static_select, {"dst": SPEC}, "select requires a typed scalar alternative"),
    (out_of_bounds, {"dst": SPEC}, "constant index is out of bounds for dimension 0"),
    (assigns_induction, {"dst": SPEC}, "cannot assign to the loop induction variable"),
    (float_predicate, {"src": SPEC, "dst": SPEC}, "if requires a boolean predicate"),
    (launches_inside, {"dst": SPEC}, "kernels cannot launch other kernels"),
])
def test_invalid_bodies_get_the_reference_diagnostics(kernel, signature, message):
    assert message in _error(kernel, signature)


@ckl.program
def uses_invalid(src: Vector, dst: Vector, count: ckl.i32) -> None:
    ckl.launch(mixed_types, src, dst, count, grid=(1,), block=(16,))


def test_invalid_bodies_fail_when_the_program_is_lowered():
    with pytest.raises(FrontendError, match="use ckl.cast explicitly"):
        uses_invalid.lower(signature={"src": SPEC, "dst": SPEC, "count": ckl.i32})


def test_nvrtc_builds_an_sm100a_cubin_and_reports_errors():
    cubin = _native.compile_cuda('extern "C" __global__ void probe(float *x) { x[0] = 1.f; }')
    assert cubin[:4] == b"\x7fELF" and b"probe" in cubin
    with pytest.raises(ValueError, match="NVRTC compilation failed"):
        _native.compile_cuda('extern "C" __global__ void broken(float *x) { x[0] = ; }')


def test_every_workload_kernel_generates_and_compiles():
    """All decoder and vector-pipeline kernel bodies translate and compile together (this is
    the program compiled with library=False)."""
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).parent))
    from oracle import decoder as ref
    from test_planner import decoder_signature
    config = ref.Config(batch=2, hidden=64, heads=4, layers=2, ffn=256, vocab=512, context=16,
                        steps=2)
    lowered = decoder.decode.lower(signature=decoder_signature(config))
    plans = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True,
                         library=False)
    assert plans.fallback is None                      # nothing to fuse: no library nodes
    assert plans.primary.nodes == 21 * config.layers + 6
    assert all(name.startswith("ckl_gen_") for name in plans.primary.node_names)
    assert plans.primary.text.count("binary hex 7f454c46") == 1
    for name in set(plans.primary.node_names):
        assert f"__global__ void {name}(" in plans.device_ir
    pipeline = vector_pipeline.lower()
    plans = plan_program(pipeline, fuse_pointwise=True, fuse_library=True, reuse_storage=True,
                         library=False)
    assert plans.primary.nodes == 2 and plans.fallback is None


@ckl.program
def mixed(src: Vector, dst: Vector, factor: ckl.f32, bias: ckl.f32) -> None:
    temp = ckl.empty_like(src)
    ckl.launch(update, src, temp, bias, grid=(1,), block=(32,))
    ckl.launch(fused_multiply_add, temp, dst, factor, bias, grid=(1,), block=(32,))


def test_plans_mix_library_and_generated_kernels():
    lowered = mixed.lower(signature={"src": SPEC, "dst": SPEC, "factor": ckl.f32,
                                     "bias": ckl.f32})
    plan = plan_program(lowered, fuse_pointwise=True, fuse_library=True,
                        reuse_storage=True).primary
    library_name, generated_name = plan.node_names
    assert library_name == "ckl.pointwise.add_scalar"
    assert generated_name.startswith("ckl_gen_fused_multiply_add_")
    assert plan.topology == {1: [], 2: [1]}
    assert "binary hex 7f454c46" in plan.text
