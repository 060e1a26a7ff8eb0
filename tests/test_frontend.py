"""Frontend behaviour: the reference workloads lower unchanged, diagnostics, kernel selection."""
from __future__ import annotations

import importlib.util
import os
from pathlib import Path

import pytest

import ckl
from ckl.compile import plan_program
from ckl.compiler import CompilationError
from ckl.library import select
from ckl.frontend import FrontendError
from ckl.frontend.analysis import canonical_key, summarize
from ckl.workloads import decoder, vector_pipeline

# A checkout of the reference project, when one is at hand (CKL_REFERENCE_CHECKOUT).
REFERENCE = Path(os.environ.get("CKL_REFERENCE_CHECKOUT", "")) \
    if os.environ.get("CKL_REFERENCE_CHECKOUT") else None
linear = decoder.linear
fill, copy, update = vector_pipeline.fill, vector_pipeline.copy, vector_pipeline.update
N = ckl.dim("N")
Vector = ckl.Buffer[ckl.f32, (N,)]
SPEC = ckl.BufferSpec((16,), ckl.f32)


def load(path):
    spec = importlib.util.spec_from_file_location(path.stem + "_under_test", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


@pytest.mark.skipif(REFERENCE is None or not REFERENCE.exists(),
                    reason="set CKL_REFERENCE_CHECKOUT to a checkout of the reference project")
def test_reference_workloads_import_lower_and_match_the_library():
    ref = load(REFERENCE / "benchmarks" / "decoder" / "workloads.py")
    for name in ("embedding", "rms_stats", "rms_apply", "linear", "rope", "append_kv",
                 "attention_scores", "softmax", "attention_values", "add", "silu", "multiply",
                 "greedy", "advance"):
        assert canonical_key(getattr(ref, name)) == canonical_key(getattr(decoder, name)), name
    pipeline = load(REFERENCE / "examples" / "vector_pipeline.py")
    assert canonical_key(pipeline.update) == canonical_key(vector_pipeline.update)
    lowered = pipeline.lower()
    plans = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True)
    assert plans.primary.nodes == 1 and plans.fallback.nodes == 2


@ckl.kernel
def unknown_kernel(src: Vector, dst: Vector) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = src[i] * src[i] + 1.0


@ckl.program
def uses_unknown(src: Vector, dst: Vector) -> None:
    ckl.launch(unknown_kernel, src, dst, grid=(1,), block=(32,))


def test_unknown_kernel_is_generated_not_emulated():
    """A kernel outside the library becomes generated sm_100a code launched with the program's
    own geometry; selection alone still refuses it."""
    lowered = uses_unknown.lower(signature={"src": SPEC, "dst": SPEC})
    with pytest.raises(CompilationError, match="no sm_100a library implementation"):
        select(lowered.trace.dispatches[0])
    plans = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True)
    (name,) = plans.primary.node_names
    assert name.startswith("ckl_gen_unknown_kernel_")
    assert f"kernel 0 {name} 1 1 1 32 1 1 0" in plans.primary.text
    assert "binary hex 7f454c46" in plans.primary.text  # an ELF CUBIN
    assert f'extern "C" __global__ void {name}(float *p_src, float *p_dst)' in plans.device_ir


@ckl.program
def short_linear(x: ckl.Buffer[ckl.f32, (2, 64)], w: ckl.Buffer[ckl.f32, (1, 64, 256)],
                 y: ckl.Buffer[ckl.f32, (2, 256)]) -> None:
    ckl.launch(linear, x, w, y, 0, grid=(1, 2), block=(64,))


def test_partial_launch_runs_generated_code_with_its_own_geometry():
    lowered = short_linear.lower(signature={"x": ckl.BufferSpec((2, 64), ckl.f32),
                                            "w": ckl.BufferSpec((1, 64, 256), ckl.f32),
                                            "y": ckl.BufferSpec((2, 256), ckl.f32)})
    with pytest.raises(CompilationError, match="does not cover"):
        select(lowered.trace.dispatches[0])
    plan = plan_program(lowered, fuse_pointwise=False, fuse_library=False,
                        reuse_storage=True).primary
    (name,) = plan.node_names
    assert name.startswith("ckl_gen_linear_")
    assert f"kernel 0 {name} 1 2 1 64 1 1 0" in plan.text


@ckl.program
def partitions(storage: Vector, output: Vector) -> None:
    middle = ckl.subview(storage, offset=2, shape=(12,))
    left = ckl.subview(middle, offset=0, shape=(4,))
    right = ckl.subview(middle, offset=4, shape=(4,))
    overlap = ckl.subview(middle, offset=3, shape=(4,))
    ckl.launch(fill, left, 1.0, grid=(1,), block=(32,))
    ckl.launch(fill, right, 2.0, grid=(1,), block=(32,))
    ckl.launch(fill, overlap, 3.0, grid=(1,), block=(32,))
    ckl.launch(copy, storage, output, grid=(1,), block=(32,))


def test_subview_regions_give_disjoint_and_overlap_edges():
    """Restates tests/Python/test_subviews.py:52-66 on the native planner."""
    lowered = partitions.lower(signature={"storage": SPEC, "output": SPEC})
    plan = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True).primary
    assert plan.topology == {0: [], 1: [], 2: [0, 1], 3: [2]}
    for offset in (8, 24, 20):
        assert f"argres 0 {offset}" in plan.text


@ckl.program
def looping(src: Vector, dst: Vector, bias: ckl.f32) -> None:
    for _ in range(3):
        ckl.launch(update, src, dst, bias, grid=(1,), block=(32,))


def test_program_loops_unroll_and_effects_are_summarized():
    lowered = looping.lower(signature={"src": SPEC, "dst": SPEC, "bias": ckl.f32})
    assert len(lowered.trace.dispatches) == 3
    spec = lowered.specializations[0]
    summary = summarize(spec.definition, spec.signature)
    assert summary.bits[:2] == [1, 2] and summary.regions[:2] == ["whole", "whole"]
    kernel = decoder.advance
    signature = ckl.frontend.checker.bind(kernel, {"pos": ckl.BufferSpec((1,), ckl.i32)}, {})
    assert summarize(kernel, signature).regions[0] == (0, 4)


@ckl.program
def computes_scalar(src: Vector, dst: Vector, bias: ckl.f32) -> None:
    ckl.launch(update, src, dst, bias + 1.0, grid=(1,), block=(32,))


@ckl.program
def too_long(src: Vector, dst: Vector, bias: ckl.f32) -> None:
    for _ in range(1025):
        ckl.launch(update, src, dst, bias, grid=(1,), block=(32,))


def test_frontend_diagnostics():
    with pytest.raises(FrontendError, match="not Python callables"):
        vector_pipeline.update(1, 2, 3)
    with pytest.raises(FrontendError, match="lower a @ckl.program"):
        vector_pipeline.update.lower(signature={})
    with pytest.raises(FrontendError, match="computed runtime host scalars"):
        computes_scalar.lower(signature={"src": SPEC, "dst": SPEC, "bias": ckl.f32})
    with pytest.raises(FrontendError, match="1024"):
        too_long.lower(signature={"src": SPEC, "dst": SPEC, "bias": ckl.f32})
    with pytest.raises(FrontendError, match="conflicts"):
        vector_pipeline.step.lower(signature={"src": SPEC, "dst": ckl.BufferSpec((8,), ckl.f32),
                                              "bias": ckl.f32})
    with pytest.raises(FrontendError, match="missing or misplaced"):
        vector_pipeline.step.lower(signature={"src": SPEC, "dst": SPEC})
    with pytest.raises(ValueError):
        ckl.BufferSpec((0,), ckl.f32)
    with pytest.raises(ValueError):
        ckl.NVIDIATarget("sm_90a").chip and vector_pipeline.lower().compile(
            target=ckl.NVIDIATarget("sm_90a"))


def test_session_inputs_equal_oracle_inputs():
    import numpy as np
    from ckl.workloads import session
    from oracle import decoder as ref
    config = ref.Config(batch=3, hidden=48, heads=3, layers=1, ffn=80, vocab=129, context=3, steps=4)
    shape = session.DecoderShape(**vars(config))
    a, rng_a = session.make_weights(shape, 7)
    b, rng_b = ref.make_weights(config, 7)
    for name in b:
        assert np.array_equal(a[name], b[name]), name
    assert np.array_equal(session.make_prompts(shape, rng_a), ref.make_prompts(config, rng_b))
