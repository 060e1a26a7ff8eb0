"""Vector pipeline on the GPU: exact results, tails, fusion/fallback, rounding, subviews.

Ports of tests/Runtime/test_frontend_runtime.py, test_pointwise_fusion.py and
test_subviews_runtime.py, plus oracle parity at a size larger than L2.
"""
from __future__ import annotations

import gc
from array import array

import numpy as np
import pytest

import ckl
from ckl.workloads import vector_pipeline
from oracle import vector_pipeline as oracle
from test_frontend import partitions

pytestmark = pytest.mark.gpu
TARGET = ckl.NVIDIATarget("sm_100a")


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


@pytest.mark.parametrize("fuse", [False, True])
def test_257_elements_tails_biases_and_replays(device, fuse):
    compiled = vector_pipeline.lower().compile(target=TARGET, fuse_pointwise=fuse)
    full, spec = ckl.BufferSpec((512,), ckl.f32), ckl.BufferSpec((257,), ckl.f32)
    input_owner, output_owner = device.empty(full), device.empty(full)
    src = device.import_buffer(input_owner.address, spec, owner=input_owner)
    dst = device.import_buffer(output_owner.address, spec, owner=output_owner)
    initial = array("f", [i * 0.25 for i in range(257)] + [-12345.] * 255)
    blank = array("f", [-12345.] * 512)
    actual = array("f", blank)
    input_owner.copy_from_host(initial)
    for bias in (0.125, -0.5):
        bound = compiled.bind(src, dst, bias)
        assert bound.node_count == (1 if fuse else 2)
        for graph in (False, True, True, True):
            output_owner.copy_from_host(blank)
            bound.run(graph=graph)
            output_owner.copy_to_host(actual)
            expected = array("f", [v + 2 * bias for v in initial[:257]] + [-12345.] * 255)
            assert actual == expected
            input_owner.copy_to_host(actual)
            assert actual == initial
        for graph in (False, True):
            burst = bound.benchmark(iterations=3, graph=graph)
            assert burst["stream_us"] > 0 and burst["wall_us"] > 0
        for mode in ("ordinary", "capture", "graph"):
            output_owner.copy_from_host(blank)
            bound.run(mode=mode, batch_size=3)
            output_owner.copy_to_host(actual)
            assert actual == expected
    # Wrong signatures fail before the native ABI; mixed devices are rejected.
    for arguments in ((src, dst), (src, dst, "bad"), (input_owner, dst, 1.0)):
        with pytest.raises(TypeError):
            compiled.bind(*arguments)
    other = ckl.Device()
    with pytest.raises(ValueError):
        compiled.bind(src, other.empty(spec), 0.125)
    # The invocation retains code, buffers and their owners after the wrappers are gone.
    bound = compiled.bind(src, dst, 0.125)
    del compiled, src, dst, input_owner
    gc.collect()
    output_owner.copy_from_host(blank)
    bound.run(graph=True)
    output_owner.copy_to_host(actual)
    assert actual[:257] == array("f", [v + 0.25 for v in initial[:257]])
    with pytest.raises(ValueError, match="one million"):
        bound.run(mode="graph", batch_size=1000001)


@pytest.mark.parametrize("n", [257, 1 << 20])
def test_fusion_overlap_fallback_and_adjacent_slices(device, n):
    spec = ckl.BufferSpec((n,), ckl.f32)
    module = vector_pipeline.step.lower(signature={"src": spec, "dst": spec, "bias": ckl.f32})
    fused = module.compile(target=TARGET)
    baseline = module.compile(target=TARGET, fuse_pointwise=False)
    src, dst = device.empty(spec), device.empty(spec)
    initial = np.array([(i % 97) / 128 for i in range(n)], np.float32)
    expected = initial + np.float32(0.25)
    actual = np.zeros(n, np.float32)
    for compiled, nodes in ((fused, 1), (baseline, 2)):
        src.copy_from_host(initial)
        invocation = compiled.bind(src, dst, 0.125)
        assert invocation.node_count == nodes
        for graph in (False, True):
            invocation.run(graph=graph)
            dst.copy_to_host(actual)
            assert np.array_equal(actual, expected)
    owner = device.empty(ckl.BufferSpec((n + 2,), ckl.f32))
    overlap = fused.bind(device.import_buffer(owner.address, spec, owner=owner),
                         device.import_buffer(owner.address + 4, spec, owner=owner), 0.125)
    assert overlap.node_count == 2
    full = np.concatenate([initial, np.float32([-12345, -12345])])
    wanted = np.concatenate([initial[:1], expected, np.float32([-12345])])
    for graph in (False, True):
        owner.copy_from_host(full)
        overlap.run(graph=graph)
        out = np.zeros(n + 2, np.float32)
        owner.copy_to_host(out)
        assert np.array_equal(out, wanted)
    adjacent_owner = device.empty(ckl.BufferSpec((2 * n,), ckl.f32))
    a_src = device.import_buffer(adjacent_owner.address, spec, owner=adjacent_owner)
    a_dst = device.import_buffer(adjacent_owner.address + 4 * n, spec, owner=adjacent_owner)
    a_src.copy_from_host(initial)
    adjacent = fused.bind(a_src, a_dst, 0.125)
    assert adjacent.node_count == 1
    adjacent.run(graph=True)
    a_dst.copy_to_host(actual)
    assert np.array_equal(actual, expected)
    exact = fused.bind(src, src, 0.125)
    assert exact.node_count == 2
    src.copy_from_host(initial)
    exact.run(graph=True)
    src.copy_to_host(actual)
    assert np.array_equal(actual, expected)


N = ckl.dim("N")
Vector = ckl.Buffer[ckl.f32, (N,)]
scale, update = vector_pipeline.scale, vector_pipeline.update


@ckl.program
def rounding(src: Vector, dst: Vector, factor: ckl.f32, bias: ckl.f32) -> None:
    temp = ckl.empty_like(src)
    ckl.launch(scale, src, temp, factor, grid=(ckl.cdiv(N, 256),), block=(256,))
    ckl.launch(update, temp, dst, bias, grid=(ckl.cdiv(N, 256),), block=(256,))


def test_fusion_keeps_float32_rounding(device):
    """Multiply-then-add through a fused chain must not contract (result exactly 0)."""
    spec = ckl.BufferSpec((257,), ckl.f32)
    p = rounding.lower(signature={"src": spec, "dst": spec, "factor": ckl.f32,
                                  "bias": ckl.f32}).compile(target=TARGET)
    src, dst = device.empty(spec), device.empty(spec)
    src.copy_from_host(np.full(257, 1 + 2 ** -23, np.float32))
    invocation = p.bind(src, dst, 1 - 2 ** -23, -1.)
    assert invocation.node_count == 1
    for graph in (False, True):
        invocation.run(graph=graph)
        out = np.ones(257, np.float32)
        dst.copy_to_host(out)
        assert out.tobytes() == np.zeros(257, np.float32).tobytes()


def test_subview_partitions(device):
    spec = ckl.BufferSpec((16,), ckl.f32)
    program = partitions.lower(signature=dict(storage=spec, output=spec)).compile(target=TARGET)
    owner = device.empty(ckl.BufferSpec((32,), ckl.f32))
    storage = owner.subview(offset=4, shape=(20,)).subview(offset=0, shape=(16,))
    output = device.empty(spec)
    expected = [-99., -99., 1., 1., 1., 3., 3., 3., 3., 2.] + [-99.] * 6
    bound = program.bind(storage, output)
    for mode in ("ordinary", "graph", "capture"):
        owner.copy_from_host(np.full(32, -99., np.float32))
        output.copy_from_host(np.full(16, -1., np.float32))
        bound.run(mode=mode, batch_size=3)
        out = np.zeros(16, np.float32)
        output.copy_to_host(out)
        assert out.tolist() == expected
        whole = np.zeros(32, np.float32)
        owner.copy_to_host(whole)
        assert whole[:4].tolist() == [-99.] * 4 and whole[20:].tolist() == [-99.] * 12
    with pytest.raises(ValueError):
        storage.subview(offset=15, shape=(2,))


def test_large_vector_matches_oracle(device):
    n = 1 << 26  # 256 MiB per buffer: larger than L2
    spec = ckl.BufferSpec((n,), ckl.f32)
    src_host = oracle.make_source(n, 1)
    expected = oracle.pipeline(src_host, 0.5)
    program = vector_pipeline.step.lower(signature={"src": spec, "dst": spec, "bias": ckl.f32})
    src, dst = device.empty(spec), device.empty(spec)
    src.copy_from_host(src_host)
    for fuse in (True, False):
        bound = program.compile(target=TARGET, fuse_pointwise=fuse).bind(src, dst, 0.5)
        bound.run(graph=True)
        out = np.empty(n, np.float32)
        dst.copy_to_host(out)
        assert out.tobytes() == expected.tobytes()
