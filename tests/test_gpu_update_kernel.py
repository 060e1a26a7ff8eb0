"""Kernel nodes of an instantiated explicit graph are updated in place.

Restates the reference's runtime validation of ``NvidiaGraphExecutable::updateKernel``
(``tests/Runtime/NvidiaRuntimeValidation.cpp:279-286``, ``lib/Runtime/NvidiaRuntime.cpp:466-496``):
a node of the cached explicit graph gets new launch parameters without re-instantiation, the
next graph launch computes with them (checked against NumPy bit for bit), a captured graph is
rejected, and an update naming an unknown node or a slot of the wrong size fails cleanly.
Here the updates change scalars, re-point a node at another buffer (running the same graph on
a new request slice without rebuilding it), update one repetition of a repeated graph, and
re-derive a tensor-core projection's TMA weight map from a new weight pointer.
"""
from __future__ import annotations

import numpy as np
import pytest

import ckl
from ckl.workloads import session as S, vector_pipeline
from oracle import decoder as ref

pytestmark = pytest.mark.gpu
N = 1 << 20


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


def buffers(device, values):
    spec = ckl.BufferSpec((N,), ckl.f32)
    src, dst, other = device.empty(spec), device.empty(spec), device.empty(spec)
    src.copy_from_host(values)
    for buffer in (dst, other):
        buffer.copy_from_host(np.zeros(N, np.float32))
    return src, dst, other


def read(buffer):
    out = np.empty(N, np.float32)
    buffer.copy_to_host(out)
    return out


def pipeline(values, *biases):
    out = values
    for bias in biases:
        out = out + np.float32(bias)
    return out


def test_fused_node_gets_new_scalars_and_output_buffer(device):
    values = np.random.default_rng(3).uniform(-1, 1, N).astype(np.float32)
    src, dst, other = buffers(device, values)
    inv = vector_pipeline.lower(N).compile(target=ckl.NVIDIATarget("sm_100a")).bind(src, dst, 0.5)
    assert inv.node_count == 1 and inv.node_names == ["ckl.pointwise.chain2"]
    inv.run(mode="graph")
    assert read(dst).tobytes() == pipeline(values, 0.5, 0.5).tobytes()
    sizes = inv.node_argument_sizes(0)
    assert sizes[:4] == [8, 8, 4, 4]
    # New biases and a new destination; the source and specialization stay.
    inv.update_kernel(0, [None, other, np.float32(0.25), np.float32(-2.0), None])
    inv.run(mode="graph")
    assert read(other).tobytes() == pipeline(values, 0.25, -2.0).tobytes()
    assert read(dst).tobytes() == pipeline(values, 0.5, 0.5).tobytes()  # untouched
    # Ordinary launches keep the bound plan (the update belongs to that graph).
    dst.copy_from_host(np.zeros(N, np.float32))
    inv.run(mode="ordinary")
    assert read(dst).tobytes() == pipeline(values, 0.5, 0.5).tobytes()


def test_unfused_node_and_repeated_graph(device):
    values = np.random.default_rng(4).uniform(-1, 1, N).astype(np.float32)
    src, dst, _ = buffers(device, values)
    inv = vector_pipeline.lower(N).compile(target=ckl.NVIDIATarget("sm_100a"),
                                           fuse_pointwise=False).bind(src, dst, 0.5)
    assert inv.node_count == 2
    inv.update_kernel(1, [None, None, np.float32(3.0), None])  # second launch's bias
    inv.run(mode="graph")
    assert read(dst).tobytes() == pipeline(values, 0.5, 3.0).tobytes()
    # Batch 3 graph: nodes 0..5; update repetition 2's first launch only.  Every repetition
    # recomputes dst from src, so the last one decides the result.
    inv.update_kernel(4, [None, None, np.float32(1.5), None], batch_size=3)
    inv.run(mode="graph", batch_size=3)
    assert read(dst).tobytes() == pipeline(values, 1.5, 0.5).tobytes()


def test_rejected_updates(device):
    values = np.zeros(N, np.float32)
    src, dst, _ = buffers(device, values)
    inv = vector_pipeline.lower(N).compile(target=ckl.NVIDIATarget("sm_100a")).bind(src, dst, 0.5)
    inv.run(mode="capture")
    with pytest.raises(ValueError, match="captured graph"):
        inv.update_kernel(0, [None] * 5, mode="capture")
    with pytest.raises(ValueError, match="explicit graph"):
        inv.update_kernel(0, [None] * 5, mode="ordinary")
    with pytest.raises(ValueError, match="unknown node"):
        inv.update_kernel(1, [None] * 5)
    with pytest.raises(ValueError, match="argument count"):
        inv.update_kernel(0, [None] * 4)
    with pytest.raises(ValueError, match="bytes"):
        inv.update_kernel(0, [None, None, np.float64(1.0), None, None])
    with pytest.raises(ValueError, match="limits"):
        inv.update_kernel(0, [None] * 5, block=(2048, 1, 1))
    with pytest.raises(TypeError):
        inv.update_kernel(0, [None, None, 1.0, None, None])
    # The graph still works after the rejected updates.
    inv.run(mode="graph")
    assert read(dst).tobytes() == pipeline(values, 0.5, 0.5).tobytes()


def test_tensor_core_projection_follows_a_new_weight_buffer(device):
    """Re-pointing a tensor-core projection at other weights re-derives its TMA weight map."""
    config = ref.Config(batch=32, hidden=128, heads=2, layers=1, ffn=160, vocab=300, context=4,
                        steps=2)
    initial, _ = ref.make_inputs(config, 9, eps=1e-6)
    session = S.DecoderSession(device, initial, epsilon=1e-6,
                               attention_scale=config.head_dim ** -0.5, whole_step=False)
    names = session.invocation.node_names
    lm_node = names.index("ckl.fused.panel_linear_argmax")
    # A second LM weight buffer; the graph's LM head is re-pointed at it.
    other_lm = np.random.default_rng(10).normal(0, 0.05, initial["lm"].shape).astype(np.float32)
    owner = device.empty(ckl.BufferSpec(other_lm.shape, ckl.f32))
    owner.copy_from_host(other_lm)
    slots = [None] * len(session.invocation.node_argument_sizes(lm_node))
    slots[1] = owner  # the LM head's slots: panel, weights, logits, partials, specialization
    session.invocation.update_kernel(lm_node, slots)
    session.step(1)
    expected = ref.expected(dict(initial, lm=other_lm), config, 1, eps=1e-6)
    assert np.array_equal(session.read("lm"), initial["lm"])  # the bound buffer is unchanged
    for name in ("tokens", "history", "position"):
        assert np.array_equal(session.read(name), expected[name]), name
    assert np.allclose(session.read("logits"), expected["logits"], rtol=1e-4, atol=1e-5)
