"""Asynchronous invocation/completion interface on the GPU.

The reference runs every invocation synchronously (``lib/Runtime/NvidiaProgram.cpp:217-229``)
and names an asynchronous completion interface with buffer-lifetime and dependency safety,
and step grouping as a completion/observation trade-off, as next work
(``benchmarks/decoder/results/deep-dive/REPORT.md:155-159``).  Checked here: grouped
asynchronous generation yields exactly the tokens of synchronous steps and leaves the same
state (against the oracle); a completion orders work across invocations; a completion keeps
its invocation's storage alive after every Python handle is gone; synchronous buffer copies
wait for in-flight submissions.
"""
from __future__ import annotations

import gc

import numpy as np
import pytest

import ckl
from ckl.workloads import vector_pipeline
from oracle import decoder as ref
from test_gpu_decoder import CFG1, open_session, verify

pytestmark = pytest.mark.gpu
TARGET = ckl.NVIDIATarget("sm_100a")
LARGE = 1 << 26


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


@pytest.mark.parametrize("group,depth", [(1, 1), (1, 3), (4, 2), (16, 1)])
def test_grouped_generation_matches_synchronous_steps(device, group, depth):
    initial, _ = ref.make_inputs(CFG1, 0, eps=1e-5)
    expected = ref.expected(initial, CFG1, CFG1.steps, eps=1e-5)
    session = open_session(device, CFG1, initial, 1e-5)
    start = int(initial["position"][0])
    observed = list(session.generate(CFG1.steps, group=group, depth=depth))
    assert [at for at, _ in observed] == list(range(start, start + CFG1.steps, group))
    tokens = np.concatenate([rows for _, rows in observed])
    assert np.array_equal(tokens, expected["history"][start:start + CFG1.steps])
    verify(session, initial, expected, CFG1)


def _vector_program(n):
    spec = ckl.BufferSpec((n,), ckl.f32)
    return vector_pipeline.step.lower(signature={"src": spec, "dst": spec, "bias": ckl.f32}) \
        .compile(target=TARGET)


def test_completion_orders_work_across_invocations(device):
    program = _vector_program(LARGE)
    values = np.linspace(-1, 1, LARGE, dtype=np.float32)
    a, b, c = (device.empty(ckl.BufferSpec((LARGE,), ckl.f32)) for _ in range(3))
    a.copy_from_host(values)
    producer = program.bind(a, b, 0.5)          # b = (a + 0.5) + 0.5
    consumer = program.bind(b, c, 0.25)         # c = (b + 0.25) + 0.25
    for _ in range(3):
        first = producer.submit(graph=True)
        second = consumer.submit(graph=True, after=[first])
        assert second.wait(timeout=60.0)
        assert first.done() and second.done()
    out = np.empty(LARGE, np.float32)
    c.copy_to_host(out)
    step1 = (values + np.float32(0.5)) + np.float32(0.5)
    assert np.array_equal(out, (step1 + np.float32(0.25)) + np.float32(0.25))


def test_completion_keeps_the_invocation_alive(device):
    program = _vector_program(LARGE)
    src = device.empty(ckl.BufferSpec((LARGE,), ckl.f32))
    src.copy_from_host(np.full(LARGE, 2.0, np.float32))
    dst = device.empty(ckl.BufferSpec((LARGE,), ckl.f32))
    observed = ckl.PinnedHostBuffer(dst.nbytes)
    invocation = program.bind(src, dst, 0.125)
    completion = invocation.submit(graph=True, observe=[(dst, observed)])
    invocation.close()
    del invocation, program, src, dst
    gc.collect()
    assert completion.wait()
    assert np.all(observed.array(np.float32, (LARGE,)) == np.float32(2.25))
    completion.close()


def test_synchronous_copies_wait_for_submissions(device):
    program = _vector_program(LARGE)
    src = device.empty(ckl.BufferSpec((LARGE,), ckl.f32))
    dst = device.empty(ckl.BufferSpec((LARGE,), ckl.f32))
    src.copy_from_host(np.full(LARGE, 1.0, np.float32))
    dst.fill_zero()
    invocation = program.bind(src, dst, 1.0)
    invocation.launch(graph=True, batch_size=4)
    out = np.empty(LARGE, np.float32)
    dst.copy_to_host(out)                       # must see the finished submission
    assert np.all(out == 3.0)
    pending = invocation.submit(graph=True)
    src.copy_from_host(np.full(LARGE, 5.0, np.float32))   # waits before overwriting src
    assert pending.done()
    dst.copy_to_host(out)
    assert np.all(out == 3.0)


@pytest.mark.parametrize("nbytes,offset", [(4, 0), (12, 4), (2048, 0), (2051, 1), (65536, 0),
                                           (65536 + 16, 0), (300000, 8)])
def test_pinned_async_copies_round_trip(device, nbytes, offset):
    """Asynchronous copies between page-locked memory and a device buffer, in stream order
    around a graph launch, for sizes from 4 bytes to 300 KB and host offsets off 16-byte
    alignment: the bytes arrive unchanged and nothing outside the range is touched."""
    count = 1 << 17
    program = _vector_program(count)
    src = device.empty(ckl.BufferSpec((count,), ckl.f32))
    dst = device.empty(ckl.BufferSpec((count,), ckl.f32))
    src.fill_zero()
    invocation = program.bind(src, dst, 1.0)
    pinned_in = ckl.PinnedHostBuffer(nbytes + 64)
    pinned_out = ckl.PinnedHostBuffer(nbytes + 64)
    data = np.random.default_rng(nbytes).integers(0, 256, nbytes, dtype=np.uint8)
    np.frombuffer(pinned_in.view(), np.uint8)[offset:offset + nbytes] = data
    np.frombuffer(pinned_out.view(), np.uint8)[:] = 7
    invocation.copy_in_async(src, pinned_in.pointer + offset, nbytes)
    invocation.launch(graph=True)                 # dst = (src + 1) + 1, in stream order
    invocation.copy_out_async(src, pinned_out.pointer + offset, nbytes)
    invocation.synchronize()
    out = np.frombuffer(pinned_out.view(), np.uint8)
    assert np.array_equal(out[offset:offset + nbytes], data)
    assert np.all(out[:offset] == 7) and np.all(out[offset + nbytes:] == 7)
    result = np.empty(count, np.float32)
    dst.copy_to_host(result)
    assert np.all(result[(nbytes + 3) // 4:] == 2.0)   # the launch saw src after the copy
