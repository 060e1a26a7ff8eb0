"""Saved programs run on the GPU: a program compiled in one process and loaded from its JSON
description (no Python source, tracing or device compilation on the loading side) produces the
results of the original, for a decoder step (library kernels) and for a plan with generated
kernels."""
from __future__ import annotations

import numpy as np
import pytest

import ckl
from ckl.workloads import decoder
from oracle import decoder as ref
from test_gpu_decoder import CFG1, open_session, verify
from test_plan_io import mixed

pytestmark = pytest.mark.gpu
TARGET = ckl.NVIDIATarget("sm_100a")


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


def test_loaded_decoder_program_matches_oracle(device, tmp_path):
    initial, _ = ref.make_inputs(CFG1, 0, eps=1e-5)
    expected = ref.expected(initial, CFG1, CFG1.steps, eps=1e-5)
    session = open_session(device, CFG1, initial, 1e-5)
    session.program.save(tmp_path / "decode.json")
    loaded = ckl.load_program(tmp_path / "decode.json")
    arguments = [session.buffers[name] for name in decoder.ARGUMENTS[:-2]]
    invocation = loaded.bind(*arguments, 1e-5, CFG1.head_dim ** -0.5)
    assert invocation.node_count == session.invocation.node_count
    for _ in range(CFG1.steps):
        invocation.run(graph=True)
    verify(session, initial, expected, CFG1)


def test_loaded_program_with_generated_kernels(device, tmp_path):
    n = 1000
    spec = ckl.BufferSpec((n,), ckl.f32)
    program = mixed.lower(signature={"src": spec, "dst": spec, "bias": ckl.f32}).compile(
        target=TARGET)
    program.save(tmp_path / "mixed.json")
    loaded = ckl.load_program(tmp_path / "mixed.json")
    values = np.linspace(-2, 2, n, dtype=np.float32)
    src, dst = device.empty(spec), device.empty(spec)
    src.copy_from_host(values)
    out = {}
    for name, p in (("original", program), ("loaded", loaded)):
        p.bind(src, dst, 0.75).run(graph=True)
        out[name] = np.empty(n, np.float32)
        dst.copy_to_host(out[name])
    temp = values + np.float32(0.75)
    assert np.array_equal(out["original"], (temp * temp) + np.float32(0.75))
    assert np.array_equal(out["loaded"], out["original"])
