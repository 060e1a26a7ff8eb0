"""The allocation-free greedy head agrees with the regular entry point.

``ckl_greedy_head_noalloc`` serves callers that cannot allocate device memory where they run
the decoder's head (a fixed memory budget owned by another allocator, a locked allocator, or
a latency-critical path that must not call cudaMalloc): its argmax partials and completion
counter live in a fixed array inside the library instead of a bind-time heap.  This test
runs the head through the regular entry point (a CKL program bound and run through the C ABI,
whose scratch comes from the planner's heap) and through the allocation-free entry point on
the same inputs, twice in a row, and requires the same logits (1e-4 relative / 1e-5
absolute), the same tokens and history rows, and the same advanced position.  Both paths
are also checked against the NumPy oracle of the head (the reference decoder's final RMSNorm,
LM projection and first-index argmax, ``benchmarks/decoder/reference.py:71-76``), including
inputs with exact ties between two columns and with a NaN logit in column 0, so that a bug
shared by both GPU paths cannot pass.  It lives in its own file, collected last, so a failure
here comes after every other test has run.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import ckl
from ckl import _native
from ckl.workloads.decoder import (FinalGain, Hidden, History, LMWeight, Logits, Position,
                                   Tokens, advance, greedy, linear, rms_apply, rms_stats, B, C as Cdim,
                                   V)
from oracle import decoder as ref

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-4, 1e-5


@ckl.program
def greedy_head(x: Hidden, final_norm: FinalGain, lm: LMWeight, logits: Logits, tokens: Tokens,
                history: History, position: Position, epsilon: ckl.f32) -> None:
    inv = ckl.empty((B,), dtype=ckl.f32)
    normed = ckl.empty_like(x)
    ckl.launch(rms_stats, x, inv, epsilon, grid=(ckl.cdiv(B, 32),), block=(32,))
    ckl.launch(rms_apply, x, inv, final_norm, normed, 0, grid=(ckl.cdiv(Cdim, 64), B), block=(64,))
    ckl.launch(linear, normed, lm, logits, 0, grid=(ckl.cdiv(V, 64), B), block=(64,))
    ckl.launch(greedy, logits, tokens, history, position, grid=(ckl.cdiv(B, 32),), block=(32,))
    ckl.launch(advance, position, grid=(1,), block=(1,))


def upload(device, array, dtype):
    buffer = device.empty(ckl.BufferSpec(array.shape, dtype))
    buffer.copy_from_host(np.ascontiguousarray(array))
    return buffer


def read(buffer, dtype):
    out = np.empty(buffer.spec.shape, dtype=dtype)
    buffer.copy_to_host(out)
    return out


def head_inputs(batch, hidden, vocab, special):
    rng = np.random.default_rng(11)
    x = rng.normal(0, 1, (batch, hidden)).astype(np.float32)
    gain = (1 + rng.normal(0, 0.02, (1, hidden))).astype(np.float32)
    lm = rng.normal(0, 0.5 / np.sqrt(hidden), (1, hidden, vocab)).astype(np.float32)
    if special == "ties":
        # Columns 3 and vocab - 2 each hold one nonzero weight, on the same (positive) input
        # column, so both logits are the same single product in any summation order and every
        # row's maximum is an exact tie, which the first index (3) must win.
        x[:, 0] = np.abs(x[:, 0]) + 1
        lm[0, :, 3] = 0.0
        lm[0, :, vocab - 2] = 0.0
        lm[0, 0, 3] = lm[0, 0, vocab - 2] = 100.0
    elif special == "nan":
        lm[0, 0, 0] = np.nan  # column 0 of every row's logits is NaN: argmax gives 0
    return x, gain, lm


def oracle_head(x, gain, lm, eps, history, position):
    """The reference decoder's head (reference.py:71-76) on the host."""
    logits = ref.rms_norm(x, gain[0], np.float32(eps)) @ lm[0]
    tokens = logits.argmax(axis=-1).astype(np.int32)
    history = history.copy()
    history[position] = tokens
    return logits, tokens, history


@pytest.mark.parametrize("batch,hidden,vocab,special", [
    (4, 64, 512, None), (512, 1024, 32000, None), (37, 96, 1000, None),
    (5, 64, 300, "ties"), (40, 128, 700, "ties"), (3, 64, 256, "nan")])
def test_noalloc_head_matches_regular_entry_point(batch, hidden, vocab, special):
    device = ckl.Device()
    capacity = 8
    x, gain, lm = head_inputs(batch, hidden, vocab, special)
    eps = 1e-6

    # Regular entry point: the head as a CKL program, bound and run twice.
    bufs = dict(x=upload(device, x, ckl.f32), final_norm=upload(device, gain, ckl.f32),
                lm=upload(device, lm, ckl.f32),
                logits=upload(device, np.zeros((batch, vocab), np.float32), ckl.f32),
                tokens=upload(device, np.zeros(batch, np.int32), ckl.i32),
                history=upload(device, np.full((capacity, batch), -1, np.int32), ckl.i32),
                position=upload(device, np.array([2], np.int32), ckl.i32))
    signature = {name: b.spec for name, b in bufs.items()}
    signature["epsilon"] = ckl.f32
    program = greedy_head.lower(signature=signature).compile(target=ckl.NVIDIATarget("sm_100a"))
    invocation = program.bind(*bufs.values(), eps)
    invocation.run(graph=True)
    logits_regular_1 = read(bufs["logits"], np.float32)
    invocation.run(graph=True)
    regular = {n: read(bufs[n], np.float32 if n == "logits" else np.int32)
               for n in ("logits", "tokens", "history", "position")}

    # Allocation-free entry point on fresh outputs, two calls in a row.
    outs = dict(logits=upload(device, np.zeros((batch, vocab), np.float32), ckl.f32),
                tokens=upload(device, np.zeros(batch, np.int32), ckl.i32),
                history=upload(device, np.full((capacity, batch), -1, np.int32), ckl.i32),
                position=upload(device, np.array([2], np.int32), ckl.i32))
    lib = _native.load()
    call = lambda: lib.ckl_greedy_head_noalloc(
        bufs["x"].address, bufs["final_norm"].address, bufs["lm"].address, C.c_float(eps),
        batch, hidden, vocab, capacity, outs["logits"].address, outs["tokens"].address,
        outs["history"].address, outs["position"].address, None)
    assert call() == 0, _native.message()
    logits_noalloc_1 = read(outs["logits"], np.float32)      # waits for the default stream
    assert call() == 0, _native.message()
    noalloc = {n: read(outs[n], np.float32 if n == "logits" else np.int32)
               for n in ("logits", "tokens", "history", "position")}

    close = dict(rtol=RTOL, atol=ATOL, equal_nan=True)
    assert np.allclose(logits_noalloc_1, logits_regular_1, **close)
    assert np.allclose(noalloc["logits"], regular["logits"], **close)
    for name in ("tokens", "history", "position"):
        assert np.array_equal(noalloc[name], regular[name]), name
    assert noalloc["position"][0] == 4
    assert np.all(noalloc["history"][2:4] >= 0) and np.all(noalloc["history"][4:] == -1)

    # Both paths against the oracle: the same inputs give the same step at positions 2 and 3.
    logits, tokens, history = oracle_head(x, gain, lm, eps, np.full((capacity, batch), -1,
                                                                     np.int32), 2)
    _, _, history = oracle_head(x, gain, lm, eps, history, 3)
    for result in (regular, noalloc):
        assert np.allclose(result["logits"], logits, **close)
        assert np.array_equal(result["tokens"], tokens)
        assert np.array_equal(result["history"], history)
    if special == "ties":
        assert np.all(tokens == 3)
    if special == "nan":
        assert np.all(tokens == 0)


def test_noalloc_head_rejects_sizes_beyond_its_scratch():
    device = ckl.Device()
    lib = _native.load()
    tiny = device.empty(ckl.BufferSpec((4,), ckl.f32))
    status = lib.ckl_greedy_head_noalloc(tiny.address, tiny.address, tiny.address, C.c_float(1e-6),
                                         100000, 64, 1000000, 8, tiny.address, tiny.address,
                                         tiny.address, tiny.address, None)
    assert status == _native.INVALID_ARGUMENT
    assert "exceed the fixed scratch" in _native.message()
