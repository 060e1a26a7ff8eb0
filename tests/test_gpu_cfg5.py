"""Parity at the benchmark's own workload: BASELINE config 5 as one 512-request GPU shard.

``bench.py``'s default line times this configuration (hidden 1024, 16 heads of 64, SwiGLU 4096,
vocabulary 32000, 4 layers, 2048-token prompts, cache capacity 2080, seed 4, epsilon 1e-6), so
its correctness is checked here at the same shapes, the same seeded weights and prompts, the
same batched prefill and the same decode graph:

* the batched prefill of the whole shard against the reference decoder's own teacher-forced
  prefill of two of its requests (``tests/golden/cfg5_prefill.npz``, made by
  ``tests/golden/make_cfg5_prefill.py`` from ``benchmarks/decoder/reference.py``): every
  prefill position's greedy token bit-exact, the appended key/value rows at positions 0, 1023
  and 2046 within the tolerance;
* four decode steps from that state (cache rows 2047..2050, attention over 2048-2051 rows) on
  the tensor-core graph and on the FFMA graph, against the oracle run on eight requests spread
  over the shard, whose state is read back from the device (requests never interact, so the
  subset's oracle state is the shard's): tokens, history and position bit-exact, logits and
  the appended cache rows within 1e-4 relative / 1e-5 absolute (the north star's tolerance,
  as ``benchmarks/decoder/run.py:107-132`` checks them).
"""
from __future__ import annotations

import numpy as np
import pytest

import ckl
from conftest import GOLDEN
from ckl.workloads import decoder, session as S
from oracle import decoder as ref

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-4, 1e-5
SHARD, CONTEXT, STEPS, SEED, EPS = 512, 2048, 32, 4, 1e-6
DIMS = dict(hidden=1024, heads=16, layers=4, ffn=4096, vocab=32000)
SUBSET = (0, 73, 146, 219, 292, 365, 438, 511)
DECODE_STEPS = 4


def request_rows(session, name, request):
    """Cache block ``[layers, heads, capacity, head_dim]`` of one request, read from the device."""
    (layers, batch, heads, capacity, dim), _ = session.shapes[name]
    block = heads * capacity * dim
    out = np.empty((layers, heads, capacity, dim), np.float32)
    for layer in range(layers):
        view = session.owners[name].subview(offset=(layer * batch + request) * block,
                                            shape=(block,))
        host = np.empty(block, np.float32)
        view.copy_to_host(host)
        out[layer] = host.reshape(heads, capacity, dim)
    return out


@pytest.fixture(scope="module")
def shard():
    """The benchmark's shard after its batched prefill, and the host copy of its weights."""
    device = ckl.Device()
    shape = S.DecoderShape(batch=SHARD, context=CONTEXT, steps=STEPS, **DIMS)
    arrays, rng = S.make_weights(shape, SEED)
    prompts = rng.integers(0, shape.vocab, (CONTEXT, SHARD), dtype=np.int32)
    cache = (shape.layers, SHARD, shape.heads, shape.capacity, shape.head_dim)
    state = dict(tokens=prompts[0].copy(), position=np.zeros(1, np.int32),
                 history=np.full((shape.capacity, SHARD), -1, np.int32),
                 kc=(cache, np.float32), vc=(cache, np.float32),
                 logits=np.zeros((SHARD, shape.vocab), np.float32))
    session = S.DecoderSession(device, {**arrays, **state}, epsilon=EPS,
                               attention_scale=shape.head_dim ** -0.5, tails=False)
    session.prefill(prompts, batched=True)
    return session, arrays, prompts


def test_batched_prefill_matches_reference_prefill(shard):
    session, _, prompts = shard
    golden = np.load(GOLDEN / "cfg5_prefill.npz")
    requests = [int(r) for r in golden["requests"]]
    assert int(session.read("position")[0]) == CONTEXT - 1
    history = session.read("history")
    tokens = session.read("tokens")
    assert np.array_equal(tokens[requests], golden["tokens"])
    assert np.array_equal(tokens, prompts[-1])
    assert np.array_equal(history[:CONTEXT - 1, requests], golden["history"])
    assert np.all(history[CONTEXT - 1:] == -1)
    positions = [int(p) for p in golden["positions"]]
    for name in ("kc", "vc"):
        expected = golden[f"{name}_rows"]  # [positions, layers, requests, heads, dim]
        for i, request in enumerate(requests):
            rows = request_rows(session, name, request)[:, :, positions, :]
            rows = np.moveaxis(rows, 2, 0)  # [positions, layers, heads, dim]
            assert np.allclose(rows, expected[:, :, i], rtol=RTOL, atol=ATOL), (name, request)


def oracle_state(session, arrays, requests):
    """Oracle state of `requests` read back from the device at the session's position."""
    tokens, history = session.read("tokens"), session.read("history")
    state = {name: arrays[name] for name in S.WEIGHTS + ("sincos",)}
    state.update(tokens=tokens[list(requests)].copy(), position=session.read("position"),
                 history=np.ascontiguousarray(history[:, list(requests)]),
                 logits=np.zeros((len(requests), DIMS["vocab"]), np.float32))
    for name in ("kc", "vc"):
        state[name] = np.stack([request_rows(session, name, r) for r in requests], axis=1)
    return state


@pytest.mark.parametrize("projections", ["tensor", "ffma"])
def test_decode_steps_at_context_2048_match_oracle(shard, projections):
    session, arrays, prompts = shard
    # Every case starts from the post-prefill state: position 2047, the last prompt tokens.
    session.write("position", np.array([CONTEXT - 1], np.int32))
    session.write("tokens", prompts[-1])
    config = ref.Config(batch=len(SUBSET), context=CONTEXT, steps=STEPS, **DIMS)
    initial = oracle_state(session, arrays, SUBSET)
    expected = ref.expected(initial, config, DECODE_STEPS, eps=EPS)
    if projections == "tensor":
        invocation = session.invocation
    else:
        program = session.lowered.compile(target=ckl.NVIDIATarget("sm_100a"), tensor_cores=False)
        invocation = program.bind(*[session.buffers[n] for n in decoder.ARGUMENTS[:-2]],
                                  float(EPS), float(session.attention_scale))
    for _ in range(DECODE_STEPS):
        invocation.run(mode="graph")
    subset = list(SUBSET)
    assert int(session.read("position")[0]) == CONTEXT - 1 + DECODE_STEPS
    assert np.array_equal(session.read("tokens")[subset], expected["tokens"])
    assert np.array_equal(session.read("history")[:, subset], expected["history"])
    assert np.allclose(session.read("logits")[subset], expected["logits"], rtol=RTOL, atol=ATOL)
    written = slice(CONTEXT - 1, CONTEXT - 1 + DECODE_STEPS)
    for name in ("kc", "vc"):
        for i, request in enumerate(SUBSET):
            rows = request_rows(session, name, request)[:, :, written]
            assert np.allclose(rows, expected[name][:, i, :, written], rtol=RTOL, atol=ATOL), \
                (name, request)
