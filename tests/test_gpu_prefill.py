"""Batched prompt prefill on the GPU against the oracle's teacher-forced prefill.

The oracle (like the reference, benchmarks/decoder/reference.py:98-108) prefills one decode step
per prompt token; the batched prefill runs the prompt positions in chunks of all requests at
once.  After it the state must be the oracle's: history, tokens and position bit-exact, the KV
rows of every prompt position and the logits within 1e-4 relative / 1e-5 absolute (with the
sentinel tails, the weights and the cache rows past the prompt untouched), and the following
greedy decode steps must reproduce the oracle's tokens.  Cases cover every head dimension, one
and several chunks with a ragged last chunk, the tensor-core path's row tiling, keys streamed
over several blocks, caches off a 16-byte boundary (the attention's plain-load path), and the
published deep-dive prompts and tokens.
"""
from __future__ import annotations

import numpy as np
import pytest

import ckl
from ckl.workloads import decoder, prefill, session as S
from oracle import decoder as ref
from test_gpu_decoder import PUBLISHED, open_session, verify

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


@pytest.mark.parametrize("batch,hidden,heads,layers,ffn,vocab,context,chunk_rows", [
    (3, 48, 3, 1, 80, 129, 6, 16384),     # head dim 16, awkward sizes, one chunk
    (1, 64, 4, 2, 256, 512, 16, 16384),   # BASELINE config 1 shape
    (1, 64, 4, 2, 256, 512, 16, 4),       # four positions per chunk, ragged last chunk
    (20, 128, 2, 1, 96, 300, 40, 64),     # head dim 64, three positions per chunk
    (64, 256, 8, 2, 1024, 512, 34, 16384),  # BASELINE config 3 shape, head dim 32
    (130, 256, 2, 1, 128, 640, 9, 300),   # head dim 128, two row tiles per position
    (8, 128, 2, 1, 96, 300, 200, 16384),  # keys streamed in four 64-row blocks, one chunk
])
def test_batched_prefill_matches_oracle(device, monkeypatch, batch, hidden, heads, layers, ffn,
                                        vocab, context, chunk_rows):
    monkeypatch.setattr(prefill, "CHUNK_ROWS", chunk_rows)
    steps = 3
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=layers, ffn=ffn,
                        vocab=vocab, context=context, steps=steps)
    empty, prompts = ref.make_inputs(config, 7, eps=1e-6, prefill=False)
    prefilled, _ = ref.make_inputs(config, 7, eps=1e-6, prefill=True)
    session = open_session(device, config, empty, 1e-6)
    session.prefill(prompts, batched=True)
    verify(session, empty, prefilled, config)
    expected = ref.expected(prefilled, config, steps, eps=1e-6)
    session.step(steps)
    verify(session, empty, expected, config)


def test_batched_prefill_with_caches_off_a_16_byte_boundary(device):
    """K/V caches bound 4 bytes past a 16-byte boundary: the prefill attention cannot stream
    their rows with 16-byte asynchronous copies and reads them with plain loads instead (its
    fallback path); the prefilled state must still be the oracle's."""
    config = ref.Config(batch=8, hidden=128, heads=2, layers=1, ffn=96, vocab=300, context=200,
                        steps=3)
    empty, prompts = ref.make_inputs(config, 7, eps=1e-6, prefill=False)
    prefilled, _ = ref.make_inputs(config, 7, eps=1e-6, prefill=True)
    session = open_session(device, config, empty, 1e-6)
    for name in ("kc", "vc"):  # views one float into their (sentinel-tailed) allocations
        session.buffers[name] = device.import_buffer(session.owners[name].address + 4,
                                                     session.buffers[name].spec,
                                                     owner=session.owners[name])
    # The prefill's last prompt position runs as an ordinary decode step: bind the session's
    # program to the same views (a binding off a 16-byte boundary takes the unfused plan).
    session.invocation = session.program.bind(
        *[session.buffers[name] for name in decoder.ARGUMENTS[:-2]], 1e-6,
        config.head_dim ** -0.5)
    session.prefill(prompts, batched=True)
    for name in ("history", "tokens", "position"):
        assert np.array_equal(session.read(name), prefilled[name]), name
    assert np.allclose(session.read("logits"), prefilled["logits"], rtol=1e-4, atol=1e-5)
    rows = config.context - 1  # the prompt positions the prefill writes
    for name in ("kc", "vc"):
        shape = session.shapes[name][0]
        size = int(np.prod(shape))
        cache = session.read(name, with_tail=True)[1:1 + size].reshape(shape)
        assert np.allclose(cache[..., :rows, :], prefilled[name][..., :rows, :], rtol=1e-4,
                           atol=1e-5), name


@pytest.mark.parametrize("case", [c for c in PUBLISHED if "deep-dive" in c["source"]],
                         ids=lambda c: c["name"])
def test_published_tokens_with_batched_prefill(device, case):
    """The published prompts, prefilled in one batch, reproduce the published tokens."""
    config = ref.Config(**case["config"])
    shape = S.DecoderShape(**case["config"])
    arrays, rng = S.make_weights(shape, case["seed"])
    prompts = S.make_prompts(shape, rng)
    assert prompts.tolist() == case["prompts"]
    arrays.update(S.initial_state(shape))
    session = open_session(device, config, arrays, 1e-5)
    session.prefill(prompts, batched=True)
    session.step(config.steps)
    history = session.read("history")
    start = config.context - 1
    assert history[start:start + config.steps].tolist() == case["generated_tokens"]
    assert int(session.read("position")[0]) == config.context - 1 + config.steps
