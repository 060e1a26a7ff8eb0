"""Split-K flash decoding (few requests, long cache) against the oracle.

Below two (request, head) pairs per SM the decode attention divides every pair's cache rows
over several CTAs and merges their softmax states in range order (``ckl.fused.attention_split``);
the reference computes the same attention serially per (request, head)
(``benchmarks/decoder/workloads.py:100-142``, the bottleneck named at ``REPORT.md:89``).

Cases:
* BASELINE config 5 dimensions (hidden 1024, 16 heads of 64, SwiGLU 4096, vocabulary 32000,
  4 layers) with 1, 3, 8 and 17 requests at context 2048 (17: tensor-core projections): the prompt is prefilled on the GPU
  (batched prefill), the state read back, and three decode steps (cache rows 2047..2049:
  2048-2050 rows per head, so the last ranges are ragged) compared with the oracle run from
  the same state, with the default projections at this hidden size (the streamed few-row FFMA
  kernel up to sixteen requests) and, for 3 requests, FFMA projections
  forced - tokens, history and position exact, logits and appended cache rows within 1e-4
  relative / 1e-5 absolute;
* a short prompt in a long cache (6 rows filled, capacity 2054): most ranges are empty;
* the same small-batch case on the tensor-core path (tensor cores are used from 17 requests:
  20 requests of 2 heads still split), which writes the context as a split-operand panel.
"""
from __future__ import annotations

import numpy as np
import pytest

import ckl
from ckl.compile import STREAMED_ROWS, attention_splits
from ckl.workloads import session as S
from oracle import decoder as ref
from test_gpu_decoder import verify

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-4, 1e-5
EPS = 1e-6
CFG5 = dict(hidden=1024, heads=16, layers=4, ffn=4096, vocab=32000)


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


def cache_rows(session, name, request):
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


@pytest.mark.parametrize("batch,tensor_cores",
                         [(1, True), (3, True), (8, True), (17, True), (3, False)])
def test_split_attention_at_context_2048_matches_oracle(device, batch, tensor_cores):
    steps = 3
    shape = S.DecoderShape(batch=batch, context=2048, steps=32, **CFG5)
    assert attention_splits(batch, shape.heads, shape.capacity) > 1
    arrays, rng = S.make_weights(shape, 4)
    prompts = rng.integers(0, shape.vocab, (shape.context, batch), dtype=np.int32)
    cache = (shape.layers, batch, shape.heads, shape.capacity, shape.head_dim)
    state = dict(tokens=prompts[0].copy(), position=np.zeros(1, np.int32),
                 history=np.full((shape.capacity, batch), -1, np.int32),
                 kc=(cache, np.float32), vc=(cache, np.float32),
                 logits=np.zeros((batch, shape.vocab), np.float32))
    session = S.DecoderSession(device, {**arrays, **state}, epsilon=EPS,
                               attention_scale=shape.head_dim ** -0.5, tails=False,
                               tensor_cores=tensor_cores)
    names = session.invocation.node_names
    assert "ckl.fused.attention_split" in names
    # Up to STREAMED_ROWS requests the streamed few-row kernel takes the projections here.
    assert ("ckl.fused.panel_linear_rope" in names) == (tensor_cores and batch > STREAMED_ROWS)
    session.prefill(prompts, batched=True)
    initial = {name: arrays[name] for name in S.WEIGHTS + ("sincos",)}
    initial.update(tokens=session.read("tokens"), position=session.read("position"),
                   history=session.read("history"),
                   logits=np.zeros((batch, shape.vocab), np.float32))
    for name in ("kc", "vc"):
        initial[name] = np.stack([cache_rows(session, name, r) for r in range(batch)], axis=1)
    config = ref.Config(batch=batch, context=2048, steps=32, **CFG5)
    expected = ref.expected(initial, config, steps, eps=EPS)
    session.step(steps)
    for name in ("tokens", "history", "position"):
        assert np.array_equal(session.read(name), expected[name]), name
    assert np.allclose(session.read("logits"), expected["logits"], rtol=RTOL, atol=ATOL)
    written = slice(2047, 2047 + steps)
    for name in ("kc", "vc"):
        for r in range(batch):
            assert np.allclose(cache_rows(session, name, r)[:, :, written],
                               expected[name][:, r, :, written], rtol=RTOL, atol=ATOL), (name, r)


@pytest.mark.parametrize("batch,heads,hidden,tensor_cores", [
    (4, 4, 128, False),   # FFMA path, head dim 32
    (20, 2, 128, True),   # tensor-core path (context written as a panel), head dim 64
    (2, 1, 128, False),   # head dim 128
])
def test_split_attention_short_prompt_in_long_cache(device, batch, heads, hidden, tensor_cores):
    """Six filled rows in a 2054-row cache: most ranges are empty, one or two hold the rows."""
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=2, ffn=160, vocab=300,
                        context=6, steps=2048)
    assert attention_splits(batch, heads, config.capacity) > 1
    initial, _ = ref.make_inputs(config, 13, eps=EPS)
    expected = ref.expected(initial, config, 3, eps=EPS)
    session = S.DecoderSession(device, initial, epsilon=EPS,
                               attention_scale=config.head_dim ** -0.5,
                               tensor_cores=tensor_cores, whole_step=False)
    assert "ckl.fused.attention_split" in session.invocation.node_names
    session.step(3)
    verify(session, initial, expected, config)
