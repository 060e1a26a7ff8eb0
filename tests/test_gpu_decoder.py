"""Decode-step parity on the GPU against the CPU oracle and the published known answers.

Tolerances: greedy tokens, history and position bit-exact; logits and
KV-cache rows within 1e-4 relative / 1e-5 absolute in float32.  Like the reference harness
(benchmarks/decoder/run.py:107-132) every check also verifies the 256-element sentinel tails,
unchanged weights and the untouched KV-cache prefix and suffix.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
import ckl
from ckl.workloads import decoder, session as S
from oracle import decoder as ref

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-4, 1e-5
PUBLISHED = json.loads((GOLDEN / "published_cases.json").read_text())["cases"]
CFG1 = ref.Config(batch=1, hidden=64, heads=4, layers=2, ffn=256, vocab=512, context=16, steps=16)


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


def open_session(device, config, arrays, eps, **kw):
    return S.DecoderSession(device, arrays, epsilon=eps, attention_scale=config.head_dim ** -0.5, **kw)


def verify(session, initial, expected, config):
    start, end = int(initial["position"][0]), int(expected["position"][0])
    for name in S.MUTABLE + S.WEIGHTS + ("sincos",):
        assert session.tail_intact(name), f"{name}: tail overwritten"
        actual = session.read(name)
        if name not in S.MUTABLE:
            assert np.array_equal(actual, initial[name]), f"{name}: weights changed"
        elif actual.dtype == np.int32:
            assert np.array_equal(actual, expected[name]), f"{name}: mismatch"
        else:
            assert np.all(np.isfinite(actual[..., :end, :] if name in ("kc", "vc") else actual))
            if name in ("kc", "vc"):
                assert np.array_equal(actual[:, :, :, :start], initial[name][:, :, :, :start])
                assert np.array_equal(actual[:, :, :, end:], initial[name][:, :, :, end:])
                assert np.allclose(actual[:, :, :, start:end], expected[name][:, :, :, start:end],
                                   rtol=RTOL, atol=ATOL), name
            else:
                assert np.allclose(actual, expected[name], rtol=RTOL, atol=ATOL), name


@pytest.mark.parametrize("fuse,whole,nodes", [(True, True, 1), (True, False, 19),
                                              (False, False, 48)],
                         ids=["whole-step", "fused-layers", "unfused"])
@pytest.mark.parametrize("eps", [1e-6, 1e-5])
def test_cfg1_sixteen_steps_match_oracle(device, fuse, whole, nodes, eps):
    initial, _ = ref.make_inputs(CFG1, 0, eps=eps)
    expected = ref.expected(initial, CFG1, CFG1.steps, eps=eps)
    session = open_session(device, CFG1, initial, eps, fuse_library=fuse, whole_step=whole)
    assert session.invocation.node_count == nodes
    session.step(CFG1.steps)
    verify(session, initial, expected, CFG1)


@pytest.mark.parametrize("mode,group", [("ordinary", 1), ("capture", 1), ("graph", 4),
                                        ("capture", 16), ("graph", 16)])
def test_modes_and_step_groups(device, mode, group):
    config = ref.Config(batch=3, hidden=48, heads=3, layers=1, ffn=80, vocab=129, context=3, steps=16)
    initial, _ = ref.make_inputs(config, 123)
    expected = ref.expected(initial, config, config.steps)
    session = open_session(device, config, initial, 1e-5)
    session.step(config.steps, mode=mode, batch_size=group)
    verify(session, initial, expected, config)


@pytest.mark.parametrize("case", [c for c in PUBLISHED if "deep-dive" in c["source"]],
                         ids=lambda c: c["name"])
def test_published_tokens_with_gpu_prefill(device, case):
    """Prompts prefilled on the GPU by teacher forcing reproduce the published tokens."""
    config = ref.Config(**case["config"])
    shape = S.DecoderShape(**case["config"])
    arrays, rng = S.make_weights(shape, case["seed"])
    prompts = S.make_prompts(shape, rng)
    assert prompts.tolist() == case["prompts"]
    arrays.update(S.initial_state(shape))
    session = open_session(device, config, arrays, 1e-5)
    session.prefill(prompts)
    session.step(config.steps)
    history = session.read("history")
    start = config.context - 1
    assert history[start:start + config.steps].tolist() == case["generated_tokens"]
    assert int(session.read("position")[0]) == config.context - 1 + config.steps


@pytest.mark.parametrize("batch,hidden,heads,layers,ffn,seed,steps", [
    (64, 256, 8, 2, 1024, 2, 4),     # cfg3 shape
    (256, 64, 4, 8, 256, 3, 3),      # cfg4 shape
    (33, 128, 2, 1, 96, 5, 3),       # ragged batch, head dim 64
])
@pytest.mark.parametrize("whole", [True, False], ids=["whole-step", "layers"])
def test_batched_shapes_match_oracle(device, batch, hidden, heads, layers, ffn, seed, steps, whole):
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=layers, ffn=ffn, vocab=512,
                        context=16, steps=steps)
    initial, _ = ref.make_inputs(config, seed, eps=1e-6)
    expected = ref.expected(initial, config, steps, eps=1e-6)
    session = open_session(device, config, initial, 1e-6, whole_step=whole)
    session.step(steps)
    verify(session, initial, expected, config)


@pytest.mark.parametrize("batch,hidden,heads,layers,ffn,vocab,context,steps", [
    (1, 64, 4, 2, 256, 512, 16, 16),       # one cluster, one request
    (7, 128, 4, 3, 512, 1024, 40, 6),      # rows per cluster 1
    (40, 64, 2, 2, 128, 8192, 20, 4),      # 256 vocabulary quads per CTA, D 32
    (200, 128, 1, 1, 256, 256, 12, 3),     # one head of dim 128, ragged last cluster
    (288, 64, 4, 1, 256, 512, 8, 3),       # 32 clusters x 9 requests, ragged last cluster
    (24, 256, 16, 2, 256, 512, 10, 3),     # two heads per CTA (16 heads)
    (16, 512, 32, 1, 256, 512, 8, 2),      # four heads per CTA (32 heads)
    (10, 512, 8, 1, 512, 512, 12, 3),      # one head of dim 64 per CTA, one-CTA-per-SM build
    (512, 64, 4, 1, 256, 512, 8, 3),       # 32 clusters x 16 requests (two row blocks)
])
def test_whole_step_kernel_matches_oracle(device, batch, hidden, heads, layers, ffn, vocab,
                                          context, steps):
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=layers, ffn=ffn,
                        vocab=vocab, context=context, steps=steps)
    initial, _ = ref.make_inputs(config, 11, eps=1e-5)
    expected = ref.expected(initial, config, steps, eps=1e-5)
    session = open_session(device, config, initial, 1e-5)
    assert session.invocation.node_names == ["ckl.fused.decode_step"]
    for mode in ("graph", "ordinary"):
        session.step(steps // 2 if mode == "graph" else steps - steps // 2, mode=mode)
    verify(session, initial, expected, config)


def test_overlapping_bindings_take_the_reference_graph(device):
    """Fused plans require distinct buffers; an aliased binding falls back to 21L+6 nodes."""
    initial, _ = ref.make_inputs(CFG1, 0)
    session = open_session(device, CFG1, initial, 1e-5)
    buffers = [session.buffers[n] for n in decoder.ARGUMENTS[:-2]]
    aliased = list(buffers)
    aliased[18] = device.import_buffer(session.buffers["vc"].address, session.buffers["logits"].spec,
                                       owner=session.owners["vc"])
    invocation = session.program.bind(*aliased, 1e-5, CFG1.head_dim ** -0.5)
    assert invocation.node_count == 21 * CFG1.layers + 6


def test_misaligned_cache_view_takes_the_reference_graph(device):
    """Fused plans access caller buffers 16 bytes at a time; a cache bound as a view one element
    into its storage (4-byte aligned) makes the binding take the 21L+6-node graph, which then
    reproduces the oracle."""
    initial, _ = ref.make_inputs(CFG1, 0)
    expected = ref.expected(initial, CFG1, 4)
    session = open_session(device, CFG1, initial, 1e-5)
    buffers = [session.buffers[n] for n in decoder.ARGUMENTS[:-2]]
    shifted = {}
    for name in ("kc", "vc"):
        values = initial[name].ravel()
        owner = device.empty(ckl.BufferSpec((values.size + 4,), ckl.f32))
        host = np.zeros(values.size + 4, np.float32)
        host[1:1 + values.size] = values
        owner.copy_from_host(host)
        view = device.import_buffer(owner.address + 4, session.buffers[name].spec, owner=owner)
        shifted[name] = (owner, view)
        buffers[decoder.ARGUMENTS.index(name)] = view
    invocation = session.program.bind(*buffers, 1e-5, CFG1.head_dim ** -0.5)
    assert invocation.node_count == 21 * CFG1.layers + 6
    for _ in range(4):
        invocation.run(mode="graph")
    start, end = int(initial["position"][0]), int(expected["position"][0])
    for name, (owner, _) in shifted.items():
        host = np.empty(initial[name].size + 4, np.float32)
        owner.copy_to_host(host)
        actual = host[1:1 + initial[name].size].reshape(initial[name].shape)
        assert np.allclose(actual[:, :, :, start:end], expected[name][:, :, :, start:end],
                           rtol=RTOL, atol=ATOL), name
    assert np.array_equal(session.read("history"), expected["history"])


@pytest.mark.parametrize("batch,options", [(2, {}), (2, {"whole_step": False}),
                                           (20, {"whole_step": False}),
                                           (2, {"fuse_library": False})],
                         ids=["whole-step", "fused-layers", "tensor-cores", "unfused"])
def test_steps_past_the_cache_capacity_write_nothing(device, batch, options):
    """The last cache row is written like any other; a step at a position at or beyond the
    capacity (where the reference indexes out of bounds) writes no cache row, no history row
    and nothing past any buffer, and still advances the position."""
    config = ref.Config(batch=batch, hidden=64, heads=4, layers=1, ffn=128, vocab=256, context=4,
                        steps=3)
    capacity = config.context + config.steps
    initial, _ = ref.make_inputs(config, 5, eps=1e-5)
    valid = capacity - int(initial["position"][0])          # steps up to the last cache row
    expected = ref.expected(initial, config, valid, eps=1e-5)
    session = open_session(device, config, initial, 1e-5, **options)
    session.step(valid)
    verify(session, initial, expected, config)
    before = {name: session.read(name) for name in ("kc", "vc", "history")}
    session.step(2)
    assert int(session.read("position")[0]) == capacity + 2
    for name in S.MUTABLE + S.WEIGHTS + ("sincos",):
        assert session.tail_intact(name), f"{name}: tail overwritten"
    for name, values in before.items():
        assert np.array_equal(session.read(name), values), f"{name} written past the capacity"


@pytest.mark.parametrize("options", [{}, {"whole_step": False}, {"fuse_library": False}],
                         ids=["whole-step", "fused-layers", "unfused"])
def test_tokens_outside_the_vocabulary_touch_nothing_past_the_buffers(device, options):
    """A token outside [0, vocab) (the reference would read past the embedding table) selects
    no embedding row; the step completes, stays inside every buffer and the other requests'
    tokens are those of a clean run."""
    config = ref.Config(batch=3, hidden=64, heads=4, layers=1, ffn=128, vocab=256, context=4,
                        steps=3)
    initial, _ = ref.make_inputs(config, 6, eps=1e-5)
    clean = open_session(device, config, initial, 1e-5, **options)
    clean.step(1)
    broken = dict(initial)
    broken["tokens"] = initial["tokens"].copy()
    broken["tokens"][0] = -1
    broken["tokens"][2] = config.vocab
    session = open_session(device, config, broken, 1e-5, **options)
    session.step(1)
    assert int(session.read("position")[0]) == int(initial["position"][0]) + 1
    for name in S.MUTABLE + S.WEIGHTS + ("sincos",):
        assert session.tail_intact(name), f"{name}: tail overwritten"
    assert session.read("tokens")[1] == clean.read("tokens")[1]
