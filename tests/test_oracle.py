"""Pin the CPU oracle: published known-answer vectors and the reference module's outputs."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import decoder as ref
from oracle import vector_pipeline

PUBLISHED = json.loads((GOLDEN / "published_cases.json").read_text())["cases"]
RUNS = json.loads((GOLDEN / "reference_runs.json").read_text())
OUTPUTS = np.load(GOLDEN / "reference_outputs.npz")


@pytest.mark.parametrize("case", PUBLISHED, ids=lambda c: f"{c['source'].split('/')[-1]}:{c['name']}")
def test_published_known_answers(case):
    """Prompts and greedy tokens equal the reference's published GPU outputs."""
    config = ref.Config(**case["config"])
    initial, prompts = ref.make_inputs(config, case["seed"])
    assert prompts.tolist() == case["prompts"]
    result = ref.expected(initial, config, config.steps)
    start = config.context - 1
    generated = result["history"][start:start + config.steps]
    assert generated.tolist() == case["generated_tokens"]


@pytest.mark.parametrize("name", sorted(RUNS))
def test_matches_reference_module_bitwise(name):
    """Every mutable output equals the reference NumPy decoder bit for bit."""
    run = RUNS[name]
    config = ref.Config(**run["config"])
    initial, prompts = ref.make_inputs(config, run["seed"], eps=run["epsilon"])
    pos0 = int(initial["position"][0])
    assert np.array_equal(prompts, OUTPUTS[f"{name}/prompts"])
    assert np.float64(initial["kc"][:, :, :, :pos0].sum()) == OUTPUTS[f"{name}/initial_kc_sum"][0]
    result = ref.expected(initial, config, run["steps"], eps=run["epsilon"])
    for key in ("history", "tokens", "position", "logits"):
        assert np.array_equal(result[key], OUTPUTS[f"{name}/{key}"]), key
    steps = run["steps"]
    assert np.array_equal(result["kc"][:, :, :, pos0:pos0 + steps], OUTPUTS[f"{name}/kc_rows"])
    assert np.array_equal(result["vc"][:, :, :, pos0:pos0 + steps], OUTPUTS[f"{name}/vc_rows"])


def test_trace_records_hidden_states():
    config = ref.Config(batch=2, hidden=32, heads=2, layers=3, ffn=48, vocab=40, context=4, steps=2)
    initial, _ = ref.make_inputs(config, 5)
    trace = ref.Trace()
    ref.expected(initial, config, 2, trace=trace)
    assert len(trace.layer_inputs) == 2 * (config.layers + 1)
    assert len(trace.final_normed) == 2
    assert trace.layer_inputs[0].shape == (2, 32)


def test_config_validation():
    with pytest.raises(ValueError):
        ref.Config(hidden=64, heads=3)
    with pytest.raises(ValueError):
        ref.Config(layers=17)
    with pytest.raises(ValueError):
        ref.Config(hidden=12, heads=4)  # odd head dimension


def test_position_capacity_guard():
    config = ref.Config(batch=1, hidden=8, heads=2, layers=1, ffn=8, vocab=8, context=1, steps=1)
    state, _ = ref.make_inputs(config, 0)
    ref.decode_step(state, config)
    ref.decode_step(state, config)
    assert int(state["position"][0]) == config.capacity
    with pytest.raises(ValueError):
        ref.decode_step(state, config)


def test_normal002_init_differs_but_is_seeded():
    config = ref.Config(batch=1, hidden=16, heads=2, layers=1, ffn=16, vocab=32, context=2, steps=2)
    a, _ = ref.make_weights(config, 3, "normal002")
    b, _ = ref.make_weights(config, 3, "normal002")
    c, _ = ref.make_weights(config, 3, "reference")
    assert np.array_equal(a["wq"], b["wq"]) and not np.array_equal(a["wq"], c["wq"])
    assert abs(float(a["wq"].std()) - 0.02) < 0.01


def test_vector_pipeline_two_roundings():
    src = np.array([1 + 2 ** -23, -0.5, 0.25], dtype=np.float32)
    out = vector_pipeline.pipeline(src, 0.125)
    expected = (src + np.float32(0.125)) + np.float32(0.125)
    assert out.tobytes() == expected.tobytes()
    assert vector_pipeline.make_source(4, 1).dtype == np.float32
