"""The reference's decoder harness flows, run against this package.

Two flows of ``benchmarks/decoder``, restated here as tests (the harness files import the
reference's MLIR compiler at import time, so they are restated rather than imported):

* ``run_case`` (``run.py:135-212``): compile the decode program with ``fuse_pointwise=False``
  for both ``reuse_storage`` values, require the same prepared device kernels for both and no
  more temporary memory with reuse, then for every execution variant (ordinary, capture,
  inferred graph, with and without storage reuse, whole-run and grouped submissions) reset the
  state, ``benchmark(iterations=1)``, verify one step (or group), reset, benchmark the whole
  run, verify, and run it again through ``run`` and verify; the tokens must be the published
  ones.  The reference asserts ``21 * layers + 6`` nodes; that count holds here for the
  unfused plan (``fuse_library=False``), and the fused plan's count is recorded beside it.
* the independent-request burst of ``experiment.py:20-70``: one invocation (own stream, own
  mutable state and scratch, shared read-only weights) per request, driven concurrently from a
  thread pool behind a barrier through ``benchmark`` (which releases the GIL), every request's
  result checked against the oracle.  Concurrent binds (the module cache) and concurrent runs
  of one invocation (serialized by its run lock) are exercised as well.

State handling follows ``run.py:81-132``: every buffer carries a 256-element sentinel tail, and
``verify`` checks tails, unchanged weights, exact tokens/history/position and the cache prefix
and suffix, with the harness tolerances (atol 2e-5, rtol 3e-4).
"""
from __future__ import annotations

import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import ckl
from ckl.plan_io import plan_stats
from ckl.workloads import decoder
from oracle import decoder as ref
from test_gpu_decoder import PUBLISHED

pytestmark = pytest.mark.gpu
TAIL, SENTINEL = 256, -12345
SEED = 123
CASES = {
    "small": ref.Config(steps=16),
    "awkward": ref.Config(batch=3, hidden=48, heads=3, layers=1, ffn=80, vocab=129, context=3,
                          steps=16),
}


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


class State:
    """Device copies of every program buffer with sentinel tails (``run.py:81-132``)."""

    def __init__(self, device, arrays, *, shared=None):
        self.initial, self.owners, self.buffers, self.host = arrays, {}, {}, {}
        for name in decoder.ARGUMENTS[:-2]:
            values = arrays[name]
            if shared is not None and name not in ref.MUTABLE:
                assert np.array_equal(values, shared.initial[name]), name
                for table in ("owners", "buffers", "host"):
                    getattr(self, table)[name] = getattr(shared, table)[name]
                continue
            host = np.full(values.size + TAIL, SENTINEL, dtype=values.dtype)
            host[:values.size] = values.ravel()
            dtype = ckl.i32 if values.dtype == np.int32 else ckl.f32
            owner = device.empty(ckl.BufferSpec(host.shape, dtype))
            owner.copy_from_host(host)
            self.owners[name], self.host[name] = owner, host
            self.buffers[name] = device.import_buffer(
                owner.address, ckl.BufferSpec(values.shape, dtype), owner=owner)

    def reset(self):
        for name in ref.MUTABLE:
            self.owners[name].copy_from_host(self.host[name])

    def verify(self, expected, config):
        start, end = int(self.initial["position"][0]), int(expected["position"][0])
        error = 0.0
        for name, owner in self.owners.items():
            actual = np.empty_like(self.host[name])
            owner.copy_to_host(actual)
            size = self.initial[name].size
            assert np.all(actual[size:] == SENTINEL), f"{name}: tail overwritten"
            actual = actual[:size].reshape(self.initial[name].shape)
            if name not in ref.MUTABLE:
                assert np.array_equal(actual, self.initial[name]), f"{name}: weights changed"
            elif actual.dtype == np.int32:
                assert np.array_equal(actual, expected[name]), f"{name}: mismatch"
            else:
                assert np.all(np.isfinite(actual)), name
                assert np.allclose(actual, expected[name], atol=2e-5, rtol=3e-4), name
                error = max(error, float(np.max(np.abs(actual - expected[name]))))
                if name in ("kc", "vc"):
                    assert np.array_equal(actual[:, :, :, :start],
                                          self.initial[name][:, :, :, :start]), name
                    assert np.array_equal(actual[:, :, :, end:],
                                          self.initial[name][:, :, :, end:]), name
        return error

    def arguments(self, config):
        return [self.buffers[name] for name in decoder.ARGUMENTS[:-2]] + [
            float(ref.REFERENCE_EPSILON), config.head_dim ** -0.5]


def variants(steps, groups=()):
    """The harness's execution variants (``run.py:24-37``)."""
    rows = [("sequential", False, "ordinary", 1), ("capture", False, "capture", 1),
            ("inferred", False, "graph", 1), ("sequential_reuse", True, "ordinary", 1),
            ("capture_reuse", True, "capture", 1), ("inferred_reuse", True, "graph", 1),
            ("batched_capture", True, "capture", steps), ("batched_inferred", True, "graph", steps)]
    for count in sorted(set(groups)):
        if 1 < count < steps and steps % count == 0:
            rows += [(f"group{count}_capture", True, "capture", count),
                     (f"group{count}_inferred", True, "graph", count)]
    return rows


@pytest.mark.parametrize("fuse_library", [False, True], ids=["unfused", "fused"])
@pytest.mark.parametrize("case", list(CASES))
def test_run_case_flow(device, case, fuse_library):
    config = CASES[case]
    rows = variants(config.steps, (4,))
    initial, prompts = ref.make_inputs(config, SEED)
    references = {count: ref.expected(initial, config, count)
                  for count in {1, config.steps, *(row[3] for row in rows)}}
    state = State(device, initial)
    signature = {name: buffer.spec for name, buffer in state.buffers.items()}
    signature.update(epsilon=ckl.f32, attention_scale=ckl.f32)
    lowered = decoder.decode.lower(signature=signature)
    programs, invocations, stats = {}, {}, {}
    for reuse in (False, True):
        program = lowered.compile(target=ckl.NVIDIATarget("sm_100a"), fuse_pointwise=False,
                                  reuse_storage=reuse, fuse_library=fuse_library)
        programs[reuse] = program
        invocations[reuse] = program.bind(*state.arguments(config))
        stats[reuse] = plan_stats(program.executable_ir)
        if not fuse_library:
            assert invocations[reuse].node_count == 21 * config.layers + 6
        else:
            assert invocations[reuse].node_count < 21 * config.layers + 6
    assert programs[False].prepared_ir == programs[True].prepared_ir
    assert stats[True]["temporary_heap_bytes"] <= stats[False]["temporary_heap_bytes"]
    for name, reuse, mode, group in rows:
        bound = invocations[reuse]
        state.reset()
        first = bound.benchmark(iterations=1, mode=mode, batch_size=group)
        assert set(first) == {"stream_us", "wall_us", "graph_setup_ms"}
        assert first["stream_us"] > 0 and first["graph_setup_ms"] >= 0
        state.verify(references[group], config)
        state.reset()
        bound.benchmark(iterations=config.steps // group, mode=mode, batch_size=group)
        state.verify(references[config.steps], config)
        state.reset()
        for _ in range(config.steps // group):
            bound.run(mode=mode, batch_size=group)
        state.verify(references[config.steps], config)
    published = next(c for c in PUBLISHED if c["name"] == case and "deep-dive" in c["source"])
    history = references[config.steps]["history"][config.context - 1:config.context - 1 + config.steps]
    assert prompts.tolist() == published["prompts"]
    assert history.tolist() == published["generated_tokens"]


def prepare(device, config, requests, *, fuse_library=True):
    """One state and invocation per request, weights shared (``experiment.py:20-38``)."""
    initial = [ref.make_inputs(config, SEED, prompt_seed=SEED + i)[0] for i in range(requests)]
    states = []
    for arrays in initial:
        states.append(State(device, arrays, shared=states[0] if states else None))
    signature = {name: buffer.spec for name, buffer in states[0].buffers.items()}
    signature.update(epsilon=ckl.f32, attention_scale=ckl.f32)
    program = decoder.decode.lower(signature=signature).compile(
        target=ckl.NVIDIATarget("sm_100a"), fuse_pointwise=False, fuse_library=fuse_library)
    references = [ref.expected(s.initial, config, config.steps) for s in states]
    return states, program, references


@pytest.mark.parametrize("mode,group", [("ordinary", 1), ("capture", 1), ("graph", 1),
                                        ("graph", 16)])
@pytest.mark.parametrize("requests", [4, 8])
def test_independent_requests_in_parallel(device, requests, mode, group):
    config = CASES["small"]
    states, program, references = prepare(device, config, requests)
    # Binds from several threads at once share the program's module cache.
    with ThreadPoolExecutor(max_workers=requests) as executor:
        invocations = list(executor.map(lambda s: program.bind(*s.arguments(config)), states))
        for _ in range(2):  # the first burst also builds every graph
            for s in states:
                s.reset()
            barrier = threading.Barrier(requests + 1)

            def worker(bound):
                barrier.wait(timeout=30)
                return bound.benchmark(iterations=config.steps // group, mode=mode,
                                       batch_size=group)

            futures = [executor.submit(worker, bound) for bound in invocations]
            barrier.wait(timeout=30)
            timings = [future.result(timeout=120) for future in futures]
            assert all(t["stream_us"] > 0 for t in timings)
            for s, expected in zip(states, references):
                s.verify(expected, config)


def test_concurrent_runs_of_one_invocation_are_serialized(device):
    """Two threads driving the same invocation: its run lock serializes whole steps, so after
    2 x 8 runs the state is exactly 16 steps on."""
    config = CASES["small"]
    (state,), program, (expected,) = prepare(device, config, 1)
    bound = program.bind(*state.arguments(config))
    barrier = threading.Barrier(2)

    def worker(mode):
        barrier.wait(timeout=30)
        for _ in range(config.steps // 2):
            bound.run(mode=mode)

    with ThreadPoolExecutor(max_workers=2) as executor:
        list(executor.map(worker, ["graph", "ordinary"]))
    state.verify(expected, config)
