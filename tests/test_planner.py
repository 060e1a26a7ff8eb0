"""Planner parity: memory planner and repeat unit cases, published decoder plans, vector plans."""
from __future__ import annotations

import ctypes as C
import json
import re

import numpy as np
import pytest

from conftest import GOLDEN
import ckl
from ckl import _native
from ckl.compile import plan_program
from ckl.workloads import decoder, vector_pipeline
from oracle import decoder as ref

PUBLISHED = json.loads((GOLDEN / "published_cases.json").read_text())["cases"]


def memory_plan(node_count, edges, resources, reuse=True):
    lib = _native.load()
    flat = [v for e in edges for v in e]
    offsets, users = [0], []
    for r in resources:
        users += r[3]
        offsets.append(len(users))
    n = len(resources)
    U64, U32 = C.c_uint64, C.c_uint32
    slots, offs = (U64 * n)(), (U64 * n)()
    base, planned = U64(), U64()
    status = lib.ckl_memory_plan(node_count, len(edges), (U32 * max(len(flat), 1))(*flat), n,
                                 (U64 * n)(*[r[0] for r in resources]), (U64 * n)(*[r[1] for r in resources]),
                                 (U32 * n)(*[r[2] for r in resources]), (U32 * (n + 1))(*offsets),
                                 (U32 * max(len(users), 1))(*users), int(reuse), C.byref(base),
                                 C.byref(planned), slots, offs)
    if status:
        raise ValueError(_native.message())
    return base.value, planned.value, list(slots)


def test_memory_planner_unit_cases():
    """Restates tests/Core/MemoryPlannerTest.cpp:18-73."""
    edges = [(0, 1), (1, 4), (2, 3), (3, 4), (4, 5), (5, 6)]
    resources = [(1024, 256, 0, [0, 1]), (512, 256, 0, [2, 3]), (768, 128, 0, [5, 6]),
                 (256, 64, 1, [0, 6]), (4096, 256, 2, [0, 6])]
    base, planned, slots = memory_plan(7, edges, resources)
    assert slots[4] == 2 ** 64 - 1                      # external: not allocated
    assert slots[0] != slots[1]                         # parallel lifetimes do not share
    assert slots[2] == slots[0]                         # ordered lifetimes share best fit
    assert slots[3] not in (slots[0], slots[1])         # persistent never recycled
    assert (base, planned) == (2560, 1792)
    base2, planned2, slots2 = memory_plan(7, edges, resources, reuse=False)
    assert planned2 == base2 and slots2[0] != slots2[2]
    _, _, s = memory_plan(2, [(0, 1)], [(64, 64, 1, [0]), (64, 64, 0, [1])])
    assert s[0] != s[1]
    with pytest.raises(ValueError, match="acyclic"):
        memory_plan(2, [(0, 1), (1, 0)], [])


def test_repeat_links_iterations():
    """Restates tests/Core/ExecutionPlanTest.cpp:34-59."""
    lib = _native.load()
    U32 = C.c_uint32
    out_off, out_deps = (U32 * 7)(), (U32 * 16)()
    assert lib.ckl_repeat_dependencies(2, (U32 * 3)(0, 0, 1), (U32 * 1)(0), 3, out_off, out_deps, 16) == 0
    deps = [list(out_deps[out_off[i]:out_off[i + 1]]) for i in range(6)]
    assert deps == [[], [0], [1], [2], [3], [4]]
    assert lib.ckl_repeat_dependencies(2, (U32 * 3)(0, 0, 1), (U32 * 1)(5), 2, out_off, out_deps, 16) != 0


def decoder_signature(config):
    arrays, _ = ref.make_inputs(config, 0, prefill=False)
    sig = {}
    for name in decoder.ARGUMENTS[:-2]:
        a = arrays[name]
        sig[name] = ckl.BufferSpec(a.shape, ckl.i32 if a.dtype == np.int32 else ckl.f32)
    sig.update(epsilon=ckl.f32, attention_scale=ckl.f32)
    return sig


def plan_stats(ir):
    """The reference harness's parser (benchmarks/decoder/run.py:66-78), restated."""
    topology = {}
    for line in ir.splitlines():
        if '"ckl_exec.kernel"' not in line:
            continue
        node = int(re.search(r"\bid = (\d+)", line).group(1))
        match = re.search(r"dependencies = array<i64(?:: ([\d, ]+))?>", line).group(1)
        topology[node] = [int(v) for v in match.split(",")] if match else []
    heaps = [l for l in ir.splitlines() if '"ckl_exec.heap"' in l]
    temporaries = [l for l in ir.splitlines()
                   if '"ckl_exec.resource"' in l and 'kind = "temporary"' in l]
    return dict(nodes=len(topology), edges=sum(map(len, topology.values())), topology=topology,
                temporary_count=len(temporaries),
                temporary_heap_bytes=sum(int(re.search(r"\bbytes = (\d+)", l).group(1)) for l in heaps))


@pytest.mark.parametrize("case", PUBLISHED, ids=lambda c: f"{c['source'].split('/')[-1]}:{c['name']}")
def test_decoder_plan_matches_published(case):
    """Nodes, reduced edges, topology, temporaries and heap bytes equal the reference's plans."""
    lowered = decoder.decode.lower(signature=decoder_signature(ref.Config(**case["config"])))
    for reuse in (False, True):
        plan = plan_program(lowered, fuse_pointwise=False, fuse_library=False, reuse_storage=reuse)
        stats = plan_stats(plan.primary.executable_ir)
        want = case["plans"][str(reuse)]
        assert stats["nodes"] == want["nodes"]
        assert stats["edges"] == want["edges"]
        assert stats["temporary_count"] == want["temporary_count"]
        assert stats["temporary_heap_bytes"] == want["temporary_heap_bytes"]
        assert {str(k): v for k, v in stats["topology"].items()} == want["topology"]


def test_fused_decoder_plan_shape():
    config = ref.Config(batch=1, hidden=64, heads=4, layers=2, ffn=256, vocab=512, context=16, steps=16)
    lowered = decoder.decode.lower(signature=decoder_signature(config))
    whole = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True)
    assert whole.primary.node_names == ["ckl.fused.decode_step"]
    assert whole.fallback.nodes == 21 * 2 + 6
    plans = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True,
                         whole_step=False)
    assert plans.primary.fused and plans.fallback is not None
    assert plans.primary.nodes == 1 + 8 * 2 + 2
    assert plans.fallback.nodes == 21 * 2 + 6
    names = plans.primary.node_names
    assert names.count("ckl.fused.attention") == 2 and names[-1] == "ckl.fused.greedy_combine"
    # Q/K/V and gate/up are independent branches of the fused graph.
    topology = plans.primary.topology
    ids = sorted(topology)
    q, k, v = ids[1], ids[2], ids[3]
    assert topology[q] == topology[k] == topology[v]
    gate, up = ids[6], ids[7]
    assert topology[gate] == topology[up]


def test_fused_qkv_node(monkeypatch):
    """cfg5-shaped layers at 512 rows plan q, k and v as one tensor-core pair launch."""
    config = ref.Config(batch=512, hidden=1024, heads=16, layers=2, ffn=4096, vocab=1000,
                        context=8, steps=8)
    lowered = decoder.decode.lower(signature=decoder_signature(config))
    plans = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True,
                         whole_step=False)
    names = plans.primary.node_names
    layer = ["ckl.fused.rms_panel", "ckl.fused.panel_qkv", "ckl.fused.attention",
             "ckl.fused.panel_linear_residual", "ckl.fused.rms_panel",
             "ckl.fused.panel_gate_up", "ckl.fused.panel_linear_residual"]
    head = ["ckl.fused.rms_panel", "ckl.fused.panel_linear_argmax", "ckl.fused.greedy_combine"]
    assert names == ["ckl.decoder.embedding"] + layer * 2 + head
    topology = plans.primary.topology
    ids = sorted(topology)
    assert topology[ids[2]] == [ids[1]] and topology[ids[3]] == [ids[2]]  # norm -> qkv -> attn
    # Pairs switched off: three projection nodes again.
    monkeypatch.setenv("CKL_B200_TC_PAIRS", "0")
    plans = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True,
                         whole_step=False)
    assert "ckl.fused.panel_qkv" not in plans.primary.node_names
    assert plans.primary.nodes == 1 + 9 * 2 + 3


def test_tensor_core_decoder_plan_shape():
    """Batches of 128+ requests: split-operand panels feed tensor-core projections."""
    config = ref.Config(batch=256, hidden=128, heads=2, layers=2, ffn=256, vocab=512, context=8,
                        steps=8)
    lowered = decoder.decode.lower(signature=decoder_signature(config))
    plans = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True,
                         whole_step=False)
    names = plans.primary.node_names
    layer = ["ckl.fused.rms_panel", "ckl.fused.panel_linear_rope",
             "ckl.fused.panel_linear_rope_append", "ckl.fused.panel_linear_append",
             "ckl.fused.attention", "ckl.fused.panel_linear_residual", "ckl.fused.rms_panel",
             "ckl.fused.panel_gate_up", "ckl.fused.panel_linear_residual"]
    head = ["ckl.fused.rms_panel", "ckl.fused.panel_linear_argmax", "ckl.fused.greedy_combine"]
    assert names == ["ckl.decoder.embedding"] + layer * 2 + head
    topology = plans.primary.topology
    ids = sorted(topology)
    norm, q, k, v = ids[1:5]
    assert topology[q] == topology[k] == topology[v] == [norm]
    gate_up, down = ids[8], ids[9]
    assert topology[gate_up] == [ids[7]] and topology[down] == [gate_up]
    # FFMA projections when tensor cores are switched off.
    ffma = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True,
                        tensor_cores=False, whole_step=False)
    assert ffma.primary.nodes == 1 + 8 * 2 + 2
    assert not any("panel" in n for n in ffma.primary.node_names)


@pytest.mark.parametrize("batch,hidden,heads,layers,ffn,vocab,context,whole", [
    (1, 64, 4, 2, 256, 512, 16, True),
    (64, 256, 8, 2, 1024, 512, 16, True),     # config 3
    (256, 64, 4, 8, 256, 512, 16, True),      # config 4
    (512, 64, 4, 1, 256, 512, 8, True),       # 32 clusters x 16 requests
    (513, 64, 4, 1, 256, 512, 8, False),      # too many requests per cluster
    (3, 48, 3, 1, 80, 129, 6, False),         # columns do not split into 8 x float4
    (33, 128, 2, 1, 96, 512, 6, True),        # three FFN quads per CTA
    (4, 1024, 16, 4, 4096, 32000, 8, False),  # weights do not stay in L2
    (24, 96, 3, 1, 256, 512, 8, False),       # three heads do not split over 8 CTAs
    (24, 256, 16, 2, 256, 512, 10, True),     # two heads per CTA
])
def test_whole_step_kernel_selection(batch, hidden, heads, layers, ffn, vocab, context, whole):
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=layers, ffn=ffn,
                        vocab=vocab, context=context, steps=4)
    lowered = decoder.decode.lower(signature=decoder_signature(config))
    plans = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True)
    assert (plans.primary.node_names == ["ckl.fused.decode_step"]) == whole
    if whole:
        # The whole step replaces every node; nothing but the cross-cluster counter persists.
        assert plans.primary.temporaries == 0 and plans.primary.edges == 0


def test_vector_pipeline_plans():
    """tests/Runtime/test_frontend_runtime.py:66-69 and test_pointwise_fusion.py:43-45."""
    lowered = vector_pipeline.lower()
    unfused = plan_program(lowered, fuse_pointwise=False, fuse_library=True, reuse_storage=True)
    assert "dependencies = array<i64: 1>" in unfused.primary.executable_ir
    assert unfused.primary.executable_ir.count('"ckl_exec.heap"') == 1
    assert unfused.primary.nodes == 2 and unfused.fallback is None
    fused = plan_program(lowered, fuse_pointwise=True, fuse_library=True, reuse_storage=True)
    assert fused.primary.executable_ir.count('"ckl_exec.kernel"') == 1
    assert '"ckl_exec.heap"' not in fused.primary.executable_ir
    assert fused.fallback.nodes == 2
    assert "@ckl_entry" in fused.host_ir and "@ckl.binary" in fused.host_ir
