"""Plan I/O (CPU): ``ckl_exec`` statistics as the reference harness computes them, the JSON
description of a compiled program, and save/load round trips (no GPU needed: programs are
built from plan text without touching a device)."""
from __future__ import annotations

import json

import ckl
from ckl import plan_io
from ckl.workloads import decoder, vector_pipeline
from oracle import decoder as ref
from test_planner import decoder_signature, plan_stats as reference_plan_stats

TARGET = ckl.NVIDIATarget("sm_100a")
N = ckl.dim("N")
Vector = ckl.Buffer[ckl.f32, (N,)]
update = vector_pipeline.update


@ckl.kernel
def square_plus(src: Vector, dst: Vector, bias: ckl.f32) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = src[i] * src[i] + bias


@ckl.program
def mixed(src: Vector, dst: Vector, bias: ckl.f32) -> None:
    temp = ckl.empty_like(src)
    ckl.launch(update, src, temp, bias, grid=(ckl.cdiv(N, 256),), block=(256,))
    ckl.launch(square_plus, temp, dst, bias, grid=(ckl.cdiv(N, 128),), block=(128,))


def programs():
    config = ref.Config(batch=2, hidden=64, heads=4, layers=2, ffn=256, vocab=512, context=16,
                        steps=2)
    spec = ckl.BufferSpec((1000,), ckl.f32)
    yield decoder.decode.lower(signature=decoder_signature(config)).compile(target=TARGET)
    yield vector_pipeline.lower(257).compile(target=TARGET)
    yield mixed.lower(signature={"src": spec, "dst": spec, "bias": ckl.f32}).compile(target=TARGET)


def test_stats_equal_the_reference_parser():
    for program in programs():
        for ir in (program.executable_ir, program.fallback_ir):
            if ir:
                assert plan_io.plan_stats(ir) == reference_plan_stats(ir)
        assert program.plan_stats == reference_plan_stats(program.executable_ir)


def test_parsed_plan_has_geometry_edges_and_resources():
    program = next(programs())
    plan = plan_io.parse_executable_ir(program.executable_ir)
    assert plan["name"].endswith(".exec")
    assert len(plan["kernels"]) == program.plans.primary.nodes
    first = plan["kernels"][0]
    assert set(first) >= {"id", "kernel", "grid", "block", "shared_memory", "dependencies", "label"}
    assert len(first["grid"]) == 3 and len(first["block"]) == 3
    assert {r["kind"] for r in plan["resources"]} <= {"external", "temporary", "persistent"}


def test_json_round_trip_rebuilds_the_same_program(tmp_path):
    for program in programs():
        document = json.loads(program.to_json())
        assert document["format"] == "ckl-b200-program"
        assert document["primary"]["stats"] == json.loads(json.dumps(program.plan_stats))
        path = tmp_path / "program.json"
        program.save(path)
        loaded = ckl.load_program(path)
        assert loaded.plans.primary.text == program.plans.primary.text
        assert loaded.executable_ir == program.executable_ir
        assert loaded.fallback_ir == program.fallback_ir
        assert loaded.signature == program.signature
        assert loaded.plan_stats == program.plan_stats


def test_generated_device_code_travels_with_the_plan():
    *_, program = programs()
    document = json.loads(program.to_json())
    assert "binary hex 7f454c46" in document["primary"]["text"]
    assert "__global__ void ckl_gen_square_plus_" in document["device_ir"]
