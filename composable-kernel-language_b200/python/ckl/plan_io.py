"""Plan input/output: ``ckl_exec`` statistics, a JSON description, and saved programs.

The reference's reporting tools read the ``ckl_exec`` text of a compiled program
(``benchmarks/decoder/run.py:66-78``, ``plan_stats``: kernel nodes with their reduced
dependencies, temporary resources, heap bytes).  This module

* parses the same text into the same statistics (:func:`plan_stats`) and into a structured
  plan (:func:`parse_executable_ir`: heaps, resources, kernels with geometry and edges);
* describes a compiled program as JSON (:func:`to_json`): its runtime signature, and for the
  primary and the fallback plan the native plan text (which embeds the device binary of any
  generated kernels), the ``ckl_exec`` text and its statistics;
* saves and loads compiled programs (:func:`save`, :func:`load`), so a program compiled once
  binds and runs elsewhere without the Python source, tracing or device compilation.
"""
from __future__ import annotations

import json
import re
from pathlib import Path

from .compile import CompiledPlans, Plan
from .frontend.checker import BoundParameter, BoundSignature
from .types import SCALAR_TYPES, BufferSpec

FORMAT = "ckl-b200-program"
VERSION = 1
_SCALARS = {t.name: t for t in SCALAR_TYPES}


def plan_stats(executable_ir: str) -> dict:
    """The reference harness's plan statistics of ``ckl_exec`` text."""
    plan = parse_executable_ir(executable_ir)
    topology = {k["id"]: list(k["dependencies"]) for k in plan["kernels"]}
    temporaries = [r for r in plan["resources"] if r["kind"] == "temporary"]
    return dict(nodes=len(topology), edges=sum(map(len, topology.values())), topology=topology,
                temporary_count=len(temporaries),
                temporary_heap_bytes=sum(h["bytes"] for h in plan["heaps"]))


_ATTRIBUTE = re.compile(r'(\w+) = ("[^"]*"|array<i64(?:: [-\d, ]+)?>|@[\w.]+|-?\d+ : i64|-?\d+)')


def _value(text: str):
    if text.startswith('"'):
        return text[1:-1]
    if text.startswith("array<i64"):
        inner = text[len("array<i64"):-1]
        return [int(v) for v in inner.lstrip(": ").split(",") if v.strip()] if inner else []
    if text.startswith("@"):
        return text[1:]
    return int(text.split(" : ")[0])


def parse_executable_ir(executable_ir: str) -> dict:
    """``{"name", "heaps", "resources", "kernels"}`` of ``ckl_exec`` text."""
    out = {"name": None, "heaps": [], "resources": [], "kernels": []}
    for line in executable_ir.splitlines():
        code, _, comment = line.partition("//")
        attributes = {m.group(1): _value(m.group(2)) for m in _ATTRIBUTE.finditer(code)}
        if '"ckl_exec.heap"' in code:
            out["heaps"].append(attributes)
        elif '"ckl_exec.resource"' in code:
            out["resources"].append(attributes)
        elif '"ckl_exec.kernel"' in code:
            attributes.setdefault("dependencies", [])
            attributes["label"] = comment.strip()
            out["kernels"].append(attributes)
        elif code.lstrip().startswith("})") and "name" in attributes:
            out["name"] = attributes["name"]
    return out


def _signature_json(signature: BoundSignature) -> list:
    out = []
    for p in signature.runtime:
        if isinstance(p.dtype, BufferSpec):
            out.append({"name": p.name, "kind": "buffer", "shape": list(p.dtype.shape),
                        "dtype": p.dtype.dtype.name})
        else:
            out.append({"name": p.name, "kind": "scalar", "dtype": p.dtype.name})
    return out


def _signature_from(entries: list, dimensions=()) -> BoundSignature:
    parameters = []
    for e in entries:
        if e["kind"] == "buffer":
            dtype = BufferSpec(tuple(int(d) for d in e["shape"]), _SCALARS[e["dtype"]])
        elif e["kind"] == "scalar":
            dtype = _SCALARS[e["dtype"]]
        else:
            raise ValueError(f"unknown signature entry kind {e['kind']!r}")
        parameters.append(BoundParameter(e["name"], dtype))
    return BoundSignature(tuple(parameters), tuple((str(n), int(v)) for n, v in dimensions))


def _plan_json(plan: Plan) -> dict:
    return {"text": plan.text, "executable_ir": plan.executable_ir, "fused": plan.fused,
            "node_names": list(plan.node_names), "stats": plan_stats(plan.executable_ir),
            "heap_bytes": plan.heap_bytes, "baseline_bytes": plan.baseline_bytes}


def _plan_from(entry: dict) -> Plan:
    stats = plan_stats(entry["executable_ir"])
    return Plan(entry["text"], entry["executable_ir"], list(entry["node_names"]), stats["nodes"],
                stats["edges"], stats["temporary_count"], int(entry["heap_bytes"]),
                int(entry["baseline_bytes"]), stats["topology"], bool(entry["fused"]))


def to_json(program) -> str:
    """JSON description of a :class:`ckl.CompiledProgram` (loadable by :func:`load`)."""
    plans = program.plans
    document = {"format": FORMAT, "version": VERSION,
                "target": program.target.chip if program.target else "sm_100a",
                "signature": _signature_json(program.signature),
                "dimensions": [list(d) for d in program.signature.dimensions],
                "primary": _plan_json(plans.primary),
                "fallback": _plan_json(plans.fallback) if plans.fallback else None,
                "device_ir": plans.device_ir, "host_ir": plans.host_ir}
    return json.dumps(document, indent=1)


def save(program, path) -> None:
    Path(path).write_text(to_json(program))


def from_json(text: str):
    """A :class:`ckl.CompiledProgram` from :func:`to_json` output."""
    from .compiler import NVIDIATarget
    from .cuda import CompiledProgram

    document = json.loads(text)
    if document.get("format") != FORMAT or document.get("version") != VERSION:
        raise ValueError("not a ckl-b200 program description (format/version mismatch)")
    plans = CompiledPlans(_plan_from(document["primary"]),
                          _plan_from(document["fallback"]) if document["fallback"] else None,
                          device_ir=document.get("device_ir", ""),
                          host_ir=document.get("host_ir", ""))
    signature = _signature_from(document["signature"], document.get("dimensions", ()))
    return CompiledProgram.from_plans(signature, plans,
                                      NVIDIATarget(document.get("target", "sm_100a")))


def load(path):
    return from_json(Path(path).read_text())
