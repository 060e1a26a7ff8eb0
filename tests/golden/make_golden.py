"""Generate the committed golden fixtures from the reference checkout.

Run in the build container (where the reference checkout exists)::

    python tests/golden/make_golden.py --reference <reference checkout>

Outputs, all small and committed beside this script:

* ``published_cases.json`` - the reference's published known-answer vectors: for every case
  of ``benchmarks/decoder/results/deep-dive/matrix.json`` and ``results/rtx5060ti.json`` the
  config, seed, prompts, generated token IDs and the plan statistics (kernel nodes,
  reduced edges, temporaries, temporary heap bytes with and without storage reuse, and the
  reduced topology).  These were produced on the reference's GPU path.
* ``reference_outputs.npz`` - outputs of the reference's own NumPy decoder
  (``benchmarks/decoder/reference.py``, imported, not copied) on the small BASELINE
  configurations: post-prefill state digests and K-step logits, KV rows, tokens and history.
  They pin the restatement in ``oracle/decoder.py`` to the reference module bit for bit.

Nothing at test time reads the reference checkout; the tests read only these files.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

# Small BASELINE shapes (seeded) that the reference NumPy decoder runs in seconds.
REFERENCE_RUNS = {
    # name: (Config kwargs, seed, epsilon, steps)
    "cfg1_eps1e-5": (dict(batch=1, hidden=64, heads=4, layers=2, ffn=256, vocab=512,
                          context=16, steps=16), 0, 1e-5, 16),
    "cfg1_eps1e-6": (dict(batch=1, hidden=64, heads=4, layers=2, ffn=256, vocab=512,
                          context=16, steps=16), 0, 1e-6, 16),
    "awkward": (dict(batch=3, hidden=48, heads=3, layers=1, ffn=80, vocab=129,
                     context=3, steps=16), 123, 1e-5, 16),
    "cfg3_b8": (dict(batch=8, hidden=256, heads=8, layers=2, ffn=1024, vocab=512,
                     context=16, steps=16), 2, 1e-6, 4),
}


def load_reference_module(root: Path):
    path = root / "benchmarks" / "decoder" / "reference.py"
    spec = importlib.util.spec_from_file_location("ckl_reference_oracle", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def published(root: Path) -> dict:
    results = root / "benchmarks" / "decoder" / "results"
    cases = []
    for source in (results / "deep-dive" / "matrix.json", results / "rtx5060ti.json"):
        data = json.loads(source.read_text())
        seed = data["configuration"]["seed"]
        names = data["configuration"].get("cases", [])
        for index, case in enumerate(data["cases"]):
            plans = {}
            for reuse, plan in case["plans"].items():
                plans[reuse] = {key: plan[key] for key in
                                ("nodes", "edges", "temporary_count", "temporary_heap_bytes",
                                 "topology")}
            cases.append({
                "source": str(source.relative_to(root)),
                "name": case.get("name") or (names[index] if index < len(names) else str(index)),
                "config": case["config"], "seed": seed,
                "prompts": case["prompts"], "generated_tokens": case["generated_tokens"],
                "plans": plans,
            })
    return {"cases": cases}


def reference_outputs(module) -> dict:
    out = {}
    for name, (kwargs, seed, eps, steps) in REFERENCE_RUNS.items():
        config = module.Config(**kwargs)
        module.EPSILON = np.float32(eps)
        initial, prompts = module.make_inputs(config, seed)
        result = module.expected(initial, config, steps)
        pos0 = int(initial["position"][0])
        out[f"{name}/prompts"] = prompts
        out[f"{name}/initial_kc_sum"] = np.array(
            [np.float64(initial["kc"][:, :, :, :pos0].sum())])
        out[f"{name}/history"] = result["history"]
        out[f"{name}/tokens"] = result["tokens"]
        out[f"{name}/position"] = result["position"]
        out[f"{name}/logits"] = result["logits"]
        # The rows written by the measured steps only (keeps the fixture small).
        out[f"{name}/kc_rows"] = result["kc"][:, :, :, pos0:pos0 + steps]
        out[f"{name}/vc_rows"] = result["vc"][:, :, :, pos0:pos0 + steps]
    module.EPSILON = np.float32(1e-5)
    return out


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    (HERE / "published_cases.json").write_text(json.dumps(published(args.reference)) + "\n")
    module = load_reference_module(args.reference)
    arrays = reference_outputs(module)
    np.savez_compressed(HERE / "reference_outputs.npz", **arrays)
    meta = {name: {"config": kwargs, "seed": seed, "epsilon": eps, "steps": steps}
            for name, (kwargs, seed, eps, steps) in REFERENCE_RUNS.items()}
    (HERE / "reference_runs.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")))


if __name__ == "__main__":
    main()
