"""Generate ``cfg5_prefill.npz``: the reference decoder's own prefill of two benchmark requests.

Run in the build container (where the reference checkout exists)::

    python tests/golden/make_cfg5_prefill.py --reference <reference checkout>

The benchmark's default workload is BASELINE config 5 as a 512-request shard per GPU: hidden
1024, 16 heads of 64, SwiGLU 4096, vocabulary 32000, 4 layers, 2048-token prompts, cache
capacity 2080, seed 4, RMSNorm epsilon 1e-6.  Its prompts are drawn for every request of the
shard after the weights (``benchmarks/decoder/reference.py:78-97``).  Requests never interact,
so the reference's teacher-forced prefill of a subset of requests gives exactly the state
those requests have in the full shard.  This script runs the reference module's own ``step``
(``reference.py:40-76``, imported from the checkout, with its ``EPSILON`` set to 1e-6) for the
2047 teacher-forced positions of requests 0 and 511 of shard 0 and stores:

* ``requests`` - the shard's request indices;
* ``history`` - the greedy token of every prefill position, ``[2047, 2]`` int32;
* ``tokens`` - the last prompt token (the first measured step's input), ``[2]``;
* ``positions`` and ``kc_rows`` / ``vc_rows`` - the appended key and value rows at cache
  positions 0, 1023 and 2046, ``[3, layers, 2, heads, head_dim]`` float32.

The weights come from ``oracle.decoder.make_weights`` (the reference draw order, pinned bit
for bit against ``reference.make_inputs`` by ``tests/test_oracle.py``).  The GPU test
``tests/test_gpu_cfg5.py`` compares the batched prefill of the full shard against this file.
About three minutes on one core.
"""
from __future__ import annotations

import argparse
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

SHARD = 512
REQUESTS = (0, 511)
POSITIONS = (0, 1023, 2046)
SHAPE = dict(hidden=1024, heads=16, layers=4, ffn=4096, vocab=32000, context=2048, steps=32)
SEED, EPSILON = 4, 1e-6


def load_reference_module(root: Path):
    path = root / "benchmarks" / "decoder" / "reference.py"
    spec = importlib.util.spec_from_file_location("ckl_reference_oracle", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    from oracle import decoder as oracle

    reference = load_reference_module(args.reference)
    reference.EPSILON = np.float32(EPSILON)
    full = oracle.Config(batch=SHARD, **SHAPE)
    arrays, rng = oracle.make_weights(full, SEED)
    prompts = rng.integers(0, full.vocab, (full.context, SHARD), dtype=np.int32)
    prompts = np.ascontiguousarray(prompts[:, list(REQUESTS)])
    config = reference.Config(batch=len(REQUESTS), **SHAPE)
    arrays.update(oracle.empty_state(oracle.Config(batch=len(REQUESTS), **SHAPE)))
    arrays["tokens"] = prompts[0].copy()
    for i in range(full.context - 1):
        reference.step(arrays, config)
        arrays["tokens"][:] = prompts[i + 1]
    rows = list(POSITIONS)
    np.savez_compressed(
        HERE / "cfg5_prefill.npz", requests=np.array(REQUESTS, np.int32),
        history=arrays["history"][:full.context - 1].copy(), tokens=arrays["tokens"].copy(),
        position=arrays["position"].copy(), positions=np.array(rows, np.int32),
        kc_rows=np.ascontiguousarray(np.moveaxis(arrays["kc"][:, :, :, rows, :], 3, 0)),
        vc_rows=np.ascontiguousarray(np.moveaxis(arrays["vc"][:, :, :, rows, :], 3, 0)))
    print("wrote", HERE / "cfg5_prefill.npz")
    return 0


if __name__ == "__main__":
    sys.exit(main())
