"""Batched projections on tcgen05 tensor cores (3xTF32) match the FP32 oracle.

The fused decoder switches to the tensor-core path at 17 or more requests: RMSNorm, attention
and SwiGLU write split operand panels and the projections read them with the FP32 weights.
These cases cover full and ragged row tiles, K not a multiple of the 32-wide slice (and not of
the 8-wide MMA step), N not a multiple of the column tile or of 4 (weights read without bulk
copies), every epilogue (RoPE, KV append, residual, argmax head), and check that no kernel
reported an expired wait or a misaligned panel.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

import ckl
from ckl import _native
from ckl.workloads import session as S
from oracle import decoder as ref
from test_gpu_decoder import verify

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


def faults():
    value = C.c_uint32()
    assert _native.load().ckl_library_faults(C.byref(value), 1) == 0
    return value.value


CASES = [
    (128, 256, 4, 2, 512, 1024, 3),    # one full row tile, head dim 64
    (300, 128, 2, 1, 96, 1000, 3),     # ragged rows, K = 96, N tails
    (512, 1024, 16, 1, 4096, 4000, 2), # cfg5 layer shapes, 4 row tiles (smaller vocab)
    (128, 1024, 16, 4, 4096, 32000, 2),  # cfg5 depth and vocabulary
    (200, 64, 2, 1, 98, 1001, 2),      # K = 98 (ragged MMA step), N % 4 != 0, head dim 32
    (129, 96, 3, 2, 160, 520, 2),      # one row in the second tile, C = 96, head dim 32
    (300, 256, 4, 2, 512, 1000, 2),    # C = 256: q/k/v as one launch when pairs are forced
]
# The same shapes with the 2-SM pair kernels taken wherever there are two row tiles: "wide"
# (CKL_B200_TC_PAIRS=2) puts every projection with 256 or more outputs on 256-wide pair tiles
# (K split over pairs of a cluster where the grid is small), "narrow" (=3) puts q/k/v/o/down
# on 128-wide ones.  Covered: odd row-tile counts (a pair whose second CTA has no rows), ragged
# K and MMA steps, N % 4 != 0 (weights read without tensor copies), outputs and vocabularies
# that end inside a tile.
PAIR_CASES = [c for c in CASES if c[0] > 128] + [
    (256, 64, 2, 1, 256, 512, 2),      # one pair, exact tiles
    (640, 128, 4, 1, 384, 32000, 2),   # five row tiles, cfg5 vocabulary
    (384, 384, 6, 1, 256, 700, 2),     # three 128-wide column tiles, K = 384
]
MODES = {"wide": "2", "narrow": "3"}


@pytest.mark.parametrize("pairs", ["heuristic", "wide", "narrow"])
@pytest.mark.parametrize("batch,hidden,heads,layers,ffn,vocab,steps", CASES)
def test_tensor_core_decoder_matches_oracle(device, monkeypatch, pairs, batch, hidden, heads,
                                            layers, ffn, vocab, steps):
    if pairs in MODES:
        if (batch, hidden, heads, layers, ffn, vocab, steps) not in PAIR_CASES:
            pytest.skip("one row tile: no pair kernel")
        monkeypatch.setenv("CKL_B200_TC_PAIRS", MODES[pairs])
    run_case(device, batch, hidden, heads, layers, ffn, vocab, steps)


@pytest.mark.parametrize("pairs", ["wide", "narrow"])
@pytest.mark.parametrize("batch,hidden,heads,layers,ffn,vocab,steps", PAIR_CASES[-3:])
def test_pair_kernel_shapes_match_oracle(device, monkeypatch, pairs, batch, hidden, heads, layers,
                                         ffn, vocab, steps):
    monkeypatch.setenv("CKL_B200_TC_PAIRS", MODES[pairs])
    run_case(device, batch, hidden, heads, layers, ffn, vocab, steps)


def run_case(device, batch, hidden, heads, layers, ffn, vocab, steps):
    import os
    forced = os.environ.get("CKL_B200_TC_PAIRS") in ("2", "3")
    faults()
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=layers, ffn=ffn,
                        vocab=vocab, context=8, steps=steps)
    initial, _ = ref.make_inputs(config, 21, eps=1e-6)
    expected = ref.expected(initial, config, steps, eps=1e-6)
    # whole_step=False: small decoders would otherwise run as one whole-step kernel.
    session = S.DecoderSession(device, initial, epsilon=1e-6,
                               attention_scale=config.head_dim ** -0.5, whole_step=False)
    names = session.invocation.node_names
    assert "ckl.fused.panel_gate_up" in names
    # q, k and v run as one pair launch when each is a whole number of 256-wide tiles and
    # there are two row tiles (always when pairs are forced; at the cfg5 layer shapes anyway).
    if hidden % 256 == 0 and batch > 128 and (forced or hidden == 1024):
        assert "ckl.fused.panel_qkv" in names and "ckl.fused.panel_linear_rope" not in names
    session.step(steps)
    verify(session, initial, expected, config)
    assert faults() == 0
