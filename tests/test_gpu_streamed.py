"""Streamed few-row projections (one to eight requests, weights of 1 MB or more) vs the oracle.

Up to eight requests, a projection whose weights are 1 MB or more runs the streamed few-row FFMA
kernel (``gemm.cuh``, configs 9-18: 8 to 64 columns per CTA by shape), with
its RMSNorm or SwiGLU prologue staged in shared memory and the fused store / residual / RoPE /
KV-append / logits + argmax epilogues.  The reference computes every projection as a plain
FP32 dot product per output (``benchmarks/decoder/workloads.py:61-69``).

Cases: hidden 512 (every projection streamed, LM head of 1000 columns: a partial last CTA)
with one to three requests (the four-row build, unused rows) and five and eight (the eight-row
build), and eleven and sixteen with FFMA projections forced (two row groups of the eight-row
build on every column block); hidden 256 with two and seven requests (q/k/v/o below the threshold on the 32-column
kernel, gate/up and the 4096-deep SwiGLU down projection streamed, a 20000-column LM head on
64-column CTAs with a partial last CTA).  Tokens, history and
position exact; logits and appended cache rows within 1e-4 relative / 1e-5 absolute.
"""
from __future__ import annotations

import pytest

import ckl
from ckl.workloads import session as S
from oracle import decoder as ref
from test_gpu_decoder import verify

pytestmark = pytest.mark.gpu
EPS = 1e-6


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


@pytest.mark.parametrize("batch,hidden,heads,ffn,vocab,layers,tensor_cores", [
    (1, 512, 8, 1408, 1000, 2, True),
    (2, 512, 8, 1408, 1000, 2, True),
    (3, 512, 8, 1408, 1000, 2, True),
    (5, 512, 8, 1408, 1000, 2, True),
    (8, 512, 8, 1408, 1000, 2, True),
    (11, 512, 8, 1408, 1000, 2, False),
    (16, 512, 8, 1408, 1000, 2, False),
    (2, 256, 4, 4096, 20000, 1, True),
    (7, 256, 4, 4096, 20000, 1, True),
])
def test_streamed_projections_match_oracle(device, batch, hidden, heads, ffn, vocab, layers,
                                           tensor_cores):
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=layers, ffn=ffn,
                        vocab=vocab, context=20, steps=3)
    initial, _ = ref.make_inputs(config, 23, eps=EPS)
    expected = ref.expected(initial, config, config.steps, eps=EPS)
    session = S.DecoderSession(device, initial, epsilon=EPS,
                               attention_scale=config.head_dim ** -0.5, whole_step=False,
                               tensor_cores=tensor_cores)
    names = session.invocation.node_names
    assert "ckl.fused.norm_linear_argmax" in names and "ckl.fused.panel_gate_up" not in names
    session.step(config.steps)
    verify(session, initial, expected, config)
