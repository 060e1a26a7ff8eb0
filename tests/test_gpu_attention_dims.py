"""Decode attention at every head dimension it is built for, against the oracle.

``ckl.fused.attention`` gives each (request, head) one CTA of eight warps that streams the K and
V rows 0..p, D/4 lanes per row and four rows deep per warp, with an online softmax merged across
lane groups and warps (the reference computes the same attention serially per (request, head),
``benchmarks/decoder/workloads.py:100-142``).  The cases keep the cache below 128 rows, so the
unsplit kernel runs whatever the batch (``attention_splits``), and 97-100 rows leave partial
rounds at each head dimension (16, 32, 64 or 128 rows per warp round); 3 requests run the FFMA
projections, 20 the tensor-core path, where attention writes the context as the o
projection's split panel.  Tokens, history and position exact; logits and appended cache rows
within 1e-4 relative / 1e-5 absolute.
"""
from __future__ import annotations

import pytest

import ckl
from ckl.compile import attention_splits
from ckl.workloads import session as S
from oracle import decoder as ref
from test_gpu_decoder import verify

pytestmark = pytest.mark.gpu
EPS = 1e-6


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


@pytest.mark.parametrize("heads,hidden", [(4, 64), (4, 128), (2, 128), (2, 256)],
                         ids=["d16", "d32", "d64", "d128"])
@pytest.mark.parametrize("batch", [3, 20], ids=["ffma", "tensor-cores"])
def test_attention_head_dims_match_oracle(device, heads, hidden, batch):
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=2, ffn=160, vocab=300,
                        context=97, steps=3)
    assert attention_splits(batch, heads, config.capacity) == 1
    initial, _ = ref.make_inputs(config, 17, eps=EPS)
    expected = ref.expected(initial, config, config.steps, eps=EPS)
    session = S.DecoderSession(device, initial, epsilon=EPS,
                               attention_scale=config.head_dim ** -0.5, whole_step=False)
    assert "ckl.fused.attention" in session.invocation.node_names
    session.step(config.steps)
    verify(session, initial, expected, config)
