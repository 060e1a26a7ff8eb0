"""An expired bounded wait in a tensor-core kernel is reported, and the context stays usable.

The tensor-core projections wait on mbarriers (copy and MMA completion) with a time limit; a
wait that expires sets bit 0 of the library's fault word, the CTA abandons its tile (draining
its own copies and MMAs, freeing its tensor memory) and returns.  The runtime reads the word
after every synchronizing call of an invocation that contains such a kernel and fails the call.
Here the failure is made on purpose without any fault on the GPU: the test hook makes every
tensor-core CTA wait on an mbarrier that nothing signals, with a one-millisecond limit.  The
step must fail with the fault reported, the word must stay set until cleared, and after the
hook is removed the same invocation must reproduce the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

import ckl
from ckl import _native
from ckl.workloads import session as S
from oracle import decoder as ref
from test_gpu_decoder import verify

pytestmark = pytest.mark.gpu
DEFAULT_LIMIT_NS = 2_000_000_000


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


@pytest.mark.parametrize("batch,hidden,heads,ffn,vocab,pairs", [
    (32, 64, 2, 96, 300, None),       # unsplit tiles
    (32, 512, 8, 1024, 1000, None),   # q/k/v/o split over 8-CTA clusters (K = 512)
    (256, 64, 2, 256, 512, "2"),      # gate/up and LM head on 2-SM CTA pairs
    (256, 512, 8, 1024, 1000, "3"),   # q/k/v/o/down on 128-wide pairs, K split over 4 pairs
])
def test_expired_wait_fails_the_step_and_the_context_recovers(device, monkeypatch, batch, hidden,
                                                              heads, ffn, vocab, pairs):
    if pairs:
        monkeypatch.setenv("CKL_B200_TC_PAIRS", pairs)
    config = ref.Config(batch=batch, hidden=hidden, heads=heads, layers=1, ffn=ffn, vocab=vocab,
                        context=4, steps=2)
    initial, _ = ref.make_inputs(config, 5, eps=1e-6)
    expected = ref.expected(initial, config, 1, eps=1e-6)
    session = S.DecoderSession(device, initial, epsilon=1e-6,
                               attention_scale=config.head_dim ** -0.5, whole_step=False)
    lib = _native.load()
    assert _native.library_faults(reset=True) == 0
    try:
        _native.check(lib.ckl_set_wait_limit(device.ordinal, 1_000_000), "wait limit")
        _native.check(lib.ckl_inject_unsignalled_wait(device.ordinal, 1), "inject")
        with pytest.raises(RuntimeError, match="bounded wait"):
            session.step(1)
        assert _native.library_faults() & 1
        # The word stays set: later synchronizing calls keep failing until it is cleared.
        with pytest.raises(RuntimeError, match="fault word"):
            session.invocation.synchronize()
    finally:
        _native.check(lib.ckl_inject_unsignalled_wait(device.ordinal, 0), "inject")
        _native.check(lib.ckl_set_wait_limit(device.ordinal, DEFAULT_LIMIT_NS), "wait limit")
        _native.library_faults(reset=True)
    session.invocation.synchronize()
    for name in S.MUTABLE:
        session.write(name, initial[name])
    session.step(1)
    verify(session, initial, expected, config)
    assert _native.library_faults() == 0
