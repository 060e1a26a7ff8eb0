"""Run the decoder program on a device: seeded inputs, persistent state, prefill and steps.

The reference harness (``benchmarks/decoder/run.py:81-132, 135-212``) keeps every program
buffer on the device with a 256-element sentinel tail, binds the compiled ``decode``
program once and replays it; prompt prefill is ``context - 1`` decode steps with the token
buffer overwritten by the next prompt token after each step (teacher forcing,
``reference.py:104-107``).  :class:`DecoderSession` does the same through the public CKL API.

:func:`make_weights` and :func:`make_prompts` produce the seeded synthetic inputs with the
reference's draw order (``reference.py:78-97``) so the device and any checker start from
identical arrays.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import ckl
from . import decoder

TAIL = 256
SENTINEL = -12345
MUTABLE = ("tokens", "position", "history", "kc", "vc", "logits")
WEIGHTS = ("emb", "norm1", "norm2", "final_norm", "wq", "wk", "wv", "wo", "wg", "wu", "wd", "lm")


@dataclass(frozen=True)
class DecoderShape:
    batch: int
    hidden: int
    heads: int
    layers: int
    ffn: int
    vocab: int
    context: int
    steps: int

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def capacity(self) -> int:
        return self.context + self.steps


def _shapes(c: DecoderShape) -> dict:
    h, l = c.hidden, c.layers
    return {"emb": (c.vocab, h), "norm1": (l, h), "norm2": (l, h), "final_norm": (1, h),
            "wq": (l, h, h), "wk": (l, h, h), "wv": (l, h, h), "wo": (l, h, h),
            "wg": (l, h, c.ffn), "wu": (l, h, c.ffn), "wd": (l, c.ffn, h), "lm": (1, h, c.vocab)}


def make_weights(c: DecoderShape, seed: int, init: str = "reference"):
    """Seeded weights + RoPE table and the generator positioned for the prompt draw."""
    rng = np.random.default_rng(seed)
    arrays = {}
    for name in WEIGHTS:
        shape = _shapes(c)[name]
        if "norm" in name:
            arrays[name] = (1 + rng.normal(0, 0.02, shape)).astype(np.float32)
        elif init == "reference":
            sigma = 0.5 if name == "emb" else 0.5 / np.sqrt(shape[-2])
            arrays[name] = rng.normal(0, sigma, shape).astype(np.float32)
        elif init == "normal002":
            arrays[name] = rng.normal(0, 0.02, shape).astype(np.float32)
        else:
            raise ValueError("init must be 'reference' or 'normal002'")
    d = c.head_dim
    angles = np.arange(c.capacity)[:, None] * (10000. ** (-np.arange(0, d, 2) / d))[None, :]
    arrays["sincos"] = np.stack((np.cos(angles), np.sin(angles)), axis=-1).astype(np.float32)
    return arrays, rng


def make_prompts(c: DecoderShape, rng) -> np.ndarray:
    return rng.integers(0, c.vocab, (c.context, c.batch), dtype=np.int32)


def initial_state(c: DecoderShape) -> dict:
    cache = (c.layers, c.batch, c.heads, c.capacity, c.head_dim)
    return {"tokens": np.zeros(c.batch, np.int32), "position": np.zeros(1, np.int32),
            "history": np.full((c.capacity, c.batch), -1, np.int32),
            "kc": np.full(cache, SENTINEL, np.float32), "vc": np.full(cache, SENTINEL, np.float32),
            "logits": np.full((c.batch, c.vocab), SENTINEL, np.float32)}


class DecoderSession:
    """Device buffers for one decoder instance, the compiled step and its bound invocation."""

    def __init__(self, device: ckl.Device, arrays: dict, *, epsilon: float, attention_scale: float,
                 fuse_library: bool = True, reuse_storage: bool = True, tails: bool = True,
                 tensor_cores: bool = True, library: bool = True, whole_step: bool = True,
                 shared_weights: "DecoderSession | None" = None):
        self.device = device
        self.epsilon, self.attention_scale = epsilon, attention_scale
        self.owners, self.buffers, self.shapes = {}, {}, {}
        self._batched_prefill = None
        self.tails = tails
        for name in decoder.ARGUMENTS[:-2]:
            values = arrays[name]
            # A (shape, numpy dtype) pair allocates zero-filled device storage without a host
            # copy (used for multi-gigabyte KV caches).
            shape, np_dtype = (values if isinstance(values, tuple) else (values.shape, values.dtype))
            size = int(np.prod(shape))
            dtype = ckl.i32 if np.dtype(np_dtype) == np.int32 else ckl.f32
            self.shapes[name] = (tuple(shape), np.dtype(np_dtype))
            if shared_weights is not None and name not in MUTABLE:
                self.owners[name] = shared_weights.owners[name]
                self.buffers[name] = shared_weights.buffers[name]
                continue
            extra = TAIL if tails else 0
            owner = device.empty(ckl.BufferSpec((size + extra,), dtype))
            if isinstance(values, tuple):
                owner.fill_zero()
            else:
                host = np.full(size + extra, SENTINEL, dtype=values.dtype)
                host[:size] = values.ravel()
                owner.copy_from_host(host)
            self.owners[name] = owner
            self.buffers[name] = device.import_buffer(owner.address, ckl.BufferSpec(tuple(shape), dtype),
                                                      owner=owner)
        signature = {name: self.buffers[name].spec for name in decoder.ARGUMENTS[:-2]}
        signature.update(epsilon=ckl.f32, attention_scale=ckl.f32)
        self.lowered = decoder.decode.lower(signature=signature)
        self.program = self.lowered.compile(target=ckl.NVIDIATarget("sm_100a"),
                                            fuse_library=fuse_library, reuse_storage=reuse_storage,
                                            tensor_cores=tensor_cores, library=library,
                                            whole_step=whole_step)
        arguments = [self.buffers[name] for name in decoder.ARGUMENTS[:-2]]
        self.invocation = self.program.bind(*arguments, float(epsilon), float(attention_scale))

    # ---- state -----------------------------------------------------------------------
    def read(self, name: str, *, with_tail: bool = False) -> np.ndarray:
        shape, dtype = self.shapes[name]
        owner = self.owners[name]
        host = np.empty(owner.nbytes // np.dtype(dtype).itemsize, dtype=dtype)
        owner.copy_to_host(host)
        if with_tail:
            return host
        return host[:int(np.prod(shape))].reshape(shape)

    def write(self, name: str, values: np.ndarray) -> None:
        shape, dtype = self.shapes[name]
        values = np.ascontiguousarray(values, dtype=dtype).reshape(shape)
        if self.tails:
            host = np.full(self.owners[name].nbytes // np.dtype(dtype).itemsize, SENTINEL, dtype)
            host[:values.size] = values.ravel()
            self.owners[name].copy_from_host(host)
        else:
            self.owners[name].copy_from_host(values)

    def tail_intact(self, name: str) -> bool:
        if not self.tails:
            return True
        host = self.read(name, with_tail=True)
        return bool(np.all(host[-TAIL:] == SENTINEL))

    # ---- execution -------------------------------------------------------------------
    def step(self, count: int = 1, *, mode: str = "graph", batch_size: int = 1) -> None:
        for _ in range(count // batch_size):
            self.invocation.run(mode=mode, batch_size=batch_size)

    def generate(self, steps: int, *, group: int = 1, depth: int = 2, mode: str = "graph"):
        """Greedy decode `steps` steps asynchronously; yields ``(position, tokens)`` per group
        of `group` steps, ``tokens[g, b]`` being request b's token at ``position + g``.

        Each group is one submission of `group` decode steps (the program repeated inside one
        graph launch: fewer submissions, later observation), followed on the same stream by a
        copy of the group's history rows into page-locked memory; up to `depth` groups are in
        flight while the host consumes earlier ones.  The device state afterwards equals
        ``step(steps)``."""
        if steps % group or group <= 0 or depth <= 0:
            raise ValueError("steps must be a positive multiple of group; depth positive")
        from collections import deque

        history = self.buffers["history"]
        capacity, batch = history.spec.shape
        position = int(self.read("position")[0])
        if position + steps > capacity:
            raise ValueError("generation would run past the history capacity")
        slots = [ckl.PinnedHostBuffer(group * batch * 4) for _ in range(depth)]
        pending = deque()
        for index in range(steps // group):
            if len(pending) == depth:
                yield self._observed(*pending.popleft())
            at = position + index * group
            rows = history.subview(offset=at * batch, shape=(group, batch))
            slot = slots[index % depth]
            completion = self.invocation.submit(mode=mode, batch_size=group,
                                                observe=[(rows, slot)])
            pending.append((completion, at, slot, group, batch))
        while pending:
            yield self._observed(*pending.popleft())

    @staticmethod
    def _observed(completion, at, slot, group, batch):
        completion.wait()
        return at, slot.array(np.int32, (group, batch)).copy()

    def prefill(self, prompts: np.ndarray, *, mode: str = "graph", batched: bool = False) -> None:
        """Teacher-forced prefill: ``context - 1`` steps, next prompt token after each.

        ``batched`` runs the prompt positions in chunks of all requests at once
        (:mod:`ckl.workloads.prefill`) instead of one decode step per position; the resulting
        state is the same up to floating-point rounding."""
        if batched:
            from .prefill import BatchedPrefill

            context = prompts.shape[0]
            if self._batched_prefill is None or self._batched_prefill.context != context:
                self._batched_prefill = BatchedPrefill(self, context)
            self._batched_prefill.run(prompts, mode=mode)
            return
        self.write("tokens", prompts[0])
        self.write("position", np.zeros(1, np.int32))
        for i in range(prompts.shape[0] - 1):
            self.invocation.run(mode=mode)
            self.write("tokens", prompts[i + 1])
