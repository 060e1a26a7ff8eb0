"""CPU oracle for the CKL decode step.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.

It restates the reference's independent NumPy decoder
(``benchmarks/decoder/reference.py``) with two changes that the reference fixes as
globals or leaves implicit:

* the RMSNorm epsilon is a parameter (the reference hard-codes ``EPSILON = 1e-5`` at
  ``reference.py:33``; the decode program receives it as a runtime scalar, ``run.py:146``);
* every step can record the residual stream entering each layer and the final normed
  hidden state, so hidden states can be compared, not only logits.

Float32 arithmetic is kept in the reference's operation order so that the greedy tokens
reproduce the reference bit for bit (pinned by ``tests/golden``: the published prompts and
generated token IDs of ``results/deep-dive/matrix.json``).

Parity of this restatement is pinned two ways: against the published token vectors and
against the reference module itself, imported in the build container by
``tests/golden/make_golden.py``.
"""
from __future__ import annotations

from dataclasses import dataclass, field
import numpy as np

#: Buffers the decode step mutates (``reference.py:32``).
MUTABLE = ("tokens", "position", "history", "kc", "vc", "logits")
#: Value of every never-written cache / logits element (``reference.py:99-101``).
SENTINEL = -12345
#: The reference's default RMSNorm epsilon (``reference.py:33``).
REFERENCE_EPSILON = 1e-5
#: Draw order of the weight tensors (``reference.py:82-92``); the RNG stream depends on it.
WEIGHT_ORDER = ("emb", "norm1", "norm2", "final_norm", "wq", "wk", "wv", "wo",
                "wg", "wu", "wd", "lm")


@dataclass(frozen=True)
class Config:
    """Decoder shape; same fields and validation as ``reference.py:7-29``."""

    batch: int = 1
    hidden: int = 64
    heads: int = 4
    layers: int = 2
    ffn: int = 128
    vocab: int = 256
    context: int = 8
    steps: int = 16

    def __post_init__(self):
        values = (self.batch, self.hidden, self.heads, self.layers, self.ffn, self.vocab,
                  self.context, self.steps)
        if min(values) <= 0 or self.hidden % self.heads or (self.hidden // self.heads) % 2:
            raise ValueError("positive dimensions and an even head dimension dividing hidden "
                             "are required")
        if self.layers > 16:
            raise ValueError("this small decoder benchmark supports at most 16 layers")

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def capacity(self) -> int:
        return self.context + self.steps


def weight_shapes(c: Config) -> dict[str, tuple[int, ...]]:
    h, l = c.hidden, c.layers
    return {"emb": (c.vocab, h), "norm1": (l, h), "norm2": (l, h), "final_norm": (1, h),
            "wq": (l, h, h), "wk": (l, h, h), "wv": (l, h, h), "wo": (l, h, h),
            "wg": (l, h, c.ffn), "wu": (l, h, c.ffn), "wd": (l, c.ffn, h),
            "lm": (1, h, c.vocab)}


def rms_norm(x: np.ndarray, gain: np.ndarray, eps: np.float32) -> np.ndarray:
    """``x * (1/sqrt(mean(x^2) + eps)) * gain`` in float32 (``reference.py:36-37``)."""
    mean_square = np.mean(x * x, axis=-1, keepdims=True)
    return x * (1 / np.sqrt(mean_square + eps)) * gain


@dataclass
class Trace:
    """Optional per-step capture of hidden states (residual stream per layer input)."""

    layer_inputs: list = field(default_factory=list)
    final_normed: list = field(default_factory=list)


def decode_step(state: dict, c: Config, eps: float = REFERENCE_EPSILON,
                trace: Trace | None = None) -> None:
    """Advance every request by one token, mutating ``state`` (``reference.py:40-76``).

    ``state`` holds the program buffers by their decode-program argument names.
    """
    eps32 = np.float32(eps)
    pos = int(state["position"][0])
    if not 0 <= pos < c.capacity:
        raise ValueError("position exceeds KV/history capacity")
    b, a, d = c.batch, c.heads, c.head_dim
    x = state["emb"][state["tokens"]].copy()
    cos = state["sincos"][pos, :, 0]
    sin = state["sincos"][pos, :, 1]
    scale = np.float32(d ** -0.5)

    def rotate(v: np.ndarray) -> np.ndarray:
        pairs = v.reshape(b, a, d // 2, 2)
        even, odd = pairs[..., 0], pairs[..., 1]
        out = np.empty_like(pairs)
        out[..., 0] = even * cos - odd * sin
        out[..., 1] = even * sin + odd * cos
        return out.reshape(b, a, d)

    kc, vc = state["kc"], state["vc"]
    for layer in range(c.layers):
        if trace is not None:
            trace.layer_inputs.append(x.copy())
        normed = rms_norm(x, state["norm1"][layer], eps32)
        q = rotate(normed @ state["wq"][layer])
        k = rotate(normed @ state["wk"][layer])
        v = (normed @ state["wv"][layer]).reshape(b, a, d)
        kc[layer, :, :, pos, :] = k
        vc[layer, :, :, pos, :] = v
        keys = kc[layer, :, :, :pos + 1, :]
        values = vc[layer, :, :, :pos + 1, :]
        scores = np.sum(q[:, :, None, :] * keys, axis=-1) * scale
        weights = np.exp(scores - scores.max(axis=-1, keepdims=True))
        weights /= weights.sum(axis=-1, keepdims=True)
        context = np.sum(weights[..., None] * values, axis=-2).reshape(b, c.hidden)
        residual = x + context @ state["wo"][layer]
        normed = rms_norm(residual, state["norm2"][layer], eps32)
        gate = normed @ state["wg"][layer]
        up = normed @ state["wu"][layer]
        x = residual + (gate / (1 + np.exp(-gate)) * up) @ state["wd"][layer]
    final = rms_norm(x, state["final_norm"][0], eps32)
    if trace is not None:
        trace.layer_inputs.append(x.copy())
        trace.final_normed.append(final.copy())
    state["logits"][:] = final @ state["lm"][0]
    state["tokens"][:] = state["logits"].argmax(axis=-1).astype(np.int32)
    state["history"][pos] = state["tokens"]
    state["position"][0] += 1


def make_weights(c: Config, seed: int, init: str = "reference") -> tuple[dict, np.random.Generator]:
    """Seeded weights and the RoPE table (``reference.py:78-94``).

    ``init="reference"`` follows the reference draw (emb ~ N(0, 0.5), projections
    ~ N(0, 0.5/sqrt(fan_in)), gains 1 + N(0, 0.02)); ``init="normal002"`` draws every
    projection and the embedding from N(0, 0.02) in the same order (BASELINE wording).
    Returns the generator so prompts continue the same stream.
    """
    if init not in ("reference", "normal002"):
        raise ValueError("init must be 'reference' or 'normal002'")
    rng = np.random.default_rng(seed)
    arrays = {}
    for name in WEIGHT_ORDER:
        shape = weight_shapes(c)[name]
        if "norm" in name:
            arrays[name] = (1 + rng.normal(0, 0.02, shape)).astype(np.float32)
        else:
            if init == "reference":
                sigma = 0.5 if name == "emb" else 0.5 / np.sqrt(shape[-2])
            else:
                sigma = 0.02
            arrays[name] = rng.normal(0, sigma, shape).astype(np.float32)
    t, d = c.capacity, c.head_dim
    inverse_frequency = 10000. ** (-np.arange(0, d, 2) / d)
    angles = np.arange(t)[:, None] * inverse_frequency[None, :]
    arrays["sincos"] = np.stack((np.cos(angles), np.sin(angles)), axis=-1).astype(np.float32)
    return arrays, rng


def empty_state(c: Config) -> dict:
    t, b = c.capacity, c.batch
    cache = (c.layers, b, c.heads, t, c.head_dim)
    return {"position": np.array([0], dtype=np.int32),
            "history": np.full((t, b), -1, dtype=np.int32),
            "kc": np.full(cache, SENTINEL, dtype=np.float32),
            "vc": np.full(cache, SENTINEL, dtype=np.float32),
            "logits": np.full((b, c.vocab), SENTINEL, dtype=np.float32)}


def make_prompts(c: Config, rng: np.random.Generator) -> np.ndarray:
    """``[context, batch]`` int32 prompts drawn after the weights (``reference.py:95-97``)."""
    return rng.integers(0, c.vocab, (c.context, c.batch), dtype=np.int32)


def make_inputs(c: Config, seed: int = 123, *, eps: float = REFERENCE_EPSILON,
                init: str = "reference", prefill: bool = True,
                prompt_seed: int | None = None):
    """Weights, prompts and (optionally) the reference prefill (``reference.py:78-108``).

    The prefill runs ``context - 1`` decode steps with teacher forcing: after each step the
    token buffer is overwritten with the next prompt token, so the last prompt token is
    the input of the first measured step.  With ``prefill=False`` the state is returned at
    position 0 with ``tokens = prompts[0]`` (the GPU runs its own prefill from there).
    """
    arrays, rng = make_weights(c, seed, init)
    prompt_rng = rng if prompt_seed is None else np.random.default_rng(prompt_seed)
    prompts = make_prompts(c, prompt_rng)
    arrays.update(empty_state(c))
    arrays["tokens"] = prompts[0].copy()
    if prefill:
        for i in range(c.context - 1):
            decode_step(arrays, c, eps)
            arrays["tokens"][:] = prompts[i + 1]
    return arrays, prompts


def expected(initial: dict, c: Config, steps: int, eps: float = REFERENCE_EPSILON,
             trace: Trace | None = None) -> dict:
    """Run ``steps`` decode steps on a copy of the mutable state (``reference.py:110-114``)."""
    result = {k: (v.copy() if k in MUTABLE else v) for k, v in initial.items()}
    for _ in range(steps):
        decode_step(result, c, eps, trace)
    return result


def top2_gap(logits: np.ndarray) -> float:
    """Smallest gap between the best and second-best logit over requests (tie fragility)."""
    part = np.sort(logits, axis=-1)
    return float(np.min(part[:, -1] - part[:, -2]))
