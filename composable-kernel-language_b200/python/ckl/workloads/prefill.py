"""Batched prompt prefill for a :class:`~ckl.workloads.session.DecoderSession`.

The reference prefills by replaying the decode step once per prompt token with the next prompt
token forced into the token buffer (``benchmarks/decoder/reference.py:98-108``): a context of
2048 tokens is 2047 dependent graph launches.  Here the prompt positions run in chunks of P
positions of all B requests at once, as one graph per chunk built directly on the library
kernels:

* ``prefill.embedding`` gathers the chunk's rows from a device copy of the prompts;
* per layer, RMSNorm into a split panel, the q/k/v tensor-core projections (their RoPE and
  KV-append epilogues place each row at its own position), ``prefill.attention`` (causal, over
  the cache rows up to each query's position), the o projection, RMSNorm, the fused
  gate/up/SwiGLU projection and the down projection;
* the head: RMSNorm, an argmax-only LM head and ``prefill.history``, which records each row's
  greedy token in ``history`` exactly as the decode step would;
* ``prefill.advance`` moves ``position`` to the next chunk.

Row m of a chunk is request ``m % B`` at position ``position[0] + m / B``.  The chunks cover
positions ``0 .. context - 3``; the last teacher-forced position (``context - 2``) then runs as
an ordinary decode step, which writes the logits, history row and position the reference
leaves behind, and the last prompt token is written to ``tokens``.
"""
from __future__ import annotations

from types import SimpleNamespace

import numpy as np

import ckl
from ..compile import (POSITION, READ, WRITE, CompiledPlans, Event, Node, Slot, _panel_floats,
                       _plan, library_accepts, library_geometry)
from ..frontend.checker import BoundParameter, BoundSignature
from ..frontend.tracer import Resource
from ..library import pack
from ..types import BufferSpec, f32, i32

# Buffers of the prefill program, in runtime-argument order (then epsilon, attention scale).
ARGUMENTS = ("prompts", "position", "history", "emb", "norm1", "norm2", "final_norm", "wq", "wk",
             "wv", "wo", "wg", "wu", "wd", "lm", "sincos", "kc", "vc")
EPSILON, SCALE = len(ARGUMENTS), len(ARGUMENTS) + 1

# Rows per chunk (positions x requests): large enough for full tensor-core tiles, small enough
# that the chunk's activations stay a few hundred megabytes.
CHUNK_ROWS = 16384


def chunk_positions(batch: int, positions: int) -> int:
    return max(1, min(positions, CHUNK_ROWS // batch))


def _gemm(M, K, N, layers, layer, A=0, D=0, T=0, tiles=0, cache=0):
    return pack(M, K, N, layers, layer, A, D, T, tiles, 0, cache or M)


def build_plan(specs: dict, positions: int):
    """The plan of one chunk of `positions` prompt positions; `specs` maps each argument name to
    its BufferSpec.  Returns (signature, plans)."""
    B = specs["history"].shape[1]
    prompts_rows = specs["prompts"].shape[0]
    L, C = specs["norm1"].shape
    F = specs["wg"].shape[2]
    V = specs["lm"].shape[2]
    _, _, A, T, D = specs["kc"].shape
    M = positions * B

    resources, events = [], []
    for index, name in enumerate(ARGUMENTS):
        resources.append(Resource(index, "argument", specs[name], argument=index, name=name))
    arg = {name: index for index, name in enumerate(ARGUMENTS)}
    allocated = []

    def temporary(shape, name, dtype=f32):
        rid = len(resources)
        resources.append(Resource(rid, "temporary", BufferSpec(tuple(shape), dtype), name=f"{name}{rid}"))
        events.append(Event("alloc", resource=rid))
        allocated.append(rid)
        return rid

    def panel(K, name):
        return temporary((_panel_floats(M, K),), name)

    R = lambda rid: Slot("resource", resource=rid)
    eps, scale = Slot("scalar", argument=EPSILON), Slot("scalar", argument=SCALE)
    position = arg["position"]
    pos_read = (position, READ, POSITION)

    def node(name, slots, spec, reads, writes, label):
        accesses = [(r, READ, "whole") for r in reads] + list(writes)
        events.append(Event("dispatch", node=Node(name, slots, spec, accesses, label)))

    x = temporary((M, C), "x")
    node("ckl.prefill.embedding", [R(arg["prompts"]), R(position), R(arg["emb"]), R(x)],
         pack(M, B, C, V, prompts_rows), [arg["prompts"], arg["emb"]],
         [pos_read, (x, WRITE, "whole")], "embedding")
    kc, vc, sincos = arg["kc"], arg["vc"], arg["sincos"]
    for layer in range(L):
        tag = f" (layer {layer})"
        x_panel = panel(C, "x_panel")
        node("ckl.fused.rms_panel", [R(x), R(arg["norm1"]), R(x_panel), eps],
             pack(M, C, L, layer), [x, arg["norm1"]], [(x_panel, WRITE, "whole")],
             "attention norm" + tag)
        q = temporary((M, C), "q")
        qkv = _gemm(M, C, C, L, layer, A, D, T, cache=B)
        if library_accepts("ckl.fused.panel_qkv", qkv):
            # q, k and v as one tensor-core pair launch (each column tile with its epilogue).
            node("ckl.fused.panel_qkv",
                 [R(x_panel), R(arg["wq"]), R(arg["wk"]), R(arg["wv"]), R(sincos), R(position),
                  R(q), R(kc), R(vc)], qkv, [x_panel, arg["wq"], arg["wk"], arg["wv"], sincos],
                 [pos_read, (q, WRITE, "whole"), (kc, WRITE, "whole"), (vc, WRITE, "whole")],
                 "q/k/v projections" + tag)
        else:
            node("ckl.fused.panel_linear_rope",
                 [R(x_panel), R(arg["wq"]), R(sincos), R(position), R(q)], qkv,
                 [x_panel, arg["wq"], sincos], [pos_read, (q, WRITE, "whole")],
                 "q projection" + tag)
            node("ckl.fused.panel_linear_rope_append",
                 [R(x_panel), R(arg["wk"]), R(sincos), R(position), R(kc)], qkv,
                 [x_panel, arg["wk"], sincos], [pos_read, (kc, WRITE, "whole")],
                 "k projection" + tag)
            node("ckl.fused.panel_linear_append", [R(x_panel), R(arg["wv"]), R(position), R(vc)],
                 qkv, [x_panel, arg["wv"]], [pos_read, (vc, WRITE, "whole")],
                 "v projection" + tag)
        context_panel = panel(C, "context_panel")
        node("ckl.prefill.attention", [R(q), R(kc), R(vc), R(position), R(context_panel), scale],
             pack(B, A, T, D, L, layer, positions), [q, kc, vc],
             [pos_read, (context_panel, WRITE, "whole")], "attention" + tag)
        residual = temporary((M, C), "residual")
        node("ckl.fused.panel_linear_residual", [R(context_panel), R(arg["wo"]), R(x), R(residual)],
             _gemm(M, C, C, L, layer), [context_panel, arg["wo"], x],
             [(residual, WRITE, "whole")], "o projection" + tag)
        r_panel = panel(C, "residual_panel")
        node("ckl.fused.rms_panel", [R(residual), R(arg["norm2"]), R(r_panel), eps],
             pack(M, C, L, layer), [residual, arg["norm2"]], [(r_panel, WRITE, "whole")],
             "mlp norm" + tag)
        p_panel = panel(F, "swiglu_panel")
        node("ckl.fused.panel_gate_up", [R(r_panel), R(arg["wg"]), R(arg["wu"]), R(p_panel)],
             _gemm(M, C, F, L, layer), [r_panel, arg["wg"], arg["wu"]],
             [(p_panel, WRITE, "whole")], "gate/up projection + swiglu" + tag)
        next_x = temporary((M, C), "x")
        node("ckl.fused.panel_linear_residual", [R(p_panel), R(arg["wd"]), R(residual), R(next_x)],
             _gemm(M, F, C, L, layer), [p_panel, arg["wd"], residual],
             [(next_x, WRITE, "whole")], "down projection" + tag)
        x = next_x

    final_panel = panel(C, "final_panel")
    node("ckl.fused.rms_panel", [R(x), R(arg["final_norm"]), R(final_panel), eps],
         pack(M, C, 1, 0), [x, arg["final_norm"]], [(final_panel, WRITE, "whole")], "final norm")
    head = _gemm(M, C, V, 1, 0)
    tiles = library_geometry("ckl.fused.panel_argmax", head)[0][0]
    partials = temporary((M, tiles, 2), "partials")
    node("ckl.fused.panel_argmax", [R(final_panel), R(arg["lm"]), R(partials)],
         _gemm(M, C, V, 1, 0, tiles=tiles), [final_panel, arg["lm"]],
         [(partials, WRITE, "whole")], "lm head (argmax only)")
    node("ckl.prefill.history", [R(partials), R(position), R(arg["history"])],
         pack(M, B, tiles, T), [partials], [pos_read, (arg["history"], WRITE, "whole")],
         "greedy tokens into history")
    node("ckl.prefill.advance", [R(position)], pack(positions), [],
         [(position, READ | WRITE, POSITION)], "advance position")
    for rid in reversed(allocated):
        events.append(Event("free", resource=rid))

    parameters = tuple(BoundParameter(name, specs[name]) for name in ARGUMENTS)
    parameters += (BoundParameter("epsilon", f32), BoundParameter("attention_scale", f32))
    signature = BoundSignature(parameters, ())
    lowered = SimpleNamespace(signature=signature, trace=SimpleNamespace(name="prefill"))
    primary = _plan(lowered, events, resources, reuse_storage=True, externals_disjoint=True,
                    fused=True)
    return signature, CompiledPlans(primary)


class BatchedPrefill:
    """Prefill programs bound to a session's buffers (one per chunk length) and a device copy of
    the prompts."""

    def __init__(self, session, context: int):
        self.session = session
        self.context = context
        history = session.buffers["history"].spec
        self.batch = history.shape[1]
        self.prompts = session.device.empty(ckl.BufferSpec((context, self.batch), ckl.i32))
        self.positions = max(context - 2, 0)
        self._bound = {}

    def _invocation(self, positions: int):
        if positions not in self._bound:
            specs = {name: self.session.buffers[name].spec for name in ARGUMENTS if name != "prompts"}
            specs["prompts"] = self.prompts.spec
            signature, plans = build_plan(specs, positions)
            program = ckl.cuda.CompiledProgram.from_plans(signature, plans)
            arguments = [self.prompts if name == "prompts" else self.session.buffers[name]
                         for name in ARGUMENTS]
            arguments += [float(self.session.epsilon), float(self.session.attention_scale)]
            self._bound[positions] = (program, program.bind(*arguments))
        return self._bound[positions][1]

    def run(self, prompts: np.ndarray, *, mode: str = "graph") -> None:
        """Prefill `prompts` [context, batch]: the state afterwards is the reference's after its
        teacher-forced prefill (position context - 1, tokens = the last prompt token)."""
        prompts = np.ascontiguousarray(prompts, dtype=np.int32)
        if prompts.shape != (self.context, self.batch):
            raise ValueError(f"prompts must have shape {(self.context, self.batch)}")
        session = self.session
        self.prompts.copy_from_host(prompts)
        session.write("position", np.zeros(1, np.int32))
        done = 0
        chunk = chunk_positions(self.batch, self.positions) if self.positions else 0
        while done < self.positions:
            count = min(chunk, self.positions - done)
            self._invocation(count).run(mode=mode)
            done += count
        if self.context >= 2:
            # The last teacher-forced position as an ordinary decode step.
            session.write("tokens", prompts[self.context - 2])
            session.invocation.run(mode=mode)
        session.write("tokens", prompts[self.context - 1])
