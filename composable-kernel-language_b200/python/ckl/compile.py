"""Lower a traced CKL program onto the sm_100a kernel library.

Stages (the reference's ``ckl-fuse-pointwise``, ``ckl-prepare-cuda``, ``ckl-build-graph`` and
``ckl-lower-graph-to-exec`` passes, ``python/ckl/_jit.py:74-154``, restated without MLIR):

1. every dispatch is resolved to a library kernel (:mod:`ckl.library`);
2. optional fusions rewrite the dispatch list:
   * pointwise fusion chains adjacent scalar pointwise launches through a single-use
     temporary (``lib/Transforms/PointwiseFusion.cpp``);
   * decoder fusion maps the decode step onto the fused decoder kernels (six graph nodes per
     layer instead of 21);
   a fused plan assumes distinct caller buffers and keeps the unfused plan as the fallback
   that binding selects when buffers overlap (``lib/Runtime/NvidiaProgram.cpp:194-205``);
3. the native planner infers dependency edges from per-operand effects, reduces them onto
   dispatches and plans temporary storage (``include/ckl_b200.h``, planning section);
4. the result is emitted as the native executable plan and as ``ckl_exec`` text.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import struct
from dataclasses import dataclass, field

from . import _native, codegen
from .compiler import CompilationError
from .frontend import analysis
from .frontend.tracer import LoweredProgram, Resource
from .library import Selection, pack, select
from .types import BufferSpec, f32, f64, i32, i64

READ, WRITE, ALLOCATE, FREE = analysis.READ, analysis.WRITE, analysis.ALLOCATE, analysis.FREE
ALIGNMENT = 256  # temporary allocation alignment (lib/Analysis/GraphAnalysis.cpp:147)
# Caller-buffer alignment the fused decoder kernels require; a binding that misses it takes the
# program's unfused fallback plan.
_FUSED_ALIGNMENT = 16
LIBRARY_BINARY = "ckl-b200:library"
POSITION = (0, 4)  # position[0] of an i32 buffer


@dataclass
class Slot:
    kind: str                 # "resource" | "scalar" | "value"
    resource: int = -1        # program resource id
    argument: int = -1        # runtime parameter position
    data: bytes = b""


@dataclass
class Node:
    """A dispatch on a library kernel, with its argument slots and memory effects."""

    name: str
    slots: list
    spec: bytes
    accesses: list            # [(resource id, bits, region)], region "whole" or (offset, length)
    label: str
    grid: tuple = (1, 1, 1)
    block: tuple = (1, 1, 1)
    shared: int = 0
    # Pointwise chain description (ops, scalar slots, n, count) when the node is one.
    chain: tuple = None
    source: object = None     # the traced dispatch (1:1 nodes)
    selection: Selection = None
    generated: object = None  # codegen.GeneratedKernel for kernels outside the library


@dataclass
class Event:
    kind: str                 # "alloc" | "dispatch" | "free"
    resource: int = -1
    node: Node = None


@dataclass
class Plan:
    """One executable plan: native text, ``ckl_exec`` text and statistics."""

    text: str
    executable_ir: str
    node_names: list
    nodes: int
    edges: int
    temporaries: int
    heap_bytes: int
    baseline_bytes: int
    topology: dict
    fused: bool = False


@dataclass
class CompiledPlans:
    primary: Plan
    fallback: Plan = None
    prepared_ir: str = ""
    device_ir: str = ""
    host_ir: str = ""


# ---------------------------------------------------------------------------------------
def _scalar_slot(operand) -> Slot:
    if operand.kind == "scalar":
        return Slot("scalar", argument=operand.argument)
    code = {f32: "<f", f64: "<d", i32: "<i", i64: "<q"}[operand.dtype]
    return Slot("value", data=struct.pack(code, operand.value))


def _one_to_one(dispatch, library: bool = True) -> Node:
    """The node of one dispatch: its library kernel when the library implements the kernel
    body over the launch's whole index space (and `library` is set), else a generated kernel
    launched with the dispatch's own geometry."""
    selection = None
    if library:
        try:
            selection = select(dispatch)
        except CompilationError:
            selection = None
    spec = dispatch.specialization
    summary = analysis.summarize(spec.definition, spec.signature)
    slots, accesses = [], []
    for position, operand in enumerate(dispatch.operands):
        if operand.kind == "resource":
            slots.append(Slot("resource", resource=operand.resource))
            bits, region = summary.bits[position], summary.regions[position]
            if bits:
                accesses.append((operand.resource, bits, region))
        else:
            slots.append(_scalar_slot(operand))
    label = f"{spec.definition.name} @ {dispatch.location}"
    if selection is None:
        kernel = codegen.generate(spec.definition, spec.signature, spec.identity)
        node = Node(kernel.symbol, slots, b"", accesses, label, source=dispatch, generated=kernel)
        node.grid, node.block, node.shared = dispatch.grid, dispatch.block, dispatch.shared_memory
        return node
    node = Node(selection.entry.native, slots, selection.spec, accesses, label, source=dispatch,
                selection=selection)
    node.grid, node.block = dispatch.grid, dispatch.block
    if selection.entry.pointwise_op >= 0 and dispatch.shared_memory == 0:
        n, count = struct.unpack("<2q", selection.spec)
        node.chain = ((selection.entry.pointwise_op,), (slots[2],), n, count)
    return node


def _resource_users(events) -> dict:
    users: dict[int, list] = {}
    for index, event in enumerate(events):
        if event.kind == "dispatch":
            for slot in event.node.slots:
                if slot.kind == "resource":
                    seen = users.setdefault(slot.resource, [])
                    if not seen or seen[-1] != index:
                        seen.append(index)
    return users


# ---- pointwise fusion ------------------------------------------------------------------
def _fuse_pointwise(events, resources) -> bool:
    """Fuse adjacent scalar pointwise chains through a single-use temporary (in place)."""
    changed = False
    while True:
        fused = False
        previous = None
        for index, event in enumerate(events):
            if event.kind == "alloc":
                continue
            if event.kind != "dispatch":
                previous = None
                continue
            node = event.node
            if previous is not None and _try_fuse_pair(events, resources, previous, index):
                fused = changed = True
                break
            previous = index
        if not fused:
            return changed


def _try_fuse_pair(events, resources, first_index, second_index) -> bool:
    first, second = events[first_index].node, events[second_index].node
    if first.chain is None or second.chain is None:
        return False
    ops1, scalars1, n1, count1 = first.chain
    ops2, scalars2, n2, count2 = second.chain
    if len(ops1) + len(ops2) > 4 or (n1, count1) != (n2, count2):
        return False
    if first.grid != second.grid or first.block != second.block or first.grid[1:] != (1, 1) \
            or first.block[1:] != (1, 1):
        return False
    src, temp = first.slots[0].resource, first.slots[1].resource
    consumed, dst = second.slots[0].resource, second.slots[1].resource
    if consumed != temp or resources[temp].kind != "temporary" or src == dst:
        return False
    users = _resource_users(events)
    if users.get(temp) != [first_index, second_index]:
        return False
    ops, scalars = ops1 + ops2, scalars1 + scalars2
    steps = len(ops)
    spec = pack(n1, count1, steps, *(list(ops) + [0] * (4 - steps)))
    regions = {}
    for rid, bits, region in first.accesses + second.accesses:
        if rid != temp:
            regions[rid] = (regions.get(rid, (0, None))[0] | bits,
                            analysis._merge(regions.get(rid, (0, None))[1], region))
    node = Node(f"ckl.pointwise.chain{steps}",
                [Slot("resource", resource=src), Slot("resource", resource=dst), *scalars],
                spec, [(rid, b, r) for rid, (b, r) in regions.items()],
                f"fused({first.label}; {second.label})",
                grid=first.grid, block=first.block, chain=(ops, scalars, n1, count1))
    events[second_index] = Event("dispatch", node=node)
    del events[first_index]
    events[:] = [e for e in events if not (e.kind in ("alloc", "free") and e.resource == temp)]
    return True


# ---- decoder fusion --------------------------------------------------------------------
_LAYER = ("rms_stats", "rms_apply", "linear", "linear", "linear", "rope", "rope", "append_kv",
          "attention_scores", "softmax", "attention_values", "linear", "add", "rms_stats",
          "rms_apply", "linear", "linear", "silu", "multiply", "linear", "add")
_HEAD = ("rms_stats", "rms_apply", "linear", "greedy", "advance")
_ATTENTION_HEAD_DIMS = (16, 32, 64, 128)
# Batches of 17 or more requests run the projections on tcgen05 tensor cores (GemmSpec config
# 0; partial 128-row tiles with split-K still beat FFMA tiles from 17 rows); up to 16 the
# few-row FFMA kernel is faster for small decoders, whose projections are latency-bound.  From
# a hidden size of 512 the weights stream from HBM (1 MB and more per projection), and up to 16
# requests the streamed few-row FFMA kernel (gemm.cuh, configs 9-18; groups of eight rows
# above eight) reads them at HBM speed: at hidden 1024 it took the step from 0.56 / 0.61 / 0.69
# / 0.78 ms on the tensor cores to 0.24 / 0.30 / 0.49 / 0.74 ms at 1 / 4 / 8 / 16 requests.
# Config 5 keeps every projection on FFMA.
_TENSOR_CORE_ROWS = 17
_TENSOR_CORE_HIDDEN = 512
STREAMED_ROWS = 16


def _panel_floats(M: int, K: int) -> int:
    """Size of a split tensor-core operand: 128-row tiles x 32-column slices x (hi, lo)."""
    return -(-M // 128) * -(-K // 32) * 2 * 128 * 32


class _NoMatch(Exception):
    pass


def _short(node: Node) -> str:
    return node.name.rsplit(".", 1)[-1] if node.name.startswith("ckl.decoder.") else node.name


def _fuse_decoder(events, resources: list, tensor_cores: bool = True,
                  whole_step: bool = True) -> bool:
    dispatches = [e.node for e in events if e.kind == "dispatch"]
    names = [_short(n) for n in dispatches]
    if len(names) < 1 + len(_LAYER) + len(_HEAD) or (len(names) - 1 - len(_HEAD)) % len(_LAYER):
        return False
    layers = (len(names) - 1 - len(_HEAD)) // len(_LAYER)
    expected = ("embedding",) + _LAYER * layers + _HEAD
    if tuple(names) != expected:
        return False
    if whole_step:
        node = _whole_step(dispatches, layers, resources)
        if node is not None:
            # The program is exactly one decode step: every temporary lives inside the kernel.
            events[:] = [Event("dispatch", node=node)]
            return True
    try:
        new_nodes, eliminated, added = _decoder_nodes(dispatches, layers, resources,
                                                      0 if tensor_cores else 5)
    except _NoMatch:
        return False
    users = _resource_users(events)
    dispatch_index = {id(e.node): i for i, e in enumerate(events) if e.kind == "dispatch"}
    for rid, allowed in eliminated.items():
        if resources[rid].kind != "temporary":
            return False
        if sorted(users.get(rid, [])) != sorted(dispatch_index[id(n)] for n in allowed):
            return False
    # Rebuild events: kept temporaries are allocated before first use; frees at the end.
    kept_allocs = [e.resource for e in events if e.kind == "alloc" and e.resource not in eliminated]
    new_events, allocated = [], set()
    for node in new_nodes:
        for slot in node.slots:
            rid = slot.resource
            if slot.kind == "resource" and rid not in allocated and \
                    resources[rid].kind == "temporary" and (rid in kept_allocs or rid in added):
                new_events.append(Event("alloc", resource=rid))
                allocated.add(rid)
        new_events.append(Event("dispatch", node=node))
    order = [rid for rid in kept_allocs + added if rid in allocated]
    for rid in reversed(order):
        new_events.append(Event("free", resource=rid))
    events[:] = new_events
    return True


# Split-K attention (csrc/kernels/decoder_fused.cu, attentionSplitKernel): below two
# (request, head) pairs per SM the cache rows of each pair are divided over several CTAs,
# aiming at about eight 4-warp CTAs per SM and keeping at least 128 cache rows (at capacity)
# per range.
_ATTENTION_UNSPLIT_PAIRS = 2 * 148
_ATTENTION_TARGET_CTAS = 8 * 148
# From 128 pairs on, fewer and longer ranges (about four CTAs per SM) measured faster: at hidden
# 1024 and context 2048, 8 requests 495 -> 479 us per step (10 -> 5 ranges), 16 requests
# 748 -> 713 us (5 -> 3 ranges), while 4 requests keep 16 ranges (302 us against 310 at 10).
_ATTENTION_WIDE_PAIRS = 128
_ATTENTION_WIDE_TARGET_CTAS = 4 * 148
_ATTENTION_MIN_SPAN = 128
_ATTENTION_MAX_SPLITS = 32


def attention_splits(B: int, A: int, T: int) -> int:
    """Cache-row ranges per (request, head) for the decode attention of B requests."""
    pairs = B * A
    if pairs >= _ATTENTION_UNSPLIT_PAIRS:
        return 1
    target = _ATTENTION_WIDE_TARGET_CTAS if pairs >= _ATTENTION_WIDE_PAIRS else _ATTENTION_TARGET_CTAS
    wanted = -(-target // pairs)
    return max(1, min(wanted, T // _ATTENTION_MIN_SPAN, _ATTENTION_MAX_SPLITS))


def _decoder_nodes(dispatches, layers, resources, config=0, collect=None):
    def op(node, i):
        return node.source.operands[i]

    def res(node, i):
        operand = op(node, i)
        if operand.kind != "resource" or resources[operand.resource].kind == "view":
            raise _NoMatch
        return operand.resource

    def const(node, i=0):
        return [p.value for p in node.source.specialization.signature.parameters if p.is_constant][i]

    def shape(rid):
        return resources[rid].spec.shape

    def same(*values):
        if any(v != values[0] for v in values):
            raise _NoMatch

    def same_shape(*rids):
        return all(shape(r) == shape(rids[0]) for r in rids)

    def gemm_spec(M, K, N, layers_, layer, A=0, D=0, T=0, tiles=0):
        return pack(M, K, N, layers_, layer, A, D, T, tiles, config, M)

    embedding = dispatches[0]
    x = res(embedding, 2)
    new_nodes = [embedding]
    added: list[int] = []

    def panel_resource(M, K, name):
        rid = _add_resource(resources, "temporary", BufferSpec((_panel_floats(M, K),), f32), name)
        added.append(rid)
        return rid

    tensor_cores = config == 0 and (shape(x)[0] >= _TENSOR_CORE_ROWS or
                                    (shape(x)[1] >= _TENSOR_CORE_HIDDEN and
                                     shape(x)[0] > STREAMED_ROWS))
    eliminated: dict[int, list] = {}
    position = sincos = kc = vc = None
    for layer_index in range(layers):
        d = dispatches[1 + layer_index * len(_LAYER):1 + (layer_index + 1) * len(_LAYER)]
        same(res(d[0], 0), res(d[1], 0), x)
        inv, normed = res(d[0], 1), res(d[1], 3)
        same(res(d[1], 1), inv)
        same(res(d[2], 0), res(d[3], 0), res(d[4], 0), normed)
        q, k, v = res(d[2], 2), res(d[3], 2), res(d[4], 2)
        wq, wk, wv = res(d[2], 1), res(d[3], 1), res(d[4], 1)
        g1 = res(d[1], 2)
        same(res(d[5], 0), q)
        same(res(d[6], 0), k)
        same(res(d[5], 1), res(d[6], 1))
        same(res(d[5], 2), res(d[6], 2), res(d[7], 4), res(d[8], 2), res(d[9], 1), res(d[10], 2))
        if position is None:
            position, sincos = res(d[5], 2), res(d[5], 1)
        same(res(d[5], 2), position)
        same(res(d[5], 1), sincos)
        qr, kr = res(d[5], 3), res(d[6], 3)
        same(res(d[7], 0), kr)
        same(res(d[7], 1), v)
        if kc is None:
            kc, vc = res(d[7], 2), res(d[7], 3)
        same(res(d[7], 2), res(d[8], 1), kc)
        same(res(d[7], 3), res(d[10], 1), vc)
        same(res(d[8], 0), qr)
        scores = res(d[8], 3)
        same(res(d[9], 0), scores)
        probs = res(d[9], 2)
        same(res(d[10], 0), probs)
        context = res(d[10], 3)
        same(res(d[11], 0), context)
        wo, projected = res(d[11], 1), res(d[11], 2)
        same(res(d[12], 0), x)
        same(res(d[12], 1), projected)
        residual = res(d[12], 2)
        same(res(d[13], 0), res(d[14], 0), residual)
        inv2, normed2 = res(d[13], 1), res(d[14], 3)
        same(res(d[14], 1), inv2)
        g2 = res(d[14], 2)
        same(res(d[15], 0), res(d[16], 0), normed2)
        wg, gate, wu, up = res(d[15], 1), res(d[15], 2), res(d[16], 1), res(d[16], 2)
        same(res(d[17], 0), gate)
        activated = res(d[17], 1)
        same(res(d[18], 0), activated)
        same(res(d[18], 1), up)
        product = res(d[18], 2)
        same(res(d[19], 0), product)
        wd, down = res(d[19], 1), res(d[19], 2)
        same(res(d[20], 0), residual)
        same(res(d[20], 1), down)
        next_x = res(d[20], 2)
        layer = const(d[1])
        same(layer, const(d[2]), const(d[3]), const(d[4]), const(d[7]), const(d[8]), const(d[10]),
             const(d[11]), const(d[14]), const(d[15]), const(d[16]), const(d[19]))
        B, Cdim = shape(x)
        L_, Bc, A, T, D = shape(kc)
        F = shape(wg)[2]
        Lw = shape(wq)[0]
        same(Bc, B)
        if D not in _ATTENTION_HEAD_DIMS or A * D != Cdim:
            raise _NoMatch
        eps1, eps2 = _scalar_slot(op(d[0], 2)), _scalar_slot(op(d[13], 2))
        scale = _scalar_slot(op(d[8], 4))

        def node(name, slots, spec, reads, writes, label):
            accesses = [(r, READ, "whole") for r in reads]
            accesses += [(r, bits, region) for r, bits, region in writes]
            return Node(name, slots, spec, accesses, f"{label} (layer {layer})")

        R = lambda r: Slot("resource", resource=r)
        pos_read = (position, READ, POSITION)

        def attention_node(qr, kc, vc, out, panel):
            splits = attention_splits(B, A, T)
            if splits == 1:
                return node("ckl.fused.attention",
                            [R(qr), R(kc), R(vc), R(position), R(out), scale],
                            pack(B, A, T, D, L_, layer, 1, 0, panel, B, 0),
                            [qr, kc, vc], [pos_read, (out, WRITE, "whole")], "attention")
            # Split-K: per-range softmax states (a node-local temporary) and one arrival
            # counter per (request, head), zeroed at allocation and re-armed by the kernel.
            states = _add_resource(resources, "temporary",
                                   BufferSpec((B * A * splits * (D + 4),), f32),
                                   "attention_states")
            added.append(states)
            arrivals = _add_resource(resources, "persistent", BufferSpec((B * A,), i32),
                                     "arrivals")
            return node("ckl.fused.attention_split",
                        [R(qr), R(kc), R(vc), R(position), R(out), R(states), R(arrivals), scale],
                        pack(B, A, T, D, L_, layer, splits, 0, panel, B, 0),
                        [qr, kc, vc], [pos_read, (out, WRITE, "whole"),
                                       (states, READ | WRITE, "whole"),
                                       (arrivals, READ | WRITE, "whole")], "attention")
        eliminated_here = [(inv, (d[0], d[1])), (normed, (d[1], d[2], d[3], d[4])),
                           (q, (d[2], d[5])), (k, (d[3], d[6])), (v, (d[4], d[7])),
                           (kr, (d[6], d[7])), (scores, (d[8], d[9])), (probs, (d[9], d[10])),
                           (projected, (d[11], d[12])), (inv2, (d[13], d[14])),
                           (normed2, (d[14], d[15], d[16])), (activated, (d[17], d[18])),
                           (product, (d[18], d[19])), (down, (d[19], d[20]))]
        if tensor_cores:
            # Each activation operand is split into a TF32 hi/lo panel once, by its producer,
            # and the projections read the panels on the tensor cores.
            x_panel = panel_resource(B, Cdim, "x_panel")
            context_panel = panel_resource(B, Cdim, "context_panel")
            r_panel = panel_resource(B, Cdim, "residual_panel")
            p_panel = panel_resource(B, F, "swiglu_panel")
            new_nodes.append(node("ckl.fused.rms_panel", [R(x), R(g1), R(x_panel), eps1],
                                  pack(B, Cdim, shape(g1)[0], layer), [x, g1],
                                  [(x_panel, WRITE, "whole")], "attention norm"))
            qkv_spec = gemm_spec(B, Cdim, Cdim, Lw, layer, A, D, T)
            if same_shape(wq, wk, wv) and library_accepts("ckl.fused.panel_qkv", qkv_spec):
                # One launch for q, k and v on tensor-core CTA pairs (each column tile takes
                # its projection's epilogue).
                new_nodes.append(node("ckl.fused.panel_qkv",
                                      [R(x_panel), R(wq), R(wk), R(wv), R(sincos), R(position),
                                       R(qr), R(kc), R(vc)], qkv_spec,
                                      [x_panel, wq, wk, wv, sincos],
                                      [pos_read, (qr, WRITE, "whole"), (kc, WRITE, "whole"),
                                       (vc, WRITE, "whole")], "q/k/v projections"))
            else:
                new_nodes.append(node("ckl.fused.panel_linear_rope",
                                      [R(x_panel), R(wq), R(sincos), R(position), R(qr)],
                                      qkv_spec, [x_panel, wq, sincos],
                                      [pos_read, (qr, WRITE, "whole")], "q projection"))
                new_nodes.append(node("ckl.fused.panel_linear_rope_append",
                                      [R(x_panel), R(wk), R(sincos), R(position), R(kc)],
                                      qkv_spec, [x_panel, wk, sincos],
                                      [pos_read, (kc, WRITE, "whole")], "k projection"))
                new_nodes.append(node("ckl.fused.panel_linear_append",
                                      [R(x_panel), R(wv), R(position), R(vc)],
                                      qkv_spec, [x_panel, wv],
                                      [pos_read, (vc, WRITE, "whole")], "v projection"))
            new_nodes.append(attention_node(qr, kc, vc, context_panel, 1))
            new_nodes.append(node("ckl.fused.panel_linear_residual",
                                  [R(context_panel), R(wo), R(x), R(residual)],
                                  gemm_spec(B, Cdim, Cdim, Lw, layer),
                                  [context_panel, wo, x], [(residual, WRITE, "whole")],
                                  "o projection"))
            new_nodes.append(node("ckl.fused.rms_panel", [R(residual), R(g2), R(r_panel), eps2],
                                  pack(B, Cdim, shape(g2)[0], layer), [residual, g2],
                                  [(r_panel, WRITE, "whole")], "mlp norm"))
            new_nodes.append(node("ckl.fused.panel_gate_up",
                                  [R(r_panel), R(wg), R(wu), R(p_panel)],
                                  gemm_spec(B, Cdim, F, shape(wg)[0], layer),
                                  [r_panel, wg, wu], [(p_panel, WRITE, "whole")],
                                  "gate/up projection + swiglu"))
            new_nodes.append(node("ckl.fused.panel_linear_residual",
                                  [R(p_panel), R(wd), R(residual), R(next_x)],
                                  gemm_spec(B, F, Cdim, shape(wd)[0], layer),
                                  [p_panel, wd, residual], [(next_x, WRITE, "whole")],
                                  "down projection"))
            eliminated_here += [(context, (d[10], d[11])), (gate, (d[15], d[17])),
                                (up, (d[16], d[18]))]
        else:
            new_nodes.append(node("ckl.fused.norm_linear_rope",
                                  [R(x), R(g1), R(wq), R(sincos), R(position), R(qr), eps1],
                                  gemm_spec(B, Cdim, Cdim, Lw, layer, A, D, T),
                                  [x, g1, wq, sincos], [pos_read, (qr, WRITE, "whole")],
                                  "q projection"))
            new_nodes.append(node("ckl.fused.norm_linear_rope_append",
                                  [R(x), R(g1), R(wk), R(sincos), R(position), R(kc), eps1],
                                  gemm_spec(B, Cdim, Cdim, Lw, layer, A, D, T),
                                  [x, g1, wk, sincos], [pos_read, (kc, WRITE, "whole")],
                                  "k projection"))
            new_nodes.append(node("ckl.fused.norm_linear_append",
                                  [R(x), R(g1), R(wv), R(position), R(vc), eps1],
                                  gemm_spec(B, Cdim, Cdim, Lw, layer, A, D, T),
                                  [x, g1, wv], [pos_read, (vc, WRITE, "whole")], "v projection"))
            new_nodes.append(attention_node(qr, kc, vc, context, 0))
            new_nodes.append(node("ckl.fused.linear_residual",
                                  [R(context), R(wo), R(x), R(residual)],
                                  gemm_spec(B, Cdim, Cdim, Lw, layer),
                                  [context, wo, x], [(residual, WRITE, "whole")], "o projection"))
            new_nodes.append(node("ckl.fused.norm_linear",
                                  [R(residual), R(g2), R(wg), R(gate), eps2],
                                  gemm_spec(B, Cdim, F, shape(wg)[0], layer),
                                  [residual, g2, wg], [(gate, WRITE, "whole")], "gate projection"))
            new_nodes.append(node("ckl.fused.norm_linear",
                                  [R(residual), R(g2), R(wu), R(up), eps2],
                                  gemm_spec(B, Cdim, F, shape(wu)[0], layer),
                                  [residual, g2, wu], [(up, WRITE, "whole")], "up projection"))
            new_nodes.append(node("ckl.fused.swiglu_linear_residual",
                                  [R(gate), R(up), R(wd), R(residual), R(next_x)],
                                  gemm_spec(B, F, Cdim, shape(wd)[0], layer),
                                  [gate, up, wd, residual], [(next_x, WRITE, "whole")],
                                  "down projection"))
        for rid, users in eliminated_here:
            eliminated[rid] = list(users)
        if collect is not None:
            collect.setdefault("layers", []).append(dict(
                layer=layer, weights=(g1, g2, wq, wk, wv, wo, wg, wu, wd),
                scalars=(eps1, eps2, scale), cache=(kc, vc), sincos=sincos, position=position))
        x = next_x
    h = dispatches[1 + layers * len(_LAYER):]
    same(res(h[0], 0), res(h[1], 0), x)
    finv, final_x = res(h[0], 1), res(h[1], 3)
    same(res(h[1], 1), finv)
    same(res(h[2], 0), final_x)
    fgain, lm, logits = res(h[1], 2), res(h[2], 1), res(h[2], 2)
    same(res(h[3], 0), logits)
    tokens, history = res(h[3], 1), res(h[3], 2)
    if position is None:
        raise _NoMatch
    same(res(h[3], 3), res(h[4], 0), position)
    same(const(h[1]), const(h[2]))
    B, Cdim = shape(x)
    V = shape(lm)[2]
    T = shape(history)[0]
    head_name = "ckl.fused.panel_linear_argmax" if tensor_cores else "ckl.fused.norm_linear_argmax"
    head_spec = gemm_spec(B, Cdim, V, shape(lm)[0], const(h[2]))
    geometry = library_geometry(head_name, head_spec)
    tiles = geometry[0][0]
    head_spec = gemm_spec(B, Cdim, V, shape(lm)[0], const(h[2]), tiles=tiles)
    partials = _add_resource(resources, "temporary", BufferSpec((B, tiles, 2), f32), "partials")
    counter = _add_resource(resources, "persistent", BufferSpec((1,), i32), "counter")
    R = lambda r: Slot("resource", resource=r)
    eps = _scalar_slot(op(h[0], 2))
    if tensor_cores:
        f_panel = panel_resource(B, Cdim, "final_panel")
        new_nodes.append(Node("ckl.fused.rms_panel", [R(x), R(fgain), R(f_panel), eps],
                              pack(B, Cdim, shape(fgain)[0], const(h[1])),
                              [(x, READ, "whole"), (fgain, READ, "whole"),
                               (f_panel, WRITE, "whole")], "final norm"))
        new_nodes.append(Node(head_name, [R(f_panel), R(lm), R(logits), R(partials)], head_spec,
                              [(f_panel, READ, "whole"), (lm, READ, "whole"),
                               (logits, WRITE, "whole"), (partials, WRITE, "whole")],
                              "lm head"))
    else:
        new_nodes.append(Node(head_name,
                              [R(x), R(fgain), R(lm), R(logits), R(partials), eps], head_spec,
                              [(x, READ, "whole"), (fgain, READ, "whole"), (lm, READ, "whole"),
                               (logits, WRITE, "whole"), (partials, WRITE, "whole")],
                              "lm head"))
    new_nodes.append(Node("ckl.fused.greedy_combine",
                          [R(partials), R(logits), R(tokens), R(history), R(position), R(counter)],
                          pack(B, tiles, T, V),
                          [(partials, READ, "whole"), (logits, READ, "whole"),
                           (tokens, WRITE, "whole"), (history, WRITE, "whole"),
                           (position, READ | WRITE, POSITION), (counter, READ | WRITE, "whole")],
                          "greedy + advance"))
    eliminated[finv] = [h[0], h[1]]
    eliminated[final_x] = [h[1], h[2]]
    if collect is not None:
        collect["head"] = dict(tokens=tokens, history=history, logits=logits, fgain=fgain, lm=lm,
                               final=const(h[1]), head=const(h[2]), eps=eps,
                               embedding=(res(embedding, 0), res(embedding, 1)))
    return new_nodes, eliminated, added + [partials]


# Whole-step kernel limits (csrc/kernels/decode_step.cu): weights small enough to stay in L2
# while every cluster streams them, at most 16 requests per 8-CTA cluster and 32 clusters (at
# two CTAs per SM 33 eight-CTA clusters are co-resident on a B200; spreading the requests over
# all of them shortens every cluster's passes: 256 requests as 32 x 8 take 205 us per step of
# an 8-layer C = 64 decoder against 309 us as 18 x 15).
_WHOLE_STEP_WEIGHT_BYTES = 24 << 20
_WHOLE_STEP_CLUSTERS = 32
_WHOLE_STEP_ROWS = 16


def _whole_step(dispatches, layers, resources):
    """One ``ckl.fused.decode_step`` node for a whole small decode step, or None."""
    info: dict = {}
    try:
        _decoder_nodes(dispatches, layers, list(resources), 5, collect=info)
    except _NoMatch:
        return None
    per_layer, head = info.get("layers", []), info.get("head")
    if head is None or len(per_layer) != layers:
        return None
    first = per_layer[0]
    for index, entry in enumerate(per_layer):
        if entry["layer"] != index or entry["weights"] != first["weights"] or \
                entry["cache"] != first["cache"] or entry["sincos"] != first["sincos"]:
            return None
        if any(not _same_slot(a, first["scalars"][0]) for a in entry["scalars"][:2]) or \
                not _same_slot(entry["scalars"][2], first["scalars"][2]):
            return None
    if not _same_slot(head["eps"], first["scalars"][0]):
        return None
    tokens, emb = head["embedding"]
    if tokens != head["tokens"]:
        return None
    g1, g2, wq, wk, wv, wo, wg, wu, wd = first["weights"]
    kc, vc = first["cache"]
    shape = lambda rid: resources[rid].spec.shape
    _, B, A, T, D = shape(kc)
    C, F, V = shape(wq)[1], shape(wg)[2], shape(head["lm"])[2]
    weight_bytes = 4 * (layers * (4 * C * C + 3 * C * F) + 2 * V * C)
    if weight_bytes > _WHOLE_STEP_WEIGHT_BYTES or B > _WHOLE_STEP_CLUSTERS * _WHOLE_STEP_ROWS:
        return None
    G = -(-B // min(_WHOLE_STEP_CLUSTERS, B))
    clusters = -(-B // G)
    spec = pack(B, C, A, D, F, V, layers, T, shape(wq)[0], shape(g1)[0], head["final"],
                head["head"], G, clusters)
    try:
        library_geometry("ckl.fused.decode_step", spec)
    except CompilationError:
        return None
    counter = _add_resource(resources, "persistent", BufferSpec((1,), i32), "counter")
    position, sincos = first["position"], first["sincos"]
    R = lambda rid: Slot("resource", resource=rid)
    operands = [tokens, position, head["history"], emb, g1, g2, head["fgain"], wq, wk, wv, wo,
                wg, wu, wd, head["lm"], sincos, kc, vc, head["logits"], counter]
    reads = [emb, g1, g2, head["fgain"], wq, wk, wv, wo, wg, wu, wd, head["lm"], sincos]
    accesses = [(r, READ, "whole") for r in reads]
    accesses += [(tokens, READ | WRITE, "whole"), (position, READ | WRITE, POSITION),
                 (head["history"], WRITE, "whole"), (kc, READ | WRITE, "whole"),
                 (vc, READ | WRITE, "whole"), (head["logits"], WRITE, "whole"),
                 (counter, READ | WRITE, "whole")]
    return Node("ckl.fused.decode_step",
                [R(r) for r in operands] + [first["scalars"][0], first["scalars"][2]], spec,
                accesses, f"whole decode step ({layers} layers, {clusters} clusters)")


def _same_slot(a, b) -> bool:
    return (a.kind, a.argument, a.data) == (b.kind, b.argument, b.data)


def _add_resource(resources, kind, spec, name) -> int:
    rid = len(resources)
    resources.append(Resource(rid, kind, spec, name=f"{name}{rid}"))
    return rid


# ---- native planning -------------------------------------------------------------------
def library_accepts(name: str, spec: bytes) -> bool:
    """Whether library kernel ``name`` has a launch geometry for this specialization."""
    try:
        library_geometry(name, spec)
    except CompilationError:
        return False
    return True


def library_geometry(name: str, spec: bytes):
    lib = _native.load()
    grid, block, shared = (C.c_uint32 * 3)(), (C.c_uint32 * 3)(), C.c_uint32()
    buffer = C.create_string_buffer(spec, len(spec)) if spec else None
    status = lib.ckl_library_geometry(name.encode(), buffer, len(spec), grid, block, C.byref(shared))
    if status:
        raise CompilationError(("ckl-b200", "geometry"), f"{name}: {_native.message()}")
    return tuple(grid), tuple(block), shared.value


def _root(resources, rid):
    r = resources[rid]
    return (r.base, r.byte_offset, r.spec.nbytes) if r.kind == "view" else (rid, 0, r.spec.nbytes)


def _region(resources, rid, region):
    root, offset, size = _root(resources, rid)
    if region == "whole":
        if resources[rid].kind == "view":
            return root, offset, size
        return root, -1, 0
    return root, offset + region[0], region[1]


def _plan(lowered: LoweredProgram, events, resources, *, reuse_storage: bool,
          externals_disjoint: bool, fused: bool, binary: bytes | None = None) -> Plan:
    lib = _native.load()
    nodes, accesses = [], []
    labels = []
    for event in events:
        first = len(accesses)
        if event.kind == "dispatch":
            for rid, bits, region in event.node.accesses:
                root, offset, length = _region(resources, rid, region)
                accesses.append(_native.GraphAccess(root, bits, offset, length))
            kind = 0
        else:
            root = _root(resources, event.resource)[0]
            accesses.append(_native.GraphAccess(root, ALLOCATE if event.kind == "alloc" else FREE,
                                                -1, 0))
            kind = 1 if event.kind == "alloc" else 2
        nodes.append(_native.GraphNode(kind, 0, first, len(accesses) - first))
        labels.append(event)
    graph_resources = []
    for r in resources:
        temporary = {"temporary": 1, "persistent": 2}.get(r.kind, 0)
        graph_resources.append(_native.GraphResource(temporary, 0, max(r.spec.nbytes, 1), ALIGNMENT))
    flags = (1 if reuse_storage else 0) | (2 if externals_disjoint else 0)
    handle = C.c_void_p()
    status = lib.ckl_graph_plan_create(
        len(nodes), (_native.GraphNode * len(nodes))(*nodes), len(accesses),
        (_native.GraphAccess * max(len(accesses), 1))(*accesses), len(graph_resources),
        (_native.GraphResource * max(len(graph_resources), 1))(*graph_resources), flags,
        C.byref(handle))
    if status:
        raise CompilationError(("ckl-b200", "plan"), _native.message())
    try:
        return _emit(lowered, lib, handle, events, resources, fused, binary)
    finally:
        lib.ckl_graph_plan_release(handle)


def _emit(lowered, lib, handle, events, resources, fused, binary=None) -> Plan:
    count = lib.ckl_graph_plan_resource_count(handle)
    order = (C.c_uint32 * max(count, 1))()
    lib.ckl_graph_plan_resources(handle, order)
    order = list(order)[:count]
    baseline, planned, heap_count = C.c_uint64(), C.c_uint64(), C.c_uint32()
    lib.ckl_graph_plan_memory(handle, C.byref(baseline), C.byref(planned), C.byref(heap_count))
    heaps = (C.c_uint64 * max(heap_count.value, 1))()
    alignments = (C.c_uint64 * max(heap_count.value, 1))()
    lib.ckl_graph_plan_heaps(handle, heaps, alignments)
    plan_index = {rid: i for i, rid in enumerate(order)}
    runtime = [p for p in lowered.signature.parameters if not p.is_constant]

    text = ["ckl-b200-plan 1"]
    ir = ['"ckl_exec.plan"() ({']
    for position, parameter in enumerate(runtime):
        if isinstance(parameter.dtype, BufferSpec):
            text.append(f"arg {position} buffer {parameter.dtype.nbytes}")
        else:
            text.append(f"arg {position} scalar {parameter.dtype.name}")
    text.append(f"binary hex {binary.hex()}" if binary else "binary library")
    if any(e.kind == "dispatch" and e.node.name.startswith("ckl.fused.") for e in events):
        # The fused decoder kernels access caller buffers 16 bytes at a time.
        text.append(f"align {_FUSED_ALIGNMENT}")
    for h in range(heap_count.value):
        text.append(f"heap {h} {heaps[h]}")
        ir.append(f'  "ckl_exec.heap"() {{id = {h} : i64, bytes = {heaps[h]} : i64, alignment = '
                  f'{alignments[h]} : i64, device = 0 : i64, address_space = "global"}} : () -> ()')
    temporaries = 0
    for i, rid in enumerate(order):
        r = resources[rid]
        if r.kind == "argument":
            text.append(f"resource {i} external {r.argument}")
            ir.append(f'  "ckl_exec.resource"() {{name = "arg{r.argument}", kind = "external", '
                      f'device = "cuda:0", address_space = "global", alignment = {ALIGNMENT} : i64}}'
                      ' : () -> ()')
            continue
        heap, offset, slot = C.c_uint64(), C.c_uint64(), C.c_uint64()
        if lib.ckl_graph_plan_assignment(handle, rid, C.byref(heap), C.byref(offset), C.byref(slot)):
            raise CompilationError(("ckl-b200", "plan"), _native.message())
        text.append(f"resource {i} temporary {heap.value} {offset.value}")
        kind = "temporary" if r.kind == "temporary" else "persistent"
        temporaries += r.kind == "temporary"
        ir.append(f'  "ckl_exec.resource"() {{name = "{r.name}", kind = "{kind}", device = '
                  f'"cuda:0", address_space = "global", alignment = {ALIGNMENT} : i64, bytes = '
                  f'{r.spec.nbytes} : i64, heap = {heap.value} : i64, offset = {offset.value} : i64}}'
                  ' : () -> ()')
    topology, names, edges = {}, [], 0
    for node_id, event in enumerate(events):
        if event.kind != "dispatch":
            continue
        node = event.node
        if node.generated is not None:
            grid, block, shared = node.grid, node.block, node.shared
        else:
            grid, block, shared = library_geometry(node.name, node.spec)
        deps_count = lib.ckl_graph_plan_dependency_count(handle, node_id)
        deps = (C.c_uint32 * max(deps_count, 1))()
        lib.ckl_graph_plan_dependencies(handle, node_id, deps)
        deps = list(deps)[:deps_count]
        topology[node_id] = deps
        edges += len(deps)
        names.append(node.name)
        text.append(f"kernel {node_id} {node.name} {grid[0]} {grid[1]} {grid[2]} {block[0]} "
                    f"{block[1]} {block[2]} {shared}")
        for slot in node.slots:
            if slot.kind == "resource":
                root, offset, _ = _root(resources, slot.resource)
                text.append(f"argres {plan_index[root]} {offset}")
            elif slot.kind == "scalar":
                text.append(f"argscalar {slot.argument}")
            else:
                text.append(f"argvalue {slot.data.hex()}")
        if node.spec:
            text.append(f"argvalue {node.spec.hex()}")
        for d in deps:
            text.append(f"dep {d}")
        dep_text = "array<i64>" if not deps else "array<i64: " + ", ".join(map(str, deps)) + ">"
        ir.append(f'  "ckl_exec.kernel"() {{id = {node_id} : i64, kernel = @{node.name}, grid = '
                  f'array<i64: {grid[0]}, {grid[1]}, {grid[2]}>, block = array<i64: {block[0]}, '
                  f'{block[1]}, {block[2]}>, shared_memory = {shared} : i64, abi = "cuda.direct", '
                  f'dependencies = {dep_text}}} : () -> ()  // {node.label}')
    text.append("end")
    ir.append(f'}}) {{backend = "cuda", name = "{lowered.trace.name}.exec"}} : () -> ()')
    return Plan("\n".join(text) + "\n", "\n".join(ir) + "\n", names, len(names), edges,
                temporaries, int(planned.value), int(baseline.value), topology, fused)


def _initial_events(lowered: LoweredProgram, library: bool = True):
    trace = lowered.trace
    resources = [Resource(r.id, r.kind, r.spec, r.argument, r.base, r.byte_offset, r.name)
                 for r in trace.resources]
    events = []
    for e in trace.events:
        if e.kind == "dispatch":
            events.append(Event("dispatch", node=_one_to_one(e.dispatch, library)))
        else:
            events.append(Event(e.kind, resource=e.resource))
    return events, resources


_BINARIES: dict = {}


def device_binary(kernels) -> tuple[str, bytes | None]:
    """The translation unit of a program's generated kernels and its sm_100a CUBIN (None when
    every dispatch runs a library kernel).  CUBINs are cached by source."""
    kernels = list(kernels)
    if not kernels:
        return "", None
    unit = codegen.translation_unit(kernels)
    key = hashlib.sha256(unit.encode()).hexdigest()
    if key not in _BINARIES:
        try:
            _BINARIES[key] = _native.compile_cuda(unit, "ckl_generated.cu")
        except (ValueError, RuntimeError) as error:
            raise CompilationError(("ckl-b200", "nvrtc", "sm_100a"), str(error)) from error
    return unit, _BINARIES[key]


def plan_program(lowered: LoweredProgram, *, fuse_pointwise: bool, fuse_library: bool,
                 reuse_storage: bool, tensor_cores: bool = True,
                 library: bool = True, whole_step: bool = True) -> CompiledPlans:
    """Plans of a lowered program.  `library=False` generates every kernel from its body (the
    reference's naive code path) instead of selecting library kernels."""
    events, resources = _initial_events(lowered, library)
    if not any(e.kind == "dispatch" for e in events):
        raise CompilationError(("ckl-b200", "plan"), "program launches no kernels")
    unit, binary = device_binary(e.node.generated for e in events
                                 if e.kind == "dispatch" and e.node.generated is not None)
    baseline = _plan(lowered, [Event(e.kind, e.resource, e.node) for e in events],
                     list(resources), reuse_storage=reuse_storage, externals_disjoint=False,
                     fused=False, binary=binary)
    fused = False
    if fuse_pointwise:
        fused |= _fuse_pointwise(events, resources)
    if fuse_library:
        fused |= _fuse_decoder(events, resources, tensor_cores, whole_step)
    plans = CompiledPlans(baseline)
    if fused:
        primary = _plan(lowered, events, resources, reuse_storage=reuse_storage,
                        externals_disjoint=True, fused=True, binary=binary)
        plans = CompiledPlans(primary, baseline)
    plans.prepared_ir = lowered.mlir
    plans.device_ir = _device_text(plans, unit)
    plans.host_ir = _host_text(plans.primary, binary)
    return plans


def _device_text(plans: CompiledPlans, generated: str = "") -> str:
    lib = _native.load()
    used = sorted(set(plans.primary.node_names) |
                  set(plans.fallback.node_names if plans.fallback else []))
    lines = ["// sm_100a kernel library entries used by this program (signature codes: "
             "P pointer, F f32, S specialization)"]
    for name in used:
        if name.startswith(codegen.SYMBOL_PREFIX):
            continue
        signature = C.create_string_buffer(64)
        lib.ckl_library_signature(name.encode(), signature, 64)
        lines.append(f"ckl.library.kernel @{name} signature \"{signature.value.decode()}\" "
                     "target \"sm_100a\"")
    if generated:
        lines += ["// generated kernels (CUDA C++, compiled by NVRTC for sm_100a):", generated]
    return "\n".join(lines) + "\n"


def _host_text(plan: Plan, binary: bytes | None = None) -> str:
    """The callback sequence the native entry replays, in LLVM-like text."""
    if binary:
        lines = [f'@ckl.binary = internal constant [{len(binary)} x i8] c"<sm_100a CUBIN>"',
                 "define void @ckl_entry(ptr %frame, ptr %arguments) {",
                 f"  call void @ckl_begin(ptr %frame, ptr @ckl.binary, i64 {len(binary)})"]
    else:
        lines = [f'@ckl.binary = internal constant [{len(LIBRARY_BINARY) + 1} x i8] '
                 f'c"{LIBRARY_BINARY}\\00"',
                 "define void @ckl_entry(ptr %frame, ptr %arguments) {",
                 f"  call void @ckl_begin(ptr %frame, ptr @ckl.binary, i64 {len(LIBRARY_BINARY)})"]
    current = None
    for line in plan.text.splitlines():
        parts = line.split()
        if not parts:
            continue
        if parts[0] in ("kernel", "end") and current is not None:
            lines.append(f"  call void @ckl_commit(ptr %frame, i64 {current})")
            current = None
        if parts[0] == "kernel":
            current = parts[1]
        if parts[0] == "heap":
            lines.append(f"  call void @ckl_heap(ptr %frame, i64 {parts[1]}, i64 {parts[2]})")
        elif parts[0] == "resource":
            if parts[2] == "external":
                lines.append(f"  call void @ckl_resource(ptr %frame, i64 {parts[1]}, i64 0, i64 0, "
                             f"ptr %arg{parts[3]})")
            else:
                lines.append(f"  call void @ckl_resource(ptr %frame, i64 {parts[1]}, i64 {parts[3]}, "
                             f"i64 {parts[4]}, ptr null)")
        elif parts[0] == "kernel":
            lines.append(f'  call void @ckl_kernel(ptr %frame, ptr @"{parts[2]}", '
                         + ", ".join(f"i64 {p}" for p in parts[3:]) + ")")
        elif parts[0] == "argres":
            lines.append(f"  call void @ckl_argument_resource(ptr %frame, i64 {parts[1]}, i64 {parts[2]})")
        elif parts[0] == "argscalar":
            lines.append(f"  call void @ckl_argument_value(ptr %frame, ptr %arg{parts[1]}, i64 ?)")
        elif parts[0] == "argvalue":
            lines.append(f"  call void @ckl_argument_value(ptr %frame, ptr x\"{parts[1]}\", "
                         f"i64 {len(parts[1]) // 2})")
        elif parts[0] == "dep":
            lines.append(f"  call void @ckl_dependency(ptr %frame, i64 {parts[1]})")
    lines += ["  ret void", "}"]
    return "\n".join(lines) + "\n"


def reference_plan_text(lowered: LoweredProgram) -> str:
    """Executable plan of the unfused program with the reference's may-alias rules."""
    return plan_program(lowered, fuse_pointwise=False, fuse_library=False,
                        reuse_storage=True).primary.executable_ir
