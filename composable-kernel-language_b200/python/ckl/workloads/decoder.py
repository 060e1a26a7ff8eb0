"""The CKL decode step, written in the CKL DSL.

This is the reference benchmark's decoder program (``benchmarks/decoder/workloads.py``): a
small Llama-style decoder whose one program invocation is one autoregressive step for a fixed
batch of requests.  The kernel bodies state the arithmetic the B200 kernel library
implements; because the library is indexed by each kernel's canonical structure, the
operations and their order here are those of the reference kernels (reordering an
expression would change float32 rounding, so it is not a free choice).

Persistent state (position, tokens, history, K/V cache) lives in the program's buffers and
is advanced by every step; temporaries are program allocations placed by the storage plan.
"""
import ckl

B, C, L, A, T, D, F, V, R = [ckl.dim(name) for name in ("B", "C", "L", "A", "T", "D", "F", "V", "R")]
W, I, O = [ckl.dim(name) for name in ("W", "I", "O")]

Hidden = ckl.Buffer[ckl.f32, (B, C)]
Rows = ckl.Buffer[ckl.f32, (B,)]
Tokens = ckl.Buffer[ckl.i32, (B,)]
Position = ckl.Buffer[ckl.i32, (1,)]
History = ckl.Buffer[ckl.i32, (T, B)]
Embedding = ckl.Buffer[ckl.f32, (V, C)]
Gain = ckl.Buffer[ckl.f32, (L, C)]
FinalGain = ckl.Buffer[ckl.f32, (1, C)]
BlockWeight = ckl.Buffer[ckl.f32, (L, C, C)]
WideWeight = ckl.Buffer[ckl.f32, (L, C, F)]
DownWeight = ckl.Buffer[ckl.f32, (L, F, C)]
LMWeight = ckl.Buffer[ckl.f32, (1, C, V)]
Cache = ckl.Buffer[ckl.f32, (L, B, A, T, D)]
SinCos = ckl.Buffer[ckl.f32, (T, R, 2)]
Scores = ckl.Buffer[ckl.f32, (B, A, T)]
Logits = ckl.Buffer[ckl.f32, (B, V)]
Input = ckl.Buffer[ckl.f32, (B, I)]
Output = ckl.Buffer[ckl.f32, (B, O)]
Matrix = ckl.Buffer[ckl.f32, (W, I, O)]


@ckl.kernel
def embedding(ids: Tokens, table: Embedding, out: Hidden) -> None:
    col = ckl.global_id(0)
    row = ckl.global_id(1)
    if col < C:
        token = ckl.cast(ids[row], ckl.index)
        out[row, col] = table[token, col]


@ckl.kernel
def rms_stats(hidden: Hidden, scale: Rows, eps: ckl.f32) -> None:
    row = ckl.global_id(0)
    if row < B:
        acc = 0.0
        for col in range(C):
            acc = acc + hidden[row, col] * hidden[row, col]
        scale[row] = ckl.rsqrt(acc / C + eps)


@ckl.kernel
def rms_apply(hidden: Hidden, scale: Rows, gains: Gain, out: Hidden,
              layer: ckl.constexpr[ckl.index]) -> None:
    col = ckl.global_id(0)
    row = ckl.global_id(1)
    if col < C:
        out[row, col] = hidden[row, col] * scale[row] * gains[layer, col]


@ckl.kernel
def linear(act: Input, weights: Matrix, out: Output, layer: ckl.constexpr[ckl.index]) -> None:
    col = ckl.global_id(0)
    row = ckl.global_id(1)
    if col < O:
        acc = 0.0
        for k in range(I):
            acc = acc + act[row, k] * weights[layer, k, col]
        out[row, col] = acc


@ckl.kernel
def rope(vec: Hidden, angles: SinCos, pos: Position, out: Hidden) -> None:
    pair = ckl.global_id(0)
    head = ckl.global_id(1)
    row = ckl.global_id(2)
    if pair < R:
        p = ckl.cast(pos[0], ckl.index)
        col = head * (2 * R) + 2 * pair
        even = vec[row, col]
        odd = vec[row, col + 1]
        cos_p = angles[p, pair, 0]
        sin_p = angles[p, pair, 1]
        out[row, col] = even * cos_p - odd * sin_p
        out[row, col + 1] = even * sin_p + odd * cos_p


@ckl.kernel
def append_kv(key: Hidden, value: Hidden, key_cache: Cache, value_cache: Cache, pos: Position,
              layer: ckl.constexpr[ckl.index]) -> None:
    lane = ckl.global_id(0)
    head = ckl.global_id(1)
    row = ckl.global_id(2)
    if lane < D:
        p = ckl.cast(pos[0], ckl.index)
        key_cache[layer, row, head, p, lane] = key[row, head * D + lane]
        value_cache[layer, row, head, p, lane] = value[row, head * D + lane]


@ckl.kernel
def attention_scores(query: Hidden, key_cache: Cache, pos: Position, out: Scores,
                     scale: ckl.f32, layer: ckl.constexpr[ckl.index]) -> None:
    t = ckl.global_id(0)
    head = ckl.global_id(1)
    row = ckl.global_id(2)
    stop = ckl.cast(pos[0], ckl.index) + 1
    if t < stop:
        acc = 0.0
        for lane in range(D):
            acc = acc + query[row, head * D + lane] * key_cache[layer, row, head, t, lane]
        out[row, head, t] = acc * scale


@ckl.kernel
def softmax(scores: Scores, pos: Position, out: Scores) -> None:
    row = ckl.global_id(0)
    head = ckl.global_id(1)
    if row < B:
        stop = ckl.cast(pos[0], ckl.index) + 1
        peak = scores[row, head, 0]
        for t in range(1, stop):
            candidate = scores[row, head, t]
            peak = ckl.select(candidate > peak, candidate, peak)
        norm = 0.0
        for t in range(stop):
            norm = norm + ckl.exp(scores[row, head, t] - peak)
        for t in range(stop):
            out[row, head, t] = ckl.exp(scores[row, head, t] - peak) / norm


@ckl.kernel
def attention_values(weights: Scores, value_cache: Cache, pos: Position, out: Hidden,
                     layer: ckl.constexpr[ckl.index]) -> None:
    lane = ckl.global_id(0)
    head = ckl.global_id(1)
    row = ckl.global_id(2)
    if lane < D:
        stop = ckl.cast(pos[0], ckl.index) + 1
        acc = 0.0
        for t in range(stop):
            acc = acc + weights[row, head, t] * value_cache[layer, row, head, t, lane]
        out[row, head * D + lane] = acc


@ckl.kernel
def add(lhs: Hidden, rhs: Hidden, out: Hidden) -> None:
    col = ckl.global_id(0)
    row = ckl.global_id(1)
    if col < C:
        out[row, col] = lhs[row, col] + rhs[row, col]


@ckl.kernel
def silu(gate: Input, out: Input) -> None:
    col = ckl.global_id(0)
    row = ckl.global_id(1)
    if col < I:
        g = gate[row, col]
        out[row, col] = g / (1.0 + ckl.exp(-g))


@ckl.kernel
def multiply(lhs: Input, rhs: Input, out: Input) -> None:
    col = ckl.global_id(0)
    row = ckl.global_id(1)
    if col < I:
        out[row, col] = lhs[row, col] * rhs[row, col]


@ckl.kernel
def greedy(logits: Logits, ids: Tokens, generated: History, pos: Position) -> None:
    row = ckl.global_id(0)
    if row < B:
        best = logits[row, 0]
        arg = ckl.cast(row, ckl.i32) * 0
        for v in range(1, V):
            cand = logits[row, v]
            better = cand > best
            arg = ckl.select(better, ckl.cast(v, ckl.i32), arg)
            best = ckl.select(better, cand, best)
        p = ckl.cast(pos[0], ckl.index)
        ids[row] = arg
        generated[p, row] = arg


@ckl.kernel
def advance(pos: Position) -> None:
    pos[0] = pos[0] + 1


@ckl.program
def decode(tokens: Tokens, position: Position, history: History,
           emb: Embedding, norm1: Gain, norm2: Gain, final_norm: FinalGain,
           wq: BlockWeight, wk: BlockWeight, wv: BlockWeight, wo: BlockWeight,
           wg: WideWeight, wu: WideWeight, wd: DownWeight, lm: LMWeight,
           sincos: SinCos, kc: Cache, vc: Cache, logits: Logits,
           epsilon: ckl.f32, attention_scale: ckl.f32) -> None:
    hidden_grid = (ckl.cdiv(C, 64), B)
    ffn_grid = (ckl.cdiv(F, 64), B)
    row_grid = (ckl.cdiv(B, 32),)
    head_grid = (ckl.cdiv(D, 32), A, B)
    x = ckl.empty((B, C), dtype=ckl.f32)
    ckl.launch(embedding, tokens, emb, x, grid=hidden_grid, block=(64,))
    for layer in range(L):
        inv = ckl.empty((B,), dtype=ckl.f32)
        normed = ckl.empty_like(x)
        ckl.launch(rms_stats, x, inv, epsilon, grid=row_grid, block=(32,))
        ckl.launch(rms_apply, x, inv, norm1, normed, layer, grid=hidden_grid, block=(64,))
        q = ckl.empty_like(x)
        k = ckl.empty_like(x)
        v = ckl.empty_like(x)
        ckl.launch(linear, normed, wq, q, layer, grid=hidden_grid, block=(64,))
        ckl.launch(linear, normed, wk, k, layer, grid=hidden_grid, block=(64,))
        ckl.launch(linear, normed, wv, v, layer, grid=hidden_grid, block=(64,))
        qr = ckl.empty_like(x)
        kr = ckl.empty_like(x)
        ckl.launch(rope, q, sincos, position, qr, grid=(ckl.cdiv(R, 32), A, B), block=(32,))
        ckl.launch(rope, k, sincos, position, kr, grid=(ckl.cdiv(R, 32), A, B), block=(32,))
        ckl.launch(append_kv, kr, v, kc, vc, position, layer, grid=head_grid, block=(32,))
        scores = ckl.empty((B, A, T), dtype=ckl.f32)
        probs = ckl.empty_like(scores)
        ckl.launch(attention_scores, qr, kc, position, scores, attention_scale, layer,
                   grid=(ckl.cdiv(T, 32), A, B), block=(32,))
        ckl.launch(softmax, scores, position, probs, grid=(ckl.cdiv(B, 32), A), block=(32,))
        context = ckl.empty_like(x)
        ckl.launch(attention_values, probs, vc, position, context, layer, grid=head_grid,
                   block=(32,))
        projected = ckl.empty_like(x)
        ckl.launch(linear, context, wo, projected, layer, grid=hidden_grid, block=(64,))
        residual = ckl.empty_like(x)
        ckl.launch(add, x, projected, residual, grid=hidden_grid, block=(64,))
        inv2 = ckl.empty((B,), dtype=ckl.f32)
        normed2 = ckl.empty_like(x)
        ckl.launch(rms_stats, residual, inv2, epsilon, grid=row_grid, block=(32,))
        ckl.launch(rms_apply, residual, inv2, norm2, normed2, layer, grid=hidden_grid, block=(64,))
        gate = ckl.empty((B, F), dtype=ckl.f32)
        up = ckl.empty_like(gate)
        ckl.launch(linear, normed2, wg, gate, layer, grid=ffn_grid, block=(64,))
        ckl.launch(linear, normed2, wu, up, layer, grid=ffn_grid, block=(64,))
        activated = ckl.empty_like(gate)
        product = ckl.empty_like(gate)
        ckl.launch(silu, gate, activated, grid=ffn_grid, block=(64,))
        ckl.launch(multiply, activated, up, product, grid=ffn_grid, block=(64,))
        down = ckl.empty_like(x)
        next_x = ckl.empty_like(x)
        ckl.launch(linear, product, wd, down, layer, grid=hidden_grid, block=(64,))
        ckl.launch(add, residual, down, next_x, grid=hidden_grid, block=(64,))
        x = next_x
    final_inv = ckl.empty((B,), dtype=ckl.f32)
    final_x = ckl.empty_like(x)
    ckl.launch(rms_stats, x, final_inv, epsilon, grid=row_grid, block=(32,))
    ckl.launch(rms_apply, x, final_inv, final_norm, final_x, 0, grid=hidden_grid, block=(64,))
    ckl.launch(linear, final_x, lm, logits, 0, grid=(ckl.cdiv(V, 64), B), block=(64,))
    ckl.launch(greedy, logits, tokens, history, position, grid=row_grid, block=(32,))
    ckl.launch(advance, position, grid=(1,), block=(1,))


#: Runtime argument order of ``decode`` (buffers by name, then the two scalars).
ARGUMENTS = ("tokens", "position", "history", "emb", "norm1", "norm2", "final_norm", "wq", "wk",
             "wv", "wo", "wg", "wu", "wd", "lm", "sincos", "kc", "vc", "logits", "epsilon",
             "attention_scale")
