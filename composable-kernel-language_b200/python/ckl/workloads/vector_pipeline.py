"""The vector pipeline in the CKL DSL: two chained pointwise launches through a temporary.

The reference's minimal program (``examples/vector_pipeline.py:9-24``): ``update`` adds a
scalar bias to every element, and ``step`` applies it twice through an ``empty_like``
temporary, so ``dst = (src + bias) + bias``.  With pointwise fusion the pair becomes one
launch and the temporary disappears.
"""
import ckl

N = ckl.dim("N")
Vector = ckl.Buffer[ckl.f32, (N,)]


@ckl.kernel
def update(src: Vector, dst: Vector, bias: ckl.f32) -> None:
    i = ckl.global_id(0)
    if i < src.shape[0]:
        dst[i] = src[i] + bias


@ckl.kernel
def scale(src: Vector, dst: Vector, factor: ckl.f32) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = src[i] * factor


@ckl.kernel
def fill(dst: Vector, value: ckl.f32) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = value


@ckl.kernel
def copy(src: Vector, dst: Vector) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = src[i]


@ckl.program
def step(src: Vector, dst: Vector, bias: ckl.f32) -> None:
    temporary = ckl.empty_like(src)
    grid = (ckl.cdiv(src.shape[0], 256),)
    block = (256,)
    ckl.launch(update, src, temporary, bias, grid=grid, block=block)
    ckl.launch(update, temporary, dst, bias, grid=grid, block=block)


def lower(n: int = 257):
    spec = ckl.BufferSpec(shape=(n,), dtype=ckl.f32)
    return step.lower(signature={"src": spec, "dst": spec, "bias": ckl.f32})
