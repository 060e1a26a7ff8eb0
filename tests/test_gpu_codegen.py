"""Generated kernels on the GPU: the reference's runtime semantic checks, restated.

* zero-trip and multi-carried f64 loops with ``select``/``exp``/``rsqrt`` in every execution
  mode and with repetition (``tests/Runtime/test_kernel_loops.py``);
* i64 constexpr and f64 runtime scalars, byte exact (``tests/Runtime/test_frontend_runtime.py``);
* no multiply-add contraction inside one kernel: (1 + 2^-23)(1 - 2^-23) - 1 is 0 in f32 with
  two roundings and -2^-46 with one (``tests/Runtime/test_pointwise_fusion.py:105-118``);
* device coordinates on three axes, integer wrap-around and conversions;
* a partial launch of the decoder's ``linear`` writes exactly its part;
* the whole decode step with every kernel generated from its body (``library=False``, the
  reference's naive code path) against the oracle, tokens bit-exact.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

import ckl
from ckl.workloads import decoder
from oracle import decoder as ref
from test_gpu_decoder import CFG1, open_session, verify

pytestmark = pytest.mark.gpu
TARGET = ckl.NVIDIATarget("sm_100a")

Doubles = ckl.Buffer[ckl.f64, (4,)]
N = ckl.dim("N")
Vector = ckl.Buffer[ckl.f32, (N,)]
linear = decoder.linear


@pytest.fixture(scope="module")
def device():
    return ckl.Device()


def upload(device, values, dtype):
    buffer = device.empty(ckl.BufferSpec(values.shape, dtype))
    buffer.copy_from_host(np.ascontiguousarray(values))
    return buffer


def download(buffer, np_dtype):
    out = np.empty(buffer.spec.shape, np_dtype)
    buffer.copy_to_host(out)
    return out


@ckl.kernel
def statistics(src: Doubles, dst: Doubles, count: ckl.i32) -> None:
    if ckl.global_id(0) == 0:
        total = src[0] * 0.0
        maximum = src[0]
        winner = count * 0
        for i in range(ckl.cast(count, ckl.index)):
            value = src[i]
            wins = value > maximum
            winner = ckl.select(wins, ckl.cast(i, ckl.i32), winner)
            maximum = ckl.select(wins, value, maximum)
            total = total + value
        dst[0] = total
        dst[1] = ckl.exp(maximum) * ckl.rsqrt(maximum * maximum + 1.0)
        dst[2] = ckl.cast(winner, ckl.f64)


@ckl.program
def statistics_entry(src: Doubles, dst: Doubles, count: ckl.i32) -> None:
    ckl.launch(statistics, src, dst, count, grid=(1,), block=(1,))


def test_loops_math_and_modes(device):
    spec = ckl.BufferSpec((4,), ckl.f64)
    src = upload(device, np.array([1., 0.25, 2., -0.5]), ckl.f64)
    dst = device.empty(spec)
    program = statistics_entry.lower(signature=dict(src=spec, dst=spec, count=ckl.i32)).compile(
        target=TARGET, fuse_pointwise=False)
    assert program.plans.primary.node_names[0].startswith("ckl_gen_statistics_")
    for count, total, maximum, winner in ((0, 0., 1., 0), (4, 2.75, 2., 2)):
        bound = program.bind(src, dst, count)
        for mode in ("capture", "ordinary", "graph"):
            dst.copy_from_host(np.full(4, -12345.))
            bound.run(mode=mode, batch_size=3)
            actual = download(dst, np.float64)
            expected = [total, math.exp(maximum) / math.sqrt(maximum * maximum + 1), winner,
                        -12345.]
            assert np.allclose(actual, expected, rtol=1e-12, atol=1e-12), (count, mode, actual)


@ckl.kernel
def integer_update(src: ckl.Buffer[ckl.i64, (4,)], dst: ckl.Buffer[ckl.i64, (4,)],
                   bias: ckl.i64) -> None:
    i = ckl.global_id(0)
    if i < 4:
        dst[i] = src[i] + bias


@ckl.program
def integer_step(src: ckl.Buffer[ckl.i64, (4,)], dst: ckl.Buffer[ckl.i64, (4,)],
                 bias: ckl.constexpr[ckl.i64]) -> None:
    ckl.launch(integer_update, src, dst, bias, grid=(1,), block=(4,))


@ckl.kernel
def double_update(src: Doubles, dst: Doubles, bias: ckl.f64) -> None:
    i = ckl.global_id(0)
    if i < 4:
        dst[i] = src[i] + bias


@ckl.program
def double_step(src: Doubles, dst: Doubles, bias: ckl.f64) -> None:
    ckl.launch(double_update, src, dst, bias, grid=(1,), block=(4,))


def test_i64_constants_and_f64_scalars_are_exact(device):
    i64 = ckl.BufferSpec((4,), ckl.i64)
    bias = -(2 ** 40 + 3)
    src = upload(device, np.arange(4, dtype=np.int64), ckl.i64)
    dst = device.empty(i64)
    program = integer_step.lower(signature={"src": i64, "dst": i64},
                                 constants={"bias": bias}).compile(target=TARGET)
    invocation = program.bind(src, dst)
    for graph in (False, True):
        invocation.run(graph=graph)
        assert download(dst, np.int64).tolist() == [v + bias for v in range(4)]
    f64 = ckl.BufferSpec((4,), ckl.f64)
    src = upload(device, np.arange(4, dtype=np.float64), ckl.f64)
    dst = device.empty(f64)
    program = double_step.lower(signature={"src": f64, "dst": f64, "bias": ckl.f64}).compile(
        target=TARGET)
    invocation = program.bind(src, dst, 2 ** -42)
    for graph in (False, True):
        invocation.run(graph=graph)
        assert download(dst, np.float64).tolist() == [v + 2 ** -42 for v in range(4)]


@ckl.kernel
def multiply_add(src: Vector, dst: Vector, factor: ckl.f32, bias: ckl.f32) -> None:
    i = ckl.global_id(0)
    if i < N:
        dst[i] = src[i] * factor + bias


@ckl.program
def rounding(src: Vector, dst: Vector, factor: ckl.f32, bias: ckl.f32) -> None:
    ckl.launch(multiply_add, src, dst, factor, bias, grid=(ckl.cdiv(N, 256),), block=(256,))


def test_no_multiply_add_contraction(device):
    spec = ckl.BufferSpec((257,), ckl.f32)
    program = rounding.lower(signature={"src": spec, "dst": spec, "factor": ckl.f32,
                                        "bias": ckl.f32}).compile(target=TARGET)
    src = upload(device, np.full(257, 1 + 2 ** -23, np.float32), ckl.f32)
    dst = upload(device, np.ones(257, np.float32), ckl.f32)
    invocation = program.bind(src, dst, 1 - 2 ** -23, -1.)
    for graph in (False, True):
        invocation.run(graph=graph)
        assert download(dst, np.float32).tobytes() == np.zeros(257, np.float32).tobytes()


Grid = ckl.Buffer[ckl.i64, (5, 3, 4, 6, 2)]


@ckl.kernel
def coordinates(out: Grid) -> None:
    x = ckl.global_id(0)
    y = ckl.global_id(1)
    z = ckl.global_id(2)
    if x < 6:
        if y < 4:
            if z < 3:
                out[0, z, y, x, 0] = ckl.cast(ckl.thread_id(0) + ckl.block_id(0) * 100, ckl.i64)
                out[0, z, y, x, 1] = ckl.cast(ckl.block_dim(0) + ckl.grid_dim(0) * 100, ckl.i64)
                out[1, z, y, x, 0] = ckl.cast(ckl.thread_id(1) + ckl.block_id(1) * 100, ckl.i64)
                out[1, z, y, x, 1] = ckl.cast(ckl.block_dim(1) + ckl.grid_dim(1) * 100, ckl.i64)
                out[2, z, y, x, 0] = ckl.cast(ckl.thread_id(2) + ckl.block_id(2) * 100, ckl.i64)
                out[2, z, y, x, 1] = ckl.cast(ckl.block_dim(2) + ckl.grid_dim(2) * 100, ckl.i64)
                out[3, z, y, x, 0] = ckl.cast(x, ckl.i64)
                out[3, z, y, x, 1] = ckl.cast(y, ckl.i64)
                out[4, z, y, x, 0] = ckl.cast(z, ckl.i64)
                out[4, z, y, x, 1] = ckl.cast(x + y * 10 + z * 100, ckl.i64)


@ckl.program
def coordinate_entry(out: Grid) -> None:
    ckl.launch(coordinates, out, grid=(2, 2, 3), block=(4, 3, 1))


def test_device_coordinates_on_three_axes(device):
    spec = ckl.BufferSpec((5, 3, 4, 6, 2), ckl.i64)
    out = upload(device, np.full(spec.shape, -1, np.int64), ckl.i64)
    program = coordinate_entry.lower(signature={"out": spec}).compile(target=TARGET)
    program.bind(out).run(graph=True)
    actual = download(out, np.int64)
    z, y, x = np.meshgrid(np.arange(3), np.arange(4), np.arange(6), indexing="ij")
    block, grid = (4, 3, 1), (2, 2, 3)
    for axis, g in enumerate((x, y, z)):
        assert np.array_equal(actual[axis, ..., 0], g % block[axis] + (g // block[axis]) * 100)
        assert np.all(actual[axis, ..., 1] == block[axis] + grid[axis] * 100)
    assert np.array_equal(actual[3, ..., 0], x) and np.array_equal(actual[3, ..., 1], y)
    assert np.array_equal(actual[4, ..., 0], z)
    assert np.array_equal(actual[4, ..., 1], x + 10 * y + 100 * z)


Ints = ckl.Buffer[ckl.i32, (6,)]
Floats = ckl.Buffer[ckl.f32, (4,)]


@ckl.kernel
def conversions(ints: Ints, floats: Floats, wide: ckl.Buffer[ckl.f64, (2,)],
                longs: ckl.Buffer[ckl.i64, (2,)]) -> None:
    if ckl.global_id(0) == 0:
        ints[0] = ints[0] + 1                                   # 2^31 - 1 + 1 wraps
        ints[1] = ints[1] * 65536                               # wraps
        ints[2] = ckl.cast(floats[0], ckl.i32)                  # fptosi truncates toward 0
        ints[3] = ckl.cast(longs[0], ckl.i32)                   # trunci keeps the low bits
        ints[4] = -ints[4]
        ints[5] = ckl.cast(ckl.cast(ints[5], ckl.index) + 7, ckl.i32)
        floats[1] = ckl.cast(ints[5], ckl.f32)                  # sitofp
        floats[2] = ckl.cast(wide[0], ckl.f32)                  # truncf rounds to nearest
        floats[3] = floats[3] / 3.0
        wide[1] = ckl.cast(floats[3], ckl.f64)                  # extf
        longs[1] = ckl.cast(ints[4], ckl.i64)                   # extsi


@ckl.program
def conversion_entry(ints: Ints, floats: Floats, wide: ckl.Buffer[ckl.f64, (2,)],
                     longs: ckl.Buffer[ckl.i64, (2,)]) -> None:
    ckl.launch(conversions, ints, floats, wide, longs, grid=(1,), block=(32,))


def test_integer_wraparound_and_conversions(device):
    ints = upload(device, np.array([2 ** 31 - 1, 40000, 0, 0, -17, 5], np.int32), ckl.i32)
    floats = upload(device, np.array([-2.7, 0, 0, 1], np.float32), ckl.f32)
    wide = upload(device, np.array([1 + 2 ** -30, 0]), ckl.f64)
    longs = upload(device, np.array([2 ** 32 + 9, 0], np.int64), ckl.i64)
    program = conversion_entry.lower(signature={
        "ints": ints.spec, "floats": floats.spec, "wide": wide.spec, "longs": longs.spec}).compile(
        target=TARGET)
    program.bind(ints, floats, wide, longs).run()
    assert download(ints, np.int32).tolist() == [-2 ** 31, 40000 * 65536 - 2 ** 32, -2, 9, 17, 12]
    f = download(floats, np.float32)
    third = np.float32(1) / np.float32(3)
    assert f[1] == 12.0 and f[2] == np.float32(1 + 2 ** -30) and f[3] == third
    assert download(wide, np.float64)[1] == float(third)
    assert download(longs, np.int64)[1] == 17


@ckl.program
def partial_linear(x: ckl.Buffer[ckl.f32, (2, 64)], w: ckl.Buffer[ckl.f32, (1, 64, 256)],
                   y: ckl.Buffer[ckl.f32, (2, 256)]) -> None:
    ckl.launch(linear, x, w, y, 0, grid=(1, 2), block=(64,))


def test_partial_launch_writes_exactly_its_part(device):
    rng = np.random.default_rng(3)
    xv = rng.standard_normal((2, 64)).astype(np.float32)
    wv = rng.standard_normal((1, 64, 256)).astype(np.float32)
    x, w = upload(device, xv, ckl.f32), upload(device, wv, ckl.f32)
    y = upload(device, np.full((2, 256), -12345., np.float32), ckl.f32)
    program = partial_linear.lower(signature={"x": x.spec, "w": w.spec, "y": y.spec}).compile(
        target=TARGET)
    program.bind(x, w, y).run(graph=True)
    actual = download(y, np.float32)
    expected = np.zeros((2, 64), np.float32)
    for i in range(64):                                   # the kernel's own summation order
        expected = (expected + (xv[:, i:i + 1] * wv[0, i:i + 1, :64])).astype(np.float32)
    assert np.array_equal(actual[:, :64], expected)
    assert np.all(actual[:, 64:] == -12345.)


@pytest.mark.parametrize("eps", [1e-6, 1e-5])
def test_decode_step_from_generated_kernels_matches_oracle(device, eps):
    """Every kernel of the decode step generated from its body (no library): the
    reference's own naive code path, on sm_100a."""
    initial, _ = ref.make_inputs(CFG1, 0, eps=eps)
    expected = ref.expected(initial, CFG1, CFG1.steps, eps=eps)
    session = open_session(device, CFG1, initial, eps, library=False)
    assert session.invocation.node_count == 21 * CFG1.layers + 6
    assert all(n.startswith("ckl_gen_") for n in session.program.plans.primary.node_names)
    session.step(CFG1.steps)
    verify(session, initial, expected, CFG1)
