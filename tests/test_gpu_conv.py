"""GPU parity of the NCHW convolution and its reverse mode.

TF32 tensor-core results (3x3 / pad 1 / stride 1 shapes) are held to the
TF32 tolerance for convolutions and their gradients, rtol 1e-3 + atol
1e-3 * max|ref|, against the oracle, and so is 2xTF32 (one operand split,
the other TF32); 3xTF32 (the same tensor-core kernels with hi/lo split
operands) and the direct path (other shapes, computing in the oracle's
order) are held to rtol 1e-5 + atol 1e-5 * max|ref|.  2xTF32 must also be
closer to the oracle than TF32 on the same data."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, to_dev, to_host
from remora_b200 import ops

pytestmark = pytest.mark.gpu


def close(got, ref, tight):
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(1.0, float(np.abs(ref).max()) if ref.size else 1.0)
    if tight:
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5 * scale)
    else:
        np.testing.assert_allclose(got, ref, rtol=1e-3, atol=1e-3 * scale)


def data(shape_x, shape_w, seed):
    rng = np.random.Generator(np.random.PCG64(seed))
    x = rng.standard_normal(shape_x).astype(np.float32)
    fan = shape_w[1] * shape_w[2] * shape_w[3]
    w = (rng.standard_normal(shape_w) * np.sqrt(2.0 / fan)).astype(np.float32)
    b = rng.standard_normal(shape_w[0]).astype(np.float32) * 0.1
    return x, w, b


def test_golden_single_channel_conv_and_grads(cuda):
    """The reference's own conv2d and tape gradients (valid 3x3 on 8x8)."""
    g = golden("conv_single")
    x, k = to_dev(g["x"][None, None], cuda), to_dev(g["k"][None, None], cuda)
    b = to_dev(np.array([g["b"]], np.float32), cuda)
    y = to_host(ops.conv2d_fwd(x, k, b, pad=0))
    close(y.reshape(-1), g["y"], True)
    cot = to_dev(g["cot"].reshape(1, 1, 6, 6), cuda)
    close(to_host(ops.conv2d_dgrad(cot, k, (1, 1, 8, 8), pad=0))[0, 0], g["dx"], True)
    close(to_host(ops.conv2d_wgrad(x, cot, (1, 1, 3, 3), pad=0))[0, 0], g["dk"], True)


@pytest.mark.parametrize("shape", [((2, 16, 64, 64), (32, 16, 3, 3)), ((3, 16, 32, 32), (32, 16, 3, 3)),
                                   ((2, 32, 32, 32), (16, 32, 3, 3)), ((2, 32, 64, 64), (16, 32, 3, 3)),
                                   ((1, 16, 7, 64), (8, 16, 3, 3)), ((2, 16, 5, 32), (32, 16, 3, 3))])
@pytest.mark.parametrize("prec", ["tf32", "3xtf32", "2xtf32"])
def test_conv_fwd_dgrad_tensor_core_shapes(cuda, oracle_mod, shape, prec):
    sx, sw = shape
    x, w, b = data(sx, sw, 11)
    dx_, dw_ = to_dev(x, cuda), to_dev(w, cuda)
    y = to_host(ops.conv2d_fwd(dx_, dw_, to_dev(b, cuda), precision=prec))
    close(y, oracle_mod.conv2d_fwd(x, w, b, nthreads=oracle_mod.max_threads()), prec == "3xtf32")
    dy = np.random.Generator(np.random.PCG64(12)).standard_normal(y.shape).astype(np.float32)
    dx = to_host(ops.conv2d_dgrad(to_dev(dy, cuda), dw_, sx, precision=prec))
    close(dx, oracle_mod.conv2d_dgrad(dy, w, sx, nthreads=oracle_mod.max_threads()), prec == "3xtf32")
    dw = to_host(ops.conv2d_wgrad(dx_, to_dev(dy, cuda), sw, precision=prec))
    close(dw, oracle_mod.conv2d_wgrad(x, dy, sw, nthreads=oracle_mod.max_threads()), prec == "3xtf32")


@pytest.mark.parametrize("shape", [((2, 16, 16, 16), (48, 16, 3, 3)), ((2, 32, 20, 128), (40, 32, 3, 3)),
                                   ((2, 64, 32, 32), (64, 64, 3, 3)), ((1, 64, 24, 64), (16, 64, 3, 3)),
                                   ((2, 16, 10, 16), (100, 16, 3, 3)), ((1, 32, 9, 128), (16, 32, 3, 3))])
@pytest.mark.parametrize("prec", ["tf32", "3xtf32", "2xtf32"])
def test_conv_wider_shapes(cuda, oracle_mod, shape, prec):
    """3x3 / pad 1 layers beyond the crater CNN's: 16-, 64- and 128-wide
    images, 16, 32 or 64 input channels, and output channels past 32, which
    the tensor-core kernels take in launches of at most 32 output channels
    each (weight gradient: 16 input channels per launch as well).  Where no
    tensor-core form exists (48 or 100 reduction channels in the input
    gradient, 3xTF32 weight gradient of 128-wide rows) the direct kernels
    run, and the same tolerances hold."""
    sx, sw = shape
    x, w, b = data(sx, sw, 21)
    dx_, dw_ = to_dev(x, cuda), to_dev(w, cuda)
    nt = oracle_mod.max_threads()
    y = to_host(ops.conv2d_fwd(dx_, dw_, to_dev(b, cuda), precision=prec))
    close(y, oracle_mod.conv2d_fwd(x, w, b, nthreads=nt), prec == "3xtf32")
    dy = np.random.Generator(np.random.PCG64(22)).standard_normal(y.shape).astype(np.float32)
    dx = to_host(ops.conv2d_dgrad(to_dev(dy, cuda), dw_, sx, precision=prec))
    close(dx, oracle_mod.conv2d_dgrad(dy, w, sx, nthreads=nt), prec == "3xtf32")
    dw = to_host(ops.conv2d_wgrad(dx_, to_dev(dy, cuda), sw, precision=prec))
    close(dw, oracle_mod.conv2d_wgrad(x, dy, sw, nthreads=nt), prec == "3xtf32")


@pytest.mark.parametrize("shape", [((2, 16, 64, 64), (32, 16, 3, 3)), ((3, 16, 32, 32), (32, 16, 3, 3)),
                                   ((2, 32, 32, 32), (16, 32, 3, 3)), ((2, 32, 64, 64), (16, 32, 3, 3))])
def test_conv_2xtf32_between_tf32_and_3xtf32(cuda, oracle_mod, shape):
    """The split operand of 2xTF32 removes its share of the TF32 error: the
    input gradient (weights split) and the weight gradient (output gradient
    split) come out closer to the oracle than plain TF32 (measured on a
    B200: 1.6x to 2.0x closer, one of the two truncated operands left)."""
    sx, sw = shape
    x, w, _ = data(sx, sw, 21)
    dx_, dw_ = to_dev(x, cuda), to_dev(w, cuda)
    oshape = (sx[0], sw[0], sx[2], sx[3])
    dy = np.random.Generator(np.random.PCG64(22)).standard_normal(oshape).astype(np.float32)
    dyd = to_dev(dy, cuda)
    nt = oracle_mod.max_threads()
    refs = {"dgrad": oracle_mod.conv2d_dgrad(dy, w, sx, nthreads=nt),
            "wgrad": oracle_mod.conv2d_wgrad(x, dy, sw, nthreads=nt)}
    err = {}
    for prec in ("tf32", "2xtf32"):
        got = {"dgrad": to_host(ops.conv2d_dgrad(dyd, dw_, sx, precision=prec)),
               "wgrad": to_host(ops.conv2d_wgrad(dx_, dyd, sw, precision=prec))}
        for k, r in refs.items():
            err[prec, k] = float(np.abs(got[k] - r).max()) / float(np.abs(r).max())
    # the weight gradient runs on the tensor cores for 16 input channels only
    for k in (("dgrad", "wgrad") if sx[1] == 16 else ("dgrad",)):
        assert err["2xtf32", k] * 1.25 <= err["tf32", k], (k, err)


@pytest.mark.parametrize("geom", [((3, 3, 10, 13), (5, 3, 3, 3), 2, 1), ((2, 1, 64, 64), (16, 1, 3, 3), 1, 1),
                                  ((1, 4, 9, 9), (2, 4, 5, 5), 1, 2), ((2, 2, 6, 6), (3, 2, 2, 2), 3, 0)])
def test_conv_direct_shapes(cuda, oracle_mod, geom):
    sx, sw, stride, pad = geom
    x, w, b = data(sx, sw, 13)
    y = to_host(ops.conv2d_fwd(to_dev(x, cuda), to_dev(w, cuda), to_dev(b, cuda), stride=stride, pad=pad,
                               precision="tf32"))
    ref = oracle_mod.conv2d_fwd(x, w, b, stride=stride, pad=pad)
    np.testing.assert_array_equal(y, ref)  # same order, same rounding
    dy = np.random.Generator(np.random.PCG64(14)).standard_normal(y.shape).astype(np.float32)
    dx = to_host(ops.conv2d_dgrad(to_dev(dy, cuda), to_dev(w, cuda), sx, stride=stride, pad=pad))
    np.testing.assert_array_equal(dx, oracle_mod.conv2d_dgrad(dy, w, sx, stride=stride, pad=pad))
    dw = to_host(ops.conv2d_wgrad(to_dev(x, cuda), to_dev(dy, cuda), sw, stride=stride, pad=pad))
    close(dw, oracle_mod.conv2d_wgrad(x, dy, sw, stride=stride, pad=pad), True)


def test_conv_benchmark_layer_full_size(cuda, oracle_mod):
    """The im2col-conv workload: x [256,16,64,64] ~ N(0,1), w [32,16,3,3] ~
    N(0, sqrt(2/144)), pad 1, cotangent dy ~ N(0,1).  The whole batch runs on
    the device; sampled images are checked against the oracle, and dw (a sum
    over every image) is checked in full."""
    rng = np.random.Generator(np.random.PCG64(1729))
    x = rng.standard_normal((256, 16, 64, 64), dtype=np.float32)
    w = (np.random.Generator(np.random.PCG64(2718)).standard_normal((32, 16, 3, 3)) * np.sqrt(2 / 144)).astype(
        np.float32)
    dy = np.random.Generator(np.random.PCG64(1731)).standard_normal((256, 32, 64, 64), dtype=np.float32)
    xd, wd, dyd = to_dev(x, cuda), to_dev(w, cuda), to_dev(dy, cuda)
    nt = oracle_mod.max_threads()
    y = to_host(ops.conv2d_fwd(xd, wd, None, precision="tf32"))
    dx = to_host(ops.conv2d_dgrad(dyd, wd, x.shape, precision="tf32"))
    for n in (0, 101, 255):
        close(y[n:n + 1], oracle_mod.conv2d_fwd(x[n:n + 1], w, None, nthreads=nt), False)
        close(dx[n:n + 1], oracle_mod.conv2d_dgrad(dy[n:n + 1], w, (1, 16, 64, 64), nthreads=nt), False)
    dw = to_host(ops.conv2d_wgrad(xd, dyd, w.shape, precision="tf32"))
    close(dw, oracle_mod.conv2d_wgrad(x, dy, w.shape, nthreads=nt), False)
