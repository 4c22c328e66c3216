"""GPU parity of scans, im2col/col2im and transpose.  i32 scans and all
layout ops are bit-exact with the oracle; f32 scans reassociate per tile and
are checked at rtol 1e-5 plus a bound scaled by the running magnitude."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, to_dev, to_host
from remora_b200 import ops
from remora_b200.codegen import scan_spec
from remora_b200.errors import RemoraUnsupportedError

pytestmark = pytest.mark.gpu


def scan_close(got, ref, x, right=False):
    ax = np.abs(x.astype(np.float64))
    mag = np.flip(np.cumsum(np.flip(ax, 0), axis=0), 0) if right else np.cumsum(ax, axis=0)
    bound = 1e-5 * np.abs(ref) + 2e-6 * (mag + 1.0)
    assert np.all(np.abs(got.astype(np.float64) - ref) <= bound)


def test_golden_scans(cuda):
    g = golden("scans")
    for tag, kw in (("inc", {}), ("exc", {"exclusive": True}), ("right", {"right": True})):
        got = to_host(ops.scan(to_dev(g["f"], cuda), init=0.5, **kw))
        np.testing.assert_allclose(got, g[f"f32_{tag}"], rtol=1e-5, atol=1e-5)
        got = to_host(ops.scan(to_dev(g["i"], cuda), init=3, **kw))
        np.testing.assert_array_equal(got, g[f"i32_{tag}"])
    np.testing.assert_array_equal(to_host(ops.scan(to_dev(np.array([2, 10, 5], np.int32), cuda))), g["small_inc"])
    g = golden("scan_rank2")
    np.testing.assert_allclose(to_host(ops.scan(to_dev(g["m"], cuda))), g["out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("n", [1, 7, 2048, 2049, 100003, 1 << 22])
@pytest.mark.parametrize("kw", [{}, {"exclusive": True}, {"right": True}, {"right": True, "exclusive": True}])
def test_rank1_scans(cuda, oracle_mod, n, kw):
    rng = np.random.default_rng(n)
    xi = rng.integers(-1000, 1000, n).astype(np.int32)
    np.testing.assert_array_equal(to_host(ops.scan(to_dev(xi, cuda), init=-5, **kw)),
                                  oracle_mod.scan(scan_spec(dtype="i32", init=-5, **kw), xi))
    xf = rng.uniform(-1, 1, n).astype(np.float32)
    scan_close(to_host(ops.scan(to_dev(xf, cuda), init=0.25, **kw)), oracle_mod.scan(scan_spec(init=0.25, **kw), xf),
               xf, right=kw.get("right", False))


@pytest.mark.parametrize("kw", [{}, {"right": True, "exclusive": True}])
@pytest.mark.parametrize("n", [100000, 100001])
def test_rank1_scan_unaligned_views_equal_contiguous_copies(cuda, oracle_mod, n, kw):
    """A view one element into its buffer (not 16-byte aligned: the tiles
    read element by element) scans to the same bits as a contiguous copy
    (read as 16-byte vectors): the combine order does not depend on how
    the elements are loaded.  i32 results equal the oracle's."""
    import torch

    rng = np.random.default_rng(n + 7)
    for dt, lo_hi in ((np.int32, (-1000, 1000)), (np.float32, None)):
        host = (rng.integers(*lo_hi, n + 1) if lo_hi else rng.uniform(-1, 1, n + 1)).astype(dt)
        buf = to_dev(host, cuda)
        view = buf[1:]
        assert view.data_ptr() % 16 != 0
        a = to_host(ops.scan(view, **kw))
        b = to_host(ops.scan(view.contiguous(), **kw))
        np.testing.assert_array_equal(a, b)
        if dt == np.int32:
            np.testing.assert_array_equal(a, oracle_mod.scan(scan_spec(dtype="i32", **kw), host[1:]))
        out = torch.zeros(n + 1, dtype=view.dtype, device=cuda)
        ops.scan(view.contiguous(), out=out[1:], **kw)  # an unaligned output view
        np.testing.assert_array_equal(to_host(out[1:]), b)


@pytest.mark.parametrize("shape", [(5, 3), (1000, 1), (4096, 16), (3, 300000), (257, 7, 5)])
def test_multirank_scans(cuda, oracle_mod, shape):
    rng = np.random.default_rng(len(shape))
    xi = rng.integers(-100, 100, shape).astype(np.int32)
    np.testing.assert_array_equal(to_host(ops.scan(to_dev(xi, cuda))), oracle_mod.scan(scan_spec(dtype="i32"), xi))
    xf = rng.uniform(-1, 1, shape).astype(np.float32)
    scan_close(to_host(ops.scan(to_dev(xf, cuda))), oracle_mod.scan(scan_spec(), xf), xf)
    with pytest.raises(RemoraUnsupportedError):
        ops.scan(to_dev(xf, cuda), exclusive=True)


def test_scan_mul_and_determinism(cuda):
    rng = np.random.default_rng(3)
    xf = rng.uniform(0.9999, 1.0001, 50000).astype(np.float32)
    d = to_dev(xf, cuda)
    a = to_host(ops.scan(d, op="*", init=1.0))
    b = to_host(ops.scan(d, op="*", init=1.0))
    np.testing.assert_array_equal(a, b)
    # f32 products of values near 1 round with a bias: sequential f32 is
    # ~1e-4 from f64 on this input, a blocked order ~3e-4
    np.testing.assert_allclose(a, np.cumprod(xf.astype(np.float64)), rtol=1e-3)


def test_im2col_col2im_golden_and_oracle(cuda, oracle_mod):
    g = golden("im2col")
    for s in (1, 2):
        np.testing.assert_array_equal(to_host(ops.im2col(to_dev(g["img"], cuda), 3, 3, s)), g[f"cols_s{s}"])
        np.testing.assert_array_equal(to_host(ops.col2im(to_dev(g[f"cin_s{s}"], cuda), (5, 6), 3, 3, s)),
                                      g[f"img_s{s}"])
    rng = np.random.default_rng(5)
    for (H, W, kh, kw, s) in ((32, 32, 3, 3, 1), (64, 48, 5, 3, 2), (9, 9, 9, 9, 1), (10, 13, 2, 4, 3)):
        img = rng.standard_normal((H, W)).astype(np.float32)
        np.testing.assert_array_equal(to_host(ops.im2col(to_dev(img, cuda), kh, kw, s)),
                                      oracle_mod.im2col(img, kh, kw, s))
        oh, ow = (H - kh) // s + 1, (W - kw) // s + 1
        cols = rng.standard_normal((oh * ow, kh * kw)).astype(np.float32)
        np.testing.assert_array_equal(to_host(ops.col2im(to_dev(cols, cuda), (H, W), kh, kw, s)),
                                      oracle_mod.col2im(cols, H, W, kh, kw, s))
    ones = to_dev(np.ones((9, 4), np.float32), cuda)
    img = to_host(ops.col2im(ones, (4, 4), 2, 2, 1))
    assert img[0, 0] == 1 and img[0, 1] == 2 and img[1, 1] == 4


def test_transpose(cuda):
    rng = np.random.default_rng(6)
    for shape in ((1, 1), (33, 65), (1024, 3), (4096, 4096)):
        a = rng.standard_normal(shape).astype(np.float32)
        np.testing.assert_array_equal(to_host(ops.transpose(to_dev(a, cuda))), a.T)
    b = rng.integers(0, 2, (70, 90)).astype(np.bool_)
    np.testing.assert_array_equal(to_host(ops.transpose(to_dev(b, cuda))), b.T)
