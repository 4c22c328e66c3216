"""GPU parity of the reference's C runtime helpers (remora/remora_rt.c) on
the device: sort, grade, filter, replicate, rotate, append.  All are integer
/ index / data-movement work and are checked bit-exact against the oracle
(itself pinned to remora_rt.c and to the reference interpreter by
tests/test_oracle_rt.py), with one documented exception: for f32 sort, -0.0
and +0.0 compare equal in the reference, whose qsort leaves their order open;
here -0.0 is placed first, so sorts containing both are compared by value."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, to_dev, to_host
from remora_b200 import ops
from remora_b200.errors import RemoraB200Error, RemoraShapeError, RemoraUnsupportedError

pytestmark = pytest.mark.gpu

OP_LT, OP_LE, OP_GT, OP_GE, OP_EQ, OP_NE = range(6, 12)
CMP = {"<": OP_LT, "<=": OP_LE, ">": OP_GT, ">=": OP_GE, "==": OP_EQ, "!=": OP_NE}


def bits_equal(a: np.ndarray, b: np.ndarray) -> None:
    assert a.shape == b.shape and a.dtype == b.dtype
    np.testing.assert_array_equal(a.view(np.uint32), b.view(np.uint32))


def test_golden_runtime_helpers(cuda):
    g = golden("rt_helpers")
    d = lambda a: to_dev(a, cuda)  # noqa: E731
    np.testing.assert_array_equal(to_host(ops.sort(d(np.array([3, 1, 4, 1], np.int32)))), g["ka_sort"])
    np.testing.assert_array_equal(to_host(ops.grade(d(np.array([3, 1, 4, 1], np.int32)))), g["ka_grade"])
    np.testing.assert_array_equal(to_host(ops.filter(d(np.array([1, -2, 3, -4], np.int32)), pred=(">", 0))),
                                  g["ka_filter"])
    assert ops.filter(d(np.array([-1, -2, -3], np.int32)), pred=(">", 0)).numel() == 0
    np.testing.assert_array_equal(to_host(ops.replicate(d(np.array([10, 20, 30], np.int32)),
                                                        d(np.array([2, 1, 3], np.int32)))), g["ka_replicate"])
    np.testing.assert_array_equal(to_host(ops.replicate(d(np.array([7, 8, 9], np.int32)),
                                                        d(np.array([0, 1, 0], np.int32)))), g["ka_replicate_zero"])
    np.testing.assert_array_equal(to_host(ops.rotate(d(np.arange(1, 6, dtype=np.int32)), 2)), g["ka_rotate"])
    np.testing.assert_array_equal(to_host(ops.rotate(d(np.arange(1, 7, dtype=np.int32).reshape(3, 2)), 1)),
                                  g["ka_rotate2"])
    np.testing.assert_array_equal(to_host(ops.append(d(np.array([[1, 2], [3, 4]], np.int32)),
                                                     d(np.array([[5, 6], [7, 8]], np.int32)))), g["ka_append"])
    f, i, m, c = g["f"], g["i"], g["m"], g["c"]
    bits_equal(to_host(ops.sort(d(f))), g["sort_f"])
    np.testing.assert_array_equal(to_host(ops.grade(d(f))), g["grade_f"])
    np.testing.assert_array_equal(to_host(ops.sort(d(i))), g["sort_i"])
    np.testing.assert_array_equal(to_host(ops.grade(d(i))), g["grade_i"])
    np.testing.assert_array_equal(to_host(ops.sort(d(m))), g["sort_m"])
    np.testing.assert_array_equal(to_host(ops.grade(d(m))), g["grade_m"])
    bits_equal(to_host(ops.filter(d(f), pred=(">", 0.25))), g["filter_f"])
    np.testing.assert_array_equal(to_host(ops.filter(d(i), pred=(">", 3))), g["filter_i"])
    bits_equal(to_host(ops.replicate(d(f), d(c))), g["replicate_f"])
    bits_equal(to_host(ops.rotate(d(f), 37)), g["rotate_f"])
    np.testing.assert_array_equal(to_host(ops.rotate(d(m), 4)), g["rotate_m"])
    bits_equal(to_host(ops.append(d(f), d(f[:41]))), g["append_f"])


SIZES = [0, 1, 5, 256, 257, 1000, 1024, 1025, 4096, 4097, 12345, 1 << 20, (1 << 22) + 3]


@pytest.mark.parametrize("n", SIZES)
def test_sort_grade_rank1(cuda, oracle_mod, n):
    rng = np.random.default_rng(n + 3)
    f = rng.standard_normal(n).astype(np.float32)
    if n > 10:
        f[::5] = f[7]  # repeated values
    wide = rng.integers(np.iinfo(np.int32).min, np.iinfo(np.int32).max, n, dtype=np.int64).astype(np.int32)
    if n >= 2:
        wide[0], wide[-1] = np.iinfo(np.int32).min, np.iinfo(np.int32).max
    ties = rng.integers(-3, 3, n).astype(np.int32)
    for x in (f, wide, ties):
        xd = to_dev(x, cuda)
        bits_equal(to_host(ops.sort(xd)), oracle_mod.sort(x))
        np.testing.assert_array_equal(to_host(ops.grade(xd)), oracle_mod.grade(x))


@pytest.mark.parametrize("shape", [(1, 1), (7, 300), (64, 1024), (33, 4096), (3, 5000), (0, 5), (4, 0), (2, 70000)])
def test_sort_grade_rows(cuda, oracle_mod, shape):
    rng = np.random.default_rng(sum(shape))
    f = rng.uniform(-4, 4, shape).astype(np.float32)
    i = rng.integers(-40, 40, shape).astype(np.int32)
    for x in (f, i):
        xd = to_dev(x, cuda)
        bits_equal(to_host(ops.sort(xd)), oracle_mod.sort(x))
        np.testing.assert_array_equal(to_host(ops.grade(xd)), oracle_mod.grade(x))


@pytest.mark.parametrize("n", [9, 6000])
def test_sort_special_floats_views_and_in_place(cuda, oracle_mod, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    x[::3] = 0.0
    x[1::3] = -0.0
    x[2] = np.inf
    x[4] = -np.inf
    xd = to_dev(x, cuda)
    got = to_host(ops.sort(xd))
    np.testing.assert_array_equal(got, oracle_mod.sort(x))  # by value: -0.0 == +0.0
    zeros = got[got == 0]
    assert np.all(np.signbit(zeros[: np.count_nonzero(np.signbit(x) & (x == 0))]))  # -0.0 first
    # grade treats -0.0 and +0.0 as equal: index order, exactly like the reference
    np.testing.assert_array_equal(to_host(ops.grade(xd)), oracle_mod.grade(x))
    # a strided view and an in-place sort
    view = xd[::2]
    np.testing.assert_array_equal(to_host(ops.sort(view)), oracle_mod.sort(x[::2]))
    y = to_dev(x, cuda)
    ops.sort(y, out=y)
    np.testing.assert_array_equal(to_host(y), oracle_mod.sort(x))
    with pytest.raises(RemoraShapeError):
        ops.sort(to_dev(x.reshape(-1, 3)[:, :, None].copy(), cuda))


@pytest.mark.parametrize("n", [0, 1, 4095, 4096, 4097, 100001, (1 << 20) + 11])
def test_filter(cuda, oracle_mod, n):
    rng = np.random.default_rng(n + 5)
    f = rng.standard_normal(n).astype(np.float32)
    i = rng.integers(-10, 10, n).astype(np.int32)
    mask = (rng.random(n) < 0.37).astype(np.int32) * rng.integers(-3, 4, n).astype(np.int32)
    for x in (f, i):
        xd = to_dev(x, cuda)
        bits_equal(to_host(ops.filter(xd, to_dev(mask, cuda))), oracle_mod.filter_(x, mask))
        bits_equal(to_host(ops.filter(xd, to_dev(mask != 0, cuda))), oracle_mod.filter_(x, mask != 0))
        for op in CMP:
            lit = 0.3 if x.dtype == np.float32 else 2
            bits_equal(to_host(ops.filter(xd, pred=(op, lit))), oracle_mod.filter_(x, pred=(CMP[op], lit)))


def test_filter_nan_capacity_and_async_count(cuda, oracle_mod):
    x = np.array([1.0, np.nan, -2.0, 3.0, np.nan, 0.5], np.float32)
    xd = to_dev(x, cuda)
    for op in CMP:  # ordered comparisons: NaN never passes, "!=" included
        bits_equal(to_host(ops.filter(xd, pred=(op, 0.5))), oracle_mod.filter_(x, pred=(CMP[op], 0.5)))
    import torch

    out = torch.full((2,), -1.0, device=cuda)
    got, count = ops.filter(xd, pred=(">", 0.0), out=out, sync=False)
    assert int(count.item()) == 3  # counted in full, written up to the capacity
    np.testing.assert_array_equal(to_host(got), [1.0, 3.0])
    with pytest.raises(RemoraB200Error):
        ops.filter(xd)


@pytest.mark.parametrize("n", [0, 1, 4096, 4097, 50000, 1 << 20])
def test_replicate(cuda, oracle_mod, n):
    rng = np.random.default_rng(n + 9)
    f = rng.standard_normal(n).astype(np.float32)
    i = rng.integers(-1000, 1000, n).astype(np.int32)
    counts = rng.integers(-1, 4, n).astype(np.int32)
    for x in (f, i):
        bits_equal(to_host(ops.replicate(to_dev(x, cuda), to_dev(counts, cuda))), oracle_mod.replicate(x, counts))


def test_replicate_skewed_sparse_and_capacity(cuda, oracle_mod):
    import torch

    rng = np.random.default_rng(77)
    n = 30000
    x = rng.integers(0, 1 << 30, n).astype(np.int32)
    skew = np.zeros(n, np.int32)
    skew[[3, 17, 29999]] = [100000, 1, 70000]  # long runs of zero counts between
    np.testing.assert_array_equal(to_host(ops.replicate(to_dev(x, cuda), to_dev(skew, cuda))),
                                  oracle_mod.replicate(x, skew))
    dense = rng.integers(0, 3, n).astype(np.int32)
    ref = oracle_mod.replicate(x, dense)
    out = torch.zeros(ref.size // 2, dtype=torch.int32, device=cuda)
    got, total = ops.replicate(to_dev(x, cuda), to_dev(dense, cuda), out=out, sync=False)
    assert int(total.item()) == ref.size
    np.testing.assert_array_equal(to_host(got), ref[: ref.size // 2])
    assert ops.replicate(to_dev(x, cuda), to_dev(np.zeros(n, np.int32), cuda)).numel() == 0


@pytest.mark.parametrize("shape", [(1,), (7,), (1000,), (12, 5), (64, 3, 7), (9, 0)])
@pytest.mark.parametrize("shift", [0, 1, -1, 4, 1003, -77])
def test_rotate(cuda, oracle_mod, shape, shift):
    rng = np.random.default_rng(len(shape) * 31 + shift % 97)
    for x in (rng.standard_normal(shape).astype(np.float32), rng.integers(-9, 9, shape).astype(np.int32),
              rng.random(shape) < 0.5):
        got = to_host(ops.rotate(to_dev(x, cuda), shift))
        np.testing.assert_array_equal(got, oracle_mod.rotate(x, shift))


def test_rotate_and_append_views(cuda, oracle_mod):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((40, 6)).astype(np.float32)
    xd = to_dev(x, cuda)
    np.testing.assert_array_equal(to_host(ops.rotate(xd[:, ::2], 3)), oracle_mod.rotate(x[:, ::2], 3))
    np.testing.assert_array_equal(to_host(ops.append(xd[::3], xd[1:5])), oracle_mod.append(x[::3], x[1:5]))
    with pytest.raises(RemoraShapeError):
        ops.append(xd, to_dev(np.zeros((2, 5), np.float32), cuda))


@pytest.mark.parametrize("na,nb", [(0, 0), (0, 5), (5, 0), (1, 1), (1000, 4097), (3, 1 << 20)])
def test_append(cuda, oracle_mod, na, nb):
    rng = np.random.default_rng(na + nb)
    for dt in (np.float32, np.int32, np.bool_):
        a = (rng.standard_normal(na) * 100).astype(dt)
        b = (rng.standard_normal(nb) * 100).astype(dt)
        np.testing.assert_array_equal(to_host(ops.append(to_dev(a, cuda), to_dev(b, cuda))), oracle_mod.append(a, b))
    a3 = rng.standard_normal((na % 7, 3, 2)).astype(np.float32)
    b3 = rng.standard_normal((nb % 5, 3, 2)).astype(np.float32)
    np.testing.assert_array_equal(to_host(ops.append(to_dev(a3, cuda), to_dev(b3, cuda))), oracle_mod.append(a3, b3))


def test_large_sort_properties(cuda):
    """At 2^25 keys: the output is non-decreasing, the grade is a permutation
    that reproduces it, and grade is stable on a small key range."""
    import torch

    n = 1 << 25
    g = torch.Generator(device=cuda).manual_seed(3)
    x = torch.randn(n, device=cuda, generator=g)
    s = ops.sort(x)
    assert bool((s[1:] >= s[:-1]).all())
    idx = ops.grade(x)
    assert torch.equal(x[idx.long()], s)
    assert torch.equal(torch.sort(idx)[0], torch.arange(n, device=cuda, dtype=torch.int32))
    t = torch.randint(0, 16, (n,), device=cuda, dtype=torch.int32, generator=g)
    gi = ops.grade(t).long()
    st = t[gi]
    assert bool((st[1:] >= st[:-1]).all())
    same = st[1:] == st[:-1]
    assert bool((gi[1:][same] > gi[:-1][same]).all())
    with pytest.raises(RemoraUnsupportedError):
        ops.sort(torch.zeros(4, dtype=torch.bool, device=cuda))
