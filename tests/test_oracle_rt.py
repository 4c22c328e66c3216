"""Pin the oracle's restatement of the reference's C runtime helpers
(remora/remora_rt.c: sort, grade, filter, replicate, rotate, append).

Two anchors: the golden fixture made by tests/golden/make_golden.py from the
reference interpreter (remora/runtime.py:1135-1189, including the known
answers of the reference's tests/test_properties.py:450-500), and remora_rt.c
itself, compiled from the reference tree into oracle/_ref/ by oracle/Makefile
(those cases are skipped where the reference tree is absent)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden

OP_GT = 8


@pytest.fixture(scope="module")
def g():
    return golden("rt_helpers")


def test_known_answers(oracle_mod, g):
    o = oracle_mod
    np.testing.assert_array_equal(o.sort(np.array([3, 1, 4, 1], np.int32)), g["ka_sort"])
    np.testing.assert_array_equal(o.grade(np.array([3, 1, 4, 1], np.int32)), g["ka_grade"])
    np.testing.assert_array_equal(o.filter_(np.array([1, -2, 3, -4], np.int32), pred=(OP_GT, 0)), g["ka_filter"])
    assert o.filter_(np.array([-1, -2, -3], np.int32), pred=(OP_GT, 0)).size == g["ka_filter_none"].size == 0
    np.testing.assert_array_equal(o.replicate(np.array([10, 20, 30], np.int32), np.array([2, 1, 3])),
                                  g["ka_replicate"])
    np.testing.assert_array_equal(o.replicate(np.array([7, 8, 9], np.int32), np.array([0, 1, 0])),
                                  g["ka_replicate_zero"])
    np.testing.assert_array_equal(o.rotate(np.arange(1, 6, dtype=np.int32), 2), g["ka_rotate"])
    np.testing.assert_array_equal(o.rotate(np.arange(1, 7, dtype=np.int32).reshape(3, 2), 1), g["ka_rotate2"])
    np.testing.assert_array_equal(o.append(np.array([[1, 2], [3, 4]], np.int32), np.array([[5, 6], [7, 8]], np.int32)),
                                  g["ka_append"])


def test_seeded_cases_match_interpreter(oracle_mod, g):
    o = oracle_mod
    f, i, m, c = g["f"], g["i"], g["m"], g["c"]
    np.testing.assert_array_equal(o.sort(f), g["sort_f"])
    np.testing.assert_array_equal(o.grade(f), g["grade_f"])
    np.testing.assert_array_equal(o.sort(i), g["sort_i"])
    np.testing.assert_array_equal(o.grade(i), g["grade_i"])
    np.testing.assert_array_equal(o.sort(m), g["sort_m"])
    np.testing.assert_array_equal(o.grade(m), g["grade_m"])
    np.testing.assert_array_equal(o.filter_(f, pred=(OP_GT, 0.25)), g["filter_f"])
    np.testing.assert_array_equal(o.filter_(i, pred=(OP_GT, 3)), g["filter_i"])
    np.testing.assert_array_equal(o.replicate(f, c), g["replicate_f"])
    np.testing.assert_array_equal(o.rotate(f, 37), g["rotate_f"])
    np.testing.assert_array_equal(o.rotate(m, 4), g["rotate_m"])
    np.testing.assert_array_equal(o.append(f, f[:41]), g["append_f"])


ref = pytest.mark.skipif("not __import__('oracle').ref_available()",
                         reason="remora_rt.c is compiled only where the reference tree is present")


@ref
@pytest.mark.parametrize("n", [0, 1, 2, 17, 1000, 65537])
def test_oracle_matches_remora_rt(oracle_mod, n):
    o = oracle_mod
    rng = np.random.default_rng(n + 11)
    f = rng.standard_normal(n).astype(np.float32)
    i = rng.integers(-50, 50, n).astype(np.int32)
    # sort: value-equal to qsort (qsort is not stable; values cannot tell)
    np.testing.assert_array_equal(o.sort(f), o.ref_sort(f))
    np.testing.assert_array_equal(o.sort(i), o.ref_sort(i))
    # grade: ties broken by index in both
    np.testing.assert_array_equal(o.grade(f), o.ref_grade(f))
    np.testing.assert_array_equal(o.grade(i), o.ref_grade(i))
    mask = (rng.random(n) < 0.4).astype(np.int32) * rng.integers(1, 5, n).astype(np.int32)
    np.testing.assert_array_equal(o.filter_(f, mask), o.ref_filter(f, mask))
    np.testing.assert_array_equal(o.filter_(i, mask), o.ref_filter(i, mask))
    counts = rng.integers(0, 4, n).astype(np.int32)
    total, rep = o.ref_replicate(f, counts)
    assert total == rep.size
    np.testing.assert_array_equal(o.replicate(f, counts), rep)
    if n:
        for k in (0, 1, n - 1, n, 3 * n + 2, -1, -n - 5):
            np.testing.assert_array_equal(o.rotate(f, k), o.ref_rotate(f, k))
    np.testing.assert_array_equal(o.append(i, i[: n // 3]), o.ref_append(i, i[: n // 3]))


@ref
def test_negative_counts_and_signed_zero(oracle_mod):
    """Deviations the restatement documents: a negative count repeats nothing
    (remora_rt.c's fill loop) although remora_replicate_*_count adds it into
    its total; -0.0 and +0.0 are equal for grade (index order wins)."""
    o = oracle_mod
    src = np.array([1.0, 2.0, 3.0], np.float32)
    counts = np.array([2, -1, 1], np.int32)
    total, rep = o.ref_replicate(src, counts)
    assert total == 2 and rep.size == 3
    np.testing.assert_array_equal(o.replicate(src, counts), rep)
    z = np.array([0.0, -0.0, 0.0, -0.0], np.float32)
    np.testing.assert_array_equal(o.grade(z), o.ref_grade(z))
    np.testing.assert_array_equal(o.grade(z), [0, 1, 2, 3])
