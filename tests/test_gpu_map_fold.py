"""GPU parity of lifted maps and folds against the oracle and the reference's
golden outputs.  Maps are bit-exact with the oracle (f32 ops rounded one by
one, no FMA contraction); f32 folds reassociate the sum, so they are checked
at rtol 1e-5 plus atol 1e-6 * max|ref|; i32 folds are bit-exact."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, to_dev, to_host
from remora_b200 import ops
from remora_b200.codegen import fold_spec
from remora_b200.program import (BinaryExpr, CmpExpr, LogicExpr, SelectExpr, UnaryExpr, compile_program, const,
                                 stable_bce, x)

pytestmark = pytest.mark.gpu

Y = BinaryExpr("+", BinaryExpr("*", x(0), const(2.5)), const(1.0))
CHAIN = SelectExpr(CmpExpr(">", Y, const(0.5)), Y, const(0.0))
SQ = BinaryExpr("*", x(0), x(0))
RTOL = 1e-5


def close(got, ref, rtol=RTOL):
    ref = np.asarray(ref, dtype=np.float64)
    atol = 1e-6 * max(1.0, float(np.abs(ref).max()) if ref.size else 1.0)
    np.testing.assert_allclose(np.asarray(got, dtype=np.float64), ref, rtol=rtol, atol=atol)


# ------------------------------------------------------------------ maps
def test_golden_maps(cuda, oracle_mod):
    g = golden("chain_map")
    out = to_host(ops.map(CHAIN, to_dev(g["x"], cuda)))
    np.testing.assert_array_equal(out, oracle_mod.run_map(compile_program(CHAIN, 1), [g["x"]], g["x"].shape,
                                                          np.float32))
    np.testing.assert_allclose(out, g["out"], rtol=2.5e-7, atol=0)
    g = golden("broadcast_add")
    out = to_host(ops.map(BinaryExpr("+", x(0), x(1)), to_dev(g["p"], cuda), to_dev(g["q"], cuda)))
    np.testing.assert_array_equal(out, g["out"])
    g = golden("i32_div")
    out = to_host(ops.map(BinaryExpr("/", x(0), x(1)), to_dev(g["a"], cuda), to_dev(g["b"], cuda), compute="f32",
                          out_dtype="f32"))
    np.testing.assert_array_equal(out, g["out"])
    g = golden("i32_add2")
    np.testing.assert_array_equal(to_host(ops.map(BinaryExpr("+", x(0), const(2)), to_dev(g["a"], cuda))), g["out"])
    g = golden("bool_and")
    out = to_host(ops.map(LogicExpr("&&", x(0), x(1)), to_dev(g["a"], cuda), to_dev(g["b"], cuda)))
    np.testing.assert_array_equal(out, g["out"])
    g = golden("f32_gt_mask")
    out = to_host(ops.map(CmpExpr(">", x(0), const(0.25)), to_dev(g["a"], cuda), out_dtype="bool"))
    np.testing.assert_array_equal(out, g["out"])


def test_known_answers(cuda):
    """The reference's GPU round-trips (tests/test_executor.py:434-770)."""
    a = to_dev(np.array([1, 2, 3, 4], np.float32), cuda)
    b = to_dev(np.array([10, 20, 30, 40], np.float32), cuda)
    np.testing.assert_array_equal(to_host(ops.map(BinaryExpr("*", x(0), const(2.0)), a)), [2, 4, 6, 8])
    np.testing.assert_array_equal(to_host(ops.map(BinaryExpr("+", x(0), x(1)), a, b)), [11, 22, 33, 44])
    assert float(to_host(ops.fold(a, mode="all"))) == 10.0
    assert float(to_host(ops.fold(a, b, mode="all", premap=BinaryExpr("*", x(0), x(1))))) == 300.0
    ai = to_dev(np.array([1, 2, 3, 4], np.int32), cuda)
    np.testing.assert_array_equal(to_host(ops.map(BinaryExpr("+", x(0), const(2)), ai)), [3, 4, 5, 6])
    assert float(to_host(ops.fold(to_dev(np.arange(10, dtype=np.float32), cuda), mode="all"))) == 45.0
    assert int(to_host(ops.fold(to_dev(np.arange(10, dtype=np.int32), cuda), mode="all"))) == 45


@pytest.mark.parametrize("shape", [(1,), (3,), (1027,), (64, 64, 64, 64), (5, 7, 9), (2, 3, 4, 5, 6, 1, 2, 2, 1, 3)])
def test_map_bit_exact_vs_oracle(cuda, oracle_mod, shape):
    rng = np.random.default_rng(7)
    xs = rng.standard_normal(shape).astype(np.float32)
    prog = compile_program(CHAIN, 1)
    out = to_host(ops.map(prog, to_dev(xs, cuda)))
    ref = oracle_mod.run_map(prog, [xs], shape, np.float32, nthreads=oracle_mod.max_threads())
    np.testing.assert_array_equal(out, ref)


def test_map_views_offsets_negative_strides(cuda, oracle_mod):
    import torch

    rng = np.random.default_rng(8)
    base = rng.standard_normal((40, 50)).astype(np.float32)
    tb = to_dev(base, cuda)
    views = [tb[3:, 5:45], tb.t(), torch.flip(tb, dims=[1])[:, 1:], tb[::3, ::2]]
    nviews = [base[3:, 5:45], base.T, base[:, ::-1][:, 1:], base[::3, ::2]]
    prog = compile_program(BinaryExpr("-", CHAIN, UnaryExpr("neg", x(0))), 1)
    for tv, nv in zip(views, nviews):
        if tv.stride(-1) < 0:
            continue  # torch has no negative strides; covered by the descriptor below
        out = to_host(ops.map(prog, tv))
        np.testing.assert_array_equal(out, oracle_mod.run_map(prog, [np.ascontiguousarray(nv)], nv.shape,
                                                              np.float32))
    # negative stride through a hand-made descriptor: reverse the columns
    import ctypes
    from remora_b200 import _lib as L
    from remora_b200.abi import make_memref_descriptor, tensor_descriptor
    from remora_b200.runtime import context

    out = torch.empty((40, 50), dtype=torch.float32, device=cuda)
    ind = make_memref_descriptor(tb.data_ptr(), (40, 50), (50, -1), None, 49)
    od = tensor_descriptor(out)
    ptrs = (ctypes.c_void_p * 1)(ctypes.addressof(ind))
    ranks = (ctypes.c_int32 * 1)(2)
    L.check(L.lib().remora_b200_map(context(0).ptr, ctypes.byref(prog), ptrs, ranks, 1, ctypes.addressof(od), 2,
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    np.testing.assert_array_equal(to_host(out), oracle_mod.run_map(prog, [np.ascontiguousarray(base[:, ::-1])],
                                                                   (40, 50), np.float32))


def test_map_prefix_broadcast_and_scalar(cuda, oracle_mod):
    rng = np.random.default_rng(9)
    a = rng.standard_normal((8, 6, 12)).astype(np.float32)
    b = rng.standard_normal((8, 6)).astype(np.float32)
    b1 = rng.standard_normal((8,)).astype(np.float32)
    s = np.array(1.75, dtype=np.float32)
    e = BinaryExpr("*", BinaryExpr("+", x(0), x(1)), BinaryExpr("-", x(2), x(3)))
    prog = compile_program(e, 4)
    out = to_host(ops.map(prog, *(to_dev(v, cuda) for v in (a, b, b1, s))))
    ref = oracle_mod.run_map(prog, [a, b, b1, s], a.shape, np.float32)
    np.testing.assert_array_equal(out, ref)
    # odd broadcast divisor (not a multiple of 4) takes the general kernel
    a = rng.standard_normal((7, 5, 3)).astype(np.float32)
    b = rng.standard_normal((7, 5)).astype(np.float32)
    prog = compile_program(BinaryExpr("/", x(0), x(1)), 2)
    np.testing.assert_array_equal(to_host(ops.map(prog, to_dev(a, cuda), to_dev(b, cuda))),
                                  oracle_mod.run_map(prog, [a, b], a.shape, np.float32))


def test_map_empty_and_errors(cuda):
    import torch

    from remora_b200.errors import RemoraShapeError

    e = to_dev(np.zeros((0, 4), np.float32), cuda)
    assert ops.map(CHAIN, e).shape == (0, 4)
    with pytest.raises(RemoraShapeError):
        ops.map(BinaryExpr("+", x(0), x(1)), to_dev(np.zeros((3, 4), np.float32), cuda),
                to_dev(np.zeros((4,), np.float32), cuda))
    del torch


def test_exp_log_bce_within_ulps(cuda, oracle_mod):
    g = golden("bce")
    out = to_host(ops.map(stable_bce(x(0), x(1)), to_dev(g["z"], cuda), to_dev(g["y"], cuda)))
    np.testing.assert_allclose(out, g["loss"], rtol=1e-6, atol=6e-7)
    rng = np.random.default_rng(10)
    z = rng.standard_normal(100000).astype(np.float32) * 5
    y = (rng.random(100000) > 0.5).astype(np.float32)
    prog = compile_program(stable_bce(x(0), x(1)), 2)
    got = to_host(ops.map(prog, to_dev(z, cuda), to_dev(y, cuda)))
    # expf/logf are CUDA's (a couple of ulps from glibc's); log(1 + exp(-|z|))
    # inherits about one ulp of 1.0 in absolute terms
    np.testing.assert_allclose(got, oracle_mod.run_map(prog, [z, y], z.shape, np.float32), rtol=2e-6, atol=6e-7)


# ----------------------------------------------------------------- folds
def test_golden_folds(cuda):
    g = golden("chained_maps")
    close(to_host(ops.fold(to_dev(g["x"], cuda), premap=CHAIN)), g["out"])
    g = golden("row_sumsq")
    sums = to_host(ops.fold(to_dev(g["x"], cuda), premap=SQ))
    close(sums, g["out"])
    norms = to_host(ops.fold(to_dev(g["x"], cuda), premap=SQ, epilogue="sqrt"))
    np.testing.assert_array_equal(norms, np.sqrt(sums))
    g = golden("fold_f32_1000")
    close(to_host(ops.fold(to_dev(g["v"], cuda), mode="all")), g["out"])
    g = golden("fold_i32_777")
    assert int(to_host(ops.fold(to_dev(g["v"], cuda), mode="all"))) == int(g["out"])
    g = golden("dot_256")
    close(to_host(ops.fold(to_dev(g["a"], cuda), to_dev(g["b"], cuda), mode="all",
                           premap=BinaryExpr("*", x(0), x(1)))), g["out"])
    g = golden("lifted_matmul")  # the dot form through a cell fold: rows of A against one column
    a, bt = g["a"], g["bt"]
    for j in range(bt.shape[0]):
        col = np.ascontiguousarray(np.broadcast_to(bt[j], a.shape))
        close(to_host(ops.fold(to_dev(a, cuda), to_dev(col, cuda), premap=BinaryExpr("*", x(0), x(1)))),
              g["out"][:, j])


def test_row_norms_full_size(cuda, oracle_mod):
    """The row_norms workload: f32[8192, 1024] ~ U[-1,1] -> sqrt(sum x*x)."""
    rng = np.random.Generator(np.random.PCG64(1729))
    xs = rng.uniform(-1, 1, (8192, 1024)).astype(np.float32)
    out = to_host(ops.fold(to_dev(xs, cuda), premap=SQ, epilogue="sqrt"))
    ref = oracle_mod.cell_fold(fold_spec(premap=SQ, epilogue="sqrt"), [xs], 1, nthreads=oracle_mod.max_threads())
    close(out, ref)


def test_chained_maps_full_size(cuda, oracle_mod):
    """The chained-map workload: f32[64,64,64,64] ~ N(0,1)."""
    rng = np.random.Generator(np.random.PCG64(1729))
    xs = rng.standard_normal((64, 64, 64, 64)).astype(np.float32)
    out = to_host(ops.fold(to_dev(xs, cuda), premap=CHAIN))
    ref = oracle_mod.cell_fold(fold_spec(premap=CHAIN), [xs], 1, nthreads=oracle_mod.max_threads())
    close(out, ref)
    # masks: exactly the same elements survive the threshold on both sides
    y = to_host(ops.map(CHAIN, to_dev(xs, cuda)))
    yo = oracle_mod.run_map(compile_program(CHAIN, 1), [xs], xs.shape, np.float32, nthreads=oracle_mod.max_threads())
    np.testing.assert_array_equal(y, yo)


@pytest.mark.parametrize("L", [1, 3, 4, 5, 33, 64, 100, 1024, 4099])
def test_cell_fold_lengths(cuda, oracle_mod, L):
    rng = np.random.default_rng(L)
    xs = rng.uniform(0, 1, (37, L)).astype(np.float32)
    close(to_host(ops.fold(to_dev(xs, cuda), premap=SQ, init=0.5)),
          oracle_mod.cell_fold(fold_spec(premap=SQ, init=0.5), [xs], 1))
    xi = rng.integers(-1000, 1000, (37, L)).astype(np.int32)
    np.testing.assert_array_equal(to_host(ops.fold(to_dev(xi, cuda), init=7)),
                                  oracle_mod.cell_fold(fold_spec(dtype="i32", init=7), [xi], 1))


def test_fold_cell_rank2_and_views(cuda, oracle_mod):
    rng = np.random.default_rng(11)
    xs = rng.uniform(0, 1, (6, 7, 8, 9)).astype(np.float32)
    close(to_host(ops.fold(to_dev(xs, cuda), cell_rank=2)),
          oracle_mod.cell_fold(fold_spec(), [xs], 2))
    t = to_dev(xs, cuda).permute(1, 0, 3, 2)
    ref = oracle_mod.cell_fold(fold_spec(), [np.ascontiguousarray(xs.transpose(1, 0, 3, 2))], 1)
    close(to_host(ops.fold(t)), ref)


def test_whole_fold_sizes_deterministic(cuda):
    rng = np.random.default_rng(12)
    for n in (0, 1, 5, 4096, 1 << 20, (1 << 24) + 3):
        xs = rng.uniform(0, 1, n).astype(np.float32)
        d = to_dev(xs, cuda)
        r1 = float(to_host(ops.fold(d, mode="all", init=1.0)))
        r2 = float(to_host(ops.fold(d, mode="all", init=1.0)))
        assert r1 == r2  # fixed combine order: bitwise reproducible
        ref = 1.0 + float(np.sum(xs.astype(np.float64)))
        assert abs(r1 - ref) <= 1e-5 * abs(ref) + 1e-6
    xi = rng.integers(-2**31, 2**31 - 1, 3_000_001, dtype=np.int64).astype(np.int32)
    got = int(to_host(ops.fold(to_dev(xi, cuda), mode="all")))
    assert got == int(np.int64(xi.astype(np.int64).sum()).astype(np.int32))
    xm = rng.uniform(0.999, 1.001, 10000).astype(np.float32)
    got = float(to_host(ops.fold(to_dev(xm, cuda), mode="all", op="*", init=1.0)))
    # f32 products of values near 1 round with a bias (sequential f32 drifts
    # ~1e-4 from f64 here too)
    assert abs(got - np.prod(xm.astype(np.float64))) <= 2e-3


def test_array_fold_and_golden(cuda, oracle_mod):
    g = golden("array_fold")
    np.testing.assert_array_equal(to_host(ops.array_fold(to_dev(g["m"], cuda), to_dev(g["init"], cuda))),
                                  oracle_mod.array_fold(fold_spec(), g["m"], g["init"]))
    close(to_host(ops.array_fold(to_dev(g["m"], cuda), to_dev(g["init"], cuda))), g["out"])
    rng = np.random.default_rng(13)
    big = rng.uniform(-1, 1, (100000, 16)).astype(np.float32)
    init = np.zeros(16, np.float32)
    close(to_host(ops.array_fold(to_dev(big, cuda), to_dev(init, cuda))),
          big.astype(np.float64).sum(0), rtol=1e-4)


def test_whole_fold_after_other_scratch_users(cuda):
    """Calls that stage data through the shared per-stream scratch (a 3xTF32
    GEMM's split operands, a scan's carries) between whole-array folds must
    not disturb the fold's block ticket."""
    import torch

    rng = np.random.default_rng(21)
    xs = rng.uniform(0, 1, 1 << 20).astype(np.float32)
    d = to_dev(xs, cuda)
    ref = float(np.sum(xs.astype(np.float64)))
    a = torch.rand(300, 200, device=cuda)
    for _ in range(3):
        ops.gemm(a, a.t(), precision="3xtf32")
        ops.scan(d)
        got = float(to_host(ops.fold(d, mode="all")))
        assert abs(got - ref) <= 1e-5 * ref
        assert float(to_host(ops.fold(to_dev(np.arange(1, 5, dtype=np.float32), cuda), mode="all"))) == 10.0


@pytest.mark.parametrize("L,n_in", [(4, 1), (64, 1), (100, 1), (1020, 1), (1024, 1), (12, 2), (512, 2)])
def test_fold_rows_independent_of_launch_geometry(cuda, oracle_mod, L, n_in):
    """A row's total depends only on the row: a ~3 MiB fold (grid-stride
    launch, ragged last row block) equals the concatenation of the folds of
    its ~200 KiB row blocks (single-pass launches) bit for bit, and the
    oracle within the fold tolerance."""
    import torch

    rng = np.random.default_rng(L + 100 * n_in)
    rows = max(4096, ((3 << 20) // (4 * L * n_in)) | 1)  # ~3 MiB, odd row count: ragged last row block
    xs = [rng.standard_normal((rows, L)).astype(np.float32) for _ in range(n_in)]
    expr, kw = (CHAIN, {}) if n_in == 1 else (stable_bce(x(0), x(1)), {})
    if n_in == 2:
        xs[1] = (xs[1] > 0).astype(np.float32)
    dev = [to_dev(a, cuda) for a in xs]
    big = to_host(ops.fold(*dev, premap=expr, **kw))
    step = max(1, (200 << 10) // (4 * L * n_in))
    parts = [to_host(ops.fold(*[d[i:i + step] for d in dev], premap=expr, **kw)) for i in range(0, rows, step)]
    np.testing.assert_array_equal(big, np.concatenate(parts))
    ref = oracle_mod.cell_fold(fold_spec(premap=expr, n_inputs=n_in), xs, 1, nthreads=oracle_mod.max_threads())
    close(big, ref)
    # i32 (exact) through the same path
    if n_in == 1:
        xi = rng.integers(-1000, 1000, (rows, L)).astype(np.int32)
        np.testing.assert_array_equal(to_host(ops.fold(to_dev(xi, cuda), init=3)),
                                      oracle_mod.cell_fold(fold_spec(dtype="i32", init=3), [xi], 1))
    torch.cuda.synchronize()
