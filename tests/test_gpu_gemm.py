"""GPU parity of the tcgen05 dense core (matmul as the lifted dot).

Every result is checked against the oracle's sequential-k f32 lifted dot at
the TF32 GEMM tolerance (rtol 1e-3 + atol 1e-3 * max|ref|).
3xTF32 is also held to the exact (f64) product at rtol 1e-5 + atol
1e-4 * max|ref| (measured worst case 3.1e-5 * max|ref| at K = 4096, from the
tensor core's f32 accumulation): ten times inside the TF32 bound."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden, to_dev, to_host
from remora_b200 import ops

pytestmark = pytest.mark.gpu


def check(got, ref, precision, exact=None):
    ref = np.asarray(ref, dtype=np.float64)
    scale = max(1.0, float(np.abs(ref).max()) if ref.size else 1.0)
    np.testing.assert_allclose(got, ref, rtol=1e-3, atol=1e-3 * scale)
    if precision == "3xtf32" and exact is not None:
        np.testing.assert_allclose(got, exact, rtol=1e-5, atol=1e-4 * scale)


def exact(a, b):
    return np.matmul(a.astype(np.float64), b.astype(np.float64))


def test_golden_lifted_matmul(cuda):
    g = golden("lifted_matmul")
    a, bt = to_dev(g["a"], cuda), to_dev(g["bt"], cuda)
    for prec in ("3xtf32", "tf32"):
        check(to_host(ops.gemm(a, bt.t(), precision=prec)), g["out"], prec,
              exact(g["a"], np.ascontiguousarray(g["bt"].T)))


@pytest.mark.parametrize("mnk", [(128, 256, 32), (128, 256, 256), (256, 512, 128), (100, 200, 40), (129, 257, 36),
                                 (300, 130, 500), (64, 64, 6), (5, 3, 1), (1, 1000, 64),
                                 (1000, 300, 3000), (512, 64, 8192), (64, 2048, 1024), (300, 40, 2000)])
@pytest.mark.parametrize("prec", ["3xtf32", "tf32"])
def test_gemm_shapes(cuda, oracle_mod, mnk, prec):
    M, N, K = mnk
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    got = to_host(ops.gemm(to_dev(a, cuda), to_dev(b, cuda), precision=prec))
    check(got, oracle_mod.matmul(a, b), prec, exact(a, b))


@pytest.mark.parametrize("layout", ["kk", "km", "mk", "mm"])
def test_gemm_operand_majors(cuda, oracle_mod, layout):
    """A K-major (rows of A contiguous) or M-major (A^T stored), B K-major (the
    reference's Bt rows) or N-major (B rows contiguous)."""
    M, N, K = 256, 512, 160
    rng = np.random.default_rng(42)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    ta = to_dev(a, cuda) if layout[0] == "k" else to_dev(a.T.copy(), cuda).t()
    tb = to_dev(b.T.copy(), cuda).t() if layout[1] == "k" else to_dev(b, cuda)
    got = to_host(ops.gemm(ta, tb, precision="3xtf32"))
    check(got, oracle_mod.matmul(a, b), "3xtf32", exact(a, b))


def test_gemm_batched_and_views(cuda, oracle_mod):
    rng = np.random.default_rng(7)
    a = rng.uniform(-1, 1, (3, 130, 68)).astype(np.float32)
    b = rng.uniform(-1, 1, (3, 68, 260)).astype(np.float32)
    for prec in ("3xtf32", "tf32"):
        check(to_host(ops.gemm(to_dev(a, cuda), to_dev(b, cuda), precision=prec)), oracle_mod.matmul(a, b), prec,
              exact(a, b))
    # strided sub-views and an output view with a row stride
    import torch

    big = to_dev(rng.uniform(-1, 1, (300, 300)).astype(np.float32), cuda)
    av, bv = big[10:138, 4:100], big[100:196, 20:276]
    out = torch.zeros((200, 400), dtype=torch.float32, device=cuda)
    ops.gemm(av, bv, precision="3xtf32", out=out[3:131, 7:263])
    ha, hb = to_host(av).copy(), to_host(bv).copy()
    check(to_host(out[3:131, 7:263]), oracle_mod.matmul(ha, hb), "3xtf32", exact(ha, hb))
    assert float(out[:3].abs().sum()) == 0.0 and float(out[:, :7].abs().sum()) == 0.0


@pytest.mark.parametrize("mnk", [(8192, 64, 512), (300, 70, 96), (130, 260, 68)])
@pytest.mark.parametrize("prec", ["3xtf32", "tf32"])
def test_gemm_output_any_strides(cuda, oracle_mod, mnk, prec):
    """C given as a column-major view (the transpose of a row-major array,
    as the CNN writes its dense layer's weight gradient), as a view with both
    strides above 1, and with a zero K: the same values as a row-major C."""
    import torch

    M, N, K = mnk
    rng = np.random.default_rng(M + N + K)
    a = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    b = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    ref, ex = oracle_mod.matmul(a, b), exact(a, b)
    ct = torch.full((N, M), 5.0, dtype=torch.float32, device=cuda)
    ops.gemm(to_dev(a, cuda), to_dev(b, cuda), precision=prec, out=ct.t())
    check(to_host(ct).T, ref, prec, ex)
    big = torch.full((2 * M + 1, 3 * N + 2), 5.0, dtype=torch.float32, device=cuda)
    view = big[1::2, 2::3]
    ops.gemm(to_dev(a, cuda), to_dev(b, cuda), precision=prec, out=view)
    check(to_host(view), ref, prec, ex)
    assert float((big[0::2] - 5.0).abs().sum()) == 0.0  # rows between the view's rows untouched
    z = torch.full((N, M), 5.0, dtype=torch.float32, device=cuda)
    ops.gemm(to_dev(a[:, :0], cuda), to_dev(b[:0], cuda), precision=prec, out=z.t())
    assert float(z.abs().sum()) == 0.0


def test_gemm_k_zero(cuda):
    import torch

    a = torch.zeros((4, 0), device=cuda)
    b = torch.zeros((0, 5), device=cuda)
    out = torch.full((4, 5), 7.0, device=cuda)
    ops.gemm(a, b, out=out)
    assert float(out.abs().sum()) == 0.0


@pytest.mark.parametrize("prec", ["3xtf32", "tf32"])
def test_gemm_4096_sampled_rows(cuda, oracle_mod, prec):
    """The dense-core workload A,B f32[4096,4096] ~ U[-1,1]: every output
    row is computed on the device; 48 sampled rows are checked against the
    oracle's sequential lifted dot."""
    ra = np.random.Generator(np.random.PCG64(1729))
    rb = np.random.Generator(np.random.PCG64(1730))
    a = ra.uniform(-1, 1, (4096, 4096)).astype(np.float32)
    b = rb.uniform(-1, 1, (4096, 4096)).astype(np.float32)
    got = to_host(ops.gemm(to_dev(a, cuda), to_dev(b, cuda), precision=prec))
    rows = np.random.default_rng(0).choice(4096, 48, replace=False)
    ref = oracle_mod.matmul(a[rows], b, nthreads=oracle_mod.max_threads())
    check(got[rows], ref, prec, exact(a[rows], b))
    assert np.isfinite(got).all()


def test_gemm_batched_full_sampled(cuda, oracle_mod):
    """The batched workload [32,1024,1024] x [32,1024,1024] (3xTF32)."""
    ra = np.random.Generator(np.random.PCG64(1729))
    a = ra.uniform(-1, 1, (32, 1024, 1024)).astype(np.float32)
    b = ra.uniform(-1, 1, (32, 1024, 1024)).astype(np.float32)
    got = to_host(ops.gemm(to_dev(a, cuda), to_dev(b, cuda), precision="3xtf32"))
    for bi in (0, 17, 31):
        rows = np.arange(bi * 13 % 1000, bi * 13 % 1000 + 24)
        check(got[bi, rows], oracle_mod.matmul(a[bi, rows], b[bi], nthreads=oracle_mod.max_threads()), "3xtf32",
              exact(a[bi, rows], b[bi]))


@pytest.mark.parametrize("shape", [(1, 2600, 2000, 520), (5, 1100, 900, 600), (1, 4096, 4096, 4096)])
@pytest.mark.parametrize("prec", ["3xtf32", "tf32"])
def test_gemm_split_last_wave_whole_output(cuda, shape, prec):
    """Launches of more tiles than SMs whose last wave is at most half full
    split those last tiles along K (partials added in split order by the
    fix-up kernel).  Every element, edge tiles and the split tiles included,
    is checked against the exact f64 product."""
    import torch

    batch, M, N, K = shape
    g = torch.Generator(device=cuda)
    g.manual_seed(M + N + K)
    a = torch.rand((batch, M, K), generator=g, device=cuda) * 2 - 1
    b = torch.rand((batch, K, N), generator=g, device=cuda) * 2 - 1
    if batch == 1:
        a, b = a[0], b[0]
    got = ops.gemm(a, b, precision=prec)
    ref = torch.matmul(a.double(), b.double())
    scale = max(1.0, float(ref.abs().max()))
    err = float((got.double() - ref).abs().max()) / scale
    assert err <= (1e-3 if prec == "tf32" else 1e-4), err
    ops.synchronize(cuda.index)
