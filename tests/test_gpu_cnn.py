"""GPU parity of the crater-CNN training step against the oracle's step
(oracle/oracle.c:oracle_cnn_step) on the same seeded images and parameters.

3xTF32 mode (split-precision tensor-core GEMMs and convs; the default) is
held to 1e-4 on the loss and rtol 1e-4 + atol 1e-4 * max|ref| per gradient
tensor, inside the 1e-3 gradient tolerance (measured: 1.1e-5 on the loss).  Plain TF32 (10-bit mantissa operands in conv2 and
the dense GEMMs) does not meet 1e-3 on every tensor: the first layer's weight
gradient, a sum over every pixel of the batch with heavy cancellation, comes
out at ~3e-2 * max|ref| (measured on B200).  Its test pins the loss at 1e-3
and every gradient at 5e-2 * max|ref|, the bound of that mode."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import to_host
from remora_b200 import crater

pytestmark = pytest.mark.gpu


def _run(cuda, oracle_mod, batch, precision, steps=1):
    import torch

    from remora_b200.cnn import CraterCNN

    params = crater.init_params()
    imgs, labels = crater.make_batch(batch)
    net = CraterCNN(cuda, batch, lr=0.01, params=params, precision=precision)
    xi, yi = torch.from_numpy(imgs).to(cuda), torch.from_numpy(labels).to(cuda)
    ref_params = params.copy()
    for _ in range(steps):
        net.forward_backward(xi, yi)
        grads = to_host(net.grads).copy()
        loss = net.loss()
        net.update()
        ref_loss, ref_grads = oracle_mod.cnn_step(ref_params, imgs, labels, lr=0.01,
                                                  nthreads=oracle_mod.max_threads())
    return loss, grads, to_host(net.params), ref_loss, ref_grads, ref_params


def _compare_from(grads, ref, tol, start):
    """_compare over the tensors that start at or after flat index `start`."""
    for name, (a, b, _) in crater.offsets().items():
        if a < start:
            continue
        r = ref[a:b].astype(np.float64)
        scale = max(float(np.abs(r).max()), 1e-12)
        err = float(np.abs(grads[a:b] - r).max()) / scale
        assert err <= tol, f"{name}: scaled error {err:.3g} > {tol}"


def _compare(grads, ref, tol):
    for name, (a, b, _) in crater.offsets().items():
        r = ref[a:b].astype(np.float64)
        scale = max(float(np.abs(r).max()), 1e-12)
        err = float(np.abs(grads[a:b] - r).max()) / scale
        assert err <= tol, f"{name}: scaled error {err:.3g} > {tol}"


@pytest.mark.parametrize("batch", [2, 8])
def test_cnn_step_3xtf32_matches_oracle(cuda, oracle_mod, batch):
    loss, grads, params, ref_loss, ref_grads, ref_params = _run(cuda, oracle_mod, batch, "3xtf32")
    assert abs(loss - ref_loss) <= 1e-4 * max(1.0, abs(ref_loss))
    _compare(grads, ref_grads, 1e-4)
    np.testing.assert_allclose(params, ref_params, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("batch, batch_total, precision", [(512, 4096, "mixed"), (4096, 4096, "mixed"),
                                                        (512, 4096, "3xtf32")])
def test_cnn_graph_step_matches_oracle_at_bench_sizes(cuda, oracle_mod, batch, batch_total, precision):
    """The step the benchmark times, at the sizes it times: 4096 images on
    one GPU, and the 512-image shard of one rank of an 8-GPU run (conv1
    split over several blocks per image, the gradient allreduced in two
    buckets; on one GPU the sum over ranks is the
    tensor itself; the dense layers' bucket is reduced and applied on the
    side stream beside the conv backward, as in a data-parallel run, with
    8 SMs left free for it).  capture() runs one eager step and records the next;
    replay() runs it from the CUDA graph.  Loss, every gradient tensor and
    the parameters after both steps are compared with two oracle steps.

    The loss and the dense layers' gradients are held to 1e-4 * max|ref|;
    the two conv layers' gradients to the 1e-3 gradient tolerance of the
    tensor-core path.  Each of those sums every pixel of the batch with
    heavy cancellation, against an oracle that accumulates in f64, while the
    tensor core accumulates a CTA's share of the batch in f32: measured on a
    B200 at 512 of 4096 in 3xTF32, 4.3e-4 * max|ref| for conv2's weight
    gradient.  The default mixed precision (2xTF32 for the conv layer's two
    gradients) adds about 4e-4 more by an f64 error study of the step."""
    import torch

    from remora_b200.cnn import CraterCNN

    params = crater.init_params()
    imgs, labels = crater.make_batch(batch)
    reduced = []

    def allreduce(t) -> None:  # one rank: the sum over ranks is the tensor itself
        reduced.append(t.numel())

    net = CraterCNN(cuda, batch, batch_total, lr=0.01, params=params, precision=precision,
                    allreduce=allreduce if batch < batch_total else None)
    xi, yi = torch.from_numpy(imgs).to(cuda), torch.from_numpy(labels).to(cuda)
    net.capture(xi, yi)
    net.replay()
    grads, got = to_host(net.grads).copy(), to_host(net.params)
    loss = net.loss()
    ref = params.copy()
    nt = oracle_mod.max_threads()
    oracle_mod.cnn_step(ref, imgs, labels, batch_total=batch_total, lr=0.01, nthreads=nt)
    ref_loss, ref_grads = oracle_mod.cnn_step(ref, imgs, labels, batch_total=batch_total, lr=0.01, nthreads=nt)
    assert abs(loss - ref_loss) <= 1e-4 * max(1.0, abs(ref_loss))
    _compare(grads, ref_grads, 1e-3)
    _compare_from(grads, ref_grads, 1e-4, crater.offsets()["w3"][0])
    np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6)
    if batch < batch_total:
        # the dense layers' bucket beside the conv backward, then the conv bucket
        assert net.overlap and reduced[-2:] == [net.bucket_dense.numel(), net.bucket_conv.numel()]


def test_cnn_step_tf32_matches_oracle(cuda, oracle_mod):
    loss, grads, params, ref_loss, ref_grads, ref_params = _run(cuda, oracle_mod, 16, "tf32")
    assert abs(loss - ref_loss) <= 1e-3 * max(1.0, abs(ref_loss))
    _compare(grads, ref_grads, 5e-2)
    np.testing.assert_allclose(params, ref_params, rtol=1e-3, atol=1e-4)


def test_cnn_training_reduces_loss_and_graph_replay(cuda):
    """A few hundred samples, several SGD steps: the loss falls (the
    reference's own training test, tests/test_crater_train.py:6-19, asks for
    the final loss below 0.95x the first); a captured CUDA-graph step gives
    the same parameters as the eager step."""
    import torch

    from remora_b200.cnn import CraterCNN

    imgs, labels = crater.make_batch(256)
    xi, yi = torch.from_numpy(imgs).to(cuda), torch.from_numpy(labels).to(cuda)
    net = CraterCNN(cuda, 256, lr=0.05)
    losses = []
    for _ in range(30):
        net.forward_backward(xi, yi)
        losses.append(net.loss())
        net.update()
    assert all(np.isfinite(losses))
    assert losses[-1] < 0.95 * losses[0], losses
    assert np.isfinite(to_host(net.params)).all()
    # graph replay == eager step
    a = CraterCNN(cuda, 256, lr=0.05)
    b = CraterCNN(cuda, 256, lr=0.05)
    a.step(xi, yi)
    b.step(xi, yi)
    b.capture(xi, yi)  # records (and runs) one step
    from remora_b200 import _lib as L

    n0 = L.launch_count()
    a.step(xi, yi)
    # one replay launches the same library kernels as one eager step
    assert L.launch_count() - n0 == b.graph_launches > 10
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_host(a.params), to_host(b.params))
    b.replay()
    a.step(xi, yi)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(to_host(a.params), to_host(b.params))


@pytest.mark.parametrize("hw", [64, 32])
def test_conv1_relu_pool_and_wgrad_layers(cuda, oracle_mod, hw):
    """The fused first layer against the oracle's conv -> ReLU -> 2x2 max-pool
    (bit-exact: same rounding order) and its weight/bias gradient against the
    oracle's conv weight gradient of the unpooled, ReLU-masked cotangent."""
    import torch

    from remora_b200.cnn import _lib
    from remora_b200.abi import tensor_descriptor
    from remora_b200.runtime import context

    lib = _lib()
    rng = np.random.default_rng(hw)
    B, K = 5, 16
    x = rng.standard_normal((B, 1, hw, hw)).astype(np.float32)
    w = (rng.standard_normal((K, 1, 3, 3)) * 0.5).astype(np.float32)
    b = (rng.standard_normal(K) * 0.1).astype(np.float32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    xd, wd, bd = dev(x), dev(w), dev(b)
    p = torch.empty((B, K, hw // 2, hw // 2), dtype=torch.float32, device=cuda)
    code = torch.empty((B, K, hw // 2, hw // 2), dtype=torch.uint8, device=cuda)
    keep = [tensor_descriptor(t) for t in (xd, wd, bd, p, code)]
    ctx = context(cuda.index)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    assert lib.remora_b200_conv1_relu_pool(ctx.ptr, *[ctypes.addressof(d) for d in keep], stream) == 0
    a1 = oracle_mod.conv2d_fwd(x, w, b)
    a1 = np.where(a1 > 0, a1, np.float32(0))
    np.testing.assert_array_equal(to_host(p), oracle_mod.maxpool2x2_fwd(a1))
    # weight gradient from a pooled cotangent
    dp = rng.standard_normal(p.shape).astype(np.float32)
    dpd = dev(dp)
    dw = torch.empty((K, 1, 3, 3), dtype=torch.float32, device=cuda)
    db = torch.empty(K, dtype=torch.float32, device=cuda)
    keep2 = [tensor_descriptor(t) for t in (xd, dpd, code, dw, db)]
    assert lib.remora_b200_conv1_wgrad_pooled(ctx.ptr, *[ctypes.addressof(d) for d in keep2], stream) == 0
    da = oracle_mod.maxpool2x2_bwd(a1, dp)
    da = np.where(a1 > 0, da, np.float32(0))
    ref_w = oracle_mod.conv2d_wgrad(x, da, (K, 1, 3, 3))
    ref_b = da.astype(np.float64).sum(axis=(0, 2, 3))
    np.testing.assert_allclose(to_host(dw), ref_w, rtol=1e-5, atol=1e-5 * float(np.abs(ref_w).max()))
    np.testing.assert_allclose(to_host(db), ref_b, rtol=1e-5, atol=1e-5 * float(np.abs(ref_b).max()))


@pytest.mark.parametrize("precision", ["tf32", "3xtf32", "2xtf32"])
def test_fused_conv2_pool_matches_unfused(cuda, precision):
    """conv2 + ReLU + max-pool in one kernel, and the conv2 gradients taken
    straight from the pooled gradient, give bit for bit what the separate
    conv2d / relu_pool / unpool calls give."""
    import torch

    from remora_b200 import _lib as L
    from remora_b200.abi import tensor_descriptor
    from remora_b200.cnn import _lib
    from remora_b200.runtime import context

    lib = _lib()
    rng = np.random.default_rng(5)
    B = 6
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    x = dev(rng.standard_normal((B, 16, 32, 32)).astype(np.float32))
    w = dev((rng.standard_normal((32, 16, 3, 3)) * 0.1).astype(np.float32))
    b = dev((rng.standard_normal(32) * 0.1).astype(np.float32))
    spec = L.RemoraConvSpec(1, 1, {"tf32": L.PREC_TF32, "3xtf32": L.PREC_3XTF32, "2xtf32": L.PREC_2XTF32}[precision],
                            0)
    ctx = context(cuda.index)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    keep = []

    def d(t):
        keep.append(tensor_descriptor(t))
        return ctypes.addressof(keep[-1])

    f32, u8 = torch.float32, torch.uint8
    a2 = torch.empty((B, 32, 32, 32), dtype=f32, device=cuda)
    p_ref, c_ref = torch.empty((B, 32, 16, 16), dtype=f32, device=cuda), torch.empty((B, 32, 16, 16), dtype=u8,
                                                                                    device=cuda)
    p_fused, c_fused = torch.empty_like(p_ref), torch.empty_like(c_ref)
    assert lib.remora_b200_conv2d_fwd(ctx.ptr, ctypes.byref(spec), d(x), d(w), d(b), d(a2), stream) == 0
    assert lib.remora_b200_relu_pool(ctx.ptr, d(a2), d(p_ref), d(c_ref), stream) == 0
    assert lib.remora_b200_conv2d_fwd_relu_pool(ctx.ptr, ctypes.byref(spec), d(x), d(w), d(b), d(p_fused),
                                                d(c_fused), stream) == 0
    np.testing.assert_array_equal(to_host(p_fused), to_host(p_ref))
    np.testing.assert_array_equal(to_host(c_fused), to_host(c_ref))
    # backward from a pooled gradient
    dp = dev(rng.standard_normal((B, 32, 16, 16)).astype(np.float32))
    da = torch.empty((B, 32, 32, 32), dtype=f32, device=cuda)
    assert lib.remora_b200_unpool(ctx.ptr, d(dp), d(c_ref), d(da), stream) == 0
    dx_ref, dx_fused = torch.empty_like(x), torch.empty_like(x)
    assert lib.remora_b200_conv2d_dgrad(ctx.ptr, ctypes.byref(spec), d(da), d(w), d(dx_ref), stream) == 0
    assert lib.remora_b200_conv2d_dgrad_unpool(ctx.ptr, ctypes.byref(spec), d(dp), d(c_ref), d(w), d(dx_fused),
                                               stream) == 0
    np.testing.assert_array_equal(to_host(dx_fused), to_host(dx_ref))
    dw_ref, dw_fused = torch.empty_like(w), torch.empty_like(w)
    db_ref, db_fused = torch.empty_like(b), torch.empty_like(b)
    assert lib.remora_b200_conv2d_wgrad_bias(ctx.ptr, ctypes.byref(spec), d(x), d(da), d(dw_ref), d(db_ref),
                                             stream) == 0
    assert lib.remora_b200_conv2d_wgrad_bias_unpool(ctx.ptr, ctypes.byref(spec), d(x), d(dp), d(c_ref),
                                                    d(dw_fused), d(db_fused), stream) == 0
    np.testing.assert_array_equal(to_host(dw_fused), to_host(dw_ref))
    np.testing.assert_array_equal(to_host(db_fused), to_host(db_ref))


def test_conv1_layers_same_for_every_block_split(cuda, oracle_mod):
    """The first layer splits an image over 1, 2 or 4 blocks depending on the
    batch (small batches use more blocks per image).  Forward outputs are
    bit for bit the same for every split; the weight gradient matches the
    oracle within the f32 tolerance for every split."""
    import torch

    from remora_b200.abi import tensor_descriptor
    from remora_b200.cnn import _lib
    from remora_b200.runtime import context

    lib = _lib()
    rng = np.random.default_rng(77)
    K, hw = 16, 64
    x = rng.standard_normal((2100, 1, hw, hw)).astype(np.float32)
    w = (rng.standard_normal((K, 1, 3, 3)) * 0.5).astype(np.float32)
    b = (rng.standard_normal(K) * 0.1).astype(np.float32)
    ctx = context(cuda.index)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    wd, bd = torch.from_numpy(w).to(cuda), torch.from_numpy(b).to(cuda)
    outs = {}
    for B in (5, 1100, 2100):  # 4, 2 and 1 blocks per image
        xd = torch.from_numpy(x[:B].copy()).to(cuda)
        p = torch.empty((B, K, 32, 32), dtype=torch.float32, device=cuda)
        code = torch.empty((B, K, 32, 32), dtype=torch.uint8, device=cuda)
        keep = [tensor_descriptor(t) for t in (xd, wd, bd, p, code)]
        assert lib.remora_b200_conv1_relu_pool(ctx.ptr, *[ctypes.addressof(d) for d in keep], stream) == 0
        outs[B] = (to_host(p), to_host(code))
        dp = torch.from_numpy(rng.standard_normal((B, K, 32, 32)).astype(np.float32)).to(cuda)
        dw = torch.empty((K, 1, 3, 3), dtype=torch.float32, device=cuda)
        db = torch.empty(K, dtype=torch.float32, device=cuda)
        keep2 = [tensor_descriptor(t) for t in (xd, dp, code, dw, db)]
        assert lib.remora_b200_conv1_wgrad_pooled(ctx.ptr, *[ctypes.addressof(d) for d in keep2], stream) == 0
        if B == 1100:
            a1 = oracle_mod.conv2d_fwd(x[:B], w, b, nthreads=oracle_mod.max_threads())
            a1 = np.where(a1 > 0, a1, np.float32(0))
            da = oracle_mod.maxpool2x2_bwd(a1, to_host(dp))
            da = np.where(a1 > 0, da, np.float32(0))
            ref_w = oracle_mod.conv2d_wgrad(x[:B], da, (K, 1, 3, 3), nthreads=oracle_mod.max_threads())
            np.testing.assert_allclose(to_host(dw), ref_w, rtol=1e-5, atol=1e-5 * float(np.abs(ref_w).max()))
    for B in (5, 1100):
        np.testing.assert_array_equal(outs[B][0], outs[2100][0][:B])
        np.testing.assert_array_equal(outs[B][1], outs[2100][1][:B])


def test_dense_bias_relu_bce_matches_unfused(cuda):
    """ReLU(hpre + b3) fused into the dense BCE kernel gives bit for bit the
    separate map + dense_bce calls."""
    import torch

    from remora_b200 import ops
    from remora_b200.abi import tensor_descriptor
    from remora_b200.cnn import _lib
    from remora_b200.program import BinaryExpr, CmpExpr, SelectExpr, const, x

    lib = _lib()
    rng = np.random.default_rng(3)
    B, D = 300, 64
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    hpre, hb = dev(rng.standard_normal((B, D)).astype(np.float32)), dev(rng.standard_normal(D).astype(np.float32))
    w4, b4 = dev((rng.standard_normal(D) * 0.2).astype(np.float32)), dev(np.array([0.05], np.float32))
    y = dev((np.arange(B) % 2).astype(np.float32))
    s = BinaryExpr("+", x(0), x(1))
    h_ref = ops.map(SelectExpr(CmpExpr(">", s, const(0.0)), s, const(0.0)), hpre, hb.unsqueeze(0).expand(B, D))
    e = lambda *sh: torch.empty(sh, dtype=torch.float32, device=cuda)  # noqa: E731
    z1, l1, g1, z2, l2, g2, h2 = e(B), e(B), e(B), e(B), e(B), e(B), e(B, D)
    ctx = __import__("remora_b200.runtime", fromlist=["context"]).context(cuda.index)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    keep = []

    def d(t):
        keep.append(tensor_descriptor(t))
        return ctypes.addressof(keep[-1])

    assert lib.remora_b200_dense_bce(ctx.ptr, d(h_ref), d(w4), d(b4), d(y), d(z1), d(l1), d(g1),
                                     ctypes.c_float(1 / B), stream) == 0
    assert lib.remora_b200_dense_bias_relu_bce(ctx.ptr, d(hpre), d(hb), d(h2), d(w4), d(b4), d(y), d(z2), d(l2),
                                               d(g2), ctypes.c_float(1 / B), stream) == 0
    for a, b_ in ((h2, h_ref), (z2, z1), (l2, l1), (g2, g1)):
        np.testing.assert_array_equal(to_host(a), to_host(b_))


def test_cnn_resume_from_checkpoint_matches_unbroken_run(cuda, tmp_path):
    """Three SGD steps on the device, against two steps, a checkpoint, a new
    model restored from it (its step captured as a CUDA graph) and one more
    step: the same parameters bit for bit (the step is deterministic)."""
    import torch

    from remora_b200.cnn import CraterCNN

    imgs, labels = crater.make_batch(64)
    xi, yi = torch.from_numpy(imgs).to(cuda), torch.from_numpy(labels).to(cuda)
    a = CraterCNN(cuda, 64, lr=0.05)
    for _ in range(3):
        a.step(xi, yi)
    b = CraterCNN(cuda, 64, lr=0.05)
    for _ in range(2):
        b.step(xi, yi)
    b.save(tmp_path / "cnn.npz", step=2)
    c = CraterCNN(cuda, 64, lr=0.05, params=np.zeros(crater.NPARAMS, np.float32))
    c.step(xi, yi)               # compile and size workspaces on throwaway parameters
    c.capture(xi, yi)            # then record the step's graph
    assert c.restore(tmp_path / "cnn.npz") == 2
    c.replay()                   # step 3 from the graph, on the restored parameters
    np.testing.assert_array_equal(to_host(c.params), to_host(a.params))


@pytest.mark.parametrize("precision", ["mixed", "3xtf32"])
def test_cnn_step_entry_point_matches_the_python_step(cuda, precision):
    """remora_b200_cnn_step, the step behind one C call, gives bit for bit
    the parameters, gradients and per-sample losses of CraterCNN.step (the
    same kernels in the same order), alone and with a one-rank NCCL
    communicator (whose allreduce leaves the gradient as it is)."""
    import torch

    from remora_b200.cnn import CraterCNN, cnn_step, nccl_comm_destroy, nccl_comm_init, nccl_unique_id

    B = 96
    imgs, labels = crater.make_batch(B)
    xi, yi = torch.from_numpy(imgs).to(cuda), torch.from_numpy(labels).to(cuda)
    ref = CraterCNN(cuda, B, lr=0.05, precision=precision)
    for _ in range(2):
        ref.step(xi, yi)
    p = torch.from_numpy(crater.init_params()).to(cuda)
    g = torch.zeros(crater.NPARAMS, dtype=torch.float32, device=cuda)
    losses = torch.empty(B, dtype=torch.float32, device=cuda)
    cnn_step(p, g, xi, yi, lr=0.05, precision=precision, losses=losses)
    comm = nccl_comm_init(1, nccl_unique_id(), 0)
    try:
        cnn_step(p, g, xi, yi, lr=0.05, precision=precision, losses=losses, comm=comm)
        torch.cuda.synchronize()
    finally:
        nccl_comm_destroy(comm)
    np.testing.assert_array_equal(to_host(p), to_host(ref.params))
    np.testing.assert_array_equal(to_host(g), to_host(ref.grads))
    np.testing.assert_array_equal(to_host(losses), to_host(ref.loss_b))
