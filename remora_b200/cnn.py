"""Crater-CNN training step on the B200 backend, data parallel over ranks.

Model (batched form of the reference's crater CNN, examples/crater_train.py):
conv3x3 1->16 + ReLU, 2x2 max-pool, conv3x3 16->32 + ReLU, 2x2 max-pool,
dense 8192->64 + ReLU, dense 64->1, stable BCE on the logit averaged over the
global batch, SGD p <- p - lr * g.  Every stage is a libremora_b200 call on
device-resident buffers: forward, backward and the update never leave the
GPU.  With several ranks each holds the full parameters and 1/world of the
global batch; the flat gradient buffer (529,217 f32) is summed with NCCL
allreduces in two buckets (the dense layers' gradients are reduced on a side
stream while the conv layers' backward still runs; the per-sample gradients
already carry 1/global_batch), so every rank applies the same update and the
replicas stay bitwise identical.

Gradient views point into one flat buffer in the parameter layout of
remora_b200.crater, so the kernels write the allreduce buffer directly.
"""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from remora_b200 import _lib as L
from remora_b200 import crater
from remora_b200.abi import tensor_descriptor
from remora_b200.program import BinaryExpr, compile_program, const, x
from remora_b200.runtime import context

_CNN_PROTOS = {
    "remora_b200_conv1_relu_pool": [ctypes.c_void_p] * 7,
    "remora_b200_relu_pool": [ctypes.c_void_p] * 5,
    "remora_b200_unpool": [ctypes.c_void_p] * 5,
    "remora_b200_dense_bce": [ctypes.c_void_p] * 8 + [ctypes.c_float, ctypes.c_void_p],
    "remora_b200_dense_bias_relu_bce": [ctypes.c_void_p] * 10 + [ctypes.c_float, ctypes.c_void_p],
    "remora_b200_dense_relu_bwd": [ctypes.c_void_p] * 9,
    "remora_b200_conv1_wgrad_pooled": [ctypes.c_void_p] * 7,
    "remora_b200_conv2d_wgrad_bias": [ctypes.c_void_p] * 7,
    "remora_b200_conv2d_fwd_relu_pool": [ctypes.c_void_p] * 8,
    "remora_b200_conv2d_dgrad_unpool": [ctypes.c_void_p] * 7,
    "remora_b200_conv2d_wgrad_bias_unpool": [ctypes.c_void_p] * 8,
}


def shard(batch_total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of `rank`'s share of a global batch split evenly over
    `world` data-parallel ranks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if batch_total % world:
        raise ValueError(f"global batch {batch_total} does not split evenly over {world} ranks")
    per = batch_total // world
    return rank * per, (rank + 1) * per


def process_group_allreduce(group=None):
    """The gradient reduction of a data-parallel step: a sum in place over
    the ranks of `group` (torch.distributed; NCCL on GPUs, gloo on CPU).
    The per-sample gradients already carry 1/global_batch, so a sum is the
    mean gradient of the global batch."""
    import torch.distributed as dist

    def allreduce(t) -> None:
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)

    return allreduce


def _lib():
    lib = L.lib()
    for name, args in _CNN_PROTOS.items():
        fn = getattr(lib, name)
        fn.restype = ctypes.c_int32
        fn.argtypes = args
    return lib


class CraterCNN:
    """Buffers and the step of one rank.  `batch` is this rank's share of
    `batch_total`; call `step(images, labels)` with device tensors
    [batch,1,64,64] and [batch]."""

    def __init__(self, device: Any, batch: int, batch_total: int | None = None, lr: float = 0.01,
                 params: np.ndarray | None = None, allreduce=None, precision: str = "3xtf32",
                 overlap_allreduce: bool | None = None) -> None:
        import torch

        self.torch = torch
        self.dev = torch.device(device)
        self.B = int(batch)
        self.B_total = int(batch_total or batch)
        self.lr = float(lr)
        self.allreduce = allreduce  # callable(tensor) summing in place over ranks, or None
        self.lib = _lib()
        self.ctx = context(self.dev.index)
        host = crater.init_params() if params is None else np.asarray(params, dtype=np.float32)
        self.params = torch.from_numpy(host.copy()).to(self.dev)
        self.grads = torch.zeros(crater.NPARAMS, dtype=torch.float32, device=self.dev)
        self.p = self._views(self.params)
        self.g = self._views(self.grads)
        B, f32, u8 = self.B, torch.float32, torch.uint8
        e = lambda *s, dt=f32: torch.empty(s, dtype=dt, device=self.dev)  # noqa: E731
        self.p1, self.code1 = e(B, 16, 32, 32), e(B, 16, 32, 32, dt=u8)
        self.p2, self.code2 = e(B, 32, 16, 16), e(B, 32, 16, 16, dt=u8)
        self.hpre, self.h = e(B, 64), e(B, 64)
        self.z, self.loss_b, self.dz = e(B), e(B), e(B)
        self.dh = e(B, 64)
        self.dp2 = e(B, 32, 16, 16)
        self.dp1 = e(B, 16, 32, 32)
        self.loss_sum = e(1).reshape(())
        # fused map: the in-place SGD update p - lr * g
        self.prog_sgd = compile_program(BinaryExpr("-", x(0), BinaryExpr("*", const(self.lr), x(1))), 2)
        # "3xtf32" (default): split-precision GEMMs and convs, gradients
        # within 1e-4 of the f32 step; "tf32": single-pass TF32 tensor-core
        # convs and GEMMs, faster, first-layer gradient off by ~3e-2 of max
        prec = {"tf32": L.PREC_TF32, "3xtf32": L.PREC_3XTF32}[precision]
        self.conv_spec = L.RemoraConvSpec(1, 1, prec, 0)
        self.gemm_spec = L.RemoraGemmSpec(prec, 0)
        self.graph = None
        self._keep: list = []
        # Two allreduce buckets: w3..b4 (the dense layers, 99 % of the
        # gradient) is final once the dense1 weight-gradient GEMM is done and
        # is reduced on a side stream while the conv layers' backward runs;
        # w1..b2 follows at the end of the backward.
        o = crater.offsets()
        split = o["w3"][0]
        self.bucket_dense = self.grads[split:]
        self.bucket_conv = self.grads[:split]
        self.comm = torch.cuda.Stream(self.dev) if allreduce is not None else None
        # False: one allreduce of the whole gradient after the backward.  By
        # default the dense bucket overlaps the conv backward only when a
        # rank holds at least 1024 images: NCCL's kernels take SMs from the
        # conv layers' persistent kernels, and with 512 images per rank on 8
        # GPUs the serial form measured faster (0.354 against 0.368 ms).
        self.overlap = self.B >= 1024 if overlap_allreduce is None else bool(overlap_allreduce)

    # ------------------------------------------------------------ helpers
    @staticmethod
    def _views(flat) -> dict:
        return {k: flat[a:b].view(*s) for k, (a, b, s) in crater.offsets().items()}

    def _d(self, t):
        d = tensor_descriptor(t)
        self._keep.append(d)
        return ctypes.addressof(d)

    def _stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream(self.dev).cuda_stream)

    def _check(self, st: int, what: str) -> None:
        if st:
            L.check(st, what)

    def _gemm(self, a, b, c) -> None:
        self._check(self.lib.remora_b200_gemm(self.ctx.ptr, ctypes.byref(self.gemm_spec), self._d(a), self._d(b),
                                              self._d(c), c.dim(), self._stream()), "gemm")

    def _map(self, prog, ins, out) -> None:
        ptrs = (ctypes.c_void_p * len(ins))(*[self._d(t) for t in ins])
        ranks = (ctypes.c_int32 * len(ins))(*[t.dim() for t in ins])
        self._check(self.lib.remora_b200_map(self.ctx.ptr, ctypes.byref(prog), ptrs, ranks, len(ins), self._d(out),
                                             out.dim(), self._stream()), "map")

    # ---------------------------------------------------------- the step
    def forward_backward(self, images, labels) -> None:
        """Loss and gradients of this rank's shard into self.grads (not yet
        reduced over ranks)."""
        lib, c, s = self.lib, self.ctx.ptr, self._stream()
        p, g = self.p, self.g
        self._keep = []
        B = self.B
        # forward
        self._check(lib.remora_b200_conv1_relu_pool(c, self._d(images), self._d(p["w1"]), self._d(p["b1"]),
                                                    self._d(self.p1), self._d(self.code1), s), "conv1")
        # conv2 + bias + ReLU + pool in one kernel: the [B,32,32,32] activation never exists
        self._check(lib.remora_b200_conv2d_fwd_relu_pool(c, ctypes.byref(self.conv_spec), self._d(self.p1),
                                                         self._d(p["w2"]), self._d(p["b2"]), self._d(self.p2),
                                                         self._d(self.code2), s), "conv2")
        p2flat = self.p2.view(B, 8192)
        self._gemm(p2flat, p["w3"].t(), self.hpre)
        # ReLU(hpre + b3), dense 64 -> 1, BCE and dlogit in one kernel
        self._check(lib.remora_b200_dense_bias_relu_bce(c, self._d(self.hpre), self._d(p["b3"]), self._d(self.h),
                                                        self._d(p["w4"]), self._d(p["b4"]), self._d(labels),
                                                        self._d(self.z), self._d(self.loss_b), self._d(self.dz),
                                                        ctypes.c_float(1.0 / self.B_total), s), "dense_bce")
        # backward
        # dense 64 -> 1 backward; also sums dh over the batch: the hidden bias gradient
        self._check(lib.remora_b200_dense_relu_bwd(c, self._d(self.h), self._d(p["w4"]), self._d(self.dz),
                                                   self._d(self.dh), self._d(g["w4"]), self._d(g["b4"]),
                                                   self._d(g["b3"]), s), "dense2 bwd")
        self._gemm(self.dh.t(), p2flat, g["w3"])
        if self.allreduce is not None and self.overlap:
            # the dense bucket is final: reduce it while the convs run
            cur = self.torch.cuda.current_stream(self.dev)
            self.comm.wait_stream(cur)
            with self.torch.cuda.stream(self.comm):
                self.allreduce(self.bucket_dense)
        self._gemm(self.dh, p["w3"], self.dp2.view(B, 8192))
        # conv2 gradients straight from the pooled gradient and the pool codes
        self._check(lib.remora_b200_conv2d_wgrad_bias_unpool(c, ctypes.byref(self.conv_spec), self._d(self.p1),
                                                             self._d(self.dp2), self._d(self.code2),
                                                             self._d(g["w2"]), self._d(g["b2"]), s), "conv2 wgrad")
        self._check(lib.remora_b200_conv2d_dgrad_unpool(c, ctypes.byref(self.conv_spec), self._d(self.dp2),
                                                        self._d(self.code2), self._d(p["w2"]), self._d(self.dp1),
                                                        s), "conv2 dgrad")
        self._check(lib.remora_b200_conv1_wgrad_pooled(c, self._d(images), self._d(self.dp1), self._d(self.code1),
                                                       self._d(g["w1"]), self._d(g["b1"]), s), "conv1 wgrad")

    def update(self) -> None:
        if self.allreduce is not None:
            cur = self.torch.cuda.current_stream(self.dev)
            self.comm.wait_stream(cur)
            with self.torch.cuda.stream(self.comm):
                self.allreduce(self.bucket_conv if self.overlap else self.grads)
            cur.wait_stream(self.comm)
        self._map(self.prog_sgd, [self.params, self.grads], self.params)

    def step(self, images, labels) -> None:
        self.forward_backward(images, labels)
        self.update()

    def loss(self) -> float:
        """This rank's share of the batch-mean loss of the last step (sum of
        its per-sample losses / global batch)."""
        from remora_b200 import ops

        ops.fold(self.loss_b, mode="all", out=self.loss_sum)
        return float(self.loss_sum.item()) / self.B_total

    # ------------------------------------------------------ graph capture
    def capture(self, images, labels) -> None:
        """Record one step (forward, backward, allreduce, update) as a CUDA
        graph on a side stream; replay() then launches it whole.  Call after
        at least one eager step (kernels compiled, workspace sized)."""
        torch = self.torch
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            self.step(images, labels)  # sizes the side stream's workspace outside capture
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        self.graph = torch.cuda.CUDAGraph()
        n0 = L.launch_count()
        with torch.cuda.graph(self.graph, stream=side):
            self.step(images, labels)
        self.graph_launches = L.launch_count() - n0  # library kernels per replay
        self._graph_keep = list(self._keep)

    def replay(self) -> None:
        self.graph.replay()
