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
    "remora_b200_cnn_step": [ctypes.c_void_p] * 9,
    "remora_b200_nccl_unique_id": [ctypes.c_void_p],
    "remora_b200_nccl_comm_init": [ctypes.c_void_p, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int32],
    "remora_b200_nccl_comm_destroy": [ctypes.c_void_p],
}

# precision codes of remora_b200_cnn_step (REMORA_CNN_* of remora_b200_cnn.h)
CNN_PRECISION = {"mixed": 0, "3xtf32": 1, "tf32": 2}


class RemoraCnnStepSpec(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("batch_total", ctypes.c_int32), ("lr", ctypes.c_float),
                ("precision", ctypes.c_int32)]


def cnn_step(params, grads, images, labels, *, batch_total: int | None = None, lr: float = 0.01,
             precision: str = "mixed", losses=None, comm: int | None = None) -> None:
    """One SGD step through the single C entry point remora_b200_cnn_step
    (the C-ABI form of CraterCNN.step): device tensors params / grads
    f32[529217], images [B,1,64,64], labels [B], optional losses [B]; `comm`
    an ncclComm_t address (nccl_comm_init) or None for one rank.  Enqueued
    on the current stream."""
    import torch

    lib = _lib()
    B = int(images.shape[0])
    spec = RemoraCnnStepSpec(B, int(batch_total or B), float(lr), CNN_PRECISION[precision])
    keep = [tensor_descriptor(t) for t in (params, grads, images, labels)]
    ld = tensor_descriptor(losses) if losses is not None else None
    stream = ctypes.c_void_p(torch.cuda.current_stream(params.device).cuda_stream)
    L.check(lib.remora_b200_cnn_step(context(params.device.index).ptr, ctypes.byref(spec),
                                     *[ctypes.addressof(d) for d in keep],
                                     ctypes.addressof(ld) if ld is not None else None,
                                     ctypes.c_void_p(comm) if comm else None, stream), "cnn_step")


def nccl_unique_id() -> bytes:
    """A new NCCL unique id (128 bytes) for nccl_comm_init, made by one rank
    and handed to the others over any host channel."""
    buf = ctypes.create_string_buffer(128)
    L.check(_lib().remora_b200_nccl_unique_id(buf), "nccl_unique_id")
    return buf.raw


def nccl_comm_init(nranks: int, uid: bytes, rank: int) -> int:
    """An ncclComm_t (as an address) of rank `rank` of `nranks` on the
    current device."""
    comm = ctypes.c_void_p()
    buf = ctypes.create_string_buffer(bytes(uid), 128)
    L.check(_lib().remora_b200_nccl_comm_init(ctypes.byref(comm), int(nranks), buf, int(rank)), "nccl_comm_init")
    return int(comm.value)


def nccl_comm_destroy(comm: int) -> None:
    L.check(_lib().remora_b200_nccl_comm_destroy(ctypes.c_void_p(comm)), "nccl_comm_destroy")


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


CHECKPOINT_FORMAT = 1


def save_checkpoint(path, params: np.ndarray, step: int, *, lr: float, batch_total: int,
                    precision: str = "mixed", data_seed: int = crater.DATA_SEED,
                    parameter_seed: int = crater.PARAMETER_SEED) -> None:
    """Write the training state of the crater CNN to `path` (.npz): the flat
    parameter vector in the layout of remora_b200.crater, the number of SGD
    steps taken, and what the run needs to continue identically (learning
    rate, global batch, precision, seeds).  The reference keeps parameter
    snapshots every K epochs in memory (examples/crater_train.py:236,263-264);
    this is their on-disk form.  The file is written under a temporary name
    and renamed, so a reader never sees a partial checkpoint."""
    import os

    flat = np.ascontiguousarray(params, dtype=np.float32).reshape(-1)
    if flat.size != crater.NPARAMS:
        raise ValueError(f"a checkpoint holds {crater.NPARAMS} parameters, got {flat.size}")
    path = os.fspath(path)
    tmp = path + ".tmp.npz"
    np.savez(tmp, params=flat, step=np.int64(step), lr=np.float64(lr), batch_total=np.int64(batch_total),
             precision=np.array(precision), data_seed=np.int64(data_seed), parameter_seed=np.int64(parameter_seed),
             layout=np.array([f"{k}:{'x'.join(map(str, sh))}" for k, sh in crater.LAYOUT]),
             format=np.int64(CHECKPOINT_FORMAT))
    os.replace(tmp, path)


def load_checkpoint(path) -> dict:
    """The state save_checkpoint wrote; raises ValueError when the file's
    parameter layout is not this model's."""
    with np.load(path) as f:
        if int(f["format"]) != CHECKPOINT_FORMAT:
            raise ValueError(f"checkpoint format {int(f['format'])}, expected {CHECKPOINT_FORMAT}")
        layout = [str(v) for v in f["layout"]]
        want = [f"{k}:{'x'.join(map(str, sh))}" for k, sh in crater.LAYOUT]
        if layout != want:
            raise ValueError(f"checkpoint layout {layout} is not the crater CNN's {want}")
        return {"params": f["params"].copy(), "step": int(f["step"]), "lr": float(f["lr"]),
                "batch_total": int(f["batch_total"]), "precision": str(f["precision"]),
                "data_seed": int(f["data_seed"]), "parameter_seed": int(f["parameter_seed"])}


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
                 params: np.ndarray | None = None, allreduce=None, precision: str = "mixed",
                 overlap_allreduce: bool | None = None, reserve_sms: int = 8) -> None:
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
        # "mixed" (default): 3xTF32 for the conv forward and every GEMM,
        # 2xTF32 (one operand split) for the conv layer's two gradients; an
        # f64 error study of the step puts every gradient within 4e-4 of
        # the f32 step (a forward in TF32 shifts ReLU masks and pool choices:
        # 1e-2).  "3xtf32": split precision everywhere, gradients within
        # 1e-4.  "tf32": single-pass TF32 everywhere, outside the 1e-3
        # gradient tolerance (first layer ~3e-2 of max): a speed reference.
        if precision not in ("mixed", "3xtf32", "tf32"):
            raise ValueError(f"unknown precision {precision!r}")
        self.precision = precision
        fwd = L.PREC_TF32 if precision == "tf32" else L.PREC_3XTF32
        bwd = {"tf32": L.PREC_TF32, "3xtf32": L.PREC_3XTF32, "mixed": L.PREC_2XTF32}[precision]
        self.conv_spec = L.RemoraConvSpec(1, 1, fwd, 0)
        self.conv_bwd_spec = L.RemoraConvSpec(1, 1, bwd, 0)
        self.gemm_spec = L.RemoraGemmSpec(fwd, 0)
        self.graph = None
        self.graphs: list = []
        self._keep: list = []
        # Two allreduce buckets: w3..b4 (the dense layers, 99 % of the
        # gradient) is final once dense1's weight gradient is done; it is
        # reduced on a side stream while dense1's input gradient and the conv
        # layers' backward run, and applied there once dense1's input
        # gradient, the last reader of those parameters, is done.  w1..b2
        # follows at the end.
        o = crater.offsets()
        split = o["w3"][0]
        self.bucket_dense = self.grads[split:]
        self.bucket_conv = self.grads[:split]
        self.params_dense = self.params[split:]
        self.params_conv = self.params[:split]
        self.comm = torch.cuda.Stream(self.dev) if allreduce is not None else None
        # False: one allreduce of the whole gradient after the backward.  By
        # default the dense bucket overlaps the conv backward: on two B200s
        # with 512 images per rank the step took 0.408 ms serial, 0.405 ms
        # overlapped, 0.399 ms overlapped with 8 SMs left to the collective.
        self.overlap = True if overlap_allreduce is None else bool(overlap_allreduce)
        # With the overlapped allreduce, the persistent kernels of the
        # backward that runs beside it (dense1's input gradient, conv2's two
        # gradients) may leave `reserve_sms` SMs to the collective's blocks.
        self.reserve_sms = int(reserve_sms) if self.overlap and allreduce is not None else 0
        self.sm_count = torch.cuda.get_device_properties(self.dev).multi_processor_count

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
    def stages(self, images, labels) -> list[tuple[str, Any]]:
        """The step's library calls up to the gradient, in order, as (name,
        callable) pairs; each callable enqueues its call on the current
        stream.  ``forward_backward`` runs them all; a benchmark may time one
        alone (it reads and writes this rank's own buffers)."""
        lib, c = self.lib, self.ctx.ptr
        p, g = self.p, self.g
        B = self.B
        d, chk, spec, bspec = self._d, self._check, self.conv_spec, self.conv_bwd_spec
        p2flat = self.p2.view(B, 8192)

        def conv1():
            chk(lib.remora_b200_conv1_relu_pool(c, d(images), d(p["w1"]), d(p["b1"]), d(self.p1), d(self.code1),
                                                self._stream()), "conv1")

        def conv2():  # conv2 + bias + ReLU + pool: the [B,32,32,32] activation never exists
            chk(lib.remora_b200_conv2d_fwd_relu_pool(c, ctypes.byref(spec), d(self.p1), d(p["w2"]), d(p["b2"]),
                                                     d(self.p2), d(self.code2), self._stream()), "conv2")

        def dense1():
            self._gemm(p2flat, p["w3"].t(), self.hpre)

        def head():  # ReLU(hpre + b3), dense 64 -> 1, BCE and dlogit
            chk(lib.remora_b200_dense_bias_relu_bce(c, d(self.hpre), d(p["b3"]), d(self.h), d(p["w4"]), d(p["b4"]),
                                                    d(labels), d(self.z), d(self.loss_b), d(self.dz),
                                                    ctypes.c_float(1.0 / self.B_total), self._stream()), "dense_bce")

        def head_bwd():  # dense 64 -> 1 backward; sums dh over the batch: the hidden bias gradient
            chk(lib.remora_b200_dense_relu_bwd(c, d(self.h), d(p["w4"]), d(self.dz), d(self.dh), d(g["w4"]),
                                               d(g["b4"]), d(g["b3"]), self._stream()), "dense2 bwd")

        def dense1_wgrad():  # as its transpose, [8192, 64] = p2^T dh: 64 row blocks, not 1
            self._gemm(p2flat.t(), self.dh, g["w3"].t())

        def dense1_dgrad():
            self._gemm(self.dh, p["w3"], self.dp2.view(B, 8192))

        def conv2_wgrad():  # straight from the pooled gradient and the pool codes
            chk(lib.remora_b200_conv2d_wgrad_bias_unpool(c, ctypes.byref(bspec), d(self.p1), d(self.dp2),
                                                         d(self.code2), d(g["w2"]), d(g["b2"]), self._stream()),
                "conv2 wgrad")

        def conv2_dgrad():
            chk(lib.remora_b200_conv2d_dgrad_unpool(c, ctypes.byref(bspec), d(self.dp2), d(self.code2), d(p["w2"]),
                                                    d(self.dp1), self._stream()), "conv2 dgrad")

        def conv1_wgrad():
            chk(lib.remora_b200_conv1_wgrad_pooled(c, d(images), d(self.dp1), d(self.code1), d(g["w1"]),
                                                   d(g["b1"]), self._stream()), "conv1 wgrad")

        return [("conv1_fwd", conv1), ("conv2_fwd", conv2), ("dense1_fwd", dense1), ("head", head),
                ("head_bwd", head_bwd), ("dense1_wgrad", dense1_wgrad), ("dense1_dgrad", dense1_dgrad),
                ("conv2_wgrad", conv2_wgrad), ("conv2_dgrad", conv2_dgrad), ("conv1_wgrad", conv1_wgrad)]

    def forward_backward(self, images, labels) -> None:
        """Loss and gradients of this rank's shard into self.grads.  With a
        data-parallel allreduce and overlap (the default), the dense layers'
        bucket is already reduced over the ranks and applied to the
        parameters on the side stream; update() finishes the conv bucket."""
        self._keep = []
        try:
            overlap = self.allreduce is not None and self.overlap
            for name, run in self.stages(images, labels):
                if name == "dense1_dgrad" and overlap and self.reserve_sms:
                    # from here on the persistent kernels run beside the allreduce
                    self._check(self.lib.remora_b200_set_persistent_sms(
                        self.ctx.ptr, max(1, self.sm_count - self.reserve_sms)), "persistent SMs")
                run()
                if name == "dense1_wgrad" and overlap:
                    # the dense bucket is final: reduce it while the rest runs
                    cur = self.torch.cuda.current_stream(self.dev)
                    self.comm.wait_stream(cur)
                    with self.torch.cuda.stream(self.comm):
                        self.allreduce(self.bucket_dense)
                elif name == "dense1_dgrad" and overlap:
                    # the last reader of the dense parameters is done: apply
                    # the reduced dense bucket beside the conv backward
                    done = self.torch.cuda.Event()
                    done.record(self.torch.cuda.current_stream(self.dev))
                    self.comm.wait_event(done)
                    with self.torch.cuda.stream(self.comm):
                        self._map(self.prog_sgd, [self.params_dense, self.bucket_dense], self.params_dense)
        finally:
            if self.reserve_sms:
                self.lib.remora_b200_set_persistent_sms(self.ctx.ptr, 0)

    def update(self) -> None:
        if self.allreduce is not None:
            cur = self.torch.cuda.current_stream(self.dev)
            self.comm.wait_stream(cur)
            with self.torch.cuda.stream(self.comm):
                self.allreduce(self.bucket_conv if self.overlap else self.grads)
            cur.wait_stream(self.comm)
        if self.allreduce is not None and self.overlap:
            # the dense layers were updated beside the conv backward
            self._map(self.prog_sgd, [self.params_conv, self.bucket_conv], self.params_conv)
        else:
            self._map(self.prog_sgd, [self.params, self.grads], self.params)

    def step(self, images, labels) -> None:
        self.forward_backward(images, labels)
        self.update()

    # -------------------------------------------------- checkpoint/resume
    def save(self, path, step: int) -> None:
        """Checkpoint this replica's parameters after `step` SGD steps (the
        replicas of a data-parallel run are identical; rank 0 writes)."""
        self.torch.cuda.synchronize(self.dev)
        save_checkpoint(path, self.params.cpu().numpy(), step, lr=self.lr, batch_total=self.B_total,
                        precision=self.precision)

    def restore(self, path) -> int:
        """Load a checkpoint's parameters into this model, in place (captured
        graphs keep reading the same buffer); returns the step it was taken
        at.  The learning rate, global batch and precision must match."""
        st = load_checkpoint(path)
        if st["batch_total"] != self.B_total or abs(st["lr"] - self.lr) > 0.0 or st["precision"] != self.precision:
            raise ValueError(f"checkpoint of lr {st['lr']}, global batch {st['batch_total']}, {st['precision']}; "
                             f"this model has lr {self.lr}, global batch {self.B_total}, {self.precision}")
        self.params.copy_(self.torch.from_numpy(st["params"]))
        self.torch.cuda.synchronize(self.dev)
        return st["step"]

    def loss(self) -> float:
        """This rank's share of the batch-mean loss of the last step (sum of
        its per-sample losses / global batch)."""
        from remora_b200 import ops

        ops.fold(self.loss_b, mode="all", out=self.loss_sum)
        return float(self.loss_sum.item()) / self.B_total

    # ------------------------------------------------------ graph capture
    def capture(self, images, labels) -> int:
        """Record one step (forward, backward, allreduce, update) on
        ``images``/``labels`` as a CUDA graph on a side stream; replay() then
        launches it whole.  Runs one eager step first (kernels compiled,
        workspace sized).  Several graphs, one per input buffer, may be
        captured (double-buffered inputs); returns this graph's index."""
        torch = self.torch
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            self.step(images, labels)  # sizes the side stream's workspace outside capture
        torch.cuda.current_stream(self.dev).wait_stream(side)
        torch.cuda.synchronize(self.dev)
        graph = torch.cuda.CUDAGraph()
        n0 = L.launch_count()
        with torch.cuda.graph(graph, stream=side):
            self.step(images, labels)
        self.graph_launches = L.launch_count() - n0  # library kernels per replay
        self.graphs.append((graph, list(self._keep)))
        self.graph = graph
        return len(self.graphs) - 1

    def replay(self, which: int | None = None) -> None:
        (self.graph if which is None else self.graphs[which][0]).replay()

    def release_graphs(self) -> None:
        """Drop every captured graph (those holding NCCL calls must go
        before the process group is destroyed)."""
        self.graph = None
        self.graphs = []

    def stage_graph(self, name: str, images, labels, reps: int):
        """One stage of the step (a name of ``stages``) repeated ``reps``
        times as a CUDA graph, for timing that stage alone."""
        torch = self.torch
        run = dict(self.stages(images, labels))[name]
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            run()  # compiles and sizes this stream's workspace outside capture
        torch.cuda.synchronize(self.dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(reps):
                run()
        return graph, list(self._keep)
