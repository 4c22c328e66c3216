"""Benchmark of the B200 backend on the Remora hot-path workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Default workload (``--config chained``): the fused chained-map fold
f32[64,64,64,64] ~ N(0,1): y = x*2.5 + 1.0, mask y > 0.5 ? y : 0, fold (+)
over the last axis -> f32[64,64,64]; metric HBM GB/s of algorithmic bytes
(67,108,864 read + 1,048,576 written per call).  One step = one pass over a
rotation of 8 distinct inputs (545 MB, more than 4x the 126 MB L2, so every
call streams from HBM).

Other configs: ``row_norms`` (f32[8192,1024] -> sqrt(sum x*x)), ``matmul``
(A,B f32[4096,4096], TF32; ``matmul_3x`` the 3xTF32 form), ``bmm``
([32,1024,1024] x [32,1024,1024], TF32), ``conv`` / ``conv_dgrad`` /
``conv_wgrad`` (x [256,16,64,64] * w [32,16,3,3], pad 1), ``cnn`` (crater-CNN
SGD step, global batch 4096, data parallel over N ranks with an NCCL
gradient allreduce: strong scaling; 3xTF32, ``cnn_tf32`` the TF32 form),
``sort`` / ``grade`` / ``filter`` (the reference's C runtime helpers on
2^26 f32 keys ~ N(0,1); filter keeps x > 0).

With N GPUs (torchrun, one process per GPU) every rank runs its own copy of
the workload (weak scaling: folds shard frames, matmuls shard rows; no
data-path collective); rank 0 prints the aggregate over max-over-ranks time.
``--impl reference`` times the CPU restatement of the reference's CPU path
(the oracle, OpenMP over all host threads) on a bounded sample of the same
workload and prints the same JSON line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC_FOLD = "map/fold HBM GB/s"
METRIC_MM = "matmul/conv TFLOP/s"
METRIC_RT = "runtime helpers HBM GB/s"


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled while the GPU is busy."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.rows: list[list[str]] = []
        self._proc = None
        self._thread = None

    def start(self) -> None:
        try:
            self._proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self._proc = None
            return

        def pump() -> None:
            assert self._proc is not None and self._proc.stdout is not None
            for line in self._proc.stdout:
                self.rows.append([c.strip() for c in line.split(",")])

        self._thread = threading.Thread(target=pump, daemon=True)
        self._thread.start()

    def stop(self) -> dict | None:
        if self._proc is None:
            return None
        self._proc.terminate()
        try:
            self._proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self._proc.kill()
        if self._thread:
            self._thread.join(timeout=2)
        busy = [r for r in self.rows if len(r) >= 10 and _num(r[4]) > 0]
        use = busy or self.rows
        if not use:
            return None
        sm = [_num(r[1]) for r in use]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in use:
            for name, v in zip(names, r[6:10]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(_num(r[2]) for r in use),
                "reasons": sorted(reasons), "samples": len(use)}


def _num(s: str) -> float:
    try:
        return float(s)
    except ValueError:
        return 0.0


def _oracle():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # noqa: E402  (checker and CPU baseline only)

    return oracle


# -------------------------------------------------------------- workloads
class FoldWorkload:
    """Cell-fold workloads: one fused map+fold kernel per call."""

    metric, unit, bound = METRIC_FOLD, "GB/s", "hbm"

    def __init__(self, name: str) -> None:
        from remora_b200.program import BinaryExpr, CmpExpr, SelectExpr, const, x

        self.name = name
        if name == "chained":
            self.shape = (64, 64, 64, 64)
            y = BinaryExpr("+", BinaryExpr("*", x(0), const(2.5)), const(1.0))
            self.premap = SelectExpr(CmpExpr(">", y, const(0.5)), y, const(0.0))
            self.epilogue = None
            self.desc = "chained_maps_fold f32[64,64,64,64] ~ N(0,1): select(x*2.5+1 > 0.5), fold + last axis"
        else:
            self.shape = (8192, 1024)
            self.premap = BinaryExpr("*", x(0), x(0))
            self.epilogue = "sqrt"
            self.desc = "row_norms f32[8192,1024] ~ U[-1,1]: sqrt(fold + (map x*x)) per row"
        self.n_in = int(np.prod(self.shape))
        self.n_out = int(np.prod(self.shape[:-1]))
        self.work_per_call = 4 * (self.n_in + self.n_out)  # algorithmic bytes
        self.rotate = 8

    def make_input(self, seed: int) -> np.ndarray:
        rng = np.random.Generator(np.random.PCG64(seed))
        if self.name == "chained":
            return rng.standard_normal(self.shape, dtype=np.float32)
        return rng.uniform(-1, 1, self.shape).astype(np.float32)

    def spec(self):
        from remora_b200.codegen import fold_spec

        return fold_spec(premap=self.premap, epilogue=self.epilogue)

    def setup(self, dev, rank: int) -> None:
        import torch

        from remora_b200 import _lib as L
        from remora_b200.abi import tensor_descriptor
        from remora_b200.runtime import context

        self.torch, self.L, self.lib = torch, L, L.lib()
        self.host = [self.make_input(1729 + 1000 * rank + k) for k in range(self.rotate)]
        self.xs = [torch.from_numpy(h).to(dev) for h in self.host]
        self.out = torch.empty(self.shape[:-1], dtype=torch.float32, device=dev)
        self.sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        self.ctx = context(dev.index)
        self._spec = self.spec()
        self.descs = [tensor_descriptor(t) for t in self.xs]
        self.out_desc = tensor_descriptor(self.out)
        self.ranks = (ctypes.c_int32 * 1)(len(self.shape))
        self.ptrs = [(ctypes.c_void_p * 1)(ctypes.addressof(d)) for d in self.descs]
        self.dev = dev

    def call(self, k: int) -> None:
        st = self.lib.remora_b200_fold(self.ctx.ptr, ctypes.byref(self._spec), self.ptrs[k], self.ranks, 1,
                                       ctypes.addressof(self.out_desc), len(self.shape) - 1, self.sptr)
        if st:
            self.L.check(st, "fold")

    def check(self) -> None:
        torch = self.torch
        self.call(0)
        torch.cuda.synchronize()
        x = self.xs[0]
        if self.name == "chained":
            y = x * 2.5 + 1.0
            ref = torch.where(y > 0.5, y, torch.zeros_like(y)).sum(-1)
        else:
            ref = (x * x).sum(-1).sqrt()
        if not torch.allclose(self.out, ref, rtol=1e-4, atol=1e-4):
            raise SystemExit("benchmark output does not match the check")

    def e2e_setup(self) -> tuple[int, int]:
        torch = self.torch
        from remora_b200.abi import tensor_descriptor

        self.pin_in = torch.from_numpy(self.host[0]).pin_memory()
        self.pin_out = torch.empty(self.shape[:-1], dtype=torch.float32).pin_memory()
        self.dbuf = torch.empty(self.shape, dtype=torch.float32, device=self.dev)
        self.dbuf_desc = tensor_descriptor(self.dbuf)
        self.dbuf_ptrs = (ctypes.c_void_p * 1)(ctypes.addressof(self.dbuf_desc))
        return self.pin_in.numel() * 4, self.pin_out.numel() * 4

    def e2e_step(self) -> None:
        L, lib = self.L, self.lib
        L.check(lib.remora_b200_memcpy_h2d(self.ctx.ptr, ctypes.c_void_p(self.dbuf.data_ptr()),
                                           ctypes.c_void_p(self.pin_in.data_ptr()), self.pin_in.numel() * 4,
                                           self.sptr))
        L.check(lib.remora_b200_fold(self.ctx.ptr, ctypes.byref(self._spec), self.dbuf_ptrs, self.ranks, 1,
                                     ctypes.addressof(self.out_desc), len(self.shape) - 1, self.sptr))
        L.check(lib.remora_b200_memcpy_d2h(self.ctx.ptr, ctypes.c_void_p(self.pin_out.data_ptr()),
                                           ctypes.c_void_p(self.out.data_ptr()), self.pin_out.numel() * 4,
                                           self.sptr))

    # ---- CPU side (oracle)
    def cpu_prepare(self) -> None:
        self.cx = self.make_input(1729)
        o = _oracle()
        self.nt = o.max_threads()
        ref = o.compiled_fold(self.name, self.cx, nthreads=self.nt)
        chk = o.cell_fold(self.spec(), [self.cx], 1, nthreads=self.nt)
        if not np.array_equal(ref, chk):
            raise SystemExit("compiled CPU loop differs from the oracle interpreter")

    def cpu_step(self) -> float:
        """One bounded CPU sample; returns the algorithmic work it covered."""
        _oracle().compiled_fold(self.name, self.cx, nthreads=self.nt)
        return float(self.work_per_call)

    cpu_sample = "full workload per sample (compiled C loop of the oracle, sequential f32 cell folds, OpenMP over frames)"


class MatmulWorkload:
    """C = A . B on tcgen05: one library call per product (A K-major, B
    N-major as given, both native operand layouts)."""

    metric, unit, bound = METRIC_MM, "TFLOP/s", "tensor"

    def __init__(self, name: str) -> None:
        self.name = name
        self.precision = "3xtf32" if name == "matmul_3x" else "tf32"
        if name == "bmm":
            self.batch, self.M, self.N, self.K = 32, 1024, 1024, 1024
            self.desc = "batched matmul [32,1024,1024] x [32,1024,1024] f32 ~ U[-1,1], TF32 tcgen05, f32 accumulate"
        else:
            self.batch, self.M, self.N, self.K = 1, 4096, 4096, 4096
            self.desc = f"matmul A,B f32[4096,4096] ~ U[-1,1], {self.precision.upper()} tcgen05, f32 accumulate"
        self.work_per_call = 2.0 * self.batch * self.M * self.N * self.K  # algorithmic flops
        self.rotate = 1

    def shapes(self):
        if self.batch > 1:
            return (self.batch, self.M, self.K), (self.batch, self.K, self.N), (self.batch, self.M, self.N)
        return (self.M, self.K), (self.K, self.N), (self.M, self.N)

    def make_inputs(self, seed: int):
        sa, sb, _ = self.shapes()
        ra = np.random.Generator(np.random.PCG64(seed))
        rb = np.random.Generator(np.random.PCG64(seed + 1))
        return ra.uniform(-1, 1, sa).astype(np.float32), rb.uniform(-1, 1, sb).astype(np.float32)

    def setup(self, dev, rank: int) -> None:
        import torch

        from remora_b200 import _lib as L
        from remora_b200.abi import tensor_descriptor
        from remora_b200.runtime import context

        self.torch, self.L, self.lib, self.dev = torch, L, L.lib(), dev
        self.ha, self.hb = self.make_inputs(1729 + 1000 * rank)
        self.a = torch.from_numpy(self.ha).to(dev)
        self.b = torch.from_numpy(self.hb).to(dev)
        self.c = torch.empty(self.shapes()[2], dtype=torch.float32, device=dev)
        self.ad, self.bd, self.cd = (tensor_descriptor(t) for t in (self.a, self.b, self.c))
        self._spec = L.RemoraGemmSpec(L.PREC_TF32 if self.precision == "tf32" else L.PREC_3XTF32, 0)
        self.sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        self.ctx = context(dev.index)
        self.rank_ = len(self.shapes()[0])

    def call(self, k: int) -> None:
        st = self.lib.remora_b200_gemm(self.ctx.ptr, ctypes.byref(self._spec), ctypes.addressof(self.ad),
                                       ctypes.addressof(self.bd), ctypes.addressof(self.cd), self.rank_, self.sptr)
        if st:
            self.L.check(st, "gemm")

    def check(self) -> None:
        torch = self.torch
        self.call(0)
        torch.cuda.synchronize()
        a64 = self.a[..., :256, :].double()
        ref = torch.matmul(a64, self.b.double())
        got = self.c[..., :256, :].double()
        tol = 1e-3 if self.precision == "tf32" else 1e-4
        err = float((got - ref).abs().max()) / max(1.0, float(ref.abs().max()))
        if not err <= tol:
            raise SystemExit(f"benchmark output does not match the check (scaled error {err:.3g})")

    def e2e_setup(self) -> tuple[int, int]:
        torch = self.torch
        self.pa = torch.from_numpy(self.ha).pin_memory()
        self.pb = torch.from_numpy(self.hb).pin_memory()
        self.pc = torch.empty(self.shapes()[2], dtype=torch.float32).pin_memory()
        return (self.pa.numel() + self.pb.numel()) * 4, self.pc.numel() * 4

    def e2e_step(self) -> None:
        L, lib, c = self.L, self.lib, self.ctx.ptr
        L.check(lib.remora_b200_memcpy_h2d(c, ctypes.c_void_p(self.a.data_ptr()), ctypes.c_void_p(self.pa.data_ptr()),
                                           self.pa.numel() * 4, self.sptr))
        L.check(lib.remora_b200_memcpy_h2d(c, ctypes.c_void_p(self.b.data_ptr()), ctypes.c_void_p(self.pb.data_ptr()),
                                           self.pb.numel() * 4, self.sptr))
        self.call(0)
        L.check(lib.remora_b200_memcpy_d2h(c, ctypes.c_void_p(self.pc.data_ptr()), ctypes.c_void_p(self.c.data_ptr()),
                                           self.pc.numel() * 4, self.sptr))

    def cpu_prepare(self) -> None:
        self.ca, self.cb = self.make_inputs(1729)
        o = _oracle()
        self.nt = o.max_threads()
        self.rows = 64 if self.batch == 1 else 16

    def cpu_step(self) -> float:
        o = _oracle()
        if self.batch == 1:
            o.matmul(self.ca[: self.rows], self.cb, nthreads=self.nt)
        else:
            o.matmul(self.ca[0, : self.rows], self.cb[0], nthreads=self.nt)
        return 2.0 * self.rows * self.N * self.K

    @property
    def cpu_sample(self) -> str:
        return (f"{self.rows} output rows of one {self.M}x{self.N}x{self.K} product per sample (oracle lifted dot, "
                "sequential f32 k order, OpenMP over rows)")


class ConvWorkload:
    """The im2col-conv layer x [256,16,64,64] * w [32,16,3,3], pad 1, stride 1:
    forward (``conv``), input gradient (``conv_dgrad``) and weight gradient
    (``conv_wgrad``) from a seeded N(0,1) cotangent.  Metric TFLOP/s; the
    layer is HBM-bound (about 48 flop/B), so the roofline is HBM GB/s of
    algorithmic bytes."""

    metric, unit = METRIC_MM, "TFLOP/s"
    bound = "hbm"

    def __init__(self, name: str) -> None:
        self.name = name
        self.kind = {"conv": "fwd", "conv_dgrad": "dgrad", "conv_wgrad": "wgrad"}[name]
        self.N, self.C, self.H, self.W, self.K = 256, 16, 64, 64, 32
        self.work_per_call = 2.0 * self.N * self.H * self.W * self.K * self.C * 9  # 9,663,676,416 flop
        x_b = 4 * self.N * self.C * self.H * self.W
        y_b = 4 * self.N * self.K * self.H * self.W
        w_b = 4 * self.K * self.C * 9
        self.bytes_per_call = x_b + y_b + w_b  # each direction reads two of x/y/w and writes the third
        self.rotate = 1
        self.precision = "tf32"
        self.desc = (f"conv2d {self.kind} x[256,16,64,64] ~ N(0,1) * w[32,16,3,3] ~ N(0,sqrt(2/144)), pad 1, "
                     "TF32 tcgen05 implicit GEMM" if self.kind != "wgrad" else
                     "conv2d wgrad x[256,16,64,64], dy[256,32,64,64] ~ N(0,1) -> dw[32,16,3,3]")

    def make_inputs(self, seed: int):
        rx = np.random.Generator(np.random.PCG64(seed))
        x = rx.standard_normal((self.N, self.C, self.H, self.W), dtype=np.float32)
        w = (np.random.Generator(np.random.PCG64(2718)).standard_normal((self.K, self.C, 3, 3))
             * np.sqrt(2 / 144)).astype(np.float32)
        dy = np.random.Generator(np.random.PCG64(seed + 2)).standard_normal((self.N, self.K, self.H, self.W),
                                                                            dtype=np.float32)
        return x, w, dy

    def setup(self, dev, rank: int) -> None:
        import torch

        from remora_b200 import _lib as L
        from remora_b200.abi import tensor_descriptor
        from remora_b200.runtime import context

        self.torch, self.L, self.lib, self.dev = torch, L, L.lib(), dev
        self.hx, self.hw, self.hdy = self.make_inputs(1729 + 1000 * rank)
        self.x, self.w, self.dy = (torch.from_numpy(a).to(dev) for a in (self.hx, self.hw, self.hdy))
        self.y = torch.empty_like(self.dy)
        self.dx = torch.empty_like(self.x)
        self.dw = torch.empty_like(self.w)
        self.d = {k: tensor_descriptor(getattr(self, k)) for k in ("x", "w", "dy", "y", "dx", "dw")}
        self._spec = L.RemoraConvSpec(1, 1, L.PREC_TF32, 0)
        self.sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        self.ctx = context(dev.index)

    def call(self, k: int) -> None:
        a = lambda n: ctypes.addressof(self.d[n])  # noqa: E731
        lib, c, s = self.lib, self.ctx.ptr, ctypes.byref(self._spec)
        if self.kind == "fwd":
            st = lib.remora_b200_conv2d_fwd(c, s, a("x"), a("w"), None, a("y"), self.sptr)
        elif self.kind == "dgrad":
            st = lib.remora_b200_conv2d_dgrad(c, s, a("dy"), a("w"), a("dx"), self.sptr)
        else:
            st = lib.remora_b200_conv2d_wgrad(c, s, a("x"), a("dy"), a("dw"), self.sptr)
        if st:
            self.L.check(st, "conv")

    def check(self) -> None:
        torch = self.torch
        self.call(0)
        torch.cuda.synchronize()
        import torch.nn.functional as F

        x64, w64, dy64 = self.x[:2].double(), self.w.double(), self.dy[:2].double()
        if self.kind == "fwd":
            got, ref = self.y[:2].double(), F.conv2d(x64, w64, padding=1)
        elif self.kind == "dgrad":
            got, ref = self.dx[:2].double(), F.conv_transpose2d(dy64, w64, padding=1)
        else:
            got = self.dw.double()
            ref = torch.nn.grad.conv2d_weight(self.x.double(), self.w.shape, self.dy.double(), padding=1)
        err = float((got - ref).abs().max()) / max(1.0, float(ref.abs().max()))
        if not err <= 1e-3:
            raise SystemExit(f"benchmark output does not match the check (scaled error {err:.3g})")

    def e2e_setup(self) -> tuple[int, int]:
        torch = self.torch
        ins = {"fwd": ("x", "w"), "dgrad": ("dy", "w"), "wgrad": ("x", "dy")}[self.kind]
        outn = {"fwd": "y", "dgrad": "dx", "wgrad": "dw"}[self.kind]
        self.pin_in = [(getattr(self, n), torch.from_numpy(getattr(self, "h" + n)).pin_memory()) for n in ins]
        self.pin_out = (getattr(self, outn), torch.empty(getattr(self, outn).shape).pin_memory())
        return sum(p.numel() * 4 for _, p in self.pin_in), self.pin_out[1].numel() * 4

    def e2e_step(self) -> None:
        L, lib, c = self.L, self.lib, self.ctx.ptr
        for dev_t, pin in self.pin_in:
            L.check(lib.remora_b200_memcpy_h2d(c, ctypes.c_void_p(dev_t.data_ptr()), ctypes.c_void_p(pin.data_ptr()),
                                               pin.numel() * 4, self.sptr))
        self.call(0)
        dev_t, pin = self.pin_out
        L.check(lib.remora_b200_memcpy_d2h(c, ctypes.c_void_p(pin.data_ptr()), ctypes.c_void_p(dev_t.data_ptr()),
                                           pin.numel() * 4, self.sptr))

    def cpu_prepare(self) -> None:
        self.cx, self.cw, self.cdy = self.make_inputs(1729)
        self.nt = _oracle().max_threads()

    def cpu_step(self) -> float:
        o = _oracle()
        if self.kind == "fwd":
            o.conv2d_fwd(self.cx[:1], self.cw, None, nthreads=self.nt)
        elif self.kind == "dgrad":
            o.conv2d_dgrad(self.cdy[:1], self.cw, (1, self.C, self.H, self.W), nthreads=self.nt)
        else:
            o.conv2d_wgrad(self.cx[:1], self.cdy[:1], self.cw.shape, nthreads=self.nt)
        return self.work_per_call / self.N

    cpu_sample = "one image of the batch per sample (oracle conv in the reference's order, OpenMP over channels)"


class CnnWorkload:
    """One SGD step of the crater CNN on a global batch of 4096 synthetic
    64x64 images (data parallel: each of N ranks takes 4096/N, one NCCL
    allreduce of the 529,217-float gradient per step).  Metric samples/s of
    the whole job; the step is one CUDA graph."""

    metric, unit, bound = "CNN train samples/s", "samples/s", "tensor"
    scaling = "strong"
    GLOBAL = 4096
    OVERLAP = None  # the step's own choice
    FLOPS_PER_SAMPLE = 33.8e6  # forward + backward, all layers

    def __init__(self, name: str) -> None:
        self.name = name
        self.rotate = 1
        self.precision = "tf32" if name == "cnn_tf32" else "3xtf32"
        self.desc = (f"crater CNN train step ({self.precision}), global batch 4096 of 64x64 synthetic images (noise 0.1, 1-3 rims r 4-16 "
                     "on positives, 50/50): conv3x3 1->16+ReLU, pool, conv3x3 16->32+ReLU, pool, dense 8192->64+ReLU, "
                     "dense 64->1, sigmoid BCE, SGD lr 0.01")

    def setup(self, dev, rank: int) -> None:
        import torch

        from remora_b200 import crater
        from remora_b200.cnn import CraterCNN

        from remora_b200.cnn import process_group_allreduce, shard

        world = getattr(self, "world", 1)
        self.torch, self.dev = torch, dev
        self.desc = self.desc.replace("global batch 4096", f"global batch {self.GLOBAL}")
        lo, hi = shard(self.GLOBAL, world, rank)
        self.B = hi - lo
        self.work_per_call = float(self.B)  # samples per rank per step; x world in the harness
        self.himg, self.hlab = crater.make_batch(self.B, start=lo)
        self.x = torch.from_numpy(self.himg).to(dev)
        self.y = torch.from_numpy(self.hlab).to(dev)
        allreduce = process_group_allreduce() if world > 1 else None
        self.net = CraterCNN(dev, self.B, self.GLOBAL, lr=0.01, allreduce=allreduce, precision=self.precision,
                             overlap_allreduce=self.OVERLAP)
        self.net.step(self.x, self.y)  # eager step: compiles map programs, sizes workspaces
        self.net.capture(self.x, self.y)
        # library kernels in one replay of the step's graph, counted at capture
        self.graph_launches_per_call = self.net.graph_launches

    def call(self, k: int) -> None:
        self.net.replay()

    def close(self) -> None:
        self.net.graph = None
        self.torch.cuda.synchronize()

    def check(self) -> None:
        self.torch.cuda.synchronize()
        if not bool(self.torch.isfinite(self.net.params).all()):
            raise SystemExit("non-finite parameters after the warm-up steps")

    def e2e_setup(self) -> tuple[int, int]:
        torch = self.torch
        self.pin_x = torch.from_numpy(self.himg).pin_memory()
        self.pin_y = torch.from_numpy(self.hlab).pin_memory()
        self.pin_loss = torch.empty(self.B, dtype=torch.float32).pin_memory()
        return (self.pin_x.numel() + self.pin_y.numel()) * 4, 4

    def e2e_step(self) -> None:
        self.x.copy_(self.pin_x, non_blocking=True)
        self.y.copy_(self.pin_y, non_blocking=True)
        self.net.replay()
        self.pin_loss[:1].copy_(self.net.loss_b[:1], non_blocking=True)  # the step's result read back

    def cpu_prepare(self) -> None:
        from remora_b200 import crater

        self.cparams = crater.init_params()
        self.cimg, self.clab = crater.make_batch(32)
        self.nt = _oracle().max_threads()

    def cpu_step(self) -> float:
        _oracle().cnn_step(self.cparams, self.cimg, self.clab, batch_total=32, nthreads=self.nt)
        return 32.0

    cpu_sample = "32 samples per SGD step (oracle CNN step: forward, backward, update; OpenMP over images)"


class RuntimeWorkload:
    """The reference's C runtime helpers (remora/remora_rt.c) on 2^26 f32
    keys ~ N(0,1) (268 MB, larger than L2): sort, grade, or filter (x > 0).
    `value` counts the bytes the operation must move at least (keys in,
    result out); the roofline counts the traffic of the implementation's
    passes (LSD sort: 4 passes, each reading the keys twice and writing them
    once, plus the indices for grade; filter: two reads, one write of the
    kept half)."""

    metric, unit, bound = METRIC_RT, "GB/s", "hbm"

    def __init__(self, name: str) -> None:
        self.name = name
        self.n = 1 << 26
        n = self.n
        if name == "sort":
            self.work_per_call = 8 * n
            self.bytes_per_call = 4 * 12 * n
        elif name == "grade":
            self.work_per_call = 8 * n
            # pass 0: 4 (count) + 4 (keys) + 8 (keys, indices out); passes 1-2:
            # 4 + 8 + 8; pass 3: 4 + 8 + 4 (indices only)
            self.bytes_per_call = 16 * n + 2 * 20 * n + 16 * n
        else:
            self.work_per_call = 4 * n + 2 * n  # read all, write the kept half
            self.bytes_per_call = 4 * n + 4 * n + 2 * n
        self.desc = f"{name} f32[{n}] ~ N(0,1)" + (" keeping x > 0" if name == "filter" else "")
        self.rotate = 1

    def setup(self, dev, rank: int) -> None:
        import torch

        from remora_b200 import _lib as L
        from remora_b200.abi import tensor_descriptor
        from remora_b200.runtime import context

        self.torch, self.L, self.lib, self.dev = torch, L, L.lib(), dev
        rng = np.random.Generator(np.random.PCG64(1729 + 1000 * rank))
        self.host = rng.standard_normal(self.n, dtype=np.float32)
        self.x = torch.from_numpy(self.host).to(dev)
        self.out = torch.empty(self.n, dtype=torch.int32 if self.name == "grade" else torch.float32, device=dev)
        self.count = torch.zeros((), dtype=torch.int64, device=dev)
        self.ctx = context(dev.index)
        self.sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        self.xd, self.od, self.cd = (tensor_descriptor(t) for t in (self.x, self.out, self.count))
        self.pred = L.RemoraFilterPred(L.OP_GT, 0.0, 0, 0)

    def _run(self, xd) -> None:
        lib, a = self.lib, ctypes.addressof
        if self.name == "sort":
            st = lib.remora_b200_sort(self.ctx.ptr, self.L.F32, a(xd), a(self.od), 1, self.sptr)
        elif self.name == "grade":
            st = lib.remora_b200_grade(self.ctx.ptr, self.L.F32, a(xd), a(self.od), 1, self.sptr)
        else:
            st = lib.remora_b200_filter(self.ctx.ptr, self.L.F32, a(xd), None, 0, ctypes.byref(self.pred), a(self.od),
                                        a(self.cd), self.sptr)
        if st:
            self.L.check(st, self.name)

    def call(self, k: int) -> None:
        self._run(self.xd)

    def check(self) -> None:
        torch = self.torch
        self.call(0)
        torch.cuda.synchronize()
        if self.name == "sort":
            ok = torch.equal(self.out, torch.sort(self.x)[0])
        elif self.name == "grade":
            ok = torch.equal(self.x[self.out.long()], torch.sort(self.x)[0])
        else:
            ref = self.x[self.x > 0]
            ok = int(self.count.item()) == ref.numel() and torch.equal(self.out[: ref.numel()], ref)
        if not ok:
            raise SystemExit("benchmark output does not match the check")

    def e2e_setup(self) -> tuple[int, int]:
        from remora_b200.abi import tensor_descriptor

        torch = self.torch
        self.pin_in = torch.from_numpy(self.host).pin_memory()
        self.pin_out = torch.empty(self.n, dtype=self.out.dtype).pin_memory()
        self.dbuf = torch.empty(self.n, dtype=torch.float32, device=self.dev)
        self.dbuf_desc = tensor_descriptor(self.dbuf)
        return self.n * 4, self.n * 4

    def e2e_step(self) -> None:
        L, lib = self.L, self.lib
        L.check(lib.remora_b200_memcpy_h2d(self.ctx.ptr, ctypes.c_void_p(self.dbuf.data_ptr()),
                                           ctypes.c_void_p(self.pin_in.data_ptr()), self.n * 4, self.sptr))
        self._run(self.dbuf_desc)
        L.check(lib.remora_b200_memcpy_d2h(self.ctx.ptr, ctypes.c_void_p(self.pin_out.data_ptr()),
                                           ctypes.c_void_p(self.out.data_ptr()), self.n * 4, self.sptr))

    # ---- CPU side: remora_rt.c itself where it was compiled, else the oracle
    def cpu_prepare(self) -> None:
        o = _oracle()
        self.o = o
        self.cn = 1 << 22
        self.cx = np.random.Generator(np.random.PCG64(1729)).standard_normal(self.cn, dtype=np.float32)
        self.cmask = (self.cx > 0).astype(np.int32)
        self.cpu_kind = "reference" if o.ref_available() else "port"
        self.nt = 1
        src = "remora_rt.c compiled from the reference source" if self.cpu_kind == "reference" else "the oracle port"
        self.cpu_sample = f"{self.cn} keys per sample ({src}, one thread, as remora_rt.c is sequential)"

    def cpu_step(self) -> float:
        o, ref = self.o, self.cpu_kind == "reference"
        if self.name == "sort":
            (o.ref_sort if ref else o.sort)(self.cx)
        elif self.name == "grade":
            (o.ref_grade if ref else o.grade)(self.cx)
        elif ref:
            o.ref_filter(self.cx, self.cmask)
        else:
            o.filter_(self.cx, self.cmask)
        return float(self.work_per_call) * self.cn / self.n


def make_workload(name: str):
    if name in ("chained", "row_norms"):
        return FoldWorkload(name)
    if name in ("cnn", "cnn_tf32"):
        return CnnWorkload(name)
    if name.startswith("conv"):
        return ConvWorkload(name)
    if name in ("sort", "grade", "filter"):
        return RuntimeWorkload(name)
    return MatmulWorkload(name)


def tf32_peak(peaks: dict, power_capped: bool = False) -> float:
    # Dense TF32 on B200 runs at half the bf16 tensor rate: peak = measured
    # cuBLAS bf16 / 2.  A kernel that ran under the power cap (sw_power_cap
    # active in the clock samples of the timed region) is held to the
    # sustained bf16 figure, one timed alone at full clocks to the burst one.
    return (peaks["bf16_tflops_sustained"] if power_capped else peaks["bf16_tflops"]) / 2.0


# --------------------------------------------------------------- harness
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    wl = make_workload(args.config)
    wl.world = world
    if isinstance(wl, CnnWorkload):
        wl.GLOBAL = args.cnn_batch
        wl.OVERLAP = False if args.cnn_serial_allreduce else None
    wl.setup(dev, rank)
    wl.check()
    stream = torch.cuda.current_stream(dev)

    for _ in range(args.warmup):
        for k in range(wl.rotate):
            wl.call(k)
    torch.cuda.synchronize()
    sampler = ClockSampler(local) if rank == 0 and not args.profile else None
    if sampler:
        sampler.start()
    # keep the GPU busy ~1 s before the timed region so clocks are steady and
    # the sampler sees the load the timed region runs under.  The number of
    # passes is agreed over the ranks first: a step may hold a collective
    # (the CNN's gradient allreduce), so every rank must run the same count.
    t0 = time.perf_counter()
    for k in range(wl.rotate):
        wl.call(k)
    torch.cuda.synchronize()
    one = max(time.perf_counter() - t0, 1e-6)
    soak = 0 if args.profile else int(min(2000, max(1, 1.0 / one)))
    if world > 1:
        n = torch.tensor([soak], dtype=torch.int64, device=dev)
        dist.all_reduce(n, op=dist.ReduceOp.MIN)
        soak = int(n.item())
    for _ in range(soak):
        for k in range(wl.rotate):
            wl.call(k)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    from remora_b200 import _lib as L

    n_launch0 = L.launch_count()
    t0.record(stream)
    for s in range(args.steps):
        ev[s][0].record(stream)
        for k in range(wl.rotate):
            wl.call(k)
        ev[s][1].record(stream)
    t1.record(stream)
    # library kernels enqueued in the timed region: counted at each launch
    # site, plus those a graph replay launches (counted when it was captured)
    n_launch = L.launch_count() - n_launch0 + args.steps * wl.rotate * getattr(wl, "graph_launches_per_call", 0)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_time(t1)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    clocks = sampler.stop() if sampler else None
    if args.profile:
        if world > 1:
            getattr(wl, "close", lambda: None)()
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"profile_run": args.config, "ms": ms, "steps": args.steps}), flush=True)
        return

    h2d, d2h = wl.e2e_setup()
    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(2):
        wl.e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        wl.e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    times = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.barrier()
    ms, e2e_ms = (float(v) for v in times.cpu())

    if rank == 0:
        peaks = measured_peaks()
        scale = {"GB/s": 1e9, "TFLOP/s": 1e12, "samples/s": 1.0}[wl.unit]
        calls = args.steps * wl.rotate
        value = wl.work_per_call * calls * world / (ms * 1e-3) / scale
        per_call_ms = float(np.mean(step_ms)) / wl.rotate
        # roofline of the dominant kernel: algorithmic bytes for HBM-bound
        # work, algorithmic flops for tensor-bound work
        capped = bool(clocks) and "sw_power_cap" in clocks.get("reasons", [])
        if wl.unit == "samples/s":
            # the whole step against the dense TF32 rate: model flops per step
            roof_unit, peak = "TFLOP/s", tf32_peak(peaks, capped)
            achieved = wl.work_per_call * wl.FLOPS_PER_SAMPLE / (per_call_ms * 1e-3) / 1e12
        elif wl.bound == "hbm":
            roof_unit, peak = "GB/s", peaks["hbm_gbs"]
            achieved = getattr(wl, "bytes_per_call", wl.work_per_call) / (per_call_ms * 1e-3) / 1e9
        else:
            roof_unit, peak = "TFLOP/s", tf32_peak(peaks, capped)
            achieved = wl.work_per_call / (per_call_ms * 1e-3) / 1e12
        e2e_value = wl.work_per_call * e2e_steps * world / (e2e_ms * 1e-3) / scale
        line = {
            "metric": wl.metric,
            "value": round(value, 2),
            "unit": wl.unit,
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True,
            "scaling": getattr(wl, "scaling", "weak"),
            "vs_baseline": None,
            "dtype": "f32" if not hasattr(wl, "precision") else f"f32 storage, {wl.precision} tensor math",
            "data": "synthetic (seeded PCG64)",
            "config": {"workload": wl.desc, "calls_per_step": wl.rotate,
                       "l2": (f"{wl.rotate} rotating inputs, {wl.rotate * wl.work_per_call / 1e6:.0f} MB > 126 MB L2"
                              if wl.unit == "GB/s" else "operands larger than the 126 MB L2"),
                       "parallelism": (f"dp{world} (NCCL gradient allreduce)" if wl.unit == "samples/s" else
                                       f"replicas x{world} (independent shards, no collective)")},
            "roofline": {"bound": wl.bound, "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": roof_unit,
                         "frac": round(achieved / peak, 4), "traffic": TRAFFIC.get(args.config),
                         "peak_source": peaks["source"] + (
                             (" bf16 sustained / 2 (ran under sw_power_cap)" if capped else " bf16 burst / 2")
                             if roof_unit == "TFLOP/s" else " HBM copy")},
            "e2e": {"value": round(e2e_value, 3), "unit": wl.unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": n_launch,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(wl, budget_s=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        getattr(wl, "close", lambda: None)()  # graphs holding NCCL calls go before the process group
        dist.barrier()
        dist.destroy_process_group()


# Per-call DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of the
# dominant kernel, from ncu captures of the same bench commands.
TRAFFIC: dict[str, float | None] = {"chained": 67_127_040 + 637_952, "row_norms": None,
                                    "matmul": 335_706_368 + 61_118_208, "matmul_3x": None, "bmm": None,
                                    "conv": 67_187_968 + 75_173_120, "conv_dgrad": 134_268_160 + 33_349_888,
                                    "conv_wgrad": 201_346_304 + 4_110_848, "cnn": None, "cnn_tf32": None,
                                    # a sort or filter call is several kernels: no single figure
                                    "sort": None, "grade": None, "filter": None}


def cpu_baseline(wl, budget_s: float = 8.0) -> dict:
    """The oracle (CPU restatement of the reference's CPU loop order), OpenMP
    over all host threads, repeated on bounded samples for ~budget_s."""
    wl.cpu_prepare()
    wl.cpu_step()
    work = 0.0
    reps = 0
    t0 = time.perf_counter()
    while True:
        work += wl.cpu_step()
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    scale = {"GB/s": 1e9, "TFLOP/s": 1e12, "samples/s": 1.0}[wl.unit]
    return {"value": round(work / el / scale, 5), "unit": wl.unit, "cores": wl.nt,
            "kind": getattr(wl, "cpu_kind", "port"),
            "sample": f"{wl.cpu_sample}; {reps} samples in {el:.1f} s"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    wl = make_workload(args.config)
    wl.cpu_prepare()
    for _ in range(max(1, args.warmup)):
        wl.cpu_step()
    work = 0.0
    t0 = time.perf_counter()
    for _ in range(args.steps):
        work += wl.cpu_step()
    el = time.perf_counter() - t0
    scale = {"GB/s": 1e9, "TFLOP/s": 1e12, "samples/s": 1.0}[wl.unit]
    value = work / el / scale
    line = {
        "metric": wl.metric, "value": round(value, 5), "unit": wl.unit,
        "n_gpus": int(os.environ.get("WORLD_SIZE", 1)), "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(el * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": getattr(wl, "scaling", "weak"),
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded PCG64)", "impl": "reference",
        "config": {"workload": wl.desc, "calls_per_step": 1},
        "cpu_baseline": {"value": round(value, 5), "unit": wl.unit, "cores": wl.nt,
                         "kind": getattr(wl, "cpu_kind", "port"),
                         "sample": f"{wl.cpu_sample}; one sample per step, {args.steps} steps"},
        "e2e": {"value": round(value, 5), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


CONFIGS = ["chained", "row_norms", "matmul", "matmul_3x", "bmm", "conv", "conv_dgrad", "conv_wgrad", "cnn", "cnn_tf32",
           "sort", "grade", "filter"]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="chained", choices=CONFIGS)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cnn-serial-allreduce", action="store_true",
                    help="CNN: always one gradient allreduce after the backward (by default the dense "
                         "layers' bucket overlaps the conv backward when a rank holds >= 1024 images)")
    ap.add_argument("--cnn-batch", type=int, default=4096,
                    help="global batch of the cnn configs (4096 is the benchmark; smaller ones show the per-rank "
                         "work of a larger data-parallel job)")
    ap.add_argument("--profile", action="store_true",
                    help="warm-up and timed steps only (no soak, e2e or CPU baseline): the ncu capture command")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
