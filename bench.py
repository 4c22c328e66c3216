"""Benchmark of the B200 backend on the Remora hot-path workloads.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

Default workload (``--config cnn``): one SGD step of the crater CNN on a
global batch of 4096 synthetic 64x64 images (conv3x3 1->16 + ReLU, pool,
conv3x3 16->32 + ReLU, pool, dense 8192->64 + ReLU, dense 64->1, sigmoid BCE,
SGD lr 0.01), in samples/s of the whole job.  Tensor-core math is mixed:
3xTF32 for the forward convolution and the dense layers, 2xTF32 for the
convolution's two gradients, every gradient within 1e-3 of the f32 step.  With
N GPUs (torchrun, one process per GPU) the batch is split 4096/N per rank and
the gradient (529,217 f32) is summed by an NCCL allreduce inside the step's
CUDA graph: strong scaling, the only workload here with a collective.  The
roofline is that of the step's dominant stage, each stage timed alone.

Other configs: ``chained`` (the fused chained-map fold f32[64,64,64,64] ~
N(0,1): y = x*2.5 + 1.0, mask y > 0.5 ? y : 0, fold (+) over the last axis,
in HBM GB/s over a rotation of 8 distinct inputs, 545 MB > 126 MB L2),
``row_norms`` (f32[8192,1024] -> sqrt(sum x*x)), ``matmul`` (A,B
f32[4096,4096], TF32; ``matmul_3x`` the 3xTF32 form), ``bmm``
([32,1024,1024] x [32,1024,1024], TF32), ``conv`` / ``conv_dgrad`` /
``conv_wgrad`` (x [256,16,64,64] * w [32,16,3,3], pad 1), ``cnn_3x`` (the
CNN step with 3xTF32 everywhere), ``cnn_tf32`` (the
CNN step in plain TF32, outside the 1e-3 gradient tolerance: a speed
reference only), ``scan`` (inclusive + scan of 2^28 f32), ``sort`` /
``grade`` / ``filter`` (the reference's C runtime helpers on 2^26 f32 keys ~
N(0,1); filter keeps x > 0).  Those run as independent replicas when N > 1
(weak scaling: folds shard frames, matmuls shard rows; no collective).

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
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "sm_max_mhz": float(d.get("sm_max_mhz", 1965.0)), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0,
            "source": "fallback"}


def simt_f32_peak(peaks: dict, sm_count: int) -> float:
    """Nominal f32 rate of the CUDA cores in TFLOP/s: 128 f32 lanes per SM,
    one fused multiply-add (2 flops) per lane and clock, at the maximum SM
    clock."""
    return sm_count * 128 * 2 * peaks["sm_max_mhz"] * 1e6 / 1e12


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
        # nvidia-smi can take a second or more to print its first line on a
        # fresh box: wait (bounded) for it, so that a short timed region
        # still falls inside the sampled window
        t0 = time.perf_counter()
        while not self.rows and time.perf_counter() - t0 < 5.0 and self._proc.poll() is None:
            time.sleep(0.05)

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
        if not self.rows:
            # the sampler printed nothing in the window: one query right
            # after the timed region is the closest record left
            try:
                out = subprocess.run(
                    ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"],
                    capture_output=True, text=True, timeout=10).stdout
                self.rows = [[c.strip() for c in line.split(",")] for line in out.splitlines() if line.strip()]
            except (FileNotFoundError, OSError, subprocess.TimeoutExpired):
                pass
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
    RESERVE = None  # SMs left to the overlapped allreduce (None: the step's own choice)
    FLOPS_PER_SAMPLE = 33.8e6  # forward + backward, all layers

    # Algorithmic work per image of each stage of the step (CraterCNN.stages):
    # (flops, bytes, runs on the tensor cores).  Bytes count each operand and
    # result once: conv2 reads p1 [16,32,32] (65,536 B) and writes the pooled
    # [32,16,16] f32 (32,768 B) plus its pool codes (8,192 B); its two
    # gradients read the pooled gradient and codes and write or read p1.
    STAGE_WORK = {
        "conv1_fwd": (2 * 4096 * 16 * 9, 16384 + 65536 + 16384, False),
        "conv2_fwd": (2 * 1024 * 32 * 144, 65536 + 32768 + 8192, True),
        "dense1_fwd": (2 * 8192 * 64, 32768 + 256, True),
        "head": (4 * 64 + 16, 256 * 2 + 16, False),
        "head_bwd": (6 * 64, 256 * 2 + 8, False),
        "dense1_wgrad": (2 * 8192 * 64, 32768 + 256, True),
        "dense1_dgrad": (2 * 8192 * 64, 32768 + 256, True),
        "conv2_wgrad": (2 * 1024 * 32 * 144, 65536 + 32768 + 8192, True),
        "conv2_dgrad": (2 * 1024 * 16 * 288, 32768 + 8192 + 65536, True),
        "conv1_wgrad": (2 * 4096 * 16 * 9, 16384 + 65536 + 16384, False),
    }

    def __init__(self, name: str) -> None:
        self.name = name
        self.rotate = 1
        self.precision = {"cnn": "mixed", "cnn_3x": "3xtf32", "cnn_tf32": "tf32"}[name]
        self.desc = (f"crater CNN train step ({self.precision}), global batch 4096 of 64x64 synthetic images (noise 0.1, 1-3 rims r 4-16 "
                     "on positives, 50/50): conv3x3 1->16+ReLU, pool, conv3x3 16->32+ReLU, pool, dense 8192->64+ReLU, "
                     "dense 64->1, sigmoid BCE, SGD lr 0.01")

    def setup(self, dev, rank: int) -> None:
        import torch

        from remora_b200 import crater
        from remora_b200.cnn import CraterCNN, process_group_allreduce, shard

        world = getattr(self, "world", 1)
        self.torch, self.dev = torch, dev
        self.desc = self.desc.replace("global batch 4096", f"global batch {self.GLOBAL}")
        lo, hi = shard(self.GLOBAL, world, rank)
        self.B = hi - lo
        self.work_per_call = float(self.B)  # samples per rank per step; x world in the harness
        self.himg, self.hlab = crater.make_batch(self.B, start=lo)
        # two input buffers: the end-to-end run copies step k+1's batch into
        # one while step k reads the other (one captured graph per buffer)
        self.xs = [torch.from_numpy(self.himg).to(dev) for _ in range(2)]
        self.ys = [torch.from_numpy(self.hlab).to(dev) for _ in range(2)]
        allreduce = process_group_allreduce() if world > 1 else None
        kw = {} if self.RESERVE is None else {"reserve_sms": self.RESERVE}
        self.net = CraterCNN(dev, self.B, self.GLOBAL, lr=0.01, allreduce=allreduce, precision=self.precision,
                             overlap_allreduce=self.OVERLAP, **kw)
        self.net.step(self.xs[0], self.ys[0])  # eager step: compiles map programs, sizes workspaces
        self.gid = [self.net.capture(self.xs[k], self.ys[k]) for k in range(2)]
        # library kernels in one replay of the step's graph, counted at capture
        self.graph_launches_per_call = self.net.graph_launches

    def call(self, k: int) -> None:
        self.net.replay(self.gid[0])

    def close(self) -> None:
        self.net.release_graphs()
        self.torch.cuda.synchronize()

    def check(self) -> None:
        self.torch.cuda.synchronize()
        if not bool(self.torch.isfinite(self.net.params).all()):
            raise SystemExit("non-finite parameters after the warm-up steps")

    def stage_times(self, peaks: dict, reps: int = 10) -> dict:
        """Each stage of the step timed alone on this rank (a CUDA graph of
        `reps` calls, CUDA events on the launching stream, after one warm-up
        replay) with its roofline: the largest of the HBM time of its bytes,
        the tensor time of its flops (tensor-core stages) and their f32 time
        on the CUDA cores (the others).  3xTF32 issues three TF32 products
        per product and 2xTF32 two, so their tensor peaks are a third and a
        half of the TF32 rate; the mixed step runs its forward and GEMMs in
        3xTF32 and the conv layer's gradients in 2xTF32."""
        torch = self.torch
        stream = torch.cuda.current_stream(self.dev)
        tf32 = tf32_peak(peaks) * 1e12
        simt = simt_f32_peak(peaks, torch.cuda.get_device_properties(self.dev).multi_processor_count) * 1e12
        out = {}
        for name, (fl, by, tensor) in self.STAGE_WORK.items():
            mult = self.tf32_products(name)
            graph, keep = self.net.stage_graph(name, self.xs[0], self.ys[0], reps)
            graph.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            graph.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            flops, nbytes = fl * self.B, by * self.B
            t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9)
            t_tc = mult * flops / tf32 if tensor else 0.0
            t_simt = 0.0 if tensor else flops / simt
            bound = "tensor" if t_tc > t_hbm else "simt" if t_simt > t_hbm else "hbm"
            if bound == "tensor":
                achieved, peak, unit = flops / (ms * 1e-3) / 1e12, tf32 / mult / 1e12, "TFLOP/s"
            elif bound == "simt":
                achieved, peak, unit = flops / (ms * 1e-3) / 1e12, simt / 1e12, "TFLOP/s"
            else:
                achieved, peak, unit = nbytes / (ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
            out[name] = {"ms": round(ms, 5), "bound": bound, "achieved": round(achieved, 1), "peak": round(peak, 1),
                         "unit": unit, "frac": round(achieved / peak, 4), "flops": flops, "bytes": nbytes}
            del graph, keep
        return out

    def tf32_products(self, stage: str) -> float:
        """TF32 tensor-core products per product of a stage's arithmetic."""
        if self.precision == "tf32":
            return 1.0
        if self.precision == "mixed" and stage in ("conv2_wgrad", "conv2_dgrad"):
            return 2.0
        return 3.0

    def e2e_setup(self) -> tuple[int, int]:
        torch = self.torch
        self.pin_x = torch.from_numpy(self.himg).pin_memory()
        self.pin_y = torch.from_numpy(self.hlab).pin_memory()
        self.pin_loss = torch.empty(2, dtype=torch.float32).pin_memory()
        self.copy_stream = torch.cuda.Stream(self.dev)
        self.e2e_k = 0
        self.step_done = [None, None]
        return (self.pin_x.numel() + self.pin_y.numel()) * 4, 4

    def _h2d(self, buf: int):
        """Host->device copy of a step's batch into input buffer `buf` on the
        copy stream, after the step that last read that buffer."""
        torch = self.torch
        with torch.cuda.stream(self.copy_stream):
            if self.step_done[buf] is not None:
                self.copy_stream.wait_event(self.step_done[buf])
            self.xs[buf].copy_(self.pin_x, non_blocking=True)
            self.ys[buf].copy_(self.pin_y, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
        return ev

    def e2e_begin(self) -> None:
        """Start of a timed end-to-end run: the first step's batch is copied
        inside the timed region like every other."""
        self.e2e_k = 0
        self.ready = self._h2d(0)

    def e2e_step(self) -> None:
        """Step k on input buffer k % 2, with step k+1's batch copied into the
        other buffer meanwhile; the step's loss is read back to host."""
        torch = self.torch
        cur = torch.cuda.current_stream(self.dev)
        buf = self.e2e_k % 2
        cur.wait_event(self.ready)
        self.net.replay(self.gid[buf])
        done = torch.cuda.Event()
        done.record(cur)
        self.step_done[buf] = done
        self.ready = self._h2d(1 - buf)
        self.pin_loss[:1].copy_(self.net.loss_b[:1], non_blocking=True)  # the step's result read back
        self.e2e_k += 1

    def cpu_prepare(self) -> None:
        from remora_b200 import crater

        self.cparams = crater.init_params()
        self.cimg, self.clab = crater.make_batch(32)
        self.nt = _oracle().max_threads()

    def cpu_step(self) -> float:
        _oracle().cnn_step(self.cparams, self.cimg, self.clab, batch_total=32, nthreads=self.nt)
        return 32.0

    cpu_sample = "32 samples per SGD step (oracle CNN step: forward, backward, update; OpenMP over images)"


class ScanWorkload:
    """Inclusive + scan of 2^28 f32 ~ U[-1,1] along the leading axis (the
    reference's rank-1 scan, remora/lowering/tensor_ops.py:2301-2482): 1 GiB
    in and 1 GiB out, larger than L2.  `value` counts the algorithmic 8 B per
    element (read once, write once); the reduce-then-scan implementation
    reads the input twice (12 B per element), which the roofline counts."""

    metric, unit, bound = METRIC_FOLD, "GB/s", "hbm"

    def __init__(self, name: str) -> None:
        self.name = name
        self.n = 1 << 28
        self.work_per_call = 8 * self.n
        self.bytes_per_call = 12 * self.n
        self.rotate = 1
        self.desc = f"inclusive + scan f32[{self.n}] ~ U[-1,1]"

    def setup(self, dev, rank: int) -> None:
        import torch

        from remora_b200 import _lib as L
        from remora_b200.abi import tensor_descriptor
        from remora_b200.codegen import scan_spec
        from remora_b200.runtime import context

        self.torch, self.L, self.lib, self.dev = torch, L, L.lib(), dev
        g = torch.Generator(device=dev)
        g.manual_seed(1729 + 1000 * rank)
        self.x = torch.rand(self.n, generator=g, device=dev, dtype=torch.float32) * 2 - 1
        self.out = torch.empty_like(self.x)
        self.ctx = context(dev.index)
        self.sptr = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        self._spec = scan_spec(op="+", init=0.0)
        self.xd, self.od = tensor_descriptor(self.x), tensor_descriptor(self.out)

    def call(self, k: int) -> None:
        st = self.lib.remora_b200_scan(self.ctx.ptr, ctypes.byref(self._spec), ctypes.addressof(self.xd),
                                       ctypes.addressof(self.od), 1, self.sptr)
        if st:
            self.L.check(st, "scan")

    def check(self) -> None:
        torch = self.torch
        self.call(0)
        torch.cuda.synchronize()
        ref = torch.cumsum(self.x[: 1 << 20].double(), 0)
        got = self.out[: 1 << 20].double()
        err = float((got - ref).abs().max())
        if not err <= 1e-5 * float(ref.abs().max()) + 1e-3:
            raise SystemExit(f"benchmark output does not match the check (error {err:.3g})")

    def e2e_setup(self) -> tuple[int, int]:
        torch = self.torch
        self.pin_in = self.x.cpu().pin_memory()
        self.pin_out = torch.empty(self.n, dtype=torch.float32).pin_memory()
        return self.n * 4, self.n * 4

    def e2e_step(self) -> None:
        L, lib = self.L, self.lib
        L.check(lib.remora_b200_memcpy_h2d(self.ctx.ptr, ctypes.c_void_p(self.x.data_ptr()),
                                           ctypes.c_void_p(self.pin_in.data_ptr()), self.n * 4, self.sptr))
        self.call(0)
        L.check(lib.remora_b200_memcpy_d2h(self.ctx.ptr, ctypes.c_void_p(self.pin_out.data_ptr()),
                                           ctypes.c_void_p(self.out.data_ptr()), self.n * 4, self.sptr))

    def cpu_prepare(self) -> None:
        from remora_b200.codegen import scan_spec

        self.cn = 1 << 24
        self.cx = np.random.Generator(np.random.PCG64(1729)).uniform(-1, 1, self.cn).astype(np.float32)
        self.cspec = scan_spec(op="+", init=0.0)
        self.nt = 1
        self.cpu_sample = f"{self.cn} elements per sample (oracle scan: the sequential f32 loop of the lowering, one thread)"

    def cpu_step(self) -> float:
        _oracle().scan(self.cspec, self.cx)
        return 8.0 * self.cn


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
    if name in ("cnn", "cnn_3x", "cnn_tf32"):
        return CnnWorkload(name)
    if name.startswith("conv"):
        return ConvWorkload(name)
    if name in ("sort", "grade", "filter"):
        return RuntimeWorkload(name)
    if name == "scan":
        return ScanWorkload(name)
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

        if args.config.startswith("cnn"):
            # the gradient allreduce runs beside the conv backward, whose
            # persistent kernels leave it 8 SMs: at most 8 NCCL channels
            os.environ.setdefault("NCCL_MAX_NCHANNELS", "8")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    wl = make_workload(args.config)
    wl.world = world
    if isinstance(wl, CnnWorkload):
        wl.GLOBAL = args.cnn_batch
        wl.OVERLAP = False if args.cnn_serial_allreduce else (True if args.cnn_overlap_allreduce else None)
        if args.cnn_reserve_sms is not None:
            wl.RESERVE = args.cnn_reserve_sms
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

    # each stage of a multi-kernel step timed alone: the dominant one gives
    # the roofline (no collective inside a stage, so ranks need not agree)
    stages = wl.stage_times(measured_peaks()) if hasattr(wl, "stage_times") else None

    h2d, d2h = wl.e2e_setup()
    e2e_steps = max(3, min(args.steps, 20))
    begin = getattr(wl, "e2e_begin", lambda: None)
    begin()
    for _ in range(2):
        wl.e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    begin()
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
        dominant = None
        if stages:
            # the stage that takes longest when timed alone
            dominant = max(stages, key=lambda k: stages[k]["ms"])
            st = stages[dominant]
            roof_unit, peak, achieved = st["unit"], st["peak"], st["achieved"]
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
                       "parallelism": (f"dp{world} (NCCL gradient allreduce, "
                                       f"{'overlapped with the conv backward' if getattr(wl, 'net', None) is not None and wl.net.overlap else 'after the backward'}"
                                       f"{', NCCL_MAX_NCHANNELS=' + os.environ['NCCL_MAX_NCHANNELS'] if world > 1 and 'NCCL_MAX_NCHANNELS' in os.environ else ''})"
                                       if wl.unit == "samples/s" else
                                       f"replicas x{world} (independent shards, no collective)")},
            "roofline": ({"kernel": dominant, "bound": stages[dominant]["bound"], "achieved": achieved,
                          "peak": peak, "unit": roof_unit, "frac": stages[dominant]["frac"],
                          "traffic": TRAFFIC.get(f"{args.config}:{dominant}"),
                          "peak_source": peaks["source"] + (
                              f" bf16 burst / 2 / {wl.tf32_products(dominant):g} (TF32 products per product)"
                              if stages[dominant]["bound"] == "tensor" else
                              " f32 CUDA-core rate at the maximum SM clock" if stages[dominant]["bound"] == "simt"
                              else " HBM copy"),
                          "timed": f"stage alone, {wl.B} images, CUDA graph of 10 calls, CUDA events"}
                         if dominant else
                         {"bound": wl.bound, "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": roof_unit,
                          "frac": round(achieved / peak, 4), "traffic": TRAFFIC.get(args.config),
                          "peak_source": peaks["source"] + (
                              (" bf16 sustained / 2 (ran under sw_power_cap)" if capped else " bf16 burst / 2")
                              if roof_unit == "TFLOP/s" else " HBM copy")}),
            "e2e": {"value": round(e2e_value, 3), "unit": wl.unit, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": n_launch,
            "clocks": clocks,
        }
        if stages:
            line["stages"] = {k: {f: v[f] for f in ("ms", "bound", "achieved", "unit", "frac")}
                              for k, v in stages.items()}
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(wl, budget_s=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        getattr(wl, "close", lambda: None)()  # graphs holding NCCL calls go before the process group
        dist.barrier()
        dist.destroy_process_group()


# Per-call DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of the
# dominant kernel, from ncu captures of the same bench commands (for the CNN
# per stage, "cnn:<stage>"; for the scan, the three kernels of one call).
TRAFFIC: dict[str, float | None] = {
    "chained": 67_117_312 + 713_728, "row_norms": 33_560_832 + 0,
    "matmul": 279_432_192 + 53_611_264, "matmul_3x": None, "bmm": None,
    "conv": 67_158_528 + 76_917_504, "conv_dgrad": 134_289_664 + 33_810_432, "conv_wgrad": 201_347_072 + 3_692_288,
    "cnn:conv1_fwd": 67_196_928 + 277_051_392, "cnn:conv2_fwd": 268_548_608 + 131_713_792,
    "cnn:dense1_fwd": 136_367_616 + 3_971_584, "cnn:dense1_wgrad": 135_338_240 + 4_023_040,
    "cnn:dense1_dgrad": 3_313_664 + 74_428_672, "cnn:conv2_wgrad": 436_544_256 + 4_085_504,
    "cnn:conv2_dgrad": 167_825_408 + 212_258_816, "cnn:conv1_wgrad": 402_680_320 + 7_718_912,
    "scan": 1_073_750_000 + 3_587_000 + 539_000 + 1_074_945_000 + 1_021_055_000,
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


CONFIGS = ["cnn", "chained", "row_norms", "matmul", "matmul_3x", "bmm", "conv", "conv_dgrad", "conv_wgrad", "cnn_3x",
           "cnn_tf32",
           "scan", "sort", "grade", "filter"]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cnn", choices=CONFIGS)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cnn-serial-allreduce", action="store_true",
                    help="CNN: one gradient allreduce after the backward (by default the dense layers' "
                         "bucket is reduced and applied while the conv backward runs)")
    ap.add_argument("--cnn-overlap-allreduce", action="store_true",
                    help="CNN: reduce the dense layers' bucket while the conv backward runs (the default)")
    ap.add_argument("--cnn-reserve-sms", type=int, default=None,
                    help="CNN, overlapped allreduce: SMs the backward's persistent kernels leave to the collective")
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
