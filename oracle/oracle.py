"""numpy wrapper of liboracle.so — TEST INFRASTRUCTURE ONLY.

The CPU restatement of the reference's CPU semantics (see oracle.h for the
reference file:line each function follows).  Used by tests/, by
__graft_entry__.smoke() and by bench.py's cpu_baseline / reference arm as the
checker and the timed CPU baseline; the product never imports it.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        newest = max((HERE / f).stat().st_mtime for f in ("oracle.c", "oracle.h"))
        if not LIB_PATH.exists() or newest > LIB_PATH.stat().st_mtime:
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.oracle_cnn_step.restype = ctypes.c_float
        _lib.oracle_max_threads.restype = ctypes.c_int
    return _lib


def _p(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def _i64(v: int) -> ctypes.c_int64:
    return ctypes.c_int64(int(v))


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def run_map(prog, inputs: list[np.ndarray], shape: tuple[int, ...], out_dtype, nthreads: int = 1) -> np.ndarray:
    """Map with prefix-frame broadcasting: input k of rank r < len(shape) is
    read at its first r indices (stride 0 on the trailing axes)."""
    rank = len(shape)
    ins = [np.asarray(a) for a in inputs]
    strides = np.zeros((max(1, len(ins)), max(1, rank)), dtype=np.int64)
    for k, a in enumerate(ins):
        es = a.dtype.itemsize
        for d in range(a.ndim):
            strides[k, d] = 0 if a.shape[d] == 1 else a.strides[d] // es
    ptrs = (ctypes.c_void_p * max(1, len(ins)))(*[a.ctypes.data for a in ins])
    out = np.empty(shape, dtype=out_dtype)
    shp = np.asarray(shape if shape else (1,), dtype=np.int64)
    lib().oracle_map(ctypes.byref(prog), len(ins), ptrs, _p(strides), _p(shp), rank, _p(out), int(nthreads))
    return out


def cell_fold(spec, inputs: list[np.ndarray], cell_rank: int, nthreads: int = 1) -> np.ndarray:
    ins = [np.ascontiguousarray(a) for a in inputs]
    frame = ins[0].shape[: ins[0].ndim - cell_rank]
    rows = int(np.prod(frame, dtype=np.int64))
    L = int(np.prod(ins[0].shape[ins[0].ndim - cell_rank:], dtype=np.int64))
    dt = np.float32 if spec.dtype == 0 else np.int32
    out = np.empty(frame, dtype=dt)
    ptrs = (ctypes.c_void_p * len(ins))(*[a.ctypes.data for a in ins])
    lib().oracle_cell_fold(ctypes.byref(spec), len(ins), ptrs, _i64(rows), _i64(L), _p(out), int(nthreads))
    return out


def compiled_fold(name: str, x: np.ndarray, nthreads: int = 1) -> np.ndarray:
    """The benchmark programs as compiled C loops ('chained' or 'row_norms')."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    L = x.shape[-1]
    rows = x.size // L
    out = np.empty(x.shape[:-1], dtype=np.float32)
    fn = {"chained": lib().oracle_chained_fold_f32, "row_norms": lib().oracle_row_norms_f32}[name]
    fn(_p(x), _i64(rows), _i64(L), _p(out), int(nthreads))
    return out


def fold_all(spec, inputs: list[np.ndarray]) -> np.ndarray:
    ins = [np.ascontiguousarray(a) for a in inputs]
    dt = np.float32 if spec.dtype == 0 else np.int32
    out = np.empty((), dtype=dt)
    ptrs = (ctypes.c_void_p * len(ins))(*[a.ctypes.data for a in ins])
    lib().oracle_fold_all(ctypes.byref(spec), len(ins), ptrs, _i64(ins[0].size), _p(out))
    return out


def array_fold(spec, x: np.ndarray, init: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    init = np.ascontiguousarray(init)
    out = np.empty(init.shape, dtype=x.dtype)
    lib().oracle_array_fold(ctypes.byref(spec), _p(x), _p(init), _i64(x.shape[0]), _i64(init.size), _p(out))
    return out


def scan(spec, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    out = np.empty_like(x)
    N = x.shape[0]
    T = x.size // max(N, 1)
    lib().oracle_scan(ctypes.byref(spec), _p(x), _i64(N), _i64(T), _p(out))
    return out


def matmul(a: np.ndarray, b: np.ndarray, rows: tuple[int, int] | None = None, nthreads: int = 1) -> np.ndarray:
    """Lifted-dot matmul of [.., M, K] x [.., K, N] (sequential k per element);
    `rows` restricts the computed rows (others are left zero)."""
    a3 = np.ascontiguousarray(a, dtype=np.float32).reshape(-1, a.shape[-2], a.shape[-1])
    b3 = np.ascontiguousarray(b, dtype=np.float32).reshape(-1, b.shape[-2], b.shape[-1])
    batch, M, K = a3.shape
    N = b3.shape[2]
    c = np.zeros((batch, M, N), dtype=np.float32)
    r0, r1 = rows if rows is not None else (0, M)
    lib().oracle_matmul(_p(a3), _p(b3), _p(c), _i64(batch), _i64(M), _i64(N), _i64(K), _i64(r0), _i64(r1),
                        int(nthreads))
    return c.reshape(*a.shape[:-1], N)


def im2col(img: np.ndarray, kh: int, kw: int, stride: int = 1) -> np.ndarray:
    img = np.ascontiguousarray(img, dtype=np.float32)
    H, W = img.shape
    oh, ow = (H - kh) // stride + 1, (W - kw) // stride + 1
    out = np.empty((oh * ow, kh * kw), dtype=np.float32)
    lib().oracle_im2col(_p(img), _i64(H), _i64(W), kh, kw, stride, _p(out))
    return out


def col2im(cols: np.ndarray, H: int, W: int, kh: int, kw: int, stride: int = 1) -> np.ndarray:
    cols = np.ascontiguousarray(cols, dtype=np.float32)
    out = np.empty((H, W), dtype=np.float32)
    lib().oracle_col2im(_p(cols), _i64(H), _i64(W), kh, kw, stride, _p(out))
    return out


def conv2d_fwd(x, w, bias=None, stride=1, pad=1, images: tuple[int, int] | None = None, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, C, H, W = x.shape
    K, _, R, S = w.shape
    OH, OW = (H + 2 * pad - R) // stride + 1, (W + 2 * pad - S) // stride + 1
    n0, n1 = images if images else (0, N)
    y = np.zeros((N, K, OH, OW), dtype=np.float32)
    b = np.ascontiguousarray(bias, dtype=np.float32) if bias is not None else None
    lib().oracle_conv2d_fwd(_p(x), _p(w), _p(b) if b is not None else None, _p(y), _i64(N), _i64(C), _i64(H),
                            _i64(W), _i64(K), R, S, stride, pad, _i64(n0), _i64(n1), int(nthreads))
    return y


def conv2d_dgrad(dy, w, input_shape, stride=1, pad=1, images=None, nthreads=1):
    dy = np.ascontiguousarray(dy, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, C, H, W = input_shape
    K, _, R, S = w.shape
    n0, n1 = images if images else (0, N)
    dx = np.zeros((N, C, H, W), dtype=np.float32)
    lib().oracle_conv2d_dgrad(_p(dy), _p(w), _p(dx), _i64(N), _i64(C), _i64(H), _i64(W), _i64(K), R, S, stride,
                              pad, _i64(n0), _i64(n1), int(nthreads))
    return dx


def conv2d_wgrad(x, dy, weight_shape, stride=1, pad=1, images=None, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    dy = np.ascontiguousarray(dy, dtype=np.float32)
    N, C, H, W = x.shape
    K, _, R, S = weight_shape
    n0, n1 = images if images else (0, N)
    dw = np.zeros(weight_shape, dtype=np.float32)
    lib().oracle_conv2d_wgrad(_p(x), _p(dy), _p(dw), _i64(N), _i64(C), _i64(H), _i64(W), _i64(K), R, S, stride,
                              pad, _i64(n0), _i64(n1), int(nthreads))
    return dw


def maxpool2x2_fwd(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    *lead, H, W = x.shape
    NC = int(np.prod(lead, dtype=np.int64))
    y = np.empty((*lead, H // 2, W // 2), dtype=np.float32)
    lib().oracle_maxpool2x2_fwd(_p(x), _p(y), _i64(NC), _i64(H), _i64(W))
    return y


def maxpool2x2_bwd(x: np.ndarray, dy: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    dy = np.ascontiguousarray(dy, dtype=np.float32)
    *lead, H, W = x.shape
    NC = int(np.prod(lead, dtype=np.int64))
    dx = np.empty_like(x)
    lib().oracle_maxpool2x2_bwd(_p(x), _p(dy), _p(dx), _i64(NC), _i64(H), _i64(W))
    return dx


CNN_NPARAMS = 529217


def cnn_step(params: np.ndarray, images: np.ndarray, labels: np.ndarray, batch_total: int | None = None,
             lr: float = 0.01, apply_sgd: bool = True, nthreads: int = 1) -> tuple[float, np.ndarray]:
    """One crater-CNN SGD step on the CPU; updates `params` in place when
    apply_sgd and returns (loss, grads)."""
    assert params.dtype == np.float32 and params.size == CNN_NPARAMS and params.flags["C_CONTIGUOUS"]
    imgs = np.ascontiguousarray(images, dtype=np.float32)
    labs = np.ascontiguousarray(labels, dtype=np.float32)
    grads = np.zeros(CNN_NPARAMS, dtype=np.float32)
    B = imgs.shape[0]
    loss = lib().oracle_cnn_step(_p(params), _p(grads), _p(imgs), _p(labs), _i64(B), _i64(batch_total or B),
                                 ctypes.c_float(lr), int(apply_sgd), int(nthreads))
    return float(loss), grads
