"""numpy wrapper of liboracle.so — TEST INFRASTRUCTURE ONLY.

The CPU restatement of the reference's CPU semantics (see oracle.h for the
reference file:line each function follows).  Used by tests/, by
__graft_entry__.smoke() and by bench.py's cpu_baseline / reference arm as the
checker and the timed CPU baseline; the product never imports it.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib = None


REF_DIR = HERE / "_ref"
REF_RT_PATH = REF_DIR / "libremora_rt.so"
# where the last build() found the reference checkout (git-ignored, like _ref/)
REF_RECORD = REF_DIR / "reference_root"


def reference_root() -> Path | None:
    """The reference checkout (the directory holding remora/): the
    REMORA_REFERENCE environment variable, else the one the last build()
    compiled the reference's C runtime from; None when neither names one."""
    cand = os.environ.get("REMORA_REFERENCE") or (REF_RECORD.read_text().strip() if REF_RECORD.exists() else "")
    if cand and (Path(cand) / "remora").is_dir():
        return Path(cand)
    return None


def build(reference: str | os.PathLike | None = None) -> Path:
    """Compile liboracle.so and, where a reference checkout is given (or
    found by reference_root), the reference's own C runtime into _ref/."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    root = Path(reference) if reference else reference_root()
    if root is not None and (root / "remora" / "remora_rt.c").exists():
        # The reference's own C runtime, compiled from its source into _ref/.
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REMORA_REFERENCE={root}"], check=True)
        REF_RECORD.write_text(str(root.resolve()) + "\n")
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


# ---- the reference's C runtime helpers (remora/remora_rt.c) ----
_F32, _I32, _BOOL = 0, 1, 2


def _code(a: np.ndarray) -> int:
    return _F32 if a.dtype == np.float32 else _I32


class FilterPred(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int32), ("lit_f", ctypes.c_float), ("lit_i", ctypes.c_int32),
                ("reserved_", ctypes.c_int32)]


def sort(x: np.ndarray, nthreads: int = 1) -> np.ndarray:
    """Ascending stable sort of a rank-1 array or of each row of a rank-2 one."""
    x = np.ascontiguousarray(x)
    out = np.empty_like(x)
    rows, length = (1, x.size) if x.ndim == 1 else x.shape
    lib().oracle_sort(_code(x), _p(x), _p(out), _i64(rows), _i64(length), int(nthreads))
    return out


def grade(x: np.ndarray, nthreads: int = 1) -> np.ndarray:
    x = np.ascontiguousarray(x)
    out = np.empty(x.shape, dtype=np.int32)
    rows, length = (1, x.size) if x.ndim == 1 else x.shape
    lib().oracle_grade(_code(x), _p(x), _p(out), _i64(rows), _i64(length), int(nthreads))
    return out


def filter_(src: np.ndarray, mask: np.ndarray | None = None, pred: tuple[int, float | int] | None = None) -> np.ndarray:
    """filter with an i32/bool mask, or with pred = (REMORA_OP_* code, literal)."""
    src = np.ascontiguousarray(src)
    dst = np.empty_like(src)
    f = lib().oracle_filter
    f.restype = ctypes.c_int64
    if pred is not None:
        pr = FilterPred(pred[0], float(pred[1]), int(pred[1]), 0)
        n = f(_code(src), _p(src), None, 0, ctypes.byref(pr), _i64(src.size), _p(dst), _i64(src.size))
    else:
        m = np.ascontiguousarray(mask)
        mdt = _BOOL if m.dtype in (np.bool_, np.uint8) else _I32
        n = f(_code(src), _p(src), _p(m), mdt, None, _i64(src.size), _p(dst), _i64(src.size))
    return dst[:n].copy()


def replicate(src: np.ndarray, counts: np.ndarray) -> np.ndarray:
    src = np.ascontiguousarray(src)
    c = np.ascontiguousarray(counts, dtype=np.int32)
    total = int(np.clip(c, 0, None).astype(np.int64).sum())
    dst = np.empty(max(total, 1), dtype=src.dtype)
    f = lib().oracle_replicate
    f.restype = ctypes.c_int64
    n = f(_code(src), _p(src), _p(c), _i64(src.size), _p(dst), _i64(total))
    assert n == total
    return dst[:total].copy()


def rotate(x: np.ndarray, shift: int) -> np.ndarray:
    """out[i] = x[(i + shift) mod N] along axis 0 (np.roll(x, -shift, 0))."""
    n = x.shape[0]
    if n == 0:
        return x.copy()
    k = shift % n
    return np.concatenate([x[k:], x[:k]], axis=0)


def append(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return np.concatenate([a, b], axis=0)


# ---- remora_rt.c itself (compiled into _ref/ where the reference is present) ----
_ref_rt = None


def ref_available() -> bool:
    return REF_RT_PATH.exists()


def ref_rt() -> ctypes.CDLL:
    global _ref_rt
    if _ref_rt is None:
        if not REF_RT_PATH.exists():
            raise FileNotFoundError(f"{REF_RT_PATH} is not built (needs the reference source tree)")
        _ref_rt = ctypes.CDLL(str(REF_RT_PATH))
        for name in ("remora_filter_i32", "remora_filter_f32", "remora_replicate_i32", "remora_replicate_f32",
                     "remora_replicate_i32_count", "remora_replicate_f32_count"):
            getattr(_ref_rt, name).restype = ctypes.c_int64
    return _ref_rt


def _mr(a: np.ndarray):
    # remora_rt.c's flattened rank-1 memref: (allocated, aligned, offset, size, stride)
    return [_p(a), _p(a), _i64(0), _i64(a.size), _i64(1)]


def _sfx(a: np.ndarray) -> str:
    return "f32" if a.dtype == np.float32 else "i32"


def ref_sort(x: np.ndarray) -> np.ndarray:
    out = np.array(x, copy=True, order="C")
    getattr(ref_rt(), f"remora_sort_{_sfx(x)}")(*_mr(out))
    return out


def ref_grade(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    out = np.empty(x.size, dtype=np.int32)
    getattr(ref_rt(), f"remora_grade_{_sfx(x)}")(*_mr(x), *_mr(out))
    return out


def ref_filter(src: np.ndarray, mask: np.ndarray) -> np.ndarray:
    src = np.ascontiguousarray(src)
    m = np.ascontiguousarray(mask, dtype=np.int32)
    dst = np.empty(src.size + 2, dtype=src.dtype)
    n = getattr(ref_rt(), f"remora_filter_{_sfx(src)}")(*_mr(src), *_mr(m), *_mr(dst))
    return dst[:n].copy()


def ref_replicate(src: np.ndarray, counts: np.ndarray) -> tuple[int, np.ndarray]:
    """(the count helper's total, the fill result)."""
    src = np.ascontiguousarray(src)
    c = np.ascontiguousarray(counts, dtype=np.int32)
    total = getattr(ref_rt(), f"remora_replicate_{_sfx(src)}_count")(*_mr(src), *_mr(c))
    dst = np.empty(max(1, int(np.clip(c, 0, None).sum())), dtype=src.dtype)
    n = getattr(ref_rt(), f"remora_replicate_{_sfx(src)}")(*_mr(src), *_mr(c), *_mr(dst))
    return int(total), dst[:n].copy()


def ref_rotate(x: np.ndarray, shift: int) -> np.ndarray:
    x = np.ascontiguousarray(x)
    k = np.array([shift], dtype=np.int32)
    out = np.empty_like(x)
    getattr(ref_rt(), f"remora_rotate_{_sfx(x)}_1d")(*_mr(x), *_mr(k), *_mr(out))
    return out


def ref_append(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    out = np.empty(a.size + b.size, dtype=a.dtype)
    getattr(ref_rt(), f"remora_append_{_sfx(a)}_1d")(*_mr(a), *_mr(b), *_mr(out))
    return out
