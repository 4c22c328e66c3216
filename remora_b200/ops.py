"""Device-tensor API over the C ABI.

Each function takes CUDA tensors (torch is only the allocator and stream
provider here), builds Remora descriptors for them — views keep their storage
base in ``aligned`` and their start in ``offset`` — and calls the matching
``remora_b200_*`` entry point on the current torch stream.  Nothing here
computes on the host.
"""

from __future__ import annotations

import ctypes
from typing import Any, Sequence

from remora_b200 import _lib as L
from remora_b200.abi import tensor_descriptor
from remora_b200.codegen import fold_spec, scan_spec
from remora_b200.errors import RemoraB200Error, RemoraShapeError
from remora_b200.program import Expr, compile_program
from remora_b200.runtime import context


def _torch():
    import torch

    return torch


def dtype_of(t) -> int:
    torch = _torch()
    if t.dtype == torch.float32:
        return L.F32
    if t.dtype == torch.int32:
        return L.I32
    if t.dtype in (torch.bool, torch.uint8):
        return L.BOOL
    raise RemoraB200Error(f"unsupported tensor dtype {t.dtype}")


def torch_dtype(code: int):
    torch = _torch()
    return {L.F32: torch.float32, L.I32: torch.int32, L.BOOL: torch.bool}[code]


def _stream(t) -> ctypes.c_void_p:
    torch = _torch()
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _ctx(t):
    return context(t.device.index if t.device.index is not None else 0)


def _check_cuda(*ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RemoraB200Error("remora_b200 ops take CUDA tensors (there is no CPU path)")


def _desc_arrays(tensors: Sequence[Any]):
    descs = [tensor_descriptor(t) for t in tensors]
    ptrs = (ctypes.c_void_p * max(1, len(descs)))()
    ranks = (ctypes.c_int32 * max(1, len(descs)))()
    for k, (d, t) in enumerate(zip(descs, tensors)):
        ptrs[k] = ctypes.addressof(d)
        ranks[k] = t.dim()
    return descs, ptrs, ranks


def frame_shape(tensors: Sequence[Any]) -> tuple[int, ...]:
    """Principal frame under prefix agreement: the highest-rank operand's
    shape, every other operand's shape being a prefix of it."""
    best = max(tensors, key=lambda t: t.dim())
    shape = tuple(best.shape)
    for t in tensors:
        if tuple(t.shape) != shape[: t.dim()]:
            raise RemoraShapeError(f"shapes {tuple(t.shape)} and {shape} do not agree on a prefix frame")
    return shape


# ------------------------------------------------------------------- maps
def map(expr_or_program: Expr | L.RemoraMapProgram, *inputs, out=None, out_dtype: object | None = None,
        compute: object | None = None):
    """Lifted map of an expression over the inputs' common prefix frame."""
    torch = _torch()
    _check_cuda(*inputs)
    if isinstance(expr_or_program, L.RemoraMapProgram):
        prog = expr_or_program
    else:
        comp = compute if compute is not None else (dtype_of(inputs[0]) if inputs else L.F32)
        if comp == L.BOOL and out_dtype is None:
            pass
        prog = compile_program(expr_or_program, len(inputs), compute=comp,
                               out=out_dtype, in_dtypes=[dtype_of(t) for t in inputs])
    if out is None:
        shape = frame_shape(inputs) if inputs else ()
        out = torch.empty(shape, dtype=torch_dtype(prog.out_dtype), device=inputs[0].device)
    _check_cuda(out)
    descs, ptrs, ranks = _desc_arrays(inputs)
    od = tensor_descriptor(out)
    L.check(L.lib().remora_b200_map(_ctx(out).ptr, ctypes.byref(prog), ptrs, ranks, len(inputs),
                                    ctypes.addressof(od), out.dim(), _stream(out)), "map")
    return out


# ------------------------------------------------------------------ folds
def fold(*inputs, op: str = "+", init: float | int = 0, mode: str = "cell", cell_rank: int = 1,
         premap: Expr | None = None, epilogue: str | None = None, out=None, dtype: object | None = None):
    """Cell-frame fold (mode='cell': fold the trailing ``cell_rank`` axes of
    every frame cell) or whole-array fold (mode='all'), optionally fused with a
    premap over one or two inputs and a sqrt epilogue."""
    torch = _torch()
    _check_cuda(*inputs)
    dt = dtype if dtype is not None else dtype_of(inputs[0])
    sp = fold_spec(op=op, init=init, mode=mode, cell_rank=cell_rank, dtype=dt, premap=premap,
                   n_inputs=len(inputs), epilogue=epilogue,
                   premap_in_dtypes=[dtype_of(t) for t in inputs] if premap is not None else None)
    if out is None:
        shape = () if mode == "all" else tuple(inputs[0].shape[: inputs[0].dim() - cell_rank])
        out = torch.empty(shape, dtype=torch_dtype(sp.dtype), device=inputs[0].device)
    descs, ptrs, ranks = _desc_arrays(inputs)
    od = tensor_descriptor(out)
    L.check(L.lib().remora_b200_fold(_ctx(out).ptr, ctypes.byref(sp), ptrs, ranks, len(inputs),
                                     ctypes.addressof(od), out.dim(), _stream(out)), "fold")
    return out


def array_fold(x, init, *, op: str = "+", out=None):
    """Leading-axis fold with an array accumulator: init op x[0] op x[1] ..."""
    torch = _torch()
    _check_cuda(x, init)
    sp = fold_spec(op=op, dtype=dtype_of(x))
    if out is None:
        out = torch.empty(tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    xd, idd, od = tensor_descriptor(x), tensor_descriptor(init), tensor_descriptor(out)
    L.check(L.lib().remora_b200_array_fold(_ctx(out).ptr, ctypes.byref(sp), ctypes.addressof(xd), x.dim(),
                                           ctypes.addressof(idd), ctypes.addressof(od), _stream(out)),
            "array_fold")
    return out


def scan(x, *, op: str = "+", init: float | int = 0, exclusive: bool = False, right: bool = False, out=None):
    torch = _torch()
    _check_cuda(x)
    sp = scan_spec(op=op, init=init, dtype=dtype_of(x), exclusive=exclusive, right=right)
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    xd, od = tensor_descriptor(x), tensor_descriptor(out)
    L.check(L.lib().remora_b200_scan(_ctx(out).ptr, ctypes.byref(sp), ctypes.addressof(xd),
                                     ctypes.addressof(od), x.dim(), _stream(out)), "scan")
    return out


# ------------------------------------------------------------- dense core
def gemm(a, b, *, precision: str = "3xtf32", out=None):
    """C = A . B (rank 2, or batched rank 3) on tcgen05 tensor cores."""
    torch = _torch()
    _check_cuda(a, b)
    prec = {"tf32": L.PREC_TF32, "3xtf32": L.PREC_3XTF32}[precision]
    if out is None:
        shape = (*a.shape[:-1], b.shape[-1])
        out = torch.empty(shape, dtype=torch.float32, device=a.device)
    spec = L.RemoraGemmSpec(prec, 0)
    ad, bd, cd = tensor_descriptor(a), tensor_descriptor(b), tensor_descriptor(out)
    L.check(L.lib().remora_b200_gemm(_ctx(out).ptr, ctypes.byref(spec), ctypes.addressof(ad),
                                     ctypes.addressof(bd), ctypes.addressof(cd), out.dim(), _stream(out)), "gemm")
    return out


# ---------------------------------------------------------- convolution
def _conv_spec(stride: int, pad: int, precision: str) -> L.RemoraConvSpec:
    return L.RemoraConvSpec(int(stride), int(pad), {"tf32": L.PREC_TF32, "3xtf32": L.PREC_3XTF32,
                                                    "2xtf32": L.PREC_2XTF32}[precision], 0)


def conv2d_fwd(x, w, bias=None, *, stride: int = 1, pad: int = 1, precision: str = "3xtf32", out=None):
    torch = _torch()
    _check_cuda(x, w, bias)
    N, C, H, W = x.shape
    K, _, R, S = w.shape
    OH, OW = (H + 2 * pad - R) // stride + 1, (W + 2 * pad - S) // stride + 1
    if out is None:
        out = torch.empty((N, K, OH, OW), dtype=torch.float32, device=x.device)
    sp = _conv_spec(stride, pad, precision)
    xd, wd, yd = tensor_descriptor(x), tensor_descriptor(w), tensor_descriptor(out)
    bd = tensor_descriptor(bias) if bias is not None else None
    L.check(L.lib().remora_b200_conv2d_fwd(_ctx(out).ptr, ctypes.byref(sp), ctypes.addressof(xd),
                                           ctypes.addressof(wd), ctypes.addressof(bd) if bd is not None else None,
                                           ctypes.addressof(yd), _stream(out)), "conv2d_fwd")
    return out


def conv2d_dgrad(dy, w, input_shape, *, stride: int = 1, pad: int = 1, precision: str = "3xtf32", out=None):
    torch = _torch()
    _check_cuda(dy, w)
    if out is None:
        out = torch.empty(tuple(input_shape), dtype=torch.float32, device=dy.device)
    sp = _conv_spec(stride, pad, precision)
    dyd, wd, dxd = tensor_descriptor(dy), tensor_descriptor(w), tensor_descriptor(out)
    L.check(L.lib().remora_b200_conv2d_dgrad(_ctx(out).ptr, ctypes.byref(sp), ctypes.addressof(dyd),
                                             ctypes.addressof(wd), ctypes.addressof(dxd), _stream(out)),
            "conv2d_dgrad")
    return out


def conv2d_wgrad(x, dy, weight_shape, *, stride: int = 1, pad: int = 1, precision: str = "3xtf32", out=None):
    torch = _torch()
    _check_cuda(x, dy)
    if out is None:
        out = torch.empty(tuple(weight_shape), dtype=torch.float32, device=x.device)
    sp = _conv_spec(stride, pad, precision)
    xd, dyd, dwd = tensor_descriptor(x), tensor_descriptor(dy), tensor_descriptor(out)
    L.check(L.lib().remora_b200_conv2d_wgrad(_ctx(out).ptr, ctypes.byref(sp), ctypes.addressof(xd),
                                             ctypes.addressof(dyd), ctypes.addressof(dwd), _stream(out)),
            "conv2d_wgrad")
    return out


# ---------------------------------------------------------------- layout
def im2col(image, kh: int, kw: int, stride: int = 1, out=None):
    torch = _torch()
    _check_cuda(image)
    H, W = image.shape
    oh, ow = (H - kh) // stride + 1, (W - kw) // stride + 1
    if out is None:
        out = torch.empty((oh * ow, kh * kw), dtype=torch.float32, device=image.device)
    sp = L.RemoraIm2colSpec(kh, kw, stride, 0)
    idd, cd = tensor_descriptor(image), tensor_descriptor(out)
    L.check(L.lib().remora_b200_im2col(_ctx(out).ptr, ctypes.byref(sp), ctypes.addressof(idd),
                                       ctypes.addressof(cd), _stream(out)), "im2col")
    return out


def col2im(cols, image_shape: tuple[int, int], kh: int, kw: int, stride: int = 1, out=None):
    torch = _torch()
    _check_cuda(cols)
    if out is None:
        out = torch.empty(tuple(image_shape), dtype=torch.float32, device=cols.device)
    sp = L.RemoraIm2colSpec(kh, kw, stride, 0)
    cd, idd = tensor_descriptor(cols), tensor_descriptor(out)
    L.check(L.lib().remora_b200_col2im(_ctx(out).ptr, ctypes.byref(sp), ctypes.addressof(cd),
                                       ctypes.addressof(idd), _stream(out)), "col2im")
    return out


def transpose(x, out=None):
    torch = _torch()
    _check_cuda(x)
    if out is None:
        out = torch.empty((x.shape[1], x.shape[0]), dtype=x.dtype, device=x.device)
    xd, od = tensor_descriptor(x), tensor_descriptor(out)
    L.check(L.lib().remora_b200_transpose(_ctx(out).ptr, dtype_of(x), ctypes.addressof(xd),
                                          ctypes.addressof(od), _stream(out)), "transpose")
    return out


def synchronize(device: int | None = None) -> None:
    """Synchronise the current stream and surface any device-side timeout."""
    torch = _torch()
    dev = torch.cuda.current_device() if device is None else device
    s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    L.check(L.lib().remora_b200_synchronize(context(dev).ptr, s), "synchronize")


def wait_check(limit_cycles: int, signal: bool = False, device: int | None = None) -> None:
    """Enqueue the bounded-wait check (remora_b200_wait_check) on the current
    stream: a wait on a barrier that only `signal` completes, given up after
    `limit_cycles`.  The next synchronize() raises RemoraTimeoutError when it
    ran out."""
    torch = _torch()
    dev = torch.cuda.current_device() if device is None else device
    s = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    L.check(L.lib().remora_b200_wait_check(context(dev).ptr, int(limit_cycles), int(bool(signal)), s), "wait_check")


# ------------------------------------------- the C runtime helpers on GPU
_CMP = {"<": L.OP_LT, "<=": L.OP_LE, ">": L.OP_GT, ">=": L.OP_GE, "==": L.OP_EQ, "!=": L.OP_NE}


def _sort_like(x, out, grade: bool):
    torch = _torch()
    _check_cuda(x)
    if x.dim() not in (1, 2):
        raise RemoraShapeError(f"{'grade' if grade else 'sort'} takes rank 1 or 2, got rank {x.dim()}")
    if out is None:
        out = torch.empty(x.shape, dtype=torch.int32 if grade else x.dtype, device=x.device)
    xd, od = tensor_descriptor(x), tensor_descriptor(out)
    fn = L.lib().remora_b200_grade if grade else L.lib().remora_b200_sort
    L.check(fn(_ctx(out).ptr, dtype_of(x), ctypes.addressof(xd), ctypes.addressof(od), x.dim(), _stream(out)),
            "grade" if grade else "sort")
    return out


def sort(x, out=None):
    """Ascending sort of a rank-1 array, or of every row of a rank-2 array
    (the reference's remora_sort_* runtime helper)."""
    return _sort_like(x, out, grade=False)


def grade(x, out=None):
    """Stable ascending argsort (int32), per row for rank 2 (remora_grade_*)."""
    return _sort_like(x, out, grade=True)


def filter(x, mask=None, *, pred: tuple[str, float | int] | None = None, out=None, count=None, sync: bool = True):
    """Keeps x[i] where mask[i] != 0 (i32 or bool mask) or where `x[i] op lit`
    for pred = (op, lit), in order (remora_filter_*).  With sync, returns the
    kept values (the count is read back to the host); otherwise returns
    (out, count) with count a device int64 scalar."""
    torch = _torch()
    _check_cuda(x)
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    if count is None:
        count = torch.zeros((), dtype=torch.int64, device=x.device)
    xd, od, cd = tensor_descriptor(x), tensor_descriptor(out), tensor_descriptor(count)
    if (mask is None) == (pred is None):
        raise RemoraB200Error("filter takes exactly one of mask and pred")
    if pred is not None:
        op, lit = pred
        pr = L.RemoraFilterPred(_CMP[op], float(lit), int(lit), 0)
        st = L.lib().remora_b200_filter(_ctx(out).ptr, dtype_of(x), ctypes.addressof(xd), None, 0,
                                        ctypes.byref(pr), ctypes.addressof(od), ctypes.addressof(cd), _stream(out))
    else:
        _check_cuda(mask)
        md = tensor_descriptor(mask)
        st = L.lib().remora_b200_filter(_ctx(out).ptr, dtype_of(x), ctypes.addressof(xd), ctypes.addressof(md),
                                        dtype_of(mask), None, ctypes.addressof(od), ctypes.addressof(cd),
                                        _stream(out))
    L.check(st, "filter")
    if not sync:
        return out, count
    return out[: int(count.item())]


def replicate(x, counts, out=None, *, total=None, sync: bool = True):
    """x[0] repeated counts[0] times, then x[1] counts[1] times, ...
    (remora_replicate_*; a negative count repeats nothing).  Without `out`
    the total is computed first and read back to size the result."""
    torch = _torch()
    _check_cuda(x, counts)
    if total is None:
        total = torch.zeros((), dtype=torch.int64, device=x.device)
    xd, cd, td = tensor_descriptor(x), tensor_descriptor(counts), tensor_descriptor(total)
    lib = L.lib()
    if out is None:
        L.check(lib.remora_b200_replicate(_ctx(x).ptr, dtype_of(x), ctypes.addressof(xd), ctypes.addressof(cd),
                                          None, ctypes.addressof(td), _stream(x)), "replicate")
        out = torch.empty((int(total.item()),), dtype=x.dtype, device=x.device)
    od = tensor_descriptor(out)
    L.check(lib.remora_b200_replicate(_ctx(x).ptr, dtype_of(x), ctypes.addressof(xd), ctypes.addressof(cd),
                                      ctypes.addressof(od), ctypes.addressof(td), _stream(x)), "replicate")
    if not sync:
        return out, total
    return out[: min(int(total.item()), out.shape[0])]


def rotate(x, shift: int, out=None):
    """out[i] = x[(i + shift) mod N] along axis 0 (remora_rotate_*)."""
    torch = _torch()
    _check_cuda(x)
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    xd, od = tensor_descriptor(x), tensor_descriptor(out)
    L.check(L.lib().remora_b200_rotate(_ctx(out).ptr, dtype_of(x), int(shift), ctypes.addressof(xd),
                                       ctypes.addressof(od), x.dim(), _stream(out)), "rotate")
    return out


def append(a, b, out=None):
    """a followed by b along axis 0 (remora_append_*)."""
    torch = _torch()
    _check_cuda(a, b)
    if out is None:
        out = torch.empty((a.shape[0] + b.shape[0], *a.shape[1:]), dtype=a.dtype, device=a.device)
    ad, bd, od = tensor_descriptor(a), tensor_descriptor(b), tensor_descriptor(out)
    L.check(L.lib().remora_b200_append(_ctx(out).ptr, dtype_of(a), ctypes.addressof(ad), ctypes.addressof(bd),
                                       ctypes.addressof(od), a.dim(), _stream(out)), "append")
    return out
