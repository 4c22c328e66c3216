"""Descriptor ABI of the Remora Dense Core, as ctypes structs.

Byte-identical to the reference's ``RemoraMemRef0..10`` (remora/abi.py:20-47,
docs/ABI.md:34-76): ``{allocated, aligned, offset, size0..sizeN-1,
stride0..strideN-1}``, offsets and strides in elements.  The layout is fixed by
the ABI, so the field list necessarily matches the reference's; the helpers
below are this package's own (numpy views and torch tensors to descriptors).
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence

import numpy as np

from remora_b200.errors import RemoraB200Error

MAX_RANK = 10


def _fields(rank: int) -> list[tuple[str, object]]:
    head = [("allocated", ctypes.c_void_p), ("aligned", ctypes.c_void_p), ("offset", ctypes.c_int64)]
    return head + [(f"size{d}", ctypes.c_int64) for d in range(rank)] + [
        (f"stride{d}", ctypes.c_int64) for d in range(rank)
    ]


DESCRIPTORS: dict[int, type[ctypes.Structure]] = {
    r: type(f"RemoraMemRef{r}", (ctypes.Structure,), {"_fields_": _fields(r), "__module__": __name__})
    for r in range(MAX_RANK + 1)
}
globals().update({cls.__name__: cls for cls in DESCRIPTORS.values()})


def memref_descriptor_type(rank: int) -> type[ctypes.Structure]:
    if rank not in DESCRIPTORS:
        raise RemoraB200Error(f"the descriptor ABI covers ranks 0 through {MAX_RANK}, not {rank}")
    return DESCRIPTORS[rank]


def descriptor_rank(desc: ctypes.Structure | type) -> int:
    """Rank of any RemoraMemRefN instance or type, including the reference's
    own classes: the struct is 24 + 16 * rank bytes."""
    size = ctypes.sizeof(desc if isinstance(desc, type) else type(desc))
    rank, rem = divmod(size - 24, 16)
    if rem or not 0 <= rank <= MAX_RANK:
        raise RemoraB200Error(f"{desc!r} is not a Remora memref descriptor ({size} bytes)")
    return rank


def descriptor_shape(desc: ctypes.Structure) -> tuple[int, ...]:
    return tuple(int(getattr(desc, f"size{d}")) for d in range(descriptor_rank(desc)))


def descriptor_strides(desc: ctypes.Structure) -> tuple[int, ...]:
    return tuple(int(getattr(desc, f"stride{d}")) for d in range(descriptor_rank(desc)))


def element_strides(array: np.ndarray) -> tuple[int, ...]:
    """numpy byte strides -> element strides (must divide evenly)."""
    arr = np.asarray(array)
    out = []
    for s in arr.strides:
        q, r = divmod(s, arr.dtype.itemsize)
        if r:
            raise RemoraB200Error(f"byte stride {s} is not a multiple of item size {arr.dtype.itemsize}")
        out.append(q)
    return tuple(out)


def make_memref_descriptor(
    ptr: int,
    shape: Sequence[int],
    strides: Sequence[int],
    dtype: object = None,
    offset: int = 0,
) -> ctypes.Structure:
    """Descriptor for a (device or host) pointer with element strides."""
    if dtype is not None:
        np.dtype(dtype)
    sizes = [int(s) for s in shape]
    st = [int(s) for s in strides]
    if len(sizes) != len(st):
        raise RemoraB200Error("shape and strides must have the same rank")
    if any(s < 0 for s in sizes):
        raise RemoraB200Error("descriptor sizes must be non-negative")
    desc = memref_descriptor_type(len(sizes))()
    desc.allocated = int(ptr)
    desc.aligned = int(ptr)
    desc.offset = int(offset)
    for d, (s, t) in enumerate(zip(sizes, st)):
        setattr(desc, f"size{d}", s)
        setattr(desc, f"stride{d}", t)
    return desc


def contiguous_strides(shape: Sequence[int]) -> tuple[int, ...]:
    out = []
    acc = 1
    for s in reversed(list(shape)):
        out.append(acc)
        acc *= int(s)
    return tuple(reversed(out))


def tensor_descriptor(t) -> ctypes.Structure:
    """Descriptor of a torch tensor view: `aligned` is the storage base and the
    view's start lives in `offset` (the ABI's view rule, docs/ABI.md:32)."""
    if t.dim() > MAX_RANK:
        raise RemoraB200Error(f"rank {t.dim()} exceeds the ABI's {MAX_RANK}")
    base = t.untyped_storage().data_ptr() if t.numel() else t.data_ptr()
    off = t.storage_offset() if t.numel() else 0
    return make_memref_descriptor(base, t.shape, t.stride(), None, off)


def numpy_descriptor(array: np.ndarray) -> ctypes.Structure:
    """Host descriptor of a numpy array or view (base allocation + offset)."""
    arr = np.asarray(array)
    base = arr
    while isinstance(base.base, np.ndarray):
        base = base.base
    byte_off = int(arr.ctypes.data) - int(base.ctypes.data)
    if byte_off % arr.dtype.itemsize:
        raise RemoraB200Error("view offset is not a whole number of elements")
    return make_memref_descriptor(
        int(base.ctypes.data), arr.shape, element_strides(arr), arr.dtype, byte_off // arr.dtype.itemsize
    )
