"""Runtime objects of the B200 backend.

``B200Runtime`` / ``B200Module`` / ``B200Kernel`` satisfy the duck type that
the reference's executor drives (remora/executor.py:20-117 over
remora/runtime.py:243-412): ``load_ptx``, ``alloc``, ``free``,
``copy_host_to_device``, ``copy_device_to_host``,
``copy_host_bytes_to_device``, ``memset_d32``, ``synchronize``, ``close``, and
``module.get_function(name).launch(grid, block, args)``.  Instead of PTX text,
``load_ptx`` takes a ``SpecModule`` (kernel name -> op spec); ``launch``
ignores the reference's grid/block numbers and calls the C-ABI entry point of
the kernel's op with the descriptor structs by host pointer (no per-launch
descriptor copy to the device, unlike remora/runtime.py:415-445).
"""

from __future__ import annotations

import atexit
import ctypes
import threading
from typing import Any

import numpy as np

from remora_b200 import _lib as L
from remora_b200.abi import descriptor_rank
from remora_b200.errors import CUDAError, RemoraExecutorError


class Context:
    """One library context (device binding + cached per-stream workspace)."""

    def __init__(self, device: int = 0) -> None:
        self.device = int(device)
        handle = ctypes.c_void_p()
        L.check(L.lib().remora_b200_init(self.device, ctypes.byref(handle)), "remora_b200_init")
        self.handle = handle

    @property
    def ptr(self) -> ctypes.c_void_p:
        if self.handle is None:
            raise CUDAError("context is closed")
        return self.handle

    def close(self) -> None:
        if self.handle is not None:
            L.lib().remora_b200_shutdown(self.handle)
            self.handle = None


_contexts: dict[int, Context] = {}
_ctx_lock = threading.Lock()


def context(device: int | None = None) -> Context:
    """Process-wide shared context for `device` (created on first use)."""
    if device is None:
        try:
            import torch

            device = torch.cuda.current_device()
        except Exception:
            device = 0
    with _ctx_lock:
        ctx = _contexts.get(int(device))
        if ctx is None:
            ctx = _contexts[int(device)] = Context(int(device))
        return ctx


@atexit.register
def _close_contexts() -> None:
    for ctx in list(_contexts.values()):
        try:
            ctx.close()
        except Exception:
            pass
    _contexts.clear()


def _addr(p: Any) -> int:
    if isinstance(p, ctypes.c_void_p):
        return int(p.value or 0)
    return int(p)


class B200Runtime:
    """Drop-in for the reference's CUDARuntime (remora/runtime.py:243-340)."""

    def __init__(self, device_idx: int = 0) -> None:
        self._ctx = context(device_idx)
        self._stream = None  # legacy default stream, as the reference uses

    @property
    def ctx(self) -> Context:
        return self._ctx

    def load_ptx(self, spec_module: Any) -> "B200Module":
        """Accepts a SpecModule in place of PTX text (remora/runtime.py:262-268)."""
        from remora_b200.codegen import SpecModule

        if not isinstance(spec_module, SpecModule):
            raise RemoraExecutorError(
                "the B200 backend loads kernel specs (remora_b200.codegen.SpecModule), not PTX text"
            )
        return B200Module(spec_module, self)

    def alloc(self, nbytes: int) -> int:
        if nbytes < 0:
            raise CUDAError("cannot allocate a negative number of bytes")
        out = ctypes.c_void_p()
        L.check(L.lib().remora_b200_malloc(self._ctx.ptr, int(nbytes), ctypes.byref(out)), "alloc")
        return int(out.value)

    def free(self, ptr: int) -> None:
        L.check(L.lib().remora_b200_free(self._ctx.ptr, ctypes.c_void_p(int(ptr))), "free")

    def copy_host_to_device(self, host_array: np.ndarray, device_ptr: int) -> None:
        arr = np.ascontiguousarray(host_array)
        self.copy_host_bytes_to_device(int(arr.ctypes.data), device_ptr, arr.nbytes)

    def copy_host_bytes_to_device(self, host_address: int, device_ptr: int, nbytes: int) -> None:
        L.check(
            L.lib().remora_b200_memcpy_h2d(self._ctx.ptr, ctypes.c_void_p(int(device_ptr)),
                                           ctypes.c_void_p(int(host_address)), int(nbytes), self._stream),
            "copy_host_to_device",
        )
        self.synchronize()

    def copy_device_to_host(self, device_ptr: int, host_array: np.ndarray) -> None:
        if not host_array.flags["C_CONTIGUOUS"]:
            raise CUDAError("copy_device_to_host needs a C-contiguous host array")
        L.check(
            L.lib().remora_b200_memcpy_d2h(self._ctx.ptr, ctypes.c_void_p(int(host_array.ctypes.data)),
                                           ctypes.c_void_p(int(device_ptr)), host_array.nbytes, self._stream),
            "copy_device_to_host",
        )
        self.synchronize()

    def memset_d32(self, device_ptr: int, value: int, count: int) -> None:
        L.check(
            L.lib().remora_b200_memset_d32(self._ctx.ptr, ctypes.c_void_p(int(device_ptr)),
                                           ctypes.c_uint32(int(value) & 0xFFFFFFFF), int(count), self._stream),
            "memset_d32",
        )

    def synchronize(self) -> None:
        L.check(L.lib().remora_b200_synchronize(self._ctx.ptr, self._stream), "synchronize")

    def close(self) -> None:
        """The shared context stays open for other runtimes of the process."""

    def __enter__(self) -> "B200Runtime":
        return self

    def __exit__(self, *_exc: object) -> None:
        self.close()


class B200Module:
    def __init__(self, spec_module: Any, runtime: B200Runtime) -> None:
        self._spec = spec_module
        self._rt = runtime

    def get_function(self, name: str) -> "B200Kernel":
        try:
            spec = self._spec.kernels[name]
        except KeyError as exc:
            raise RemoraExecutorError(f"unknown kernel {name}") from exc
        return B200Kernel(spec, self._rt)

    def close(self) -> None:
        pass


class B200Kernel:
    """Launch adapter: descriptor structs in, C-ABI call out."""

    def __init__(self, spec: Any, runtime: B200Runtime) -> None:
        self.spec = spec
        self._rt = runtime

    def launch(self, grid: tuple, block: tuple, args: list, *, shared_mem: int = 0, stream: int = 0) -> None:
        del grid, block, shared_mem  # the library sizes its own launches
        descs = [a for a in args if isinstance(a, ctypes.Structure)]
        scalars = [a for a in args if not isinstance(a, ctypes.Structure)]
        if scalars:
            raise RemoraExecutorError("B200 kernels take descriptor arguments only")
        self.spec.launch(self._rt.ctx, descs[:-1], descs[-1], ctypes.c_void_p(int(stream)) if stream else None)


def desc_ptr_array(descs: list[ctypes.Structure]) -> tuple[ctypes.Array, ctypes.Array]:
    """(void* array, int32 rank array) for a list of descriptor structs."""
    ptrs = (ctypes.c_void_p * max(1, len(descs)))()
    ranks = (ctypes.c_int32 * max(1, len(descs)))()
    for k, d in enumerate(descs):
        ptrs[k] = ctypes.addressof(d)
        ranks[k] = descriptor_rank(d)
    return ptrs, ranks
