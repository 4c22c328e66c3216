"""High-level execution of descriptor-ABI kernels on the B200 backend.

``B200Executor.execute`` keeps the contract of the reference's
``RemoraExecutor.execute`` (remora/executor.py:34-117): the same arity and
output shape/dtype rules, per-call host-to-device copies, an optional
caller-supplied arena for the output, descriptors built from the host arrays'
shapes and element strides, launch, synchronise, device-to-host copy, free in
``finally``.  The reference's own ``RemoraExecutor`` also runs unchanged on a
``B200Runtime`` given a ``SpecModule``; this class exists so the backend does
not depend on the reference package being importable.
"""

from __future__ import annotations

from typing import Any

import numpy as np

from remora_b200.abi import element_strides, make_memref_descriptor
from remora_b200.codegen import KernelMeta, SpecModule
from remora_b200.errors import RemoraExecutorError
from remora_b200.runtime import B200Runtime


class B200Executor:
    def __init__(self, spec_module: SpecModule, kernels: list[KernelMeta],
                 runtime: B200Runtime | None = None) -> None:
        self._rt = B200Runtime() if runtime is None else runtime
        self._module = self._rt.load_ptx(spec_module)
        self._meta = {k.name: k for k in kernels}
        self._kernels = {k.name: self._module.get_function(k.name) for k in kernels}

    def execute(self, kernel_name: str, inputs: list[np.ndarray], *, arena: Any | None = None) -> np.ndarray:
        try:
            meta = self._meta[kernel_name]
            kernel = self._kernels[kernel_name]
        except KeyError as exc:
            raise RemoraExecutorError(f"unknown kernel {kernel_name}") from exc
        if meta.num_outputs != 1:
            raise RemoraExecutorError("only single-output kernels are supported")
        if meta.num_inputs != len(inputs):
            raise RemoraExecutorError(f"kernel {kernel_name} expects {meta.num_inputs} inputs, got {len(inputs)}")
        host = [np.ascontiguousarray(a) for a in inputs]
        out_shape = compute_output_shape(meta, host)
        out_dtype = kernel_output_dtype(meta, host)
        output = np.empty(out_shape, dtype=out_dtype)
        dev: list[int] = []
        out_ptr: int | None = None
        try:
            for a in host:
                p = self._rt.alloc(a.nbytes)
                dev.append(p)
                self._rt.copy_host_to_device(a, p)
            out_ptr = arena.alloc(output.nbytes) if arena is not None else self._rt.alloc(output.nbytes)
            in_descs = [make_memref_descriptor(p, a.shape, element_strides(a), a.dtype) for p, a in zip(dev, host)]
            out_desc = make_memref_descriptor(out_ptr, output.shape, element_strides(output), output.dtype)
            kernel.launch((1, 1, 1), (1, 1, 1), [*in_descs, out_desc])
            self._rt.synchronize()
            self._rt.copy_device_to_host(out_ptr, output)
        finally:
            for p in dev:
                self._rt.free(p)
            if out_ptr is not None and arena is None:
                self._rt.free(out_ptr)
        return output

    def execute_main(self, inputs: list[np.ndarray] | None = None, *, arena: Any | None = None) -> np.ndarray:
        if "main" in self._kernels:
            name = "main"
        elif len(self._kernels) == 1:
            name = next(iter(self._kernels))
        else:
            raise RemoraExecutorError("execute_main requires a kernel named main or exactly one compiled kernel")
        return self.execute(name, [] if inputs is None else inputs, arena=arena)

    def close(self) -> None:
        self._module.close()

    def __enter__(self) -> "B200Executor":
        return self

    def __exit__(self, *_exc: object) -> None:
        self.close()


def compute_output_shape(meta: KernelMeta, inputs: list[np.ndarray]) -> tuple[int, ...]:
    """Same rule as remora/executor.py:309-315."""
    if meta.output_shape is not None:
        return tuple(int(d) for d in meta.output_shape)
    if inputs:
        return tuple(int(d) for d in inputs[0].shape)
    return ()


_NAMES = {"i1": np.bool_, "bool": np.bool_, "i8": np.bool_, "i32": np.int32, "int32": np.int32,
          "f32": np.float32, "float32": np.float32}


def kernel_output_dtype(meta: KernelMeta, inputs: list[np.ndarray]) -> np.dtype:
    """Same rule as remora/executor.py:318-341."""
    if meta.output_dtype is not None:
        return np.dtype(_NAMES.get(meta.output_dtype, meta.output_dtype))
    if meta.output_elem_types:
        return np.dtype(_NAMES.get(meta.output_elem_types[0], meta.output_elem_types[0]))
    if inputs:
        return np.dtype(inputs[0].dtype)
    return np.dtype(np.float32)
