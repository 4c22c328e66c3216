"""Exceptions of the B200 backend.

The names mirror the reference's error surface so callers can catch the same
classes: ``RemoraExecutorError`` (remora/executor.py:13-14) and
``RuntimeUnavailable`` / ``CUDAError`` (remora/runtime.py:110-115).
"""


class RemoraB200Error(Exception):
    """Base class for every error raised by the B200 backend."""


class RuntimeUnavailable(RemoraB200Error):
    """The backend cannot run here (no library, no sm_100 device)."""


class CUDAError(RuntimeUnavailable):
    """A CUDA runtime call inside the backend failed."""


class RemoraExecutorError(RemoraB200Error):
    """High-level execution cannot proceed (arity, unknown kernel, ...)."""


class RemoraShapeError(RemoraB200Error):
    """Ranks or sizes of the operands disagree."""


class RemoraUnsupportedError(RemoraB200Error):
    """The op / dtype / layout combination is not provided."""


class RemoraTimeoutError(RemoraB200Error):
    """A bounded device-side wait ran out; the affected results are invalid."""


class RemoraLimitError(RemoraB200Error):
    """A request exceeds a documented maximum size."""
