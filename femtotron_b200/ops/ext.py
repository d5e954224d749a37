"""Loader for the sm_100a native extension ``femtotron_b200._C``.

CUDA tensors always run through the hand-written kernels of the extension.  When the
extension is missing on a machine with a GPU, every CUDA op raises instead of silently
falling back to PyTorch.  CPU tensors (unit tests, gloo ranks) use the plain PyTorch
restatement of each op in this package.
"""
from __future__ import annotations

import torch

_C = None
_IMPORT_ERROR: Exception | None = None

# Number of native kernel launches issued through this module.  Read by the benchmark.
LAUNCHES = [0]

# Kernels launched per call of an entry point when it is not exactly one: the flash backward
# runs three (delta/LSE pre-pass, main, fp32 -> bf16 convert); the memory-management and
# stream-memory-operation entry points launch none (copy engines, cuStreamWriteValue32).
KERNELS_PER_CALL = {
    "flash_bwd": 3,
    "symm_alloc": 0, "ipc_handle": 0, "ipc_open": 0, "ipc_close": 0, "tensor_at": 0,
    "copy_from_ptrs": 0, "stream_write": 0,
}


class _Counted:
    """Proxy of the extension module that counts kernel launches."""

    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        n = KERNELS_PER_CALL.get(name, 1)

        def wrapped(*a, **k):
            LAUNCHES[0] += n
            return fn(*a, **k)
        wrapped.__name__ = name
        return wrapped


def native():
    """Return the compiled extension module, raising a clear error if it is not built."""
    global _C, _IMPORT_ERROR
    if _C is None:
        try:
            from femtotron_b200 import _C as mod  # type: ignore[attr-defined]
        except ImportError as e:  # pragma: no cover - depends on the build
            _IMPORT_ERROR = e
            raise RuntimeError(
                "femtotron_b200 native extension is not built; run "
                "`python setup.py build_ext --inplace` (sm_100a) before using CUDA tensors"
            ) from e
        _C = _Counted(mod)
    return _C


def has_native() -> bool:
    try:
        native()
        return True
    except RuntimeError:
        return False


_ERR: dict[int, torch.Tensor] = {}


def error_flag(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that bounded device-side waits write on timeout."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _ERR.get(idx)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _ERR[idx] = t
    return t


class KernelTimeoutError(RuntimeError):
    """A native kernel gave up on a bounded wait (see the error code)."""


def check_kernel_errors(device: torch.device | None = None) -> None:
    """Raise KernelTimeoutError if any native kernel on `device` reported a bounded-wait
    timeout since the last check (reads one int from the device; synchronises)."""
    devs = [device] if device is not None else [torch.device("cuda", i) for i in _ERR]
    for d in devs:
        t = _ERR.get(d.index if d.index is not None else torch.cuda.current_device())
        if t is None:
            continue
        code = int(t.item())
        if code != 0:
            t.zero_()
            raise KernelTimeoutError(f"native kernel reported bounded-wait timeout, code {code}")
