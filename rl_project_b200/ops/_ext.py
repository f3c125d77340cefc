"""Loader for the in-tree sm_100a extension ``rl_project_b200._C``.

On a CUDA tensor every op in this package runs its native kernel; if the
extension is missing there, ``native()`` raises instead of silently falling
back to an eager PyTorch path.  CPU tensors use the plain-PyTorch reference
implementation of the same op (the numerics oracle and the CPU training path).
"""

from __future__ import annotations

import os
from typing import Any, Optional

import torch

_C: Optional[Any] = None
_err: Optional[BaseException] = None

try:  # pragma: no cover - depends on the build
    from rl_project_b200 import _C as _C  # type: ignore[no-redef]
except BaseException as exc:  # noqa: BLE001
    _C = None
    _err = exc


# kernels launched by each binding (launch accounting for benchmarks)
_LAUNCHES = {"rmsnorm_bwd": 2, "grad_norm": 2, "adam_chunk_size": 0, "adam_tensor_desc_bytes": 0, "bounds_status": 0}


class _Counted:
    """Forwards to the extension module and counts the kernels each call launches."""

    def __init__(self, mod: Any):
        self._mod = mod
        self._fns: dict = {}
        self.launches = 0

    def __getattr__(self, name: str):
        fns = self.__dict__["_fns"]
        if name not in fns:
            fn = getattr(self.__dict__["_mod"], name)
            if not callable(fn):
                return fn
            n = _LAUNCHES.get(name, 1)

            def call(*a, __fn=fn, __n=n, **k):
                self.launches += __n
                return __fn(*a, **k)

            fns[name] = call
        return fns[name]


_counted = _Counted(_C) if _C is not None else None


def available() -> bool:
    return _C is not None


def native() -> Any:
    if _counted is None:
        raise RuntimeError(
            "rl_project_b200._C (the sm_100a kernel library) is not built or failed to load: "
            f"{_err!r}. Build it with `python setup.py build_ext --inplace`."
        )
    return _counted


def launch_count() -> int:
    """Native kernels launched so far in this process (through the bindings)."""
    return _counted.launches if _counted is not None else 0


def count_launches(n: int) -> None:
    """Record launches made outside the counted bindings (e.g. extensions built separately)."""
    if _counted is not None:
        _counted.launches += n


def on_gpu(t: torch.Tensor) -> bool:
    return t.is_cuda


_SMS: dict = {}


def sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def debug_checks() -> bool:
    return os.environ.get("RLB_DEBUG_BOUNDS", "0") == "1"


def bounds_code(device: torch.device, clear: bool = True) -> int:
    """The shared index-error word of ``device`` (0: no kernel skipped an out-of-range index).
    Synchronises with the device; ``clear`` resets the word after reading it."""
    return int(native().bounds_status(int(torch.device(device).index or 0), clear))


def raise_bounds_error(code: int) -> None:
    """Raise the ``KernelError`` that a non-zero index-error word stands for (no-op for 0)."""
    from rl_project_b200.core.errors import KernelError

    if code:
        raise KernelError(f"a kernel reported an out-of-range index (status {code})",
                          hint="A position, token or block id exceeded its table; the affected rows were skipped.")


def check_bounds(device: torch.device, clear: bool = True) -> None:
    """Raise ``KernelError`` if a kernel on ``device`` reported an out-of-range index into the shared
    index-error word (RoPE positions outside the cos / sin table).  Synchronises with the device."""
    raise_bounds_error(bounds_code(device, clear))
