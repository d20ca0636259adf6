"""Data wrapper, device/stream plumbing and profiling hooks.

Mirrors the parts of rdv/core/_core.py the hot path exposes:

* ``RDVObject`` / ``wrap`` (rdv/core/_core.py:273-380): wrap any tensor; a
  tensor already on the GPU is aliased (no copy), a host tensor is copied to
  the current CUDA device. ``device_ptr``, ``shape``, ``as_tensor(backend)``.
* ``profiling`` / ``reset_submit_times`` / ``profiling_submit_times``
  (rdv/core/_core.py:54-59, 2877-2886, 3179-3188). The reference sums the
  wall time of its blocking ``vk.submit_and_wait``; here, with profiling on,
  each launch is bracketed by CUDA events on the launch stream and the call
  waits for them, so the sum is device time in seconds.

Device memory and streams come from PyTorch: work is enqueued on
``torch.cuda.current_stream()``, so results are ordered with the caller's
own torch work on that stream.
"""
from __future__ import annotations

import contextlib
import math

import torch

__PROFILING__ = False
__submit_times__ = 0.0


def profiling(enable: bool = True) -> None:
    global __PROFILING__
    __PROFILING__ = bool(enable)


def reset_submit_times() -> None:
    global __submit_times__
    __submit_times__ = 0.0


def profiling_submit_times() -> float:
    return __submit_times__


@contextlib.contextmanager
def _timed():
    """Context around one operator's launches: with profiling on, records CUDA
    events on the current stream and adds the elapsed seconds to the
    submit-time total (synchronizing on the end event, like the reference's
    blocking submit)."""
    if not __PROFILING__:
        yield
        return
    global __submit_times__
    s = torch.cuda.current_stream()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(s)
    yield
    end.record(s)
    end.synchronize()
    __submit_times__ += start.elapsed_time(end) / 1000.0


def current_device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("rdv_project_b200 needs a CUDA device (B200, sm_100a); none is available")
    return torch.device("cuda", torch.cuda.current_device())


def stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


class RDVObject:
    """Wraps a tensor-like object as device memory of the current CUDA device.

    A CUDA tensor is aliased (so later in-place edits are seen by operators
    that read it again, as with the reference's aliasing wrap,
    rdv/core/_core.py:278-283); anything else (a CPU tensor, a numpy array,
    nested lists) is converted to a torch tensor and copied to the device."""

    def __init__(self, data):
        if isinstance(data, RDVObject):
            data = data._tensor
        if not isinstance(data, torch.Tensor):
            data = torch.as_tensor(data)
        # Without a CUDA device the data stays where it is: construction and
        # shape validation still work, and every operator call then raises.
        if torch.cuda.is_available():
            dev = torch.device("cuda", torch.cuda.current_device())
            if data.device != dev:
                data = data.to(dev, non_blocking=data.device.type == "cpu" and data.is_pinned())
        self._data = data
        self._tensor = data
        self._tensor_cache = {}

    @property
    def device_ptr(self) -> int:
        return self._tensor.data_ptr()

    @property
    def device_index(self) -> int:
        return self._tensor.device.index

    @property
    def shape(self):
        return tuple(self._tensor.shape)

    @property
    def scalar_type(self):
        return self._tensor.dtype

    @property
    def is_direct(self) -> bool:
        return True

    def as_tensor(self, backend: str = "torch"):
        if backend not in ("torch", "jax", "numpy", "cupy", "tensorflow"):
            raise NotImplementedError(
                f"Unknown backend {backend}. Supported backends are: torch, jax, numpy, cupy, tensorflow.")
        if backend == "torch":
            return self._tensor
        if backend == "numpy":
            return self._tensor.detach().cpu().numpy()
        raise NotImplementedError(f"backend {backend} is not available in this build")

    def as_type(self, backend: str = "torch"):
        return self.as_tensor(backend)

    def host(self) -> "RDVObject":
        out = RDVObject.__new__(RDVObject)
        out._data = out._tensor = self._tensor.detach().cpu()
        out._tensor_cache = {}
        return out

    def device(self) -> "RDVObject":
        return RDVObject(self._tensor.clone())

    def __repr__(self):
        return f"RDVObject(shape={self.shape}, dtype={self._tensor.dtype}, device={self._tensor.device})"


def wrap(data) -> RDVObject:
    if isinstance(data, RDVObject):
        return data
    return RDVObject(data)


def as_device_tensor(x) -> torch.Tensor:
    """Tensor view of an RDVObject / tensor on the current device
    (host data is copied)."""
    if isinstance(x, RDVObject):
        return x._tensor
    return wrap(x)._tensor


def numel_of(shape) -> int:
    return int(math.prod(shape)) if len(shape) else 1
