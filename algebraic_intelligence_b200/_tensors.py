"""Host-side array plumbing shared by the operator modules.

The operators accept CUDA tensors (the normal case: inputs already resident in
HBM) and, for host callers, NumPy arrays or CPU tensors, which are copied to the
current CUDA device and whose results are copied back. Nothing is ever computed
on the host.
"""
from __future__ import annotations

import numpy as np
import torch


class Staged:
    """Moves host inputs to the GPU and results back to the caller's kind."""

    def __init__(self, *arrays):
        self.kind = "torch"
        self.host_device = None
        tensors = []
        for a in arrays:
            if isinstance(a, np.ndarray) or np.isscalar(a):
                self.kind = "numpy"
                a = torch.from_numpy(np.ascontiguousarray(a))
            elif not isinstance(a, torch.Tensor):
                a = torch.as_tensor(a)
            tensors.append(a)
        dev = next((t.device for t in tensors if t.is_cuda), None)
        if dev is None:
            if not torch.cuda.is_available():
                raise RuntimeError("a CUDA device is required: this library has no CPU execution path")
            dev = torch.device("cuda", torch.cuda.current_device())
            if self.kind == "torch":
                self.host_device = tensors[0].device if tensors else None
        self.device = dev
        self.tensors = [t.to(dev, non_blocking=False).contiguous() for t in tensors]

    def back(self, t):
        if t is None:
            return None
        if self.kind == "numpy":
            return t.cpu().numpy()
        if self.host_device is not None:
            return t.to(self.host_device)
        return t


def host_checks_float(*arrays) -> None:
    """TypeError for non-floating inputs (src/primitives.py:19-20)."""
    for a in arrays:
        dt = a.dtype
        if isinstance(a, np.ndarray):
            ok = np.issubdtype(dt, np.floating)
        else:
            ok = dt.is_floating_point
        if not ok:
            raise TypeError("expected a floating point array")
