"""Device settings, chosen once: the same Backend object and preset names as the reference's src/trnopt/backend.py,
plus the "cuda-fused" preset that selects this package's fused CUDA half-step.

The reference's presets (backend.py:33-45) are kept so code that builds them still constructs the same objects,
but this package runs only the fused sm_100a kernels: sinkhorn() accepts a backend on a CUDA device in float32
(what "cuda-fused" gives) and raises ValueError for anything else, as the reference's kernel selection does for an
impossible request (sinkhorn.py:196-208). There is no CPU path here.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np
import torch


@dataclass(frozen=True)
class Backend:
    device: str = "cpu"
    dtype: torch.dtype = torch.float64
    compile: bool = False
    compile_backend: str | None = None

    @classmethod
    def preset(cls, name: str, **overrides) -> "Backend":
        """Named starting points; any field can be overridden, e.g. Backend.preset("cuda-fused", device="cuda:1")."""
        table = {
            "cpu": cls(),
            "cpu-float32": cls(dtype=torch.float32),
            "cuda": cls(device="cuda"),
            # This package's preset: the fused sm_100a half-step (kernel="auto" or "cuda" in SinkhornOptions).
            "cuda-fused": cls(device="cuda", dtype=torch.float32),
            "neuron": cls(device="neuron", dtype=torch.float32, compile=True, compile_backend="neuron"),
            "emulate-neuron": cls(device="cpu", dtype=torch.float32, compile=True),
            "mps": cls(device="mps", dtype=torch.float32),
        }
        if name not in table:
            raise ValueError(f"unknown backend preset {name!r}; choose from {sorted(table)}")
        return replace(table[name], **overrides)

    @property
    def is_cuda_fused(self) -> bool:
        return self.device.startswith("cuda") and self.dtype == torch.float32

    def torch_device(self) -> torch.device:
        dev = torch.device(self.device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        return dev

    def tensor(self, a) -> torch.Tensor:
        """Host array -> tensor of this backend's dtype on its device (converted on the host first)."""
        return torch.as_tensor(np.asarray(a), dtype=self.dtype).to(self.torch_device())
