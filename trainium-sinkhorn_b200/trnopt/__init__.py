"""trnopt (B200 build): entropic optimal transport with the Sinkhorn half-step fused into sm_100a CUDA kernels.

A drop-in for the hot path of evandiewald/trainium-sinkhorn's trnopt package: the same Backend, SinkhornOptions,
SinkhornResult, sinkhorn and transport_plan, with Backend.preset("cuda-fused") selecting the fused kernels, plus
the plan evaluated from potentials on the GPU (trnopt.plan: rows, marginals, pull-back).
"""

from .backend import Backend
from .sinkhorn import SinkhornOptions, SinkhornResult, sinkhorn, transport_plan

__all__ = ["Backend", "SinkhornOptions", "SinkhornResult", "sinkhorn", "transport_plan"]
