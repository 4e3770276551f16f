"""s_salaad_b200 — B200-native (sm_100a) sparse-plus-low-rank linear for S-SALAAD.

``y = x · Sᵀ + (x · Bᵀ) · Aᵀ + bias`` with S block-sparse (BSR), run by the
hand-written CUDA kernels of ``libslr_b200.so`` (C ABI: include/slr_b200.h).
The package mirrors the reference's module and operator API
(``efficient.LRSLinear``, ``efficient.dense_to_bsr``,
``efficient.build_efficient_model``, ``cuda_sparse.register_reference_op``);
``ops.LayerGroup`` runs layers that read one input together and ``shard``
splits a layer by block-rows over several GPUs.  CUDA only; no CPU fallback.
"""
from . import ops
from ._lib import LIB_PATH, load

__all__ = ["ops", "load", "LIB_PATH"]
