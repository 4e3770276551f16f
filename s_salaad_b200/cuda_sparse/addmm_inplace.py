"""The in-place BSR addmm operator, under the reference's operator name.

The reference defines ``ssalaad::tilelang_bsr_addmm_inplace_dense_`` in
``ssalaad/tilelang_sparse/addmm_inplace.py:130-141`` with a TileLang CUDA
implementation and a fake (meta) implementation.  :func:`register_reference_op`
defines the same schema with the libslr_b200 kernel as its CUDA
implementation, so ``_LRSLinearLRBlockCUDA.forward``-style callers
(``torch.ops.ssalaad.tilelang_bsr_addmm_inplace_dense_(y, x, crow, col,
values, active_rows)``) run unchanged.  It must be called in a process that
has not imported the reference's TileLang module (both would define the op).
"""
from __future__ import annotations

import torch

from .. import ops

_SCHEMA = ("tilelang_bsr_addmm_inplace_dense_(Tensor(a!) out_inplace, Tensor x, Tensor crow_indices, "
           "Tensor col_indices, Tensor values, Tensor active_rows) -> ()")
_lib = None


def get_tuned_config(block_p: int, block_q: int) -> dict:
    """Row multiple the caller may pad M to (reference: addmm_inplace.py:36-38).

    The B200 kernels take any M, so no padding is required: BM = 1.  The
    warp-tile keys are kept for callers that read them.
    """
    return {"BM": 1, "WARP_TILE_M": 16, "WARP_TILE_N": int(block_p)}


def _impl(out_inplace, x, crow_indices, col_indices, values, active_rows) -> None:
    ops.bsr_addmm_inplace_(out_inplace, x, crow_indices, col_indices, values, active_rows)


def register_reference_op() -> bool:
    """Define ``ssalaad::tilelang_bsr_addmm_inplace_dense_`` (CUDA + fake).

    Returns False if the operator already exists in this process.
    """
    global _lib
    if _lib is not None:
        return True
    try:
        torch.ops.ssalaad.tilelang_bsr_addmm_inplace_dense_  # noqa: B018
        return False
    except (AttributeError, RuntimeError):
        pass
    lib = torch.library.Library("ssalaad", "DEF")
    lib.define(_SCHEMA)
    lib.impl("tilelang_bsr_addmm_inplace_dense_", _impl, "CUDA")

    @torch.library.register_fake("ssalaad::tilelang_bsr_addmm_inplace_dense_", lib=lib)
    def _fake(out_inplace, x, crow_indices, col_indices, values, active_rows) -> None:
        return None

    _lib = lib
    return True
