"""The in-place BSR addmm operator, under the reference's operator name.

The reference defines ``ssalaad::tilelang_bsr_addmm_inplace_dense_`` in
``ssalaad/tilelang_sparse/addmm_inplace.py:130-141`` with a TileLang CUDA
implementation and a fake (meta) implementation.  :func:`register_reference_op`
defines the same schema with the libslr_b200 kernel as its CUDA
implementation, so ``_LRSLinearLRBlockCUDA.forward``-style callers
(``torch.ops.ssalaad.tilelang_bsr_addmm_inplace_dense_(y, x, crow, col,
values, active_rows)``) run unchanged.  It must be called in a process that
has not imported the reference's TileLang module (both would define the op).
It also defines the fused layer as ``ssalaad::slr_linear``.
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


# The fused layer as one functional operator: y = x·Sᵀ + (x·Bᵀ)·Aᵀ + bias on
# the layer's buffers (S as int32 S_crow / S_col and S_values [nnz, bq, bp],
# absent for a low-rank-only layer).  No reference counterpart.
_LINEAR_SCHEMA = ("slr_linear(Tensor x, Tensor A, Tensor B, Tensor? bias, Tensor? S_crow, Tensor? S_col, "
                  "Tensor? S_values, int block_p, int block_q) -> Tensor")
_descs: dict = {}
_MAX_DESCS = 256


def _linear_impl(x, A, B, bias, S_crow, S_col, S_values, block_p, block_q):
    sparse = S_col is not None and S_col.numel() > 0
    key = tuple(None if t is None else (t.data_ptr(), tuple(t.shape), t.dtype)
                for t in (A, B, bias, S_crow, S_col, S_values)) + (block_p, block_q)
    desc = _descs.get(key)
    if desc is None:
        if len(_descs) >= _MAX_DESCS:
            _descs.pop(next(iter(_descs)))
        order = None
        if sparse:
            order = torch.from_numpy(ops.plan_row_order(S_crow)).to(S_crow.device)
        desc = ops.LayerDesc(A=A, B=B, bias=bias, crow=S_crow if sparse else None, col=S_col if sparse else None,
                             values=S_values if sparse else None, row_order=order,
                             in_features=int(B.shape[1]), out_features=int(A.shape[0]),
                             block_p=int(block_p) if sparse else 0, block_q=int(block_q) if sparse else 0)
        _descs[key] = desc
    return ops.lrs_linear_forward(desc, x)


def register_reference_op() -> bool:
    """Define ``ssalaad::tilelang_bsr_addmm_inplace_dense_`` (CUDA + fake) and
    the fused ``ssalaad::slr_linear``.

    Returns False if the operators already exist in this process.
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
    lib.define(_LINEAR_SCHEMA)
    lib.impl("slr_linear", _linear_impl, "CUDA")

    @torch.library.register_fake("ssalaad::tilelang_bsr_addmm_inplace_dense_", lib=lib)
    def _fake(out_inplace, x, crow_indices, col_indices, values, active_rows) -> None:
        return None

    @torch.library.register_fake("ssalaad::slr_linear", lib=lib)
    def _fake_linear(x, A, B, bias, S_crow, S_col, S_values, block_p, block_q):
        return x.new_empty(*x.shape[:-1], A.shape[0])

    _lib = lib
    return True
