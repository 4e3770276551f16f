"""S+LR linear modules on B200, with the reference's module API.

Mirrors ``ssalaad/efficient/ls_linear.py`` of S-SALAAD: the same class names,
constructor arguments, registered buffers (``A``, ``B``, ``bias``,
``S_crow``, ``S_col``, ``S_values``, ``S_active_rows``, so state dicts are
interchangeable) and exceptions, with the forward routed to the fused CUDA
kernels of libslr_b200 instead of F.linear + TileLang:

* :class:`_LRSLinearLR` (reference :47-54) — ``S == 0``: the fused kernel
  with no sparse term.
* :class:`_LRSLinearLRBlockBase` (reference :57-104) — BSR buffers.
* :class:`_LRSLinearLRBlockCUDA` (reference :107-137) — one fused launch pair
  (``x·Bᵀ`` then sparse + up-projection + bias) instead of pad, two cuBLAS
  calls, the in-place TileLang kernel and a bias pass.
* :func:`LRSLinear` (reference :227-285) — the factory.

* :class:`_LRSLinearLRNM` (reference :167-224) — S 2:4 sparse along K: the
  sparse product on the sparse tensor cores (mma.sp) fused with the
  up-projection and the bias, instead of cuSPARSELt plus addmm and a bias pass.

There is no CPU path: CPU tensors are rejected with ValueError (the
reference's CPU kernel stays the oracle).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .. import ops


class _LRSLinearBase(nn.Module):
    kind: str = ""

    def __init__(self, A: torch.Tensor, B: torch.Tensor, *, in_features: int, out_features: int,
                 bias: torch.Tensor | None = None) -> None:
        super().__init__()
        (n, r) = A.shape
        (rB, m) = B.shape
        if rB != r:
            raise ValueError(f"A.shape[1]={r} must match B.shape[0]={rB}")
        if (n, m) != (out_features, in_features):
            raise ValueError(
                f"L = A·B shape ({n},{m}) must equal (out_features={out_features}, in_features={in_features})")
        self.in_features = in_features
        self.out_features = out_features
        self.r = int(r)
        self.register_buffer("B", B.contiguous())
        self.register_buffer("A", A.contiguous())
        if bias is not None:
            self.register_buffer("bias", bias.contiguous().to(A.dtype))
        else:
            self.bias = None
        self._desc: ops.LayerDesc | None = None
        self._group = None  # set by efficient.model.group_projections
        self._group_index = 0

    # ------------------------------------------------------------ kernels --
    def _check_device(self) -> None:
        if not self.A.is_cuda:
            raise ValueError("s_salaad_b200 layers require CUDA tensors (no CPU path).")
        if self.A.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            raise ValueError("s_salaad_b200 layers require fp16, bf16 or fp32.")

    def _desc_tensors(self) -> dict:
        return dict(A=self.A, B=self.B, bias=self.bias)

    def _layer_desc(self) -> ops.LayerDesc:
        t = self._desc_tensors()
        key = tuple(None if v is None else v.data_ptr() for v in t.values())
        d = self._desc
        if d is None or d.key != key or d.dtype != self.A.dtype:
            d = ops.LayerDesc(in_features=self.in_features, out_features=self.out_features,
                              block_p=getattr(self, "block_p", 0), block_q=getattr(self, "block_q", 0), **t)
            self._desc = d
        return d

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._group is not None and x.is_cuda and x.dtype == self.A.dtype:
            return self._group.output(self._group_index, x)
        return ops.lrs_linear_forward(self._layer_desc(), x)


class _LRSLinearLR(_LRSLinearBase):
    kind = "lr_only"

    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        self._check_device()

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, rank={self.r}, "
                f"S=zero (skipped), bias={self.bias is not None}")


class _LRSLinearLRBlockBase(_LRSLinearBase):
    """Block-sparse S in BSR layout (same buffers as the reference)."""

    kind = "block_sparse"

    def __init__(self, A: torch.Tensor, B: torch.Tensor, S_sparse: torch.Tensor, *, in_features: int,
                 out_features: int, bias: torch.Tensor | None, block_p: int, block_q: int) -> None:
        super().__init__(A, B, in_features=in_features, out_features=out_features, bias=bias)
        if tuple(S_sparse.shape) != (out_features, in_features):
            raise ValueError(f"S shape {tuple(S_sparse.shape)} must equal "
                             f"(out_features, in_features)=({out_features},{in_features})")
        self.block_p = int(block_p)
        self.block_q = int(block_q)
        self.S_nnz = int(S_sparse._nnz())
        crow = S_sparse.crow_indices()
        self.register_buffer("S_crow", crow.to(torch.int32).clone())
        self.register_buffer("S_col", S_sparse.col_indices().to(torch.int32).clone())
        self.register_buffer("S_values", S_sparse.values().transpose(1, 2).contiguous().clone().to(A.dtype))
        active = (crow[1:] - crow[:-1]).nonzero(as_tuple=False).squeeze(-1)
        self.register_buffer("S_active_rows", active.to(torch.int32).clone())

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, rank={self.r}, "
                f"S_nnz={self.S_nnz}, block=({self.block_p}×{self.block_q}), bias={self.bias is not None}")


class _LRSLinearLRBlockCUDA(_LRSLinearLRBlockBase):
    """Fused sm_100a block-sparse + low-rank kernels of libslr_b200."""

    def __init__(self, *args, **kwargs) -> None:
        super().__init__(*args, **kwargs)
        if self.S_values.device.type != "cuda":
            raise ValueError("The B200 block kernel requires CUDA.")
        mult = 8 if self.S_values.dtype == torch.float32 else 16
        if self.block_p % mult or self.block_q % mult:
            raise ValueError(f"The B200 block kernel requires block dimensions divisible by {mult}.")
        if self.S_values.dtype not in (torch.float16, torch.bfloat16, torch.float32):
            raise ValueError("The B200 block kernel requires fp16, bf16 or fp32.")
        # One device-side structure check at load time; the forward trusts it.
        ops.validate_bsr(self.S_crow, self.S_col, self.in_features // self.block_q, self.S_active_rows)
        # Heaviest block-rows first (persistent-schedule order).
        order = ops.plan_row_order(self.S_crow)
        self.register_buffer("_row_order", torch.from_numpy(order).to(self.S_crow.device), persistent=False)

    def _desc_tensors(self) -> dict:
        return dict(A=self.A, B=self.B, bias=self.bias, crow=self.S_crow, col=self.S_col,
                    values=self.S_values, row_order=self._row_order)


class _LRSLinearLRNM(_LRSLinearBase):
    """S with at most 2 nonzeros in every aligned group of 4 input features.

    Same constructor arguments, persistent buffers (``A``, ``B``, ``bias``)
    and ``S_nnz`` (kept entries, K/2 per row) as the reference class
    (ls_linear.py:167-190); S may be given dense or as a torch sparse tensor
    (the reference takes torch's semi-structured packing of it).  S is kept in
    the library's compressed layout (``_nm_values`` [N, K/2] and ``_nm_meta``
    [N, K/32], non-persistent like the reference's packed buffers)."""

    kind = "nm"

    def __init__(self, A: torch.Tensor, B: torch.Tensor, S: torch.Tensor, *, in_features: int, out_features: int,
                 bias: torch.Tensor | None = None) -> None:
        super().__init__(A, B, in_features=in_features, out_features=out_features, bias=bias)
        self._check_device()
        if A.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("The B200 N:M kernel requires fp16 or bf16.")
        dense = S.to_dense() if S.layout != torch.strided else S
        if tuple(dense.shape) != (out_features, in_features):
            raise ValueError(f"S shape {tuple(dense.shape)} must equal "
                             f"(out_features, in_features)=({out_features},{in_features})")
        values, meta = ops.nm_compress(dense.to(device=A.device, dtype=A.dtype))
        self.S_nnz = int(values.numel())
        self.register_buffer("_nm_values", values, persistent=False)
        self.register_buffer("_nm_meta", meta, persistent=False)
        self._nm_desc: ops.NmLayerDesc | None = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        t = (self._nm_values, self._nm_meta, self.A, self.B, self.bias)
        key = tuple(None if v is None else v.data_ptr() for v in t)
        d = self._nm_desc
        if d is None or getattr(d, "key", None) != key:
            d = ops.NmLayerDesc(values=self._nm_values, meta=self._nm_meta, A=self.A, B=self.B, bias=self.bias,
                                in_features=self.in_features, out_features=self.out_features)
            d.key = key
            self._nm_desc = d
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        return d.forward(x2).reshape(*shape[:-1], self.out_features)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, rank={self.r}, "
                f"S_nnz={self.S_nnz}, N:M 2:4 (sparse tensor cores), bias={self.bias is not None}")


def LRSLinear(A, B, S_sparse, *, in_features, out_features, bias=None, block_p=None, block_q=None,
              nm_n=None, nm_m=None):
    """Compute ``x @ (A @ B + S).T + bias`` with the B200 kernels.

    Same dispatch as the reference factory (ls_linear.py:227-285): LR-only
    when S has no stored entry, the N:M 2:4 kernel when ``nm_n``/``nm_m`` are
    given, the block kernel for BSR S.  CPU tensors are rejected (ValueError)
    — this package is the CUDA path only.
    """
    if S_sparse.layout == torch.strided:
        nnz = int(torch.count_nonzero(S_sparse))
    else:
        nnz = S_sparse._nnz()
    kwargs = dict(in_features=in_features, out_features=out_features, bias=bias)
    if not A.is_cuda:
        raise ValueError("s_salaad_b200.LRSLinear requires CUDA tensors (the CPU path is the reference's).")
    if nnz == 0:
        return _LRSLinearLR(A, B, **kwargs)
    if nm_n is not None:
        if (nm_n, nm_m) != (2, 4):
            raise ValueError("N:M inference requires CUDA and a 2:4 mask.")
        return _LRSLinearLRNM(A, B, S_sparse, **kwargs)
    if block_p is None or block_q is None:
        raise ValueError("Sparse S needs a recorded block shape to pick a kernel.")
    if S_sparse.layout == torch.strided:
        from .artifact import dense_to_bsr
        S_sparse = dense_to_bsr(S_sparse, int(block_p), int(block_q))
    return _LRSLinearLRBlockCUDA(A, B, S_sparse, block_p=block_p, block_q=block_q, **kwargs)
