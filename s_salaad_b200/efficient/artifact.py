"""BSR conversion on the GPU, bit-exact with the reference.

Mirrors ``dense_to_bsr`` of ``ssalaad/efficient/artifact.py:20-37``: same
name, arguments, ValueError text and result (a ``torch.sparse_bsr_tensor``
with int64 crow/col and blocks in row-major order), computed by the
libslr_b200 kernels for CUDA tensors.  The bundle format itself
(save/load_artifact) is not part of this package.
"""
from __future__ import annotations

import torch

from .. import ops


def dense_to_bsr(S: torch.Tensor, block_p: int, block_q: int) -> torch.Tensor:
    (n, m) = S.shape
    if n % block_p or m % block_q:
        raise ValueError(f"shape ({n}, {m}) not divisible by block ({block_p}, {block_q})")
    crow, col, values = ops.dense_to_bsr_cuda(S, int(block_p), int(block_q))
    return torch.sparse_bsr_tensor(crow, col, values, size=(n, m))


def module_buffers(S: torch.Tensor, block_p: int, block_q: int):
    """The layer buffers of ls_linear.py:86-97 straight from dense S:
    int32 crow/col, values ``[nnz, bq, bp]``, int32 active rows."""
    crow, col, values = ops.dense_to_bsr_cuda(S, int(block_p), int(block_q), transpose=True)
    active = (crow[1:] - crow[:-1]).nonzero(as_tuple=False).squeeze(-1)
    return crow.to(torch.int32), col.to(torch.int32), values, active.to(torch.int32)
