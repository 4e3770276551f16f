"""Multi-GPU S+LR layer: block-row shards plus an all-gather of y.

Rank p of P owns the contiguous block-rows [bounds[p], bounds[p+1]) chosen
by ``slr_plan_shards`` so that every rank gets a nearly equal share of the
per-token cost ``nnz_i*bp*bq + bp*r`` (the Zipf-skewed rows of a layer do not
all land on one rank).  Each rank keeps the rebased crow/col/values slice,
its rows of A and bias, and the whole of B (``x·Bᵀ`` is recomputed per rank,
2*T*r*K flops, instead of exchanging it).  After the local fused forward,
one NCCL all-gather assembles y on every rank.

The reference runs on one device only; this module has no reference
counterpart and follows the single-device arithmetic exactly (each output
element is computed by exactly one rank with the single-GPU kernels).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import ops


def shard_bounds(crow: np.ndarray, block_p: int, block_q: int, rank_r: int, world: int) -> np.ndarray:
    return ops.plan_shards(np.asarray(crow, dtype=np.int32), block_p, block_q, rank_r, world)


def shard_tensors(t: dict, crow: np.ndarray, block_p: int, bounds: np.ndarray, rank: int) -> dict:
    """Slice a layer's tensors (from ``LayerSpec.tensors``) to rank's block-rows."""
    r0, r1 = int(bounds[rank]), int(bounds[rank + 1])
    j0, j1 = int(crow[r0]), int(crow[r1])
    dev = t["A"].device
    crow_p = torch.from_numpy((np.asarray(crow[r0:r1 + 1]) - j0).astype(np.int32)).to(dev)
    out = dict(A=t["A"][r0 * block_p:r1 * block_p].contiguous(), B=t["B"],
               bias=None if t["bias"] is None else t["bias"][r0 * block_p:r1 * block_p].contiguous(),
               S_crow=crow_p, S_col=t["S_col"][j0:j1].contiguous(), S_values=t["S_values"][j0:j1].contiguous())
    active = (crow_p[1:] - crow_p[:-1]).nonzero().squeeze(-1).to(torch.int32)
    out["S_active_rows"] = active
    return out


class ShardedLayer:
    """One rank's part of a block-row-sharded S+LR layer."""

    def __init__(self, t: dict, crow: np.ndarray, *, in_features: int, out_features: int, block_p: int,
                 block_q: int, rank: int, world: int, group=None):
        self.rank, self.world, self.group = rank, world, group
        r = int(t["A"].shape[1])
        self.bounds = shard_bounds(crow, block_p, block_q, r, world)
        self.widths = (np.diff(self.bounds) * block_p).astype(np.int64)
        self.wmax = int(self.widths.max())
        self.n0 = int(self.bounds[rank]) * block_p
        self.width = int(self.widths[rank])
        self.out_features = out_features
        self.in_features = in_features
        self.dtype = t["A"].dtype
        self.device = t["A"].device
        self.desc = None
        if self.width:
            p = shard_tensors(t, crow, block_p, self.bounds, rank)
            order = torch.from_numpy(ops.plan_row_order(p["S_crow"].cpu().numpy())).to(self.device)
            nnz = int(p["S_col"].numel())
            self.desc = ops.LayerDesc(A=p["A"], B=p["B"], bias=p["bias"],
                                      crow=p["S_crow"] if nnz else None, col=p["S_col"] if nnz else None,
                                      values=p["S_values"] if nnz else None, row_order=order if nnz else None,
                                      in_features=in_features, out_features=self.width, block_p=block_p,
                                      block_q=block_q)
        self._buf: torch.Tensor | None = None

    def gather_buffer(self, T: int) -> torch.Tensor:
        if self._buf is None or self._buf.shape[1] != T:
            self._buf = torch.empty(self.world, T, self.wmax, dtype=self.dtype, device=self.device)
        return self._buf

    def local(self, x2: torch.Tensor) -> torch.Tensor:
        """This rank's columns of y, written into its slot of the gather buffer."""
        buf = self.gather_buffer(x2.shape[0])
        if self.desc is not None:
            self.desc.forward(x2, out=buf[self.rank][:, :self.width])
        return buf

    def gather(self, buf: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """All-gather every rank's slot and assemble y [T, N] in column order."""
        if self.world > 1:
            dist.all_gather_into_tensor(buf.view(-1), buf[self.rank].view(-1), group=self.group)
        T = buf.shape[1]
        if out is None:
            out = torch.empty(T, self.out_features, dtype=self.dtype, device=self.device)
        parts = [buf[p][:, :int(w)] for p, w in enumerate(self.widths) if w]
        torch.cat(parts, dim=1, out=out)
        return out

    def forward(self, x2: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return self.gather(self.local(x2), out)
