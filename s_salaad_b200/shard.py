"""Multi-GPU S+LR layer: block-row shards plus an all-gather of y.

Rank p of P owns the contiguous block-rows [bounds[p], bounds[p+1]) chosen
by ``slr_plan_shards`` so that every rank gets a nearly equal share of the
per-token cost ``nnz_i*bp*bq + bp*r`` (the Zipf-skewed rows of a layer do not
all land on one rank).  Each rank keeps the rebased crow/col/values slice,
its rows of A and bias, and the whole of B; ``x·Bᵀ`` is recomputed by every
rank (optionally split by tokens with an all-gather of H).  After the local
fused forward into its slot of a ``[P, T, Nmax]`` buffer, one all-gather
(NCCL on GPUs) gives every rank all slots and the columns are assembled
into y.

The reference runs on one device only; this module has no reference
counterpart and keeps the single-device arithmetic exactly (each output
element is computed by exactly one rank with the single-GPU kernels).

:class:`ShardPlan` is device-agnostic (bounds, slicing, gather, assembly);
:class:`ShardedLayer` adds the CUDA compute.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import ops


def shard_bounds(crow: np.ndarray, block_p: int, block_q: int, rank_r: int, world: int) -> np.ndarray:
    return ops.plan_shards(np.asarray(crow, dtype=np.int32), block_p, block_q, rank_r, world)


class ShardPlan:
    """Which block-rows rank `rank` owns, and how y is reassembled."""

    def __init__(self, crow: np.ndarray, *, out_features: int, block_p: int, block_q: int, rank_r: int,
                 rank: int, world: int, group=None):
        self.crow = np.asarray(crow, dtype=np.int64)
        self.rank, self.world, self.group = rank, world, group
        self.block_p = block_p
        self.out_features = out_features
        self.bounds = shard_bounds(self.crow, block_p, block_q, rank_r, world)
        self.widths = (np.diff(self.bounds) * block_p).astype(np.int64)
        self.wmax = int(self.widths.max())
        self.n0 = int(self.bounds[rank]) * block_p
        self.width = int(self.widths[rank])

    def slice(self, t: dict) -> dict:
        """This rank's part of a layer's tensors (keys of ``LayerSpec.tensors``)."""
        r0, r1 = int(self.bounds[self.rank]), int(self.bounds[self.rank + 1])
        j0, j1 = int(self.crow[r0]), int(self.crow[r1])
        bp = self.block_p
        dev = t["A"].device
        crow_p = torch.from_numpy((self.crow[r0:r1 + 1] - j0).astype(np.int32)).to(dev)
        return dict(A=t["A"][r0 * bp:r1 * bp].contiguous(), B=t["B"],
                    bias=None if t.get("bias") is None else t["bias"][r0 * bp:r1 * bp].contiguous(),
                    S_crow=crow_p, S_col=t["S_col"][j0:j1].contiguous(),
                    S_values=t["S_values"][j0:j1].contiguous(),
                    S_active_rows=(crow_p[1:] - crow_p[:-1]).nonzero().squeeze(-1).to(torch.int32))

    def gather_buffer(self, T: int, dtype, device) -> torch.Tensor:
        return torch.empty(self.world, T, self.wmax, dtype=dtype, device=device)

    def gather(self, buf: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """All-gather every rank's slot of `buf` and assemble y [T, N] in column order."""
        if self.world > 1:
            dist.all_gather_into_tensor(buf.view(-1), buf[self.rank].view(-1), group=self.group)
        T = buf.shape[1]
        if out is None:
            out = torch.empty(T, self.out_features, dtype=buf.dtype, device=buf.device)
        parts = [buf[p][:, :int(w)] for p, w in enumerate(self.widths) if w]
        torch.cat(parts, dim=1, out=out)
        return out


class ShardedLayer(ShardPlan):
    """One rank's part of a block-row-sharded S+LR layer on CUDA.

    ``x·Bᵀ`` is recomputed by every rank by default.  With
    ``split_lowrank=True`` (and T divisible by the world size) each rank
    writes the H rows of its token slice straight into its row range of the
    layer workspace and an in-place all-gather (on ``group_h``) completes H on
    every rank; on B200 the collective's latency exceeds the GEMM time it
    saves at these sizes, so it is off by default.  The y
    all-gather runs asynchronously on ``group_y`` (a second communicator, so
    it overlaps the next layer's H exchange and kernels): :meth:`start`
    returns a handle, :meth:`finish` waits and assembles y.
    """

    def __init__(self, t: dict, crow: np.ndarray, *, in_features: int, out_features: int, block_p: int,
                 block_q: int, rank: int, world: int, group=None, group_h=None, split_lowrank: bool = False):
        super().__init__(crow, out_features=out_features, block_p=block_p, block_q=block_q,
                         rank_r=int(t["A"].shape[1]), rank=rank, world=world, group=group)
        self.group_h = group_h  # None: the default process group
        self.split_lowrank = split_lowrank
        self.in_features = in_features
        self.rank_r = int(t["A"].shape[1])
        self.dtype = t["A"].dtype
        self.device = t["A"].device
        self.desc = None
        if self.width:
            p = self.slice(t)
            nnz = int(p["S_col"].numel())
            order = torch.from_numpy(ops.plan_row_order(p["S_crow"].cpu().numpy())).to(self.device)
            self.desc = ops.LayerDesc(A=p["A"], B=p["B"], bias=p["bias"],
                                      crow=p["S_crow"] if nnz else None, col=p["S_col"] if nnz else None,
                                      values=p["S_values"] if nnz else None, row_order=order if nnz else None,
                                      in_features=in_features, out_features=self.width, block_p=block_p,
                                      block_q=block_q)
        self._buf: torch.Tensor | None = None

    def local_buffer(self, T: int) -> torch.Tensor:
        if self._buf is None or self._buf.shape[1] != T:
            self._buf = self.gather_buffer(T, self.dtype, self.device)
        return self._buf

    def _lowrank(self, x2: torch.Tensor) -> None:
        """H = x2·Bᵀ into the layer workspace, token-split across ranks when possible."""
        T = x2.shape[0]
        d = self.desc
        ws = d.workspace(T)
        if self.rank_r == 0 or ws is None:
            return
        tp = T // self.world
        # token split only on the tensor-core path (>= 128 rows per rank): the small-M
        # path keeps split-K counters after its H rows, which the H all-gather would overwrite
        if self.split_lowrank and self.world > 1 and T % self.world == 0 and tp >= 128 and x2.stride(1) == 1:
            ldh = (self.rank_r + 63) // 64 * 64
            hbytes = T * ldh * x2.element_size()
            off = self.rank * tp * ldh * x2.element_size()
            if off % 256 == 0:
                # room for the slice call's own layout (H rows, then its scratch) at the offset
                ws = d.workspace(T, at_least=off + d.workspace_bytes(tp))
                import ctypes

                from . import _lib

                xs = x2[self.rank * tp:(self.rank + 1) * tp]
                rc = _lib.load().slr_lrs_linear_lowrank(
                    ctypes.byref(d.struct), xs.data_ptr(), xs.stride(0), tp, ws.data_ptr() + off, ws.numel() - off,
                    torch.cuda.current_stream(self.device).cuda_stream)
                _lib.check(rc, "lrs_linear_lowrank (token shard)")
                h = ws[:hbytes]
                dist.all_gather_into_tensor(h, h[off:off + tp * ldh * x2.element_size()], group=self.group_h)
                return
        d.lowrank(x2)

    def start(self, x2: torch.Tensor):
        """Local shard of y plus an asynchronous all-gather; returns a handle for finish()."""
        T = x2.shape[0]
        buf = self.local_buffer(T)
        if self.desc is not None:
            self._lowrank(x2)
            self.desc.combine(x2, buf[self.rank][:, :self.width])
        work = None
        if self.world > 1:
            work = dist.all_gather_into_tensor(buf.view(-1), buf[self.rank].view(-1), group=self.group,
                                               async_op=True)
        return work, buf

    def finish(self, handle, out: torch.Tensor | None = None) -> torch.Tensor:
        work, buf = handle
        if work is not None:
            work.wait()
        T = buf.shape[1]
        if out is None:
            out = torch.empty(T, self.out_features, dtype=buf.dtype, device=buf.device)
        parts = [buf[p][:, :int(w)] for p, w in enumerate(self.widths) if w]
        torch.cat(parts, dim=1, out=out)
        return out

    def forward(self, x2: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        return self.finish(self.start(x2), out)
