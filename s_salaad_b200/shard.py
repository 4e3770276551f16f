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

With :class:`PeerOutputs` the all-gather disappears: every rank owns a full
y, the other ranks' y are mapped into its address space (CUDA IPC), and the
combine kernel's epilogue stores each output tile into all of them over
NVLink while it computes; a wait kernel ends the call once every rank's
tiles have landed.

The reference runs on one device only; this module has no reference
counterpart and keeps the single-device arithmetic exactly (each output
element is computed by exactly one rank with the single-GPU kernels).

:class:`ShardPlan` is device-agnostic (bounds, slicing, gather, assembly);
:class:`ShardedLayer` adds the CUDA compute.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib, ops


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
                                      block_q=block_q, route_out_features=out_features)
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
        # token split only on the tensor-core path (>= 128 rows per rank): there the H
        # of a token slice equals those rows of the whole H bit for bit (the small-M
        # kernel splits K by the token count)
        if self.split_lowrank and self.world > 1 and T % self.world == 0 and tp >= 128 and x2.stride(1) == 1:
            ldh = (self.rank_r + 63) // 64 * 64
            hbytes = T * ldh * x2.element_size()
            off = self.rank * tp * ldh * x2.element_size()
            if off % 256 == 0:
                # room for the slice call's own layout (H rows, then its scratch) at the offset
                ws = d.workspace(T, at_least=off + d.workspace_bytes(tp))
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
            if T <= _lib.SLR_DECODE_MAX_TOKENS:
                # decode sizes: the single-launch kernel when it applies (as the whole layer's forward)
                self.desc.forward(x2, buf[self.rank][:, :self.width])
            else:
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

    # ---------------------------------------------- y written into peer memory
    def peers_supported(self, x2: torch.Tensor) -> bool:
        """Whether this rank's combine can store into peers (a rank without
        rows only takes part in the signals).  All ranks must agree before
        :meth:`start_peers` is used: see :func:`all_ranks`."""
        if self.desc is None:
            return True
        return bool(_lib.load().slr_lrs_linear_peers_supported(
            ctypes.byref(self.desc.struct), x2.data_ptr(), ops.LayerDesc._ld(x2), x2.shape[0]))

    def start_peers(self, x2: torch.Tensor, po: "PeerOutputs") -> None:
        """x·Bᵀ, then the combine with every output tile stored into all ranks' y."""
        if self.desc is None:
            return
        self._lowrank(x2)
        self.start_peers_combine(x2, po)

    def start_peers_combine(self, x2: torch.Tensor, po: "PeerOutputs") -> None:
        """The combine alone (after the x·Bᵀ phase) into all ranks' y."""
        if self.desc is None:
            return
        d = self.desc
        ws = d.workspace(x2.shape[0])
        with ops._DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_combine_peers(
                ctypes.byref(d.struct), x2.data_ptr(), ops.LayerDesc._ld(x2), po.ldy, x2.shape[0],
                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), ctypes.byref(po.struct),
                torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc, "lrs_linear_combine_peers")

    def h_address(self, T: int) -> tuple[int, int] | None:
        """(device address, row stride) of the H that :meth:`_lowrank` leaves
        in this rank's layer workspace for T tokens; None without rows or rank."""
        if self.desc is None or self.rank_r == 0:
            return None
        return self.desc.workspace(T).data_ptr(), (self.rank_r + 63) // 64 * 64

    def finish_peers(self, po: "PeerOutputs") -> torch.Tensor:
        """Wait (on the stream) until every rank's columns are in po.y."""
        po.wait(empty_shard=self.desc is None)
        return po.y


def start_set_peers(layers: list[ShardedLayer], xs: list[torch.Tensor], pos: list["PeerOutputs"],
                    hs: list[tuple[int, int] | None], sync: "PeerOutputs") -> bool:
    """The combines of a set of sharded layers (after their x·Bᵀ phases) in
    ONE launch of the 2-SM kernel, every output tile stored into every rank's
    y (layer i's into ``pos[i].y``); the launch's arrival and completion
    signals use ``sync``'s slot (``slr_lrs_linear_multi_combine_peers``).
    ``hs[i]`` is (address, row stride) of layer i's H (:meth:`ShardedLayer.h_address`,
    :meth:`s_salaad_b200.ops.LayerGroup.h_of`).  Returns False, launching
    nothing, when this rank holds no rows of any of the layers.  Every rank
    calls it with the same layers and ``sync``, in the same order, and ends the
    call with :func:`finish_set_peers`."""
    idx = [i for i, L in enumerate(layers) if L.desc is not None]
    if not idx:
        return False
    n = len(idx)
    T = xs[idx[0]].shape[0]
    structs = (_lib.SlrLayer * n)(*[layers[i].desc.struct for i in idx])
    xp = (ctypes.c_void_p * n)(*[xs[i].data_ptr() for i in idx])
    lx = (ctypes.c_int64 * n)(*[ops.LayerDesc._ld(xs[i]) for i in idx])
    hp = (ctypes.c_void_p * n)(*[hs[i][0] if hs[i] else None for i in idx])
    lh = (ctypes.c_int64 * n)(*[hs[i][1] if hs[i] else 0 for i in idx])
    ly = (ctypes.c_int64 * n)(*[pos[i].ldy for i in idx])
    ps = (_lib.SlrPeers * n)(*[pos[i].struct for i in idx])
    with ops._DeviceGuard(sync.device):
        rc = _lib.load().slr_lrs_linear_multi_combine_peers(
            structs, n, xp, lx, hp, lh, ly, T, ps, ctypes.byref(sync.struct),
            torch.cuda.current_stream(sync.device).cuda_stream)
    _lib.check(rc, "lrs_linear_multi_combine_peers")
    return True


def finish_set_peers(sync: "PeerOutputs", launched: bool) -> None:
    """Ends a :func:`start_set_peers` call: once it returns (on the stream)
    every rank's tiles of every layer of the set are in this rank's y."""
    sync.wait(empty_shard=not launched)


def all_ranks(flag: bool, device, group=None) -> bool:
    """True when `flag` holds on every rank of the group."""
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t.item())


class PeerOutputs:
    """The full y [T, N] of one sharded layer on this rank, with the y and
    signal slot of every other rank mapped in (collective: every rank of the
    group constructs it for the same layer, in the same order).

    ``struct`` is the ``slr_peers`` argument of the combine: y of rank p
    advanced to this rank's first column ``n0``.
    """

    def __init__(self, plan: ShardPlan, T: int, dtype, device, group=None):
        self.world, self.rank = plan.world, plan.rank
        if not 2 <= self.world <= _lib.SLR_MAX_RANKS:
            raise ValueError(f"peer outputs need 2..{_lib.SLR_MAX_RANKS} ranks")
        self.device = device
        self.y = torch.empty(T, plan.out_features, dtype=dtype, device=device)
        self.ldy = plan.out_features
        self.signal = torch.zeros(_lib.SLR_SIGNAL_WORDS, dtype=torch.int64, device=device)
        lib = _lib.load()
        hb = _lib.SLR_IPC_HANDLE_BYTES
        mine = np.zeros(2 * (hb + 8), dtype=np.uint8)
        with ops._DeviceGuard(device):
            for k, t in enumerate((self.y, self.signal)):
                h = (ctypes.c_uint8 * hb)()
                off = ctypes.c_int64()
                _lib.check(lib.slr_ipc_export(t.data_ptr(), h, ctypes.byref(off)), "ipc_export")
                base = k * (hb + 8)
                mine[base:base + hb] = np.frombuffer(bytes(h), dtype=np.uint8)
                mine[base + hb:base + hb + 8] = np.frombuffer(np.int64(off.value).tobytes(), dtype=np.uint8)
        local = torch.from_numpy(mine).to(device)
        every = torch.empty(self.world * mine.size, dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(every, local, group=group)
        every = every.cpu().numpy().reshape(self.world, -1)
        self._imported: list[bytes] = []
        st = _lib.SlrPeers()
        st.world, st.rank = self.world, self.rank
        col_bytes = plan.n0 * self.y.element_size()
        with ops._DeviceGuard(device):
            for p in range(self.world):
                ptrs = []
                for k, t in enumerate((self.y, self.signal)):
                    if p == self.rank:
                        ptrs.append(t.data_ptr())
                        continue
                    base = k * (hb + 8)
                    h = bytes(every[p, base:base + hb])
                    off = int(np.frombuffer(every[p, base + hb:base + hb + 8].tobytes(), dtype=np.int64)[0])
                    out = ctypes.c_void_p()
                    _lib.check(lib.slr_ipc_import(h, off, ctypes.byref(out)), "ipc_import")
                    self._imported.append(h)
                    ptrs.append(out.value)
                st.y[p] = ptrs[0] + col_bytes
                st.signal[p] = ptrs[1]
        self.struct = st

    def wait(self, empty_shard: bool = False) -> None:
        with ops._DeviceGuard(self.device):
            rc = _lib.load().slr_peers_wait(ctypes.byref(self.struct), 1 if empty_shard else 0,
                                            torch.cuda.current_stream(self.device).cuda_stream)
        _lib.check(rc, "peers_wait")

    def close(self) -> None:
        """Drop the mappings of the other ranks' buffers (after all use)."""
        lib = _lib.load()
        for h in self._imported:
            lib.slr_ipc_release(h)
        self._imported = []
