"""Tensor-level entry points over the C ABI (CUDA tensors only).

* :func:`bsr_addmm_inplace_`  — in-place ``out += x @ S.T`` for BSR S; the
  implementation behind the ``ssalaad::tilelang_bsr_addmm_inplace_dense_``
  operator (reference: ssalaad/tilelang_sparse/addmm_inplace.py:88-141).
* :class:`LayerDesc` / :func:`lrs_linear_forward` — the fused S+LR forward
  ``y = x @ S.T + (x @ B.T) @ A.T + bias`` (reference:
  ssalaad/efficient/ls_linear.py:124-137); :class:`LayerGroup` for layers
  that read one input, :class:`LayerSet` for independent layers side by side.
  Within :func:`single_launch_decode` (off by default), calls of 1 to 32
  tokens run the single-launch decode kernel (``slr_lrs_linear_decode``).
"""
from __future__ import annotations

import contextlib
import ctypes

import numpy as np
import torch

from . import _lib

_DTYPES = {torch.float32: _lib.SLR_F32, torch.float16: _lib.SLR_F16, torch.bfloat16: _lib.SLR_BF16}


def slr_dtype(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise TypeError(f"s_salaad_b200 supports float32/float16/bfloat16, got {dtype}") from None


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """The current CUDA stream of `device` as a raw handle (the cheap path
    when torch provides it: this runs once per library call)."""
    if _raw_stream is not None:
        return _raw_stream(device.index if device.index is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (s_salaad_b200 has no CPU path)")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


class _DeviceGuard:
    """Make `device` current for the C call (cheap when it already is)."""

    __slots__ = ("dev", "prev")

    def __init__(self, device: torch.device):
        self.dev = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.dev:
            self.prev = cur
            torch.cuda.set_device(self.dev)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


# --------------------------------------------------------------- addmm --

def bsr_addmm_inplace_(out, x, crow_indices, col_indices, values, active_rows) -> None:
    """In place ``out += x @ S.T`` (S in BSR with values ``[nnz, bq, bp]``).

    Same contract as ``ssalaad::tilelang_bsr_addmm_inplace_dense_``
    (addmm_inplace.py:130-141): ``out``/``x`` contiguous 2-D of one dtype,
    int32 ``crow``/``col``/``active_rows``, all on one CUDA device; only the
    block-rows in ``active_rows`` are touched.  Unlike the reference, M needs
    no padding, and float32 is accepted (bit-identical to the AVX2 kernel).
    """
    lib = _lib.load()
    dtype = slr_dtype(out.dtype)
    if x.dtype != out.dtype or values.dtype != out.dtype:
        raise TypeError(f"out/x/values dtypes differ: {out.dtype}, {x.dtype}, {values.dtype}")
    for name, t in (("out", out), ("x", x), ("crow", crow_indices), ("col", col_indices),
                    ("values", values), ("active_rows", active_rows)):
        _require_cuda(name, t)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    for name, t in (("crow", crow_indices), ("col", col_indices), ("active_rows", active_rows)):
        if t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32, got {t.dtype}")
    if out.dim() != 2 or x.dim() != 2 or values.dim() != 3:
        raise ValueError("out and x must be 2-D and values 3-D (nnz, block_q, block_p)")
    M, K = x.shape
    bq, bp = int(values.shape[1]), int(values.shape[2])
    NB = crow_indices.numel() - 1
    if out.shape[0] != M or out.shape[1] != NB * bp:
        raise ValueError(f"out shape {tuple(out.shape)} does not match ({M}, {NB * bp})")
    if values.shape[0] != col_indices.numel():
        raise ValueError("values nnz must match col nnz")
    with _DeviceGuard(out.device):
        rc = lib.slr_bsr_addmm_inplace(
            out.data_ptr(), x.data_ptr(), M, K, crow_indices.data_ptr(), NB,
            col_indices.data_ptr(), values.data_ptr(), values.shape[0], bp, bq,
            active_rows.data_ptr(), active_rows.numel(), dtype, _stream(out.device))
    _lib.check(rc, "bsr_addmm_inplace_")


def validate_bsr(crow, col, nbk: int, active_rows) -> None:
    """Device-side structure check (raises ValueError on a bad index)."""
    lib = _lib.load()
    with _DeviceGuard(crow.device):
        rc = lib.slr_validate_bsr(crow.data_ptr(), crow.numel() - 1, col.data_ptr(), col.numel(), nbk,
                                  active_rows.data_ptr(), active_rows.numel(), _stream(crow.device))
    _lib.check(rc, "validate_bsr")


# ------------------------------------------------------------ S+LR layer --

# ------------------------------------------------------- decode path --

# Off by default: on B200 the two-launch path (x·Bᵀ, then the combine as a
# programmatic dependent) is as fast or faster except for large layer sets.
_single_launch = False


@contextlib.contextmanager
def single_launch_decode(enabled: bool):
    """Within the block, calls of 1..32 tokens take (enabled) or skip the
    single-launch decode kernel; skipped (the default), they run x·Bᵀ and the
    combine as two launches (``slr_lrs_linear_forward`` and its group / multi
    forms)."""
    global _single_launch
    prev, _single_launch = _single_launch, bool(enabled)
    try:
        yield
    finally:
        _single_launch = prev


def decode_supported(descs: list["LayerDesc"], xs: list[torch.Tensor]) -> bool:
    """Whether these layers on these inputs (1..32 rows) can run on the
    single-launch decode kernel (it does so within single_launch_decode(True))."""
    n = len(descs)
    arr = (_lib.SlrLayer * n)(*[d.struct for d in descs])
    xp = (ctypes.c_void_p * n)(*[x.data_ptr() for x in xs])
    lx = (ctypes.c_int64 * n)(*[LayerDesc._ld(x) for x in xs])
    return bool(_lib.load().slr_lrs_linear_decode_supported(arr, n, xp, lx, xs[0].shape[0]))


class _DecodeState:
    """Control block (zeroed once; each call leaves it zero) and workspace of
    ``slr_lrs_linear_decode`` for one owner of descriptors.  An owner's calls
    must not run on two streams at once (they share the control block)."""

    __slots__ = ("ctrl", "ws", "ok", "sizes")

    def __init__(self):
        self.ctrl: torch.Tensor | None = None
        self.ws: torch.Tensor | None = None
        self.ok: dict = {}
        self.sizes: dict = {}

    def run(self, arr, blob: bytes, n: int, xs: list[torch.Tensor], ys: list[torch.Tensor], M: int,
            device: torch.device) -> bool:
        """Runs the call on the decode kernel if it qualifies; False if not."""
        if not _single_launch or not 1 <= M <= _lib.SLR_DECODE_MAX_TOKENS:
            return False
        lib = _lib.load()
        xp = (ctypes.c_void_p * n)(*[x.data_ptr() for x in xs])
        lx = (ctypes.c_int64 * n)(*[LayerDesc._ld(x) for x in xs])
        key = (blob, M, tuple(x.data_ptr() % 16 for x in xs), tuple(lx))
        ok = self.ok.get(key)
        if ok is None:
            if len(self.ok) > 256:
                self.ok.clear()
            ok = self.ok[key] = bool(lib.slr_lrs_linear_decode_supported(arr, n, xp, lx, M))
        if not ok:
            return False
        need = self.sizes.get((blob, M))
        if need is None:
            if len(self.sizes) > 256:
                self.sizes.clear()
            need = self.sizes[(blob, M)] = int(lib.slr_lrs_linear_decode_workspace_size(arr, n, M))
        if self.ctrl is None or self.ctrl.device != device:
            self.ctrl = torch.zeros(_lib.SLR_DECODE_CTRL_BYTES // 4, dtype=torch.int32, device=device)
        if need and (self.ws is None or self.ws.numel() < need or self.ws.device != device):
            self.ws = torch.empty(need, dtype=torch.uint8, device=device)
        yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
        ly = (ctypes.c_int64 * n)(*[LayerDesc._ld(y) for y in ys])
        with _DeviceGuard(device):
            rc = lib.slr_lrs_linear_decode(arr, n, xp, lx, yp, ly, M, None if not need else self.ws.data_ptr(),
                                           need, self.ctrl.data_ptr(), _stream(device))
        _lib.check(rc, "lrs_linear_decode")
        return True


class LayerDesc:
    """Owns an ``slr_layer`` descriptor plus the layer's workspace.

    The descriptor holds raw device pointers of the tensors given here; call
    :meth:`refresh` (or construct anew) whenever those tensors move.
    """

    def __init__(self, *, A, B, bias=None, crow=None, col=None, values=None, row_order=None,
                 in_features: int, out_features: int, block_p: int = 0, block_q: int = 0, flags: int = 0,
                 route_out_features: int = 0):
        self.tensors = dict(A=A, B=B, bias=bias, crow=crow, col=col, values=values, row_order=row_order)
        self.flags = int(flags)  # slr_layer.flags: SLR_FLAG_PAIR_MMA | SLR_FLAG_STRICT_ORDER
        # a block-row shard: kernels chosen as for the whole layer of this width
        self.route_out_features = int(route_out_features)
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        self.block_p = int(block_p)
        self.block_q = int(block_q)
        self.struct = _lib.SlrLayer()
        self._ws: torch.Tensor | None = None
        self._ws_sizes: dict = {}
        self._plan_key = None
        self._plan = None
        self._decode = _DecodeState()
        self.refresh()

    def refresh(self, **tensors) -> None:
        self.tensors.update(tensors)
        t = self.tensors
        A = t["A"]
        s = self.struct
        s.in_features = self.in_features
        s.out_features = self.out_features
        s.rank = int(A.shape[1])
        nnz = 0 if t["col"] is None else int(t["col"].numel())
        s.nnz = nnz
        s.block_p = self.block_p if nnz else 0
        s.block_q = self.block_q if nnz else 0
        s.crow = _ptr(t["crow"]) if nnz else None
        s.col = _ptr(t["col"]) if nnz else None
        s.values = _ptr(t["values"]) if nnz else None
        s.row_order = _ptr(t["row_order"]) if nnz else None
        s.A = A.data_ptr() if A.numel() else None
        s.B = t["B"].data_ptr() if t["B"].numel() else None
        s.bias = _ptr(t["bias"])
        s.dtype = slr_dtype(A.dtype)
        s.flags = self.flags
        s.route_out_features = self.route_out_features
        self.device = A.device
        self.dtype = A.dtype
        self.key = tuple(_ptr(v) for v in t.values())
        # column schedule of the tensor-core path, rebuilt when the indices move
        pk = (_ptr(t["crow"]), _ptr(t["col"]), _ptr(t["row_order"]), self.block_p) if nnz else None
        if pk != self._plan_key:
            self._plan_key = pk
            self._plan = None
            if nnz and A.dtype != torch.float32:
                p = plan_stages(t["crow"], t["col"], self.block_p, t["row_order"])
                if p is not None:
                    self._plan = tuple(torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a).to(A.device)
                                       for a in p)
        s.stage_plan = self._plan[0].data_ptr() if self._plan is not None else None
        s.stage_start = self._plan[1].data_ptr() if self._plan is not None else None

    def workspace_bytes(self, M: int) -> int:
        key = (bytes(self.struct), M)  # the size depends on the descriptor and M only
        need = self._ws_sizes.get(key)
        if need is None:
            need = int(_lib.load().slr_lrs_linear_workspace_size(ctypes.byref(self.struct), M))
            if len(self._ws_sizes) > 64:
                self._ws_sizes.clear()
            self._ws_sizes[key] = need
        return need

    def workspace(self, M: int, at_least: int = 0) -> torch.Tensor | None:
        need = max(self.workspace_bytes(M), at_least)
        if need == 0:
            return None
        if self._ws is None or self._ws.numel() < need or self._ws.device != self.device:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    @staticmethod
    def _ld(t: torch.Tensor) -> int:
        if t.dim() != 2 or t.stride(1) != 1:
            raise ValueError("x/out must be 2-D with unit stride in the last dimension")
        return t.stride(0)

    def forward(self, x2: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """y = x2 @ S.T + (x2 @ B.T) @ A.T + bias; x2/out may be row-strided."""
        lib = _lib.load()
        M = x2.shape[0]
        if out is None:
            out = torch.empty(M, self.out_features, dtype=self.dtype, device=self.device)
        if self._decode.run(ctypes.byref(self.struct), bytes(self.struct), 1, [x2], [out], M, self.device):
            return out
        ws = self.workspace(M)
        with _DeviceGuard(self.device):
            rc = lib.slr_lrs_linear_forward(
                ctypes.byref(self.struct), x2.data_ptr(), self._ld(x2), out.data_ptr(), self._ld(out), M,
                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
                _stream(self.device))
        _lib.check(rc, "lrs_linear_forward")
        return out

    def lowrank(self, x2: torch.Tensor) -> None:
        """Phase 1 alone: H = x2 @ B.T into this layer's workspace."""
        M = x2.shape[0]
        ws = self.workspace(M)
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_lowrank(
                ctypes.byref(self.struct), x2.data_ptr(), self._ld(x2), M,
                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _stream(self.device))
        _lib.check(rc, "lrs_linear_lowrank")

    def combine(self, x2: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Phase 2 alone: out = x2 @ S.T + H @ A.T + bias (H from lowrank())."""
        M = x2.shape[0]
        ws = self.workspace(M)
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_combine(
                ctypes.byref(self.struct), x2.data_ptr(), self._ld(x2), out.data_ptr(), self._ld(out), M,
                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _stream(self.device))
        _lib.check(rc, "lrs_linear_combine")
        return out


class LayerGroup:
    """Layers that read the same input (q/k/v, gate/up): one grouped call.

    ``forward(x)`` returns each layer's ``y`` exactly as
    :meth:`LayerDesc.forward` would; the ``x · Bᵀ`` products run as one
    launch over the stacked ``B`` matrices (a tensor-core GEMM from 128 tokens
    on) and, below 128 tokens, the combine phases of all layers as one launch
    when their block shapes allow.
    """

    def __init__(self, descs: list[LayerDesc]):
        if not 1 <= len(descs) <= 4:
            raise ValueError("a group holds 1 to 4 layers")
        if len({d.in_features for d in descs}) != 1 or len({d.dtype for d in descs}) != 1:
            raise ValueError("grouped layers must share in_features and dtype")
        self.descs = list(descs)
        self.device = descs[0].device
        self.dtype = descs[0].dtype
        self._ws: torch.Tensor | None = None
        self._decode = _DecodeState()

    def _structs(self):
        """The members' descriptors as one C array (rebuilt when one changes)."""
        blob = b"".join(bytes(d.struct) for d in self.descs)
        if blob != getattr(self, "_blob", None):
            arr = (_lib.SlrLayer * len(self.descs))()
            ctypes.memmove(arr, blob, len(blob))
            self._arr, self._blob, self._ws_sizes = arr, blob, {}
        return self._arr

    def workspace(self, M: int) -> torch.Tensor | None:
        arr = self._structs()
        need = self._ws_sizes.get(M)
        if need is None:
            need = self._ws_sizes[M] = int(_lib.load().slr_lrs_linear_group_workspace_size(arr, len(self.descs), M))
        if need == 0:
            return None
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, x2: torch.Tensor, outs: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
        M = x2.shape[0]
        n = len(self.descs)
        if outs is None:
            outs = [torch.empty(M, d.out_features, dtype=self.dtype, device=self.device) for d in self.descs]
        arr = self._structs()
        if self._decode.run(arr, self._blob, n, [x2] * n, outs, M, self.device):
            return outs
        ws = self.workspace(M)
        ys = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
        lds = (ctypes.c_int64 * n)(*[LayerDesc._ld(o) for o in outs])
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_forward_group(
                self._structs(), n, x2.data_ptr(), LayerDesc._ld(x2), ys, lds, M,
                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _stream(self.device))
        _lib.check(rc, "lrs_linear_forward_group")
        return outs

    def lowrank(self, x2: torch.Tensor) -> None:
        """Phase 1 alone: every layer's x2 @ B.T into the group workspace."""
        M = x2.shape[0]
        ws = self.workspace(M)
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_group_lowrank(
                self._structs(), len(self.descs), x2.data_ptr(), LayerDesc._ld(x2), M,
                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _stream(self.device))
        _lib.check(rc, "lrs_linear_group_lowrank")

    def h_row_bytes(self) -> int:
        """Bytes of one token's row of the group's H (x2 @ [B_0; ...].T)."""
        esize = torch.finfo(self.dtype).bits // 8
        return sum((d.struct.rank + 63) // 64 * 64 for d in self.descs) * esize

    def h_of(self, i: int, M: int) -> tuple[int, int]:
        """(device address, row stride in elements) of layer i's H after
        :meth:`lowrank` or :meth:`lowrank_rows` on M >= 128 tokens: its
        columns of the group H [M, sum of round_up(rank, 64)] at the start of
        the workspace (the layout of the tensor-core path)."""
        if M < 128 or self.dtype == torch.float32:
            raise ValueError("the shared-H layout is the 16-bit tensor-core path's (M >= 128)")
        esize = torch.finfo(self.dtype).bits // 8
        widths = [(d.struct.rank + 63) // 64 * 64 for d in self.descs]
        return self.workspace(M).data_ptr() + sum(widths[:i]) * esize, sum(widths)

    def lowrank_rows(self, x2: torch.Tensor, row0: int, rows: int) -> torch.Tensor:
        """Phase 1 for tokens [row0, row0 + rows) of x2 only, written into their
        rows of the group H of all x2.shape[0] tokens (that layout depends on
        the token count alone); returns the whole H region of the workspace as
        bytes, e.g. for an all-gather of the other ranks' rows."""
        M = x2.shape[0]
        if row0 < 0 or rows <= 0 or row0 + rows > M:
            raise ValueError("token rows out of range")
        # the shared-H layout needs the tensor-core x*B^T for every layer and both token counts
        if rows < 128 or self.dtype == torch.float32 or any(
                d.struct.rank < 64 or d.in_features < 64 or d.in_features % 8 for d in self.descs):
            raise ValueError("lowrank_rows needs >= 128 rows, 16-bit layers with rank >= 64 and K % 8 == 0")
        ws = self.workspace(M)
        off = row0 * self.h_row_bytes()
        if off % 256:
            raise ValueError("row0 * H row bytes must be a multiple of 256 (workspace alignment)")
        xs = x2[row0:row0 + rows]
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_group_lowrank(
                self._structs(), len(self.descs), xs.data_ptr(), LayerDesc._ld(x2), rows,
                ws.data_ptr() + off, ws.numel() - off, _stream(self.device))
        _lib.check(rc, "lrs_linear_group_lowrank")
        return ws[:M * self.h_row_bytes()]

    def combine_peers(self, i: int, x2: torch.Tensor, po) -> None:
        """Phase 2 of layer i with its output stored into every rank's y
        (``po``: a :class:`s_salaad_b200.shard.PeerOutputs` of that layer)."""
        M = x2.shape[0]
        ws = self.workspace(M)
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_group_combine_peers(
                self._structs(), len(self.descs), i, x2.data_ptr(), LayerDesc._ld(x2), po.ldy, M,
                None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), ctypes.byref(po.struct),
                _stream(self.device))
        _lib.check(rc, "lrs_linear_group_combine_peers")

    def combine(self, i: int, x2: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Phase 2 of layer i (after lowrank() on the same x2)."""
        M = x2.shape[0]
        ws = self.workspace(M)
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_group_combine(
                self._structs(), len(self.descs), i, x2.data_ptr(), LayerDesc._ld(x2), out.data_ptr(),
                LayerDesc._ld(out), M, None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
                _stream(self.device))
        _lib.check(rc, "lrs_linear_group_combine")
        return out


class LayerSet:
    """Independent layers run side by side, each on its own input (one
    ``slr_lrs_linear_forward_multi`` call): ``forward(xs)`` returns what
    :meth:`LayerDesc.forward` gives for each layer, bit for bit.  Up to 127
    tokens every layer's ``x · Bᵀ`` is one launch and the combine phases one
    more (two launches for the whole set instead of two per layer)."""

    def __init__(self, descs: list[LayerDesc]):
        if not 1 <= len(descs) <= 8:
            raise ValueError("a layer set holds 1 to 8 layers")
        if len({d.dtype for d in descs}) != 1:
            raise ValueError("the layers of a set must share one dtype")
        self.descs = list(descs)
        self.device = descs[0].device
        self.dtype = descs[0].dtype
        self._ws: torch.Tensor | None = None
        self._decode = _DecodeState()

    def _structs(self):
        """The members' descriptors as one C array (rebuilt when one changes)."""
        blob = b"".join(bytes(d.struct) for d in self.descs)
        if blob != getattr(self, "_blob", None):
            arr = (_lib.SlrLayer * len(self.descs))()
            ctypes.memmove(arr, blob, len(blob))
            self._arr, self._blob, self._ws_sizes = arr, blob, {}
        return self._arr

    def workspace(self, M: int) -> torch.Tensor | None:
        arr = self._structs()
        need = self._ws_sizes.get(M)
        if need is None:
            need = self._ws_sizes[M] = int(_lib.load().slr_lrs_linear_multi_workspace_size(arr, len(self.descs), M))
        if need == 0:
            return None
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, xs: list[torch.Tensor], outs: list[torch.Tensor] | None = None) -> list[torch.Tensor]:
        n = len(self.descs)
        if len(xs) != n:
            raise ValueError(f"{n} layers need {n} inputs")
        M = xs[0].shape[0]
        if any(x.shape[0] != M for x in xs):
            raise ValueError("every input of a layer set has the same number of rows")
        if outs is None:
            outs = [torch.empty(M, d.out_features, dtype=self.dtype, device=self.device) for d in self.descs]
        arr = self._structs()
        if self._decode.run(arr, self._blob, n, xs, outs, M, self.device):
            return outs
        ws = self.workspace(M)
        xp = (ctypes.c_void_p * n)(*[x.data_ptr() for x in xs])
        lx = (ctypes.c_int64 * n)(*[LayerDesc._ld(x) for x in xs])
        yp = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
        ly = (ctypes.c_int64 * n)(*[LayerDesc._ld(o) for o in outs])
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_forward_multi(
                self._structs(), n, xp, lx, yp, ly, M, None if ws is None else ws.data_ptr(),
                0 if ws is None else ws.numel(), _stream(self.device))
        _lib.check(rc, "lrs_linear_forward_multi")
        return outs

    def _ptrs(self, xs, outs=None):
        n = len(self.descs)
        xp = (ctypes.c_void_p * n)(*[x.data_ptr() for x in xs])
        lx = (ctypes.c_int64 * n)(*[LayerDesc._ld(x) for x in xs])
        if outs is None:
            return xp, lx, None, None
        yp = (ctypes.c_void_p * n)(*[o.data_ptr() for o in outs])
        ly = (ctypes.c_int64 * n)(*[LayerDesc._ld(o) for o in outs])
        return xp, lx, yp, ly

    def lowrank(self, xs: list[torch.Tensor]) -> None:
        """Phase 1 alone: every layer's x @ B.T into the set's workspace."""
        M = xs[0].shape[0]
        ws = self.workspace(M)
        xp, lx, _, _ = self._ptrs(xs)
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_multi_lowrank(
                self._structs(), len(self.descs), xp, lx, M, None if ws is None else ws.data_ptr(),
                0 if ws is None else ws.numel(), _stream(self.device))
        _lib.check(rc, "lrs_linear_multi_lowrank")

    def h_addresses(self, xs: list[torch.Tensor]) -> list[tuple[int, int] | None]:
        """(device address, row stride) of each layer's H that :meth:`lowrank`
        leaves in the set's workspace for these inputs (None without rank)."""
        M = xs[0].shape[0]
        ws = self.workspace(M)
        n = len(self.descs)
        xp, lx, _, _ = self._ptrs(xs)
        hp = (ctypes.c_void_p * n)()
        lh = (ctypes.c_int64 * n)()
        rc = _lib.load().slr_lrs_linear_multi_h(self._structs(), n, xp, lx, M, None if ws is None else ws.data_ptr(),
                                                0 if ws is None else ws.numel(), hp, lh)
        _lib.check(rc, "lrs_linear_multi_h")
        return [(int(hp[i]), int(lh[i])) if hp[i] else None for i in range(n)]

    def combine(self, xs: list[torch.Tensor], outs: list[torch.Tensor]) -> list[torch.Tensor]:
        """Phase 2 alone (after lowrank() on the same inputs): every layer's y."""
        M = xs[0].shape[0]
        ws = self.workspace(M)
        xp, lx, yp, ly = self._ptrs(xs, outs)
        with _DeviceGuard(self.device):
            rc = _lib.load().slr_lrs_linear_multi_combine(
                self._structs(), len(self.descs), xp, lx, yp, ly, M, None if ws is None else ws.data_ptr(),
                0 if ws is None else ws.numel(), _stream(self.device))
        _lib.check(rc, "lrs_linear_multi_combine")
        return outs


# ------------------------------------------------ N:M 2:4 + low-rank --

def nm_compress(S: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Dense 2:4-sparse S [N, K] (CUDA, fp16/bf16) -> (values [N, K/2],
    meta [N, K/32] int32 view of the uint32 words), the layout of
    ``slr_nm_compress``.  ValueError if S is not 2:4 sparse."""
    _require_cuda("S", S)
    if S.dim() != 2:
        raise ValueError("S must be 2-D")
    N, K = S.shape
    if K % 32:
        raise ValueError(f"N:M layer: in_features {K} must be a multiple of 32")
    S = S.contiguous()
    values = torch.empty(N, K // 2, dtype=S.dtype, device=S.device)
    meta = torch.empty(N, K // 32, dtype=torch.int32, device=S.device)
    with _DeviceGuard(S.device):
        rc = _lib.load().slr_nm_compress(S.data_ptr(), N, K, slr_dtype(S.dtype), values.data_ptr(),
                                         meta.data_ptr(), _stream(S.device))
    _lib.check(rc, "nm_compress")
    return values, meta


def nm_expand(values: torch.Tensor, meta: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`nm_compress` (host-side torch ops): the dense S."""
    N, half = values.shape
    K = 2 * half
    words = meta.to(torch.int64) & 0xFFFFFFFF                        # [N, K/32]
    shifts = torch.arange(8, device=meta.device) * 4
    nib = (words.unsqueeze(-1) >> shifts) & 0xF                       # [N, K/32, 8]
    first, second = nib & 3, nib >> 2
    base = (torch.arange(K // 4, device=meta.device) * 4).view(K // 32, 8)
    pos = torch.stack((first + base, second + base), dim=-1).reshape(N, K // 2)
    S = torch.zeros(N, K, dtype=values.dtype, device=values.device)
    S.scatter_(1, pos, values)
    return S


class NmLayerDesc:
    """Owns an ``slr_nm_layer`` descriptor plus its workspace (the N:M 2:4 +
    low-rank layer: values/meta from :func:`nm_compress`, A [N, r], B [r, K])."""

    def __init__(self, *, values, meta, A, B, bias=None, in_features: int, out_features: int, flags: int = 0):
        self.tensors = dict(values=values, meta=meta, A=A, B=B, bias=bias)
        self.in_features, self.out_features = int(in_features), int(out_features)
        s = self.struct = _lib.SlrNmLayer()
        s.in_features, s.out_features, s.rank = self.in_features, self.out_features, int(A.shape[1])
        s.values, s.meta = values.data_ptr(), meta.data_ptr()
        s.A, s.B, s.bias = A.data_ptr(), B.data_ptr(), _ptr(bias)
        s.dtype, s.flags = slr_dtype(A.dtype), int(flags)
        self.device, self.dtype = A.device, A.dtype
        self._ws: torch.Tensor | None = None

    def forward(self, x2: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        lib = _lib.load()
        M = x2.shape[0]
        if out is None:
            out = torch.empty(M, self.out_features, dtype=self.dtype, device=self.device)
        need = int(lib.slr_nm_linear_workspace_size(ctypes.byref(self.struct), M))
        if need and (self._ws is None or self._ws.numel() < need):
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        ws = self._ws if need else None
        with _DeviceGuard(self.device):
            rc = lib.slr_nm_linear_forward(ctypes.byref(self.struct), x2.data_ptr(), LayerDesc._ld(x2),
                                           out.data_ptr(), LayerDesc._ld(out), M,
                                           None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
                                           _stream(self.device))
        _lib.check(rc, "nm_linear_forward")
        return out


def lrs_linear_forward(desc: LayerDesc, x: torch.Tensor) -> torch.Tensor:
    """``y = x @ S.T + (x @ B.T) @ A.T + bias`` for x of shape ``[..., in]``."""
    _require_cuda("x", x)
    if x.dtype != desc.dtype:
        raise TypeError(f"x dtype {x.dtype} does not match the layer dtype {desc.dtype}")
    shape = x.shape
    if shape[-1] != desc.in_features:
        raise ValueError(f"x last dim {shape[-1]} != in_features {desc.in_features}")
    x2 = x.reshape(-1, shape[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    return desc.forward(x2).reshape(*shape[:-1], desc.out_features)


# ---------------------------------------------------------- dense -> BSR --

def dense_to_bsr_cuda(S: torch.Tensor, block_p: int, block_q: int, *, transpose: bool = False,
                      index_dtype=torch.int64):
    """GPU ``dense_to_bsr`` (artifact.py:20-37), bit-exact.

    Returns ``(crow, col, values)`` on S's device: int64 indices (or
    ``index_dtype``) and values ``[nnz, bp, bq]`` (``[nnz, bq, bp]`` when
    ``transpose``).  Raises ValueError like the reference when the shape is
    not divisible by the block shape.
    """
    lib = _lib.load()
    _require_cuda("S", S)
    if S.dim() != 2:
        raise ValueError("S must be 2-D")
    n, m = S.shape
    if n % block_p or m % block_q:
        raise ValueError(f"shape ({n}, {m}) not divisible by block ({block_p}, {block_q})")
    S = S.contiguous()
    dtype = slr_dtype(S.dtype)
    rb, cb = n // block_p, m // block_q
    dev = S.device
    mask = torch.empty(rb * cb, dtype=torch.uint8, device=dev)
    crow = torch.empty(rb + 1, dtype=torch.int64, device=dev)
    stream = _stream(dev)
    with _DeviceGuard(dev):
        _lib.check(lib.slr_dense_to_bsr_mask(S.data_ptr(), n, m, block_p, block_q, dtype,
                                             mask.data_ptr(), crow.data_ptr(), stream), "dense_to_bsr")
        nnz = int(crow[-1].item())
        col = torch.empty(nnz, dtype=torch.int64, device=dev)
        shape = (nnz, block_q, block_p) if transpose else (nnz, block_p, block_q)
        values = torch.empty(shape, dtype=S.dtype, device=dev)
        _lib.check(lib.slr_dense_to_bsr_fill(S.data_ptr(), n, m, block_p, block_q, dtype, mask.data_ptr(),
                                             crow.data_ptr(), col.data_ptr(), values.data_ptr(),
                                             int(transpose), stream), "dense_to_bsr")
    if index_dtype != torch.int64:
        crow, col = crow.to(index_dtype), col.to(index_dtype)
    return crow, col, values


# ---------------------------------------------------------------- plans --

def plan_row_order(crow) -> np.ndarray:
    """Block-rows heaviest first (ties by index), from the host planner."""
    c = np.ascontiguousarray(np.asarray(crow.cpu() if hasattr(crow, "cpu") else crow), dtype=np.int32)
    NB = c.shape[0] - 1
    out = np.empty(max(NB, 0), dtype=np.int32)
    _lib.check(_lib.load().slr_plan_row_order(c.ctypes.data, NB, out.ctypes.data), "plan_row_order")
    return out


def plan_stages(crow, col, block_p: int, row_order=None) -> tuple[np.ndarray, np.ndarray] | None:
    """Column schedule of the tensor-core path (``slr_plan_stages``): the plan
    words and the per-group stage starts, or None when the layer has no such
    path (block_p not 16/32/64, or a column index above 65535)."""
    host = lambda t: np.ascontiguousarray(np.asarray(t.cpu() if hasattr(t, "cpu") else t), dtype=np.int32)  # noqa: E731
    c, k = host(crow), host(col)
    o = None if row_order is None else host(row_order)
    NB = c.shape[0] - 1
    if block_p not in (16, 32, 64) or NB <= 0 or int(c[-1]) == 0:
        return None
    lib = _lib.load()
    n = ctypes.c_int64(0)
    args = (c.ctypes.data, k.ctypes.data, NB, None if o is None else o.ctypes.data, block_p)
    if lib.slr_plan_stages(*args, None, None, 0, ctypes.byref(n)) != _lib.SLR_OK:
        return None
    G = 256 // block_p
    words = np.empty(max(n.value, 1), dtype=np.uint32)
    starts = np.empty((NB + G - 1) // G + 1, dtype=np.int32)
    _lib.check(lib.slr_plan_stages(*args, words.ctypes.data, starts.ctypes.data, words.shape[0], ctypes.byref(n)),
               "plan_stages")
    return words[:n.value], starts


def plan_shards(crow, block_p: int, block_q: int, rank: int, world: int) -> np.ndarray:
    """Contiguous, cost-balanced block-row ranges: bounds[world+1]."""
    c = np.ascontiguousarray(np.asarray(crow.cpu() if hasattr(crow, "cpu") else crow), dtype=np.int32)
    NB = c.shape[0] - 1
    out = np.empty(world + 1, dtype=np.int64)
    _lib.check(_lib.load().slr_plan_shards(c.ctypes.data, NB, block_p, block_q, rank, world, out.ctypes.data),
               "plan_shards")
    return out
