"""ctypes binding of libslr_b200.so (the C ABI in include/slr_b200.h).

The shared library is built in-tree by ``make -C s_salaad_b200/csrc`` (see
``__graft_entry__.build``).  There is no fallback: if the library is missing
or cannot be loaded, every entry point raises ``RuntimeError``.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libslr_b200.so"

# slr_status codes (include/slr_b200.h)
ABI_VERSION = 8  # SLR_ABI_VERSION of include/slr_b200.h
SLR_OK = 0
# slr_layer.flags bits (include/slr_b200.h)
SLR_FLAG_PAIR_MMA = 1
SLR_FLAG_STRICT_ORDER = 2
SLR_ERR_INVALID_ARGUMENT = 1
SLR_ERR_UNSUPPORTED_DTYPE = 2
SLR_ERR_UNSUPPORTED = 3
SLR_ERR_CUDA = 4
SLR_ERR_WORKSPACE = 5
SLR_ERR_BAD_INDEX = 6
SLR_ERR_TIMEOUT = 7

SLR_F32, SLR_F16, SLR_BF16 = 0, 1, 2

# Every function the header declares, for the symbol test.
EXPORTED = (
    "slr_abi_version",
    "slr_set_sm_limit",
    "slr_status_string",
    "slr_last_error",
    "slr_device_status",
    "slr_bsr_addmm_inplace",
    "slr_validate_bsr",
    "slr_lrs_linear_workspace_size",
    "slr_lrs_linear_forward",
    "slr_lrs_linear_lowrank",
    "slr_lrs_linear_combine",
    "slr_lrs_linear_forward_noalloc",
    "slr_lrs_linear_group_workspace_size",
    "slr_lrs_linear_forward_group",
    "slr_lrs_linear_group_lowrank",
    "slr_lrs_linear_group_combine",
    "slr_dense_to_bsr_mask",
    "slr_dense_to_bsr_fill",
    "slr_plan_stages",
    "slr_plan_row_order",
    "slr_plan_shards",
    "slr_ipc_export",
    "slr_ipc_import",
    "slr_ipc_release",
    "slr_lrs_linear_peers_supported",
    "slr_lrs_linear_combine_peers",
    "slr_lrs_linear_group_combine_peers",
    "slr_lrs_linear_multi_combine_peers",
    "slr_lrs_linear_multi_h",
    "slr_peers_wait",
    "slr_set_wait_limit_ns",
    "slr_lrs_linear_multi_workspace_size",
    "slr_lrs_linear_forward_multi",
    "slr_lrs_linear_multi_lowrank",
    "slr_lrs_linear_multi_combine",
    "slr_lrs_linear_decode_supported",
    "slr_lrs_linear_decode_workspace_size",
    "slr_lrs_linear_decode",
    "slr_nm_compress",
    "slr_nm_linear_workspace_size",
    "slr_nm_linear_forward",
)

SLR_MAX_RANKS = 8
SLR_IPC_HANDLE_BYTES = 64
SLR_SIGNAL_WORDS = 32
SLR_DECODE_CTRL_BYTES = 4096
SLR_DECODE_MAX_TOKENS = 32

i64, i32, vp, sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t


class SlrLayer(ctypes.Structure):
    """Mirror of ``struct slr_layer``."""

    _fields_ = [
        ("in_features", ctypes.c_int64),
        ("out_features", ctypes.c_int64),
        ("rank", ctypes.c_int64),
        ("block_p", ctypes.c_int64),
        ("block_q", ctypes.c_int64),
        ("nnz", ctypes.c_int64),
        ("crow", ctypes.c_void_p),
        ("col", ctypes.c_void_p),
        ("values", ctypes.c_void_p),
        ("row_order", ctypes.c_void_p),
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("stage_plan", ctypes.c_void_p),
        ("stage_start", ctypes.c_void_p),
        ("route_out_features", ctypes.c_int64),
    ]


class SlrNmLayer(ctypes.Structure):
    """Mirror of ``struct slr_nm_layer``."""

    _fields_ = [
        ("in_features", ctypes.c_int64),
        ("out_features", ctypes.c_int64),
        ("rank", ctypes.c_int64),
        ("values", ctypes.c_void_p),
        ("meta", ctypes.c_void_p),
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("flags", ctypes.c_int32),
    ]


class SlrPeers(ctypes.Structure):
    """Mirror of ``struct slr_peers``."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("y", ctypes.c_void_p * SLR_MAX_RANKS),
        ("signal", ctypes.c_void_p * SLR_MAX_RANKS),
    ]


_SIGS = {
    "slr_abi_version": ([], i32),
    "slr_set_sm_limit": ([i32], i32),
    "slr_status_string": ([i32], ctypes.c_char_p),
    "slr_last_error": ([], ctypes.c_char_p),
    "slr_device_status": ([ctypes.POINTER(ctypes.c_int)], i32),
    "slr_bsr_addmm_inplace": ([vp, vp, i64, i64, vp, i64, vp, vp, i64, i64, i64, vp, i64, i32, vp], i32),
    "slr_validate_bsr": ([vp, i64, vp, i64, i64, vp, i64, vp], i32),
    "slr_lrs_linear_workspace_size": ([ctypes.POINTER(SlrLayer), i64], sz),
    "slr_lrs_linear_forward": ([ctypes.POINTER(SlrLayer), vp, i64, vp, i64, i64, vp, sz, vp], i32),
    "slr_lrs_linear_lowrank": ([ctypes.POINTER(SlrLayer), vp, i64, i64, vp, sz, vp], i32),
    "slr_lrs_linear_combine": ([ctypes.POINTER(SlrLayer), vp, i64, vp, i64, i64, vp, sz, vp], i32),
    "slr_lrs_linear_forward_noalloc": ([ctypes.POINTER(SlrLayer), vp, i64, vp, i64, i64, vp], i32),
    "slr_lrs_linear_group_workspace_size": ([ctypes.POINTER(SlrLayer), i32, i64], sz),
    "slr_lrs_linear_forward_group": ([ctypes.POINTER(SlrLayer), i32, vp, i64, ctypes.POINTER(vp),
                                      ctypes.POINTER(i64), i64, vp, sz, vp], i32),
    "slr_lrs_linear_group_lowrank": ([ctypes.POINTER(SlrLayer), i32, vp, i64, i64, vp, sz, vp], i32),
    "slr_lrs_linear_group_combine": ([ctypes.POINTER(SlrLayer), i32, i32, vp, i64, vp, i64, i64, vp, sz, vp], i32),
    "slr_dense_to_bsr_mask": ([vp, i64, i64, i64, i64, i32, vp, vp, vp], i32),
    "slr_dense_to_bsr_fill": ([vp, i64, i64, i64, i64, i32, vp, vp, vp, vp, i32, vp], i32),
    "slr_plan_stages": ([vp, vp, i64, vp, i64, vp, vp, i64, ctypes.POINTER(i64)], i32),
    "slr_plan_row_order": ([vp, i64, vp], i32),
    "slr_plan_shards": ([vp, i64, i64, i64, i64, i32, vp], i32),
    "slr_ipc_export": ([vp, vp, ctypes.POINTER(i64)], i32),
    "slr_ipc_import": ([vp, i64, ctypes.POINTER(vp)], i32),
    "slr_ipc_release": ([vp], i32),
    "slr_lrs_linear_peers_supported": ([ctypes.POINTER(SlrLayer), vp, i64, i64], i32),
    "slr_lrs_linear_combine_peers": ([ctypes.POINTER(SlrLayer), vp, i64, i64, i64, vp, sz,
                                      ctypes.POINTER(SlrPeers), vp], i32),
    "slr_lrs_linear_group_combine_peers": ([ctypes.POINTER(SlrLayer), i32, i32, vp, i64, i64, i64, vp, sz,
                                            ctypes.POINTER(SlrPeers), vp], i32),
    "slr_lrs_linear_multi_combine_peers": ([ctypes.POINTER(SlrLayer), i32, ctypes.POINTER(vp), ctypes.POINTER(i64),
                                            ctypes.POINTER(vp), ctypes.POINTER(i64), ctypes.POINTER(i64), i64,
                                            ctypes.POINTER(SlrPeers), ctypes.POINTER(SlrPeers), vp], i32),
    "slr_lrs_linear_multi_h": ([ctypes.POINTER(SlrLayer), i32, ctypes.POINTER(vp), ctypes.POINTER(i64), i64, vp, sz,
                                ctypes.POINTER(vp), ctypes.POINTER(i64)], i32),
    "slr_peers_wait": ([ctypes.POINTER(SlrPeers), i32, vp], i32),
    "slr_set_wait_limit_ns": ([ctypes.c_uint64], i32),
    "slr_lrs_linear_multi_workspace_size": ([ctypes.POINTER(SlrLayer), i32, i64], sz),
    "slr_lrs_linear_forward_multi": ([ctypes.POINTER(SlrLayer), i32, ctypes.POINTER(vp), ctypes.POINTER(i64),
                                      ctypes.POINTER(vp), ctypes.POINTER(i64), i64, vp, sz, vp], i32),
    "slr_lrs_linear_multi_lowrank": ([ctypes.POINTER(SlrLayer), i32, ctypes.POINTER(vp), ctypes.POINTER(i64), i64,
                                      vp, sz, vp], i32),
    "slr_lrs_linear_multi_combine": ([ctypes.POINTER(SlrLayer), i32, ctypes.POINTER(vp), ctypes.POINTER(i64),
                                      ctypes.POINTER(vp), ctypes.POINTER(i64), i64, vp, sz, vp], i32),
    "slr_lrs_linear_decode_supported": ([ctypes.POINTER(SlrLayer), i32, ctypes.POINTER(vp), ctypes.POINTER(i64),
                                         i64], i32),
    "slr_lrs_linear_decode_workspace_size": ([ctypes.POINTER(SlrLayer), i32, i64], sz),
    "slr_lrs_linear_decode": ([ctypes.POINTER(SlrLayer), i32, ctypes.POINTER(vp), ctypes.POINTER(i64),
                               ctypes.POINTER(vp), ctypes.POINTER(i64), i64, vp, sz, vp, vp], i32),
    "slr_nm_compress": ([vp, i64, i64, i32, vp, vp, vp], i32),
    "slr_nm_linear_workspace_size": ([ctypes.POINTER(SlrNmLayer), i64], sz),
    "slr_nm_linear_forward": ([ctypes.POINTER(SlrNmLayer), vp, i64, vp, i64, i64, vp, sz, vp], i32),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load_sm_count() -> int:
    """Streaming multiprocessors of the current CUDA device."""
    import torch

    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def load(path: Path | str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library; raises RuntimeError if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.is_file():
            raise RuntimeError(
                f"s_salaad_b200: CUDA library {p} is not built; run "
                "`make -C s_salaad_b200/csrc` (or __graft_entry__.build()). "
                "There is no CPU fallback."
            )
        try:
            lib = ctypes.CDLL(str(p))
        except OSError as exc:  # pragma: no cover - depends on the machine
            raise RuntimeError(f"s_salaad_b200: cannot load {p}: {exc}") from exc
        for name, (args, res) in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        if lib.slr_abi_version() != ABI_VERSION:
            raise RuntimeError("s_salaad_b200: libslr_b200.so ABI version mismatch")
        if path is None:
            _lib = lib
        return lib


def last_error() -> str:
    return (load().slr_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str = "") -> None:
    """Map an slr_status to the reference's exception classes."""
    if rc == SLR_OK:
        return
    msg = last_error()
    text = f"{what}: {msg}" if what else msg
    if rc == SLR_ERR_UNSUPPORTED_DTYPE:
        raise TypeError(text)
    if rc in (SLR_ERR_INVALID_ARGUMENT, SLR_ERR_BAD_INDEX, SLR_ERR_WORKSPACE):
        raise ValueError(text)
    raise RuntimeError(f"{text} [{load().slr_status_string(rc).decode()}]")
