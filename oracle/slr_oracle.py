"""TEST INFRASTRUCTURE — CPU oracle for the S+LR linear and its BSR format.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module, and only as the checker (or as the timed CPU baseline);
the product package ``s_salaad_b200`` never imports it.

Parity pin: tests/test_oracle.py checks every function here against the
golden vectors in tests/golden/, which tests/golden/make_golden.py produced by
running the S-SALAAD reference itself (its AVX2 kernel, ``dense_to_bsr`` and
``_LRSLinearLRBlockCPU``) on seeded inputs.

Restated reference functions (paths within the S-SALAAD project):

* ``bsr_addmm_f32_``      ssalaad/cpu_sparse/bsr_addmm_avx2.cpp:67-174
                          (C: oracle/slr_oracle.c, bit-exact fmaf chain)
* ``dense_to_bsr``        ssalaad/efficient/artifact.py:20-37
* ``module_buffers``      ssalaad/efficient/ls_linear.py:86-97
* ``lrs_forward_f32``     ssalaad/efficient/ls_linear.py:155-164 (+ :38-44)
* ``lr_forward_f32``      ssalaad/efficient/ls_linear.py:47-51
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB_PATH = HERE / "_build" / "libslr_oracle.so"
_lib = None


def build() -> Path:
    """Compile oracle/slr_oracle.c (make, a few seconds)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.is_file():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        i64, p = ctypes.c_int64, ctypes.c_void_p
        L.oracle_bsr_addmm_f32.argtypes = [p, p, p, p, p, p] + [i64] * 7
        L.oracle_bsr_addmm_f32.restype = ctypes.c_int
        L.oracle_block_mask_f32.argtypes = [p, i64, i64, i64, i64, p]
        L.oracle_block_mask_f32.restype = ctypes.c_int
        L.oracle_block_mask_u16.argtypes = [p, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int, p]
        L.oracle_block_mask_u16.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data


def _np(t):
    """torch tensor or array-like -> numpy (no copy for contiguous CPU tensors)."""
    if hasattr(t, "detach"):
        t = t.detach()
        if t.device.type != "cpu":
            t = t.cpu()
        return t.contiguous().numpy()
    return np.ascontiguousarray(t)


# --------------------------------------------------------------- BSR addmm --

def bsr_addmm_f32_(out, x, crow, col, values, active_rows) -> None:
    """In place ``out += x @ S.T`` for BSR ``S`` (values stored ``[nnz, bq, bp]``).

    Same argument meaning as the reference ``bsr_addmm_avx2_``
    (ssalaad/cpu_sparse/bsr_addmm_avx2.py:53-68); ``out`` must be a writable
    float32 numpy array (or CPU tensor sharing memory with one).
    """
    o = _np(out)
    if o.dtype != np.float32:
        raise TypeError("oracle bsr_addmm: out must be float32")
    xs = np.ascontiguousarray(_np(x), dtype=np.float32)
    cr = np.ascontiguousarray(_np(crow), dtype=np.int32)
    cl = np.ascontiguousarray(_np(col), dtype=np.int32)
    vals = np.ascontiguousarray(_np(values), dtype=np.float32)
    act = np.ascontiguousarray(_np(active_rows), dtype=np.int32)
    nnz, bq, bp = vals.shape
    M, K = xs.shape
    NB = cr.shape[0] - 1
    if o.shape != (M, NB * bp):
        raise ValueError(f"oracle bsr_addmm: out shape {o.shape} != ({M}, {NB * bp})")
    rc = lib().oracle_bsr_addmm_f32(_ptr(o), _ptr(xs), _ptr(cr), _ptr(cl), _ptr(vals), _ptr(act),
                                    M, K, NB, nnz, act.shape[0], bp, bq)
    if rc != 0:
        raise ValueError("oracle bsr_addmm: invalid BSR structure")
    if hasattr(out, "detach") and out.data_ptr() != o.ctypes.data:
        import torch
        out.copy_(torch.from_numpy(o))


# ------------------------------------------------------------ dense -> BSR --

_U16_FORMATS = {"bfloat16": (8, 7), "float16": (5, 10)}


def block_mask(S, bp: int, bq: int, fmt: str | None = None) -> np.ndarray:
    """Live-block mask ``[n/bp, m/bq]`` (artifact.py:26-29: block L1 > 0).

    ``S`` is float32/float64 numpy, a torch tensor, or uint16 bit patterns with
    ``fmt`` in {"bfloat16", "float16"}.
    """
    if hasattr(S, "detach"):
        import torch
        if S.dtype in (torch.bfloat16, torch.float16):
            fmt = "bfloat16" if S.dtype == torch.bfloat16 else "float16"
            S = S.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
        else:
            S = S.detach().cpu().contiguous().to(torch.float32).numpy()
    n, m = S.shape
    if n % bp or m % bq:
        raise ValueError(f"shape ({n}, {m}) not divisible by block ({bp}, {bq})")
    mask = np.zeros((n // bp, m // bq), dtype=np.uint8)
    if fmt is not None:
        e, man = _U16_FORMATS[fmt]
        a = np.ascontiguousarray(S, dtype=np.uint16)
        rc = lib().oracle_block_mask_u16(_ptr(a), n, m, bp, bq, e, man, _ptr(mask))
    else:
        a = np.ascontiguousarray(S, dtype=np.float32)
        rc = lib().oracle_block_mask_f32(_ptr(a), n, m, bp, bq, _ptr(mask))
    if rc != 0:
        raise ValueError("oracle block_mask: bad arguments")
    return mask.astype(bool)


def dense_to_bsr(S, bp: int, bq: int):
    """Restates ``dense_to_bsr`` (artifact.py:20-37) in numpy.

    Returns ``(crow int64 [rb+1], col int64 [nnz], values [nnz, bp, bq])`` with
    blocks in row-major (block-row, then block-column) order, exactly the
    order ``torch.nonzero(mask)`` yields.  ``values`` keeps the input's
    element type (uint16 bit patterns for 16-bit torch inputs).
    """
    raw = S
    if hasattr(S, "detach"):
        import torch
        if S.dtype in (torch.bfloat16, torch.float16):
            raw = S.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
        else:
            raw = S.detach().cpu().contiguous().numpy()
    mask = block_mask(S, bp, bq)
    n, m = raw.shape
    rb, cb = n // bp, m // bq
    blocks = raw.reshape(rb, bp, cb, bq).transpose(0, 2, 1, 3)
    counts = mask.sum(axis=1).astype(np.int64)
    crow = np.concatenate([np.zeros(1, np.int64), np.cumsum(counts)])
    rows, cols = np.nonzero(mask)  # row-major order
    values = np.ascontiguousarray(blocks[rows, cols])
    return crow, cols.astype(np.int64), values


def module_buffers(crow, col, values_pq):
    """Restates ls_linear.py:86-97: int32 indices, blocks transposed to
    ``[nnz, bq, bp]``, and the int32 list of nonempty block-rows."""
    crow = np.asarray(crow)
    S_crow = crow.astype(np.int32)
    S_col = np.asarray(col).astype(np.int32)
    S_values = np.ascontiguousarray(np.asarray(values_pq).transpose(0, 2, 1))
    S_active_rows = np.nonzero(crow[1:] - crow[:-1])[0].astype(np.int32)
    return S_crow, S_col, S_values, S_active_rows


# ---------------------------------------------------------- S+LR forward --

def lrs_forward_f32(x, A, B, S_crow, S_col, S_values, S_active_rows, bias=None):
    """Restates ``_LRSLinearLRBlockCPU.forward`` (ls_linear.py:155-164).

    ``y = F.linear(F.linear(x, B), A)`` on the CPU (the same library calls the
    reference makes), then the in-place sparse accumulate above, then
    ``y += bias`` (ls_linear.py:41-44).  All float32; returns a torch tensor
    shaped like ``x[..., :out]``.
    """
    import torch
    import torch.nn.functional as F

    x = torch.as_tensor(_np(x)).float()
    A = torch.as_tensor(_np(A)).float()
    B = torch.as_tensor(_np(B)).float()
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    y = F.linear(F.linear(x2, B), A).contiguous()
    if S_col is not None and np.asarray(_np(S_col)).size:
        yn = y.numpy()
        bsr_addmm_f32_(yn, x2.numpy(), S_crow, S_col, S_values, S_active_rows)
    if bias is not None:
        y.add_(torch.as_tensor(_np(bias)).float())
    return y.reshape(*shape[:-1], A.shape[0])


def lr_forward_f32(x, A, B, bias=None):
    """Restates ``_LRSLinearLR.forward`` (ls_linear.py:47-51): no sparse term."""
    return lrs_forward_f32(x, A, B, None, None, None, None, bias)


def nm_project_2_4(R):
    """Keep the 2 largest-magnitude entries of every aligned group of 4 along
    the last axis (the reference's projection onto the 2:4 set,
    ssalaad/inference/egar.py:285-291); returns a torch tensor like R."""
    import torch

    R = torch.as_tensor(_np(R))
    n, k = R.shape
    g = R.reshape(n, k // 4, 4)
    keep = torch.zeros_like(g, dtype=torch.bool)
    keep.scatter_(-1, g.abs().topk(2, dim=-1).indices, True)
    return torch.where(keep, g, torch.zeros_like(g)).reshape(n, k)


def nm_forward_f32(x, A, B, S, bias=None):
    """Restates ``_LRSLinearLRNM.forward`` (ls_linear.py:210-221) in float32
    on the CPU: ``latent = F.linear(x, B)``; ``y = F.linear(x, S)`` with S the
    dense 2:4 matrix; ``y += latent @ A.T``; then the bias (:41-44)."""
    import torch
    import torch.nn.functional as F

    x = torch.as_tensor(_np(x)).float()
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    latent = F.linear(x2, torch.as_tensor(_np(B)).float())
    y = F.linear(x2, torch.as_tensor(_np(S)).float())
    y.addmm_(latent, torch.as_tensor(_np(A)).float().t())
    if bias is not None:
        y.add_(torch.as_tensor(_np(bias)).float())
    return y.reshape(*shape[:-1], y.shape[-1])


def ref_avx2_module():
    """The reference's own AVX2 kernel compiled by oracle/build_ref.py, or None."""
    try:
        import build_ref  # type: ignore
    except ImportError:
        import importlib.util
        spec = importlib.util.spec_from_file_location("slr_build_ref", HERE / "build_ref.py")
        build_ref = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(build_ref)
    try:
        return build_ref.load()
    except (FileNotFoundError, OSError, ImportError):
        return None


def lrs_forward_f32_ref_kernel(x, A, B, S_crow, S_col, S_values, S_active_rows, bias=None, mod=None):
    """Same as :func:`lrs_forward_f32` but the sparse step runs the reference's
    own compiled AVX2 kernel (the "reference" CPU baseline)."""
    import torch
    import torch.nn.functional as F

    mod = mod or ref_avx2_module()
    if mod is None:
        raise RuntimeError("reference AVX2 kernel not built (oracle/build_ref.py)")
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).contiguous()
    y = F.linear(F.linear(x2, B), A).contiguous()
    if S_col is not None and S_col.numel():
        mod.bsr_addmm_avx2_(y, x2, S_crow, S_col, S_values, S_active_rows)
    if bias is not None:
        y.add_(bias)
    return y.reshape(*shape[:-1], A.shape[0])


def max_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
