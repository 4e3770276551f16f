"""The allocation-free forward, slr_lrs_linear_forward_noalloc.

Callers that cannot allocate device memory (a plugin inside a framework that
owns every allocation, code running under another component's stream
capture, a serving loop that must never enter the allocator) use this entry
point: it takes no workspace and keeps its scratch in a fixed array inside
the library.  These tests call it through the C ABI and check that it gives
the same output as slr_lrs_linear_forward (which uses a caller workspace),
call after call, and that a request larger than the array is refused before
anything runs.  The file sorts last so a failure here leaves every other test
already run.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from s_salaad_b200 import _lib, ops, workloads

pytestmark = pytest.mark.gpu


def _layer(device, T_seed: int):
    crow, col = workloads.bernoulli_structure(384 // 32, 512 // 32, 0.3, seed=31)
    spec = workloads.LayerSpec("noalloc", 384, 512, 64, 32, 32, crow, col, seed=32, bias_std=0.01)
    t = spec.tensors(device, torch.bfloat16)
    order = torch.from_numpy(ops.plan_row_order(crow.astype(np.int32))).to(device)
    return spec, ops.LayerDesc(A=t["A"], B=t["B"], bias=t["bias"], crow=t["S_crow"], col=t["S_col"],
                               values=t["S_values"], row_order=order, in_features=512, out_features=384,
                               block_p=32, block_q=32)


def _close(y: torch.Tensor, ref: torch.Tensor) -> None:
    """The 16-bit bound of the parity tests: 2e-2 * RMS(ref) + half an ulp of |ref|."""
    y, ref = y.float(), ref.float()
    rms = float(ref.pow(2).mean().sqrt())
    half_ulp = torch.pow(2.0, torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - 8)
    assert torch.isfinite(y).all()
    assert bool(((y - ref).abs() <= 2e-2 * rms + half_ulp + 1e-6).all())


@pytest.mark.parametrize("T", [7, 300])  # split-K small-batch path, and the tcgen05 path
def test_noalloc_forward_matches_workspace_forward_twice(cuda, T):
    lib = _lib.load()
    spec, desc = _layer(cuda, T)
    x = workloads.tokens(T, 512, seed=T, device=cuda, dtype=torch.bfloat16)
    ref = desc.forward(x)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for _ in range(2):  # the array keeps the previous call's contents
        y = torch.full_like(ref, float("nan"))
        rc = lib.slr_lrs_linear_forward_noalloc(ctypes.byref(desc.struct), x.data_ptr(), 512, y.data_ptr(), 384,
                                                T, stream)
        _lib.check(rc, "slr_lrs_linear_forward_noalloc")
        torch.cuda.synchronize()
        _close(y, ref)


def test_noalloc_refuses_requests_beyond_its_array(cuda):
    lib = _lib.load()
    spec, desc = _layer(cuda, 0)
    M = 1 << 20  # 1M tokens x 64 rank columns x 2 bytes = 128 MiB of scratch
    rc = lib.slr_lrs_linear_forward_noalloc(ctypes.byref(desc.struct), 16, 512, 16, 384, M, None)
    assert rc == _lib.SLR_ERR_WORKSPACE
    assert "bytes of scratch" in _lib.last_error()


def test_noalloc_size_limit_is_exact(cuda):
    """The largest token count whose scratch fits the 16 MiB array runs and
    matches the workspace forward; one token more is refused."""
    lib = _lib.load()
    spec, desc = _layer(cuda, 0)
    limit = 16 << 20
    M = limit // (64 * 2)  # H = x * B^T: 64 rank columns of 2 bytes per token
    assert desc.workspace_bytes(M) <= limit < desc.workspace_bytes(M + 1)
    x = workloads.tokens(M, 512, seed=11, device=cuda, dtype=torch.bfloat16)
    ref = desc.forward(x)
    y = torch.full_like(ref, float("nan"))
    stream = torch.cuda.current_stream(cuda).cuda_stream
    _lib.check(lib.slr_lrs_linear_forward_noalloc(ctypes.byref(desc.struct), x.data_ptr(), 512, y.data_ptr(), 384,
                                                  M, stream), "slr_lrs_linear_forward_noalloc")
    torch.cuda.synchronize()
    _close(y, ref)
    rc = lib.slr_lrs_linear_forward_noalloc(ctypes.byref(desc.struct), x.data_ptr(), 512, y.data_ptr(), 384,
                                            M + 1, stream)
    assert rc == _lib.SLR_ERR_WORKSPACE
