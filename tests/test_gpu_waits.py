"""Bounded waits on other ranks (the multi-GPU y assembly), on one GPU.

A wait that no rank answers gives up after the limit set by
``slr_set_wait_limit_ns`` and reports ``SLR_ERR_TIMEOUT`` through
``slr_device_status``; the GPU stays usable.  Both "ranks" of a call are this
process's own buffers: rank 0 is the library under test, and rank 1's words
in rank 0's signal slot are written from the host (or never written).  No
wait here is unbounded: each gives up after 50 ms.

Signal slot words (``SLR_SIGNAL_WORDS`` uint64 per layer and rank):
arrivals [0, 8), completions [8, 16), failed-call marks [16, 24), and the
rank's own call count at 24.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from s_salaad_b200 import _lib, ops, workloads

pytestmark = pytest.mark.gpu

ARRIVE, DONE, FAIL, CALLS = 0, 8, 16, 24
UNIT = 1 << 32  # completion count of one rank per call
LIMIT_NS = 50_000_000


@pytest.fixture
def lib(cuda):
    lib = _lib.load()
    lib.slr_set_wait_limit_ns(LIMIT_NS)
    yield lib
    lib.slr_set_wait_limit_ns(0)  # back to the 2 s default


def _status(lib) -> int:
    st = ctypes.c_int(-1)
    _lib.check(lib.slr_device_status(ctypes.byref(st)))
    return st.value


def _peers(cuda, y: torch.Tensor):
    mine = torch.zeros(_lib.SLR_SIGNAL_WORDS, dtype=torch.int64, device=cuda)
    theirs = torch.zeros_like(mine)  # rank 1's slot: rank 0 signals into it, nobody waits on it
    y_theirs = torch.zeros_like(y)
    st = _lib.SlrPeers()
    st.world, st.rank = 2, 0
    for p, (slot, yy) in enumerate(((mine, y), (theirs, y_theirs))):
        st.y[p] = yy.data_ptr()
        st.signal[p] = slot.data_ptr()
    return st, mine, theirs


def test_peer_wait_times_out_then_resynchronises(cuda, lib):
    assert _status(lib) == _lib.SLR_OK
    y = torch.zeros(8, 64, dtype=torch.bfloat16, device=cuda)
    st, mine, theirs = _peers(cuda, y)
    stream = torch.cuda.current_stream(cuda).cuda_stream

    def call() -> int:  # rank 0 without rows of the layer: announce, wait, count
        t0 = time.perf_counter()
        _lib.check(lib.slr_peers_wait(ctypes.byref(st), 1, stream), "peers_wait")
        s = _status(lib)
        assert time.perf_counter() - t0 < 5.0
        return s

    # call 1: rank 1 never arrives -> timeout; the call is marked failed at
    # both ranks and still counted, so the counts stay in step
    assert call() == _lib.SLR_ERR_TIMEOUT
    m, t = mine.cpu(), theirs.cpu()
    assert (int(m[CALLS]), int(m[ARRIVE]), int(m[FAIL]), int(m[DONE])) == (1, 1, 1, UNIT)
    assert (int(t[ARRIVE]), int(t[FAIL]), int(t[DONE])) == (1, 1, UNIT)
    # rank 1 catches up with call 1 only: its words for call 1 must not let call 2 pass
    mine[ARRIVE + 1] = 1
    mine[DONE + 1] = UNIT
    assert call() == _lib.SLR_ERR_TIMEOUT
    assert int(mine[CALLS].item()) == 2
    # rank 1 makes call 3 on time: the layer is synchronised again
    mine[ARRIVE + 1] = 3
    mine[DONE + 1] = 3 * UNIT
    assert call() == _lib.SLR_OK
    # rank 1 a call ahead (it skipped one): call 4 reports a timeout instead of passing
    mine[ARRIVE + 1] = 5
    mine[DONE + 1] = 5 * UNIT
    assert call() == _lib.SLR_ERR_TIMEOUT
    assert _status(lib) == _lib.SLR_OK  # reading the status cleared it


def test_peer_epilogue_times_out_keeps_local_result(cuda, lib):
    """The 2-SM combine kernel with a peer that never arrives: its epilogue
    waits give up, the local y is still written, and the call reports a
    timeout (the peer's y is left alone)."""
    n, k, b, r, T = 1024, 512, 64, 64, 512
    crow, col = workloads.bernoulli_structure(n // b, k // b, 0.3, seed=5)
    spec = workloads.LayerSpec("waits", n, k, r, b, b, crow, col, seed=6, bias_std=0.01)
    t = spec.tensors(cuda, torch.bfloat16)
    order = torch.from_numpy(ops.plan_row_order(crow.astype(np.int32))).to(cuda)
    d = ops.LayerDesc(A=t["A"], B=t["B"], bias=t["bias"], crow=t["S_crow"], col=t["S_col"], values=t["S_values"],
                      row_order=order, in_features=k, out_features=n, block_p=b, block_q=b)
    x = workloads.tokens(T, k, seed=9, device=cuda, dtype=torch.bfloat16)
    ref = d.forward(x)
    assert lib.slr_lrs_linear_peers_supported(ctypes.byref(d.struct), x.data_ptr(), k, T) == 1
    y = torch.full_like(ref, float("nan"))
    st, mine, theirs = _peers(cuda, y)
    ws = d.workspace(T)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    assert _status(lib) == _lib.SLR_OK
    d.lowrank(x)
    _lib.check(lib.slr_lrs_linear_combine_peers(ctypes.byref(d.struct), x.data_ptr(), k, n, T, ws.data_ptr(),
                                                ws.numel(), ctypes.byref(st), stream), "combine_peers")
    _lib.check(lib.slr_peers_wait(ctypes.byref(st), 0, stream), "peers_wait")
    assert _status(lib) == _lib.SLR_ERR_TIMEOUT
    assert torch.equal(y, ref)  # the local tiles were stored
    assert int(mine[FAIL].item()) == 1 and int(theirs[FAIL].item()) == 1
    # the GPU is still usable and the library's status is clean again
    assert torch.equal(d.forward(x), ref)
    assert _status(lib) == _lib.SLR_OK
