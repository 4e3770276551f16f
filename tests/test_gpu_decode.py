"""The single-launch decode kernel (slr_lrs_linear_decode): x·Bᵀ and the
combine of up to eight layers in one persistent launch, 1..32 tokens.

Reference: _LRSLinearLRBlockCUDA.forward (ssalaad/efficient/ls_linear.py:
124-137); the oracle is its fp32 restatement (oracle/slr_oracle.py).
Tolerance: the 16-bit bound of the other parity tests, |y - y_ref| <=
2e-2 * RMS(y_ref) + half an ulp of y_ref elementwise.  Bit-exact claims:
the result of a layer does not depend on the token count (<= 32), on the
other layers of the call, on the grid or on graph capture.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from s_salaad_b200 import _lib, ops, workloads
from test_gpu_parity import assert_16bit_close, desc_for, oracle_layer, random_layer

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _single_launch():
    """The library's calls of 1..32 tokens take the single-launch kernel
    (opt-in; the two-launch path is the default)."""
    with ops.single_launch_decode(True):
        yield

SHAPES = [
    # n, k, bp, bq, r, density: K below and above one 1024-wide H chunk, every block size
    (256, 512, 16, 16, 32, 0.3),
    (512, 2048, 32, 32, 256, 0.3),
    (384, 1536, 64, 64, 512, 0.2),
    (320, 1100 // 16 * 16, 16, 16, 16, 0.4),   # K = 1088: a ragged last chunk
    (256, 768, 32, 16, 48, 0.5),
    (192, 256, 64, 32, 64, 0.0),               # low-rank only (nnz = 0)
]


def _status() -> int:
    st = ctypes.c_int(-1)
    _lib.check(_lib.load().slr_device_status(ctypes.byref(st)), "device_status")
    return st.value


def _layer(cuda, shape, seed, dtype=torch.bfloat16):
    n, k, bp, bq, r, dens = shape
    spec = random_layer(n, k, bp, bq, r, dens, seed=seed)
    t = spec.tensors("cpu", dtype)
    return spec, t, desc_for(t, spec, cuda, dtype)


def _supported(d: ops.LayerDesc, x: torch.Tensor) -> bool:
    xp = (ctypes.c_void_p * 1)(x.data_ptr())
    lx = (ctypes.c_int64 * 1)(x.stride(0))
    return bool(_lib.load().slr_lrs_linear_decode_supported(ctypes.byref(d.struct), 1, xp, lx, x.shape[0]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("T", [1, 7, 8, 9, 16, 17, 32])
def test_decode_matches_oracle(cuda, oracle, dtype, shape, T):
    spec, t, d = _layer(cuda, shape, seed=sum(shape[:5]) + T, dtype=dtype)
    x = workloads.tokens(T, spec.in_features, seed=T, dtype=dtype).to(cuda)
    assert _supported(d, x)
    y = d.forward(x)
    assert_16bit_close(y, oracle_layer(oracle, t, x.cpu()))


def test_decode_is_batch_invariant_and_call_invariant(cuda):
    """A token's output is the same bit for bit whatever the other tokens of
    the call (1, 5, 16 or 32 rows) and whatever the other layers of a set."""
    layers = [_layer(cuda, s, seed=40 + i) for i, s in enumerate(SHAPES)]
    xs = [workloads.tokens(32, s.in_features, seed=3 + i, dtype=torch.bfloat16).to(cuda)
          for i, (s, _, _) in enumerate(layers)]
    full = [d.forward(x) for (_, _, d), x in zip(layers, xs)]
    for T in (1, 5, 16):
        for (_, _, d), x, y32 in zip(layers, xs, full):
            assert torch.equal(d.forward(x[:T].contiguous()), y32[:T])
    descs = [d for _, _, d in layers]
    ys = ops.LayerSet(descs).forward(xs)
    for y, y32 in zip(ys, full):
        assert torch.equal(y, y32)


def test_decode_differs_from_two_launch_path_only_by_rounding(cuda, oracle):
    """Both paths meet the bound; they need not agree bit for bit (x·Bᵀ is
    split over K differently)."""
    spec, t, d = _layer(cuda, (512, 2048, 32, 32, 256, 0.3), seed=5)
    x = workloads.tokens(4, 2048, seed=4, dtype=torch.bfloat16).to(cuda)
    ref = oracle_layer(oracle, t, x.cpu())
    y1 = d.forward(x)
    with ops.single_launch_decode(False):
        y2 = d.forward(x)
    assert_16bit_close(y1, ref)
    assert_16bit_close(y2, ref)


def test_decode_control_block_is_left_zero_and_graph_replays(cuda):
    specs = [(512, 2048, 32, 32, 256, 0.3), (1376, 512, 16, 16, 64, 0.5), (512, 1376, 16, 16, 64, 0.5)]
    layers = [_layer(cuda, s, seed=60 + i) for i, s in enumerate(specs)]
    lset = ops.LayerSet([d for _, _, d in layers])
    xs = [workloads.tokens(3, s.in_features, seed=i, dtype=torch.bfloat16).to(cuda)
          for i, (s, _, _) in enumerate(layers)]
    ref = [y.clone() for y in lset.forward(xs)]
    torch.cuda.synchronize()
    assert int(lset._decode.ctrl.abs().sum()) == 0
    outs = [torch.empty_like(y) for y in ref]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        lset.forward(xs, outs)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            lset.forward(xs, outs)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(5):
        for o in outs:
            o.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        for o, r in zip(outs, ref):
            assert torch.equal(o, r)
    assert int(lset._decode.ctrl.abs().sum()) == 0
    assert _status() == _lib.SLR_OK
    del g


def test_decode_wait_for_h_times_out_then_recovers(cuda):
    """A tile counter that can never reach its target (planted in the
    control block) keeps the layer's H from being published: every CTA's
    wait for H gives up after the limit, the call reports SLR_ERR_TIMEOUT,
    the last CTA still leaves the control block zero, and the next call is
    correct.  No wait here lasts longer than 50 ms."""
    lib = _lib.load()
    spec, t, d = _layer(cuda, (512, 2048, 32, 32, 256, 0.3), seed=9)  # K = 2048: two chunks per tile
    x = workloads.tokens(2, 2048, seed=2, dtype=torch.bfloat16).to(cuda)
    ref = d.forward(x)
    torch.cuda.synchronize()
    assert _status() == _lib.SLR_OK
    lib.slr_set_wait_limit_ns(50_000_000)
    try:
        ctrl = d._decode.ctrl
        ctrl[16] = 1 << 20  # tile 0 of the layer: the last-chunk test never matches
        d.forward(x)
        torch.cuda.synchronize()
        assert _status() == _lib.SLR_ERR_TIMEOUT
        assert int(ctrl.abs().sum()) == 0
        assert torch.equal(d.forward(x), ref)
        assert _status() == _lib.SLR_OK
    finally:
        lib.slr_set_wait_limit_ns(0)


def test_decode_falls_back_outside_its_shapes(cuda, oracle):
    """rank % 16 != 0 and more than 32 tokens take the two-launch path."""
    spec, t, d = _layer(cuda, (256, 256, 32, 32, 24, 0.5), seed=3)
    x = workloads.tokens(4, 256, seed=1, dtype=torch.bfloat16).to(cuda)
    assert not _supported(d, x)
    assert_16bit_close(d.forward(x), oracle_layer(oracle, t, x.cpu()))
    spec, t, d = _layer(cuda, (256, 256, 32, 32, 64, 0.5), seed=4)
    x = workloads.tokens(33, 256, seed=1, dtype=torch.bfloat16).to(cuda)
    assert not _supported(d, x)
    assert_16bit_close(d.forward(x), oracle_layer(oracle, t, x.cpu()))


def test_decode_rows_without_blocks_and_ragged_low_rank_tiles(cuda, oracle):
    """Block-rows with no blocks get the low-rank term and bias only; a
    low-rank-only layer whose width is not a multiple of its 64-feature tiles."""
    n, k = 256, 512
    crow = np.zeros(n // 32 + 1, dtype=np.int64)
    col = []
    for i in range(n // 32):
        cols = [] if i % 3 == 0 else list(range(i % 4, k // 32, 3))
        col += cols
        crow[i + 1] = crow[i] + len(cols)
    spec = workloads.LayerSpec("holes", n, k, 64, 32, 32, crow, np.asarray(col, dtype=np.int64), seed=8)
    t = spec.tensors("cpu", torch.bfloat16)
    d = desc_for(t, spec, cuda, torch.bfloat16)
    x = workloads.tokens(5, k, seed=5, dtype=torch.bfloat16).to(cuda)
    assert _supported(d, x)
    assert_16bit_close(d.forward(x), oracle_layer(oracle, t, x.cpu()))
    spec = random_layer(200, 256, 16, 16, 32, 0.0, seed=11)
    t = spec.tensors("cpu", torch.bfloat16)
    d = desc_for(t, spec, cuda, torch.bfloat16)
    x = workloads.tokens(3, 256, seed=6, dtype=torch.bfloat16).to(cuda)
    assert _supported(d, x)
    ref = oracle.lr_forward_f32(x.cpu().float(), t["A"].float(), t["B"].float(), t["bias"].float())
    assert_16bit_close(d.forward(x), ref)
