"""The N:M 2:4 + low-rank layer on the sparse tensor cores.

Reference: _LRSLinearLRNM (ssalaad/efficient/ls_linear.py:167-224), forward
at :210-221 (cuSPARSELt semi-structured S, then addmm of the low-rank term,
then the bias).  The oracle restates that forward in fp32 on fp32 copies of
the 16-bit tensors (oracle/slr_oracle.py: nm_forward_f32).

Tolerances: the 2:4 packing round trip is bit-exact; the layer's output
|y - y_ref| <= 2e-2 * RMS(y_ref) + half an ulp of y_ref elementwise (the
16-bit bound of the other parity tests).
"""
from __future__ import annotations

import pytest
import torch

from s_salaad_b200 import ops, workloads
from s_salaad_b200.efficient import LRSLinear, _LRSLinearLRNM
from test_gpu_parity import assert_16bit_close, rms

pytestmark = pytest.mark.gpu


def sparse_2_4(n, k, seed, std=0.02, dtype=torch.bfloat16, partial=True):
    """A random 2:4 matrix: N(0, std) projected to the 2 largest of each group
    of 4 (the reference's projection), and (partial) some groups holding one
    or no entry."""
    import slr_oracle

    g = torch.Generator().manual_seed(seed)
    R = torch.randn(n, k, generator=g) * std
    S = slr_oracle.nm_project_2_4(R)
    if partial:
        groups = S.view(n, k // 4, 4)
        drop = torch.rand(n, k // 4, generator=g)
        groups[drop < 0.1] = 0.0                       # empty groups
        one = (drop >= 0.1) & (drop < 0.2)             # groups with one entry
        first = groups[one].clone()
        keep = first.abs().argmax(-1, keepdim=True)
        groups[one] = torch.zeros_like(first).scatter_(-1, keep, first.gather(-1, keep))
    assert not bool((S == 0).logical_and(S.signbit()).any())  # every dropped entry is +0
    return S.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_nm_compress_round_trip_bit_exact(cuda, dtype):
    S = sparse_2_4(96, 256, seed=1, dtype=dtype).to(cuda)
    values, meta = ops.nm_compress(S)
    assert values.shape == (96, 128) and meta.shape == (96, 8)
    assert torch.equal(ops.nm_expand(values, meta).view(torch.int16), S.view(torch.int16))
    # positions are ordered within every group (first < second)
    words = meta.to(torch.int64) & 0xFFFFFFFF
    nib = (words.unsqueeze(-1) >> (torch.arange(8, device=cuda) * 4)) & 0xF
    assert bool(((nib & 3) < (nib >> 2)).all())


def test_nm_compress_rejects_dense_groups(cuda):
    S = sparse_2_4(32, 64, seed=2).to(cuda)
    S[5, 8:11] = 1.0  # three entries in one group of 4
    with pytest.raises(ValueError, match="2:4"):
        ops.nm_compress(S)
    with pytest.raises(ValueError):
        ops.nm_compress(torch.zeros(16, 48, dtype=torch.bfloat16, device=cuda))  # K % 32 != 0


NM_SHAPES = [  # out, in, rank, bias
    (256, 512, 64, True),
    (384, 256, 32, False),
    (512, 1024, 128, True),
    (128, 2048, 256, True),
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", NM_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("T", [1, 7, 16, 33, 64, 127, 128, 300])
def test_nm_forward_matches_oracle(cuda, oracle, dtype, shape, T):
    n, k, r, has_bias = shape
    g = torch.Generator().manual_seed(n + k + r + T)
    S = sparse_2_4(n, k, seed=n + r + T, dtype=dtype)
    A = (torch.randn(n, r, generator=g) * 0.02).to(dtype)
    B = (torch.randn(r, k, generator=g) * 0.02).to(dtype)
    bias = (torch.randn(n, generator=g) * 0.01).to(dtype) if has_bias else None
    x = workloads.tokens(T, k, seed=T, dtype=dtype)
    layer = LRSLinear(A.to(cuda), B.to(cuda), S.to(cuda), in_features=k, out_features=n,
                      bias=None if bias is None else bias.to(cuda), nm_n=2, nm_m=4)
    assert isinstance(layer, _LRSLinearLRNM)
    y = layer(x.to(cuda))
    ref = oracle.nm_forward_f32(x.float(), A.float(), B.float(), S.float(), None if bias is None else bias.float())
    assert_16bit_close(y, ref)


def test_nm_module_api_mirrors_reference(cuda):
    n, k, r = 256, 512, 64
    S = sparse_2_4(n, k, seed=9).to(cuda)
    A = torch.randn(n, r, device=cuda, dtype=torch.bfloat16) * 0.02
    B = torch.randn(r, k, device=cuda, dtype=torch.bfloat16) * 0.02
    bias = torch.zeros(n, device=cuda, dtype=torch.bfloat16)
    layer = LRSLinear(A, B, S.to_sparse_csr(), in_features=k, out_features=n, bias=bias, nm_n=2, nm_m=4)
    assert layer.kind == "nm" and layer.S_nnz == n * k // 2
    assert set(layer.state_dict()) == {"A", "B", "bias"}  # packed S is not persistent, as in the reference
    with pytest.raises(ValueError, match="2:4"):
        LRSLinear(A, B, S, in_features=k, out_features=n, nm_n=2, nm_m=8)
    with pytest.raises(ValueError):
        LRSLinear(A.cpu(), B.cpu(), S.cpu(), in_features=k, out_features=n, nm_n=2, nm_m=4)
    x = torch.randn(3, 5, k, device=cuda, dtype=torch.bfloat16)
    assert layer(x).shape == (3, 5, n)


@pytest.mark.parametrize("T", [1, 32, 4096])
def test_nm_full_size_matches_torch_fp32(cuda, T, parity_log):
    """A LLaMA-7B-shaped MLP projection (11008 x 4096, rank 512) with 2:4 S
    against a plain PyTorch fp32 reference on the GPU (TF32 off)."""
    n, k, r = 11008, 4096, 512
    g = torch.Generator(device="cpu").manual_seed(T)
    S = sparse_2_4(n, k, seed=T, partial=False).to(cuda)
    A = (torch.randn(n, r, generator=g) * (0.02 / 8)).to(cuda, torch.bfloat16)
    B = (torch.randn(r, k, generator=g) * (0.02 / 8)).to(cuda, torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.01).to(cuda, torch.bfloat16)
    x = workloads.tokens(T, k, seed=T, device=cuda, dtype=torch.bfloat16)
    layer = LRSLinear(A, B, S, in_features=k, out_features=n, bias=bias, nm_n=2, nm_m=4)
    y = layer(x)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        xf = x.float()
        ref = xf @ S.float().T + (xf @ B.float().T) @ A.float().T + bias.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    parity_log(f"nm24 T={T} 11008x4096 r512", y, ref)
    assert_16bit_close(y, ref)
    assert rms(ref) > 0


@pytest.mark.parametrize("T", [255, 256, 1000])
def test_nm_prefill_route(cuda, oracle, T):
    """From 256 tokens (out, in and rank multiples of 64) S is unpacked per
    call into full-density 64 x 64 blocks and the layer runs on the 2-SM
    tensor-core combine: the workspace then holds the unpacked S, and the
    result meets the same bound against the fp32 oracle as the mma.sp kernel's
    below 256 tokens."""
    import ctypes

    from s_salaad_b200 import _lib

    n, k, r = 512, 1024, 128
    dtype = torch.bfloat16
    g = torch.Generator().manual_seed(T)
    S = sparse_2_4(n, k, seed=T, dtype=dtype)
    A = (torch.randn(n, r, generator=g) * 0.02).to(dtype)
    B = (torch.randn(r, k, generator=g) * 0.02).to(dtype)
    bias = (torch.randn(n, generator=g) * 0.01).to(dtype)
    values, meta = ops.nm_compress(S.to(cuda))
    desc = ops.NmLayerDesc(values=values, meta=meta, A=A.to(cuda), B=B.to(cuda), bias=bias.to(cuda),
                           in_features=k, out_features=n)
    lib = _lib.load()
    ws = int(lib.slr_nm_linear_workspace_size(ctypes.byref(desc.struct), T))
    ws_h = int(lib.slr_nm_linear_workspace_size(ctypes.byref(desc.struct), 255))
    if T >= 256:
        assert ws >= ws_h + n * k * 2  # the unpacked S
    x = workloads.tokens(T, k, seed=T, dtype=dtype)
    y = desc.forward(x.to(cuda))
    ref = oracle.nm_forward_f32(x.float(), A.float(), B.float(), S.float(), bias.float())
    assert_16bit_close(y, ref)
    # a second call reuses the workspace (the blocks and the schedule are rewritten)
    assert torch.equal(desc.forward(x.to(cuda)), y)
