"""The CPU oracle against the golden vectors produced by the reference itself.

Bit-exact where the reference is deterministic integer/order-fixed work (the
AVX2 kernel's FMA chain, dense_to_bsr); within fp32 rounding for the layer,
whose low-rank step is a BLAS call.
"""
from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import load_golden
from s_salaad_b200 import workloads


@pytest.mark.parametrize("block", [8, 16, 32, 64])
def test_oracle_addmm_is_bit_exact_with_reference_avx2(oracle, block):
    g = load_golden(f"avx2_block{block}")
    for start, key in ((np.zeros_like(g["out_zero"]), "out_zero"), (g["out0"], "out_acc")):
        out = start.copy()
        oracle.bsr_addmm_f32_(out, g["x"], g["crow"], g["col"], g["values"], g["active_rows"])
        assert np.array_equal(out.view(np.uint32), g[key].view(np.uint32)), key


@pytest.mark.parametrize("block", [8, 16, 32, 64])
def test_golden_matches_dense_matmul(block):
    """The reference test's own check (tests/test_ssalaad.py:320-327)."""
    g = load_golden(f"avx2_block{block}")
    ref = torch.from_numpy(g["x"]) @ torch.from_numpy(g["dense_S"]).T
    torch.testing.assert_close(torch.from_numpy(g["out_zero"]), ref, rtol=0, atol=1e-4)


def test_oracle_leaves_empty_block_rows_untouched(oracle):
    g = load_golden("avx2_empty_rows")
    out = np.full_like(g["out"], 7.0)
    oracle.bsr_addmm_f32_(out, g["x"], g["crow"], g["col"], g["values"], g["active_rows"])
    assert np.array_equal(out.view(np.uint32), g["out"].view(np.uint32))
    assert np.all(out[:, :32] == 7.0)


def test_reference_kernel_build_matches_golden():
    """oracle/_ref (the reference .cpp compiled by oracle/build_ref.py) is the
    same arithmetic as the reference's own JIT build that made the goldens."""
    import slr_oracle

    mod = slr_oracle.ref_avx2_module()
    if mod is None:
        pytest.skip("oracle/_ref not built (reference sources absent when building)")
    for block in (8, 16, 32, 64):
        g = load_golden(f"avx2_block{block}")
        out = torch.from_numpy(g["out0"].copy())
        mod.bsr_addmm_avx2_(out, torch.from_numpy(g["x"]), torch.from_numpy(g["crow"]),
                            torch.from_numpy(g["col"]), torch.from_numpy(g["values"]),
                            torch.from_numpy(g["active_rows"]))
        assert torch.equal(out.view(torch.int32), torch.from_numpy(g["out_acc"]).view(torch.int32))


def test_oracle_rejects_out_of_range_col(oracle):
    g = load_golden("avx2_block16")
    col = g["col"].copy()
    col[0] = 99
    with pytest.raises(ValueError):
        oracle.bsr_addmm_f32_(np.zeros_like(g["out_zero"]), g["x"], g["crow"], col, g["values"],
                              g["active_rows"])


def _d2b_cases():
    with np.load("tests/golden/dense_to_bsr.npz") as z:
        keys = sorted({k.split("__")[0] for k in z.files})
    return keys


@pytest.fixture(scope="module")
def d2b():
    from conftest import GOLDEN

    with np.load(GOLDEN / "dense_to_bsr.npz") as z:
        data = {}
        for k in z.files:
            case, f = k.split("__")
            data.setdefault(case, {})[f] = z[k]
    return data


def _block_shape(case: str, values: np.ndarray, S: np.ndarray):
    if values.ndim == 3 and values.shape[0]:
        return values.shape[1], values.shape[2]
    if case.endswith(("zero", "full")):
        return 16, 16
    bp, bq = case.split("_")[-1].split("x")
    return int(bp), int(bq)


def test_oracle_dense_to_bsr_is_bit_exact(oracle, d2b):
    assert len(d2b) >= 10
    for case, g in d2b.items():
        bp, bq = _block_shape(case, g["values"], g["S"])
        fmt = "bfloat16" if case.startswith("d2b_bf16") else None
        S = g["S"]
        if fmt:
            mask = oracle.block_mask(S, bp, bq, fmt)
            raw = S
        else:
            mask = oracle.block_mask(S, bp, bq)
            raw = S
        crow, col, values = oracle.dense_to_bsr(torch.from_numpy(S) if fmt is None else _bf16(S), bp, bq)
        assert np.array_equal(crow, g["crow"]), case
        assert np.array_equal(col, g["col"]), case
        assert values.shape == g["values"].shape, case
        assert np.array_equal(values.view(np.uint8), np.ascontiguousarray(g["values"]).view(np.uint8)), case
        assert mask.sum() == g["col"].shape[0]
        del raw


def _bf16(u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(u16.view(np.int16).copy()).view(torch.bfloat16)


def test_dense_to_bsr_edge_semantics(d2b):
    """-0.0 and NaN blocks are dropped, inf and subnormal blocks kept."""
    for case in ("d2b_f32_16x16", "d2b_bf16_16x16"):
        g = d2b[case]
        col, crow = g["col"], g["crow"]
        row_cols = lambda i: set(col[crow[i]:crow[i + 1]].tolist())  # noqa: E731
        assert 0 not in row_cols(0)      # all -0.0
        assert 0 not in row_cols(1)      # NaN + 1.0
        assert 1 in row_cols(2)          # inf
        assert 2 in row_cols(3)          # subnormal


def _digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        if hasattr(a, "detach"):
            a = a.detach().cpu().contiguous()
            if a.dtype == torch.bfloat16:
                a = a.view(torch.int16)
            a = a.numpy()
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_oracle_layer_matches_reference_cfg1(oracle):
    g = load_golden("lrs_cfg1_T32")
    spec = workloads.cfg1_layer(0)
    t = spec.tensors("cpu", torch.float32)
    x = workloads.tokens(32, spec.in_features, seed=5)
    assert _digest(t["A"], t["B"], t["bias"], t["values_pq"], spec.crow, spec.col, x) == str(g["inputs_sha256"])
    torch.set_num_threads(1)
    y = oracle.lrs_forward_f32(x, t["A"], t["B"], t["S_crow"], t["S_col"], t["S_values"], t["S_active_rows"],
                               t["bias"])
    ref = torch.from_numpy(g["y"])
    # Same library calls in the same order as the reference: identical bits
    # on one thread; allow fp32 rounding in case the BLAS build differs.
    torch.testing.assert_close(y, ref, rtol=1e-6, atol=1e-7)


def test_oracle_layer_matches_reference_bf16_values(oracle):
    g = load_golden("lrs_b32_bf16vals")
    crow, col = workloads.bernoulli_structure(256 // 32, 512 // 32, 0.3, seed=21)
    spec = workloads.LayerSpec("b32", 256, 512, 64, 32, 32, crow, col, seed=22)
    t = spec.tensors("cpu", torch.bfloat16)
    x = workloads.tokens(16, 512, seed=23, dtype=torch.bfloat16)
    assert _digest(t["A"], t["B"], t["values_pq"], spec.crow, spec.col, x) == str(g["inputs_sha256"])
    y = oracle.lrs_forward_f32(x.float(), t["A"].float(), t["B"].float(), t["S_crow"], t["S_col"],
                               t["S_values"].float(), t["S_active_rows"])
    torch.testing.assert_close(y, torch.from_numpy(g["y"]), rtol=1e-6, atol=1e-7)


def test_oracle_tiny_rank4_layer(oracle):
    g = load_golden("lrs_tiny_rank4")
    crow, col, vals = oracle.dense_to_bsr(torch.from_numpy(g["S"]), 16, 16)
    S_crow, S_col, S_values, active = oracle.module_buffers(crow, col, vals)
    y = oracle.lrs_forward_f32(g["x"], g["A"], g["B"], S_crow, S_col, S_values, active)
    torch.testing.assert_close(y, torch.from_numpy(g["y"]), rtol=1e-6, atol=1e-8)
