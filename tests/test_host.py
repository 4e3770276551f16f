"""Host-side logic that needs no GPU: the C ABI library loads and exports
every declared symbol, argument validation maps to the reference's exception
classes, the planners, and the synthetic workload generators."""
from __future__ import annotations

import ctypes
import re
import subprocess

import numpy as np
import pytest
import torch

from conftest import REPO
from s_salaad_b200 import _lib, ops, workloads


def _declared_symbols() -> set[str]:
    text = (REPO / "include" / "slr_b200.h").read_text()
    return set(re.findall(r"^SLR_API\s+[\w\s\*]+?\b(slr_\w+)\(", text, flags=re.M))


def test_header_and_binding_agree():
    assert _declared_symbols() == set(_lib.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    for name in _declared_symbols():
        assert name in exported, name
        assert getattr(lib, name) is not None
    assert lib.slr_abi_version() == _lib.ABI_VERSION == 8


def test_library_is_built_for_sm100a():
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", str(_lib.LIB_PATH)],
                         capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    assert "sm_100a" in out.stdout


def test_status_strings():
    lib = _lib.load()
    assert lib.slr_status_string(0) == b"SLR_OK"
    assert lib.slr_status_string(7) == b"SLR_ERR_TIMEOUT"


def test_addmm_argument_errors_need_no_gpu():
    lib = _lib.load()
    # bad dtype -> TypeError class
    rc = lib.slr_bsr_addmm_inplace(None, None, 4, 32, None, 2, None, None, 0, 16, 16, None, 1, 9, None)
    assert rc == _lib.SLR_ERR_UNSUPPORTED_DTYPE
    with pytest.raises(TypeError):
        _lib.check(rc)
    # block not divisible by 16 for bf16 -> RuntimeError class (reference: ValueError at construction)
    rc = lib.slr_bsr_addmm_inplace(None, None, 4, 32, None, 2, None, None, 0, 8, 16, None, 1, _lib.SLR_BF16, None)
    assert rc == _lib.SLR_ERR_UNSUPPORTED
    # K not divisible by block_q
    rc = lib.slr_bsr_addmm_inplace(None, None, 4, 33, None, 2, None, None, 0, 16, 16, None, 1, _lib.SLR_BF16, None)
    assert rc == _lib.SLR_ERR_INVALID_ARGUMENT
    assert "divisible" in _lib.last_error()
    # null pointers with work to do
    rc = lib.slr_bsr_addmm_inplace(None, None, 4, 32, None, 2, None, None, 1, 16, 16, None, 1, _lib.SLR_BF16, None)
    assert rc == _lib.SLR_ERR_INVALID_ARGUMENT
    # nothing to do: OK without touching the device
    rc = lib.slr_bsr_addmm_inplace(None, None, 0, 32, None, 2, None, None, 0, 16, 16, None, 0, _lib.SLR_BF16, None)
    assert rc == _lib.SLR_OK


def test_layer_descriptor_validation_needs_no_gpu():
    lib = _lib.load()
    L = _lib.SlrLayer(in_features=64, out_features=64, rank=8, block_p=16, block_q=16, nnz=0, dtype=_lib.SLR_BF16)
    # rank > 0 without A/B
    fwd = lambda x, y, M, ldx=0, ldy=0: lib.slr_lrs_linear_forward(  # noqa: E731
        ctypes.byref(L), x, ldx, y, ldy, M, None, 0, None)
    assert fwd(1, 1, 4) == _lib.SLR_ERR_INVALID_ARGUMENT
    L.A, L.B = 0x1000, 0x2000
    L.flags = 8
    assert fwd(1, 1, 4) == _lib.SLR_ERR_INVALID_ARGUMENT
    L.flags = 0
    L.dtype = 5
    assert fwd(1, 1, 4) == _lib.SLR_ERR_UNSUPPORTED_DTYPE
    L.dtype = _lib.SLR_BF16
    # workspace is required for rank > 0
    need = lib.slr_lrs_linear_workspace_size(ctypes.byref(L), 4)
    assert need > 0 and need % 256 == 0
    assert fwd(0x100, 0x200, 4) == _lib.SLR_ERR_WORKSPACE
    assert lib.slr_lrs_linear_lowrank(ctypes.byref(L), 0x100, 0, 4, None, 0, None) == _lib.SLR_ERR_WORKSPACE
    # strides below the row length are rejected
    assert fwd(0x100, 0x200, 4, ldx=32) == _lib.SLR_ERR_INVALID_ARGUMENT
    # M == 0 is a no-op
    assert fwd(0x100, 0x200, 0) == _lib.SLR_OK


def test_stage_schedule_matches_a_python_merge():
    for bp, bq, dens, seed in [(32, 32, 0.3, 1), (16, 16, 0.05, 2), (64, 64, 0.5, 3)]:
        crow, col = workloads.bernoulli_structure(1024 // bp, 2048 // bq, dens, seed)
        crow, col = crow.astype(np.int32), col.astype(np.int32)
        order = ops.plan_row_order(crow)
        words, starts = ops.plan_stages(crow, col, bp, order)
        G = 256 // bp
        NB = crow.shape[0] - 1
        recs, blks = [], []
        for gi in range((NB + G - 1) // G):
            assert starts[gi] == len(recs)
            rows = [int(order[r]) for r in range(gi * G, min(NB, gi * G + G))]
            ptr = [int(crow[r]) for r in rows]
            end = [int(crow[r + 1]) for r in rows]
            while any(p < e for p, e in zip(ptr, end)):
                c = min(int(col[p]) for p, e in zip(ptr, end) if p < e)
                mask, first = 0, len(blks)
                for j in range(len(rows)):
                    if ptr[j] < end[j] and int(col[ptr[j]]) == c:
                        mask |= 1 << j
                        blks.append(ptr[j])
                        ptr[j] += 1
                recs.append((c | (mask << 16), first))
        n = len(recs)
        assert starts[-1] == n
        got = words.tolist()
        assert got[2 * n:] == blks
        assert [(got[2 * i], got[2 * i + 1] - 2 * n) for i in range(n)] == recs
        # every block appears exactly once
        assert sorted(blks) == list(range(int(crow[-1])))
    # no tensor-core schedule for other block heights
    assert ops.plan_stages(np.array([0, 1], np.int32), np.array([0], np.int32), 8) is None


def test_group_call_validation_needs_no_gpu():
    lib = _lib.load()
    arr = (_lib.SlrLayer * 5)()
    for i in range(5):
        arr[i] = _lib.SlrLayer(in_features=64, out_features=64, rank=64, block_p=16, block_q=16, nnz=0,
                               A=0x1000, B=0x2000, dtype=_lib.SLR_BF16)
    ys = (ctypes.c_void_p * 5)(*([0x3000] * 5))
    grp = lambda n, M=4: lib.slr_lrs_linear_forward_group(arr, n, 0x100, 0, ys, None, M, None, 0, None)  # noqa: E731
    # size: the larger of H [M, 64 + 64] (grouped call) and one workspace per layer (fallback)
    one = lib.slr_lrs_linear_workspace_size(ctypes.byref(arr[0]), 4)
    two = lib.slr_lrs_linear_group_workspace_size(arr, 2, 4)
    assert two == max(2 * one, 256) and two % 256 == 0
    big = lib.slr_lrs_linear_group_workspace_size(arr, 2, 4096)
    assert big >= 4096 * 128 * 2
    assert grp(2) == _lib.SLR_ERR_WORKSPACE
    assert grp(0) == _lib.SLR_ERR_INVALID_ARGUMENT
    assert grp(5) == _lib.SLR_ERR_INVALID_ARGUMENT
    assert lib.slr_lrs_linear_group_workspace_size(arr, 5, 4) == 0
    arr[1].in_features = 128  # layers of a group read one x
    assert grp(2) == _lib.SLR_ERR_INVALID_ARGUMENT
    assert "in_features" in _lib.last_error()
    arr[1].in_features = 64
    arr[1].dtype = _lib.SLR_F16
    assert grp(2) == _lib.SLR_ERR_INVALID_ARGUMENT
    arr[1].dtype = _lib.SLR_BF16
    assert grp(2, M=0) == _lib.SLR_OK


def test_dense_to_bsr_shape_error_text_matches_reference():
    lib = _lib.load()
    rc = lib.slr_dense_to_bsr_mask(None, 30, 32, 16, 16, _lib.SLR_F32, None, None, None)
    assert rc == _lib.SLR_ERR_INVALID_ARGUMENT
    assert "not divisible by block (16, 16)" in _lib.last_error()


def test_row_order_is_heaviest_first_and_stable():
    crow = np.array([0, 2, 2, 7, 8, 11, 13], dtype=np.int32)  # counts 2,0,5,1,3,2
    order = ops.plan_row_order(crow)
    assert order.tolist() == [2, 4, 0, 5, 3, 1]


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_are_contiguous_and_balanced(world):
    spec = workloads.layer_set("cfg4")[0]
    crow = spec.crow.astype(np.int32)
    b = ops.plan_shards(crow, 64, 64, 512, world)
    assert b[0] == 0 and b[-1] == spec.nb and np.all(np.diff(b) >= 0)
    cost = np.diff(crow) * 64 * 64 + 64 * 512
    parts = np.array([cost[b[p]:b[p + 1]].sum() for p in range(world)])
    # no shard exceeds the ideal share by more than one (the heaviest) row
    assert parts.max() <= cost.sum() / world + cost.max()


def test_zipf_generator_properties():
    rng = np.random.Generator(np.random.PCG64(3))
    counts = workloads.zipf_counts(64, 64, 0.2, 1.1, rng)
    assert counts.sum() == round(0.2 * 64 * 64)
    assert counts.max() == 64  # the head is capped at NB_K
    assert counts.min() >= 0
    crow, col = workloads.zipf_structure(172, 64, 0.2, 1.1, 0)
    for i in range(172):
        c = col[crow[i]:crow[i + 1]]
        assert np.all(np.diff(c) > 0) and (c.size == 0 or (c.min() >= 0 and c.max() < 64))


def test_band_generator_density():
    crow, col = workloads.band_structure(512, 512, 32, 0.04, 0.01, 0)
    nnz = col.shape[0]
    assert abs(nnz / (512 * 512) - 0.05) < 0.003
    rows = np.repeat(np.arange(512), np.diff(crow))
    d = col - rows
    band = (d >= -32) & (d < 32)
    assert abs(band.sum() / (512 * 512) - 0.04) < 0.003


def test_generators_are_deterministic():
    a = workloads.layer_set("cfg3", seed=0)
    b = workloads.layer_set("cfg3", seed=0)
    assert [x.structure_digest() for x in a] == [y.structure_digest() for y in b]
    t1 = a[0].tensors("cpu", torch.bfloat16)
    t2 = b[0].tensors("cpu", torch.bfloat16)
    assert torch.equal(t1["A"], t2["A"]) and torch.equal(t1["values_pq"], t2["values_pq"])


def test_layer_api_rejects_cpu_tensors():
    from s_salaad_b200.efficient import LRSLinear

    A, B = torch.randn(64, 8), torch.randn(8, 96)
    S = torch.zeros(64, 96)
    S[:16, 16:32] = 1.0
    with pytest.raises(ValueError, match="CUDA"):
        LRSLinear(A, B, S.to_sparse_bsr(blocksize=(16, 16)), in_features=96, out_features=64, block_p=16,
                  block_q=16)


def test_bundle_round_trip_and_errors(tmp_path):
    """save_artifact / load_artifact keep the reference's bundle format
    (ssalaad/efficient/artifact.py:78-118) and its error messages."""
    from s_salaad_b200.efficient import export_model_config, load_artifact, save_artifact

    model = torch.nn.Sequential(torch.nn.Linear(32, 16), torch.nn.Linear(16, 8))
    S = torch.zeros(16, 32)
    S[:16, 16:32] = 0.5
    layers = {"0": {"A": torch.randn(16, 4), "B": torch.randn(4, 32), "S": S.to_sparse_bsr(blocksize=(16, 16)),
                    "block_p": 16, "block_q": 16}}
    config = {"model_type": "llama", "hidden_size": 32, "run_name": "dropped", "tokenizer_id": str(tmp_path)}
    path = tmp_path / "sub" / "bundle.pt"
    save_artifact(path, layers, {"mode": "x", "step": 3}, model=model, model_config=config)
    p = load_artifact(path)
    assert p["format_version"] == 1 and p["meta"] == {"mode": "x"}
    assert p["model_config"] == {"model_type": "llama", "hidden_size": 32}
    assert set(p["base_state_dict"]) == {"0.bias", "1.weight", "1.bias"}
    assert torch.equal(p["layers"]["0"]["S"].to_dense(), S)
    assert export_model_config({"tokenizer_id": "org/name", "foo": 1}) == {"tokenizer_id": "org/name"}
    torch.save({"format_version": 1}, tmp_path / "partial.pt")
    with pytest.raises(ValueError, match="complete model bundle"):
        load_artifact(tmp_path / "partial.pt")
    torch.save({**p, "format_version": 2}, tmp_path / "v2.pt")
    with pytest.raises(ValueError, match="Unsupported model bundle version"):
        load_artifact(tmp_path / "v2.pt")


def test_efficient_model_requires_cuda(tmp_path):
    from s_salaad_b200.efficient import build_efficient_model

    with pytest.raises(ValueError, match="CUDA"):
        build_efficient_model(tmp_path / "missing.pt", device="cpu")


def test_peer_call_validation_needs_no_gpu():
    """slr_peers arguments are checked before anything touches a GPU."""
    lib = _lib.load()
    L = _lib.SlrLayer(in_features=256, out_features=256, rank=64, block_p=64, block_q=64, nnz=0,
                      A=0x1000, B=0x2000, dtype=_lib.SLR_BF16)
    P = _lib.SlrPeers()
    call = lambda: lib.slr_lrs_linear_combine_peers(ctypes.byref(L), 0x100, 0, 256, 512, None, 0,  # noqa: E731
                                                    ctypes.byref(P), None)
    P.world, P.rank = 1, 0
    assert call() == _lib.SLR_ERR_INVALID_ARGUMENT and "world" in _lib.last_error()
    P.world, P.rank = 2, 2
    assert call() == _lib.SLR_ERR_INVALID_ARGUMENT
    P.rank = 0
    assert call() == _lib.SLR_ERR_INVALID_ARGUMENT and "NULL" in _lib.last_error()
    P.y[0], P.y[1], P.signal[0], P.signal[1] = 0x10000, 0x20008, 0x30000, 0x40000
    assert call() == _lib.SLR_ERR_INVALID_ARGUMENT and "aligned" in _lib.last_error()
    assert lib.slr_peers_wait(None, 0, None) == _lib.SLR_ERR_INVALID_ARGUMENT
    assert lib.slr_lrs_linear_peers_supported(ctypes.byref(L), 0x100, 0, 0) == 0
    h = (ctypes.c_uint8 * _lib.SLR_IPC_HANDLE_BYTES)()
    off = ctypes.c_int64()
    assert lib.slr_ipc_export(None, h, ctypes.byref(off)) == _lib.SLR_ERR_INVALID_ARGUMENT
    assert lib.slr_ipc_release(bytes(_lib.SLR_IPC_HANDLE_BYTES)) == _lib.SLR_ERR_INVALID_ARGUMENT


def test_operators_register_with_shapes_on_meta_tensors():
    """ssalaad::tilelang_bsr_addmm_inplace_dense_ and ssalaad::slr_linear are
    defined with fake (meta) implementations, so tracing needs no GPU."""
    from s_salaad_b200.cuda_sparse import register_reference_op

    register_reference_op()
    x = torch.empty(3, 5, 64, device="meta", dtype=torch.bfloat16)
    A = torch.empty(32, 8, device="meta", dtype=torch.bfloat16)
    B = torch.empty(8, 64, device="meta", dtype=torch.bfloat16)
    y = torch.ops.ssalaad.slr_linear(x, A, B, None, None, None, None, 0, 0)
    assert y.shape == (3, 5, 32) and y.dtype == torch.bfloat16


def test_synthetic_bundle_is_a_loadable_cfg2_model(tmp_path):
    """The cfg2 bundle writer produces a reference-format bundle whose layers
    rebuild the dense weights A·B + S it returns (CPU only; one layer)."""
    from s_salaad_b200 import workloads
    from s_salaad_b200.efficient import load_artifact

    path = tmp_path / "cfg2.pt"
    dense = workloads.compressed_bundle(path, n_layers=1)
    p = load_artifact(path)
    assert set(p["layers"]) == set(dense) and len(dense) == 7
    assert p["model_config"]["num_hidden_layers"] == 1 and p["model_config"]["hidden_size"] == 512
    for name, data in p["layers"].items():
        W = data["A"] @ data["B"] + data["S"].to_dense()
        assert torch.equal(W, dense[name])
        assert (data["block_p"], data["block_q"]) == (16, 16)
    assert not any(k.endswith("q_proj.weight") for k in p["base_state_dict"])
