"""Generate the golden vectors in tests/golden/ by running the S-SALAAD
reference itself (CPU parts) on seeded inputs.

Run where the reference sources exist (read-only); ``--ref`` gives the root
directory of the reference project:

    python tests/golden/make_golden.py --ref DIR

What is run, all from the reference, unmodified:
  * ``ssalaad.cpu_sparse.bsr_addmm_avx2_`` (its AVX2 kernel, built by the
    reference's own loader on first import),
  * ``ssalaad.efficient.artifact.dense_to_bsr``,
  * ``ssalaad.efficient.ls_linear._LRSLinearLRBlockCPU`` / ``LRSLinear``.

Small cases store inputs and outputs.  The cfg1-sized cases store only the
outputs plus a SHA-256 of the inputs, which the tests regenerate from the
same seeds with s_salaad_b200.workloads and check against the digest before
comparing.  The GPU box never runs this script (the reference is absent there).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from s_salaad_b200 import workloads  # noqa: E402


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = a.detach().cpu().contiguous() if hasattr(a, "detach") else np.ascontiguousarray(a)
        if hasattr(a, "numpy"):
            if a.dtype == torch.bfloat16:
                a = a.view(torch.int16)
            a = a.numpy()
        h.update(a.tobytes())
    return h.hexdigest()


def block_sparse(n, m, block, coords, seed=0):
    """Same construction as the reference test helper (tests/test_ssalaad.py:307-317
    builds S this way): standard-normal blocks at the given block coordinates."""
    g = torch.Generator().manual_seed(seed)
    S = torch.zeros(n, m)
    for br, bc in coords:
        S[br * block:(br + 1) * block, bc * block:(bc + 1) * block] = torch.randn(block, block, generator=g)
    return S


def layer_buffers(S, bp, bq):
    bsr = S.to_sparse_bsr(blocksize=(bp, bq))
    crow = bsr.crow_indices().to(torch.int32)
    return (crow, bsr.col_indices().to(torch.int32), bsr.values().transpose(1, 2).contiguous(),
            (crow[1:] - crow[:-1]).nonzero().squeeze(-1).to(torch.int32))


def t2n(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root directory of the S-SALAAD reference project")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from ssalaad.cpu_sparse import SUPPORTED_BLOCK_SIZES, bsr_addmm_avx2_
    from ssalaad.efficient.artifact import dense_to_bsr
    from ssalaad.efficient.ls_linear import LRSLinear, _LRSLinearLRBlockCPU

    torch.set_num_threads(1)  # fixes the MKL summation order of the LR step
    manifest = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__,
                "numpy": np.__version__, "cases": {}}

    # 1. AVX2 kernel vs the reference test's own construction, blocks 8/16/32/64,
    #    from zero and from a nonzero `out` (pins in-place accumulation).
    for block in SUPPORTED_BLOCK_SIZES:
        S = block_sparse(block * 4, block * 6, block, [(0, 1), (1, 0), (1, 3), (2, 5), (3, 2)], seed=block)
        g = torch.Generator().manual_seed(100 + block)
        x = torch.randn(5, block * 6, generator=g)
        out0 = torch.randn(5, block * 4, generator=g)
        crow, col, vals, active = layer_buffers(S, block, block)
        out_zero = torch.zeros(5, block * 4)
        bsr_addmm_avx2_(out_zero, x.contiguous(), crow, col, vals, active)
        out_acc = out0.clone()
        bsr_addmm_avx2_(out_acc, x.contiguous(), crow, col, vals, active)
        name = f"avx2_block{block}"
        np.savez_compressed(HERE / f"{name}.npz", x=t2n(x), out0=t2n(out0), crow=t2n(crow), col=t2n(col),
                            values=t2n(vals), active_rows=t2n(active), out_zero=t2n(out_zero),
                            out_acc=t2n(out_acc), dense_S=t2n(S))
        manifest["cases"][name] = "reference bsr_addmm_avx2_; out_zero from zeros, out_acc from out0"

    # 2. Empty block-rows stay untouched (reference test :330-337 construction).
    block = 16
    S = block_sparse(block * 3, block * 3, block, [(2, 0)], seed=7)
    x = torch.randn(3, block * 3, generator=torch.Generator().manual_seed(8))
    out = torch.full((3, block * 3), 7.0)
    crow, col, vals, active = layer_buffers(S, block, block)
    bsr_addmm_avx2_(out, x.contiguous(), crow, col, vals, active)
    np.savez_compressed(HERE / "avx2_empty_rows.npz", x=t2n(x), crow=t2n(crow), col=t2n(col), values=t2n(vals),
                        active_rows=t2n(active), out=t2n(out))
    manifest["cases"]["avx2_empty_rows"] = "reference bsr_addmm_avx2_ with out=7.0 and two empty block-rows"

    # 3. dense_to_bsr: patterns incl. -0.0, NaN, inf, subnormal blocks; fp32 and bf16;
    #    square and rectangular blocks.
    d2b = {}
    g = torch.Generator().manual_seed(11)
    for dt_name, dt in (("f32", torch.float32), ("bf16", torch.bfloat16)):
        for (bp, bq) in ((16, 16), (8, 16), (32, 32), (16, 8)):
            n, m = 4 * bp, 6 * bq
            S = torch.randn(n, m, generator=g)
            keep = torch.rand(n // bp, m // bq, generator=g) < 0.5
            S = S * keep.repeat_interleave(bp, 0).repeat_interleave(bq, 1)
            # special blocks (block-row, block-col) -> content
            S[0:bp, 0:bq] = -0.0                              # all negative zero: dropped
            S[bp:2 * bp, 0:bq] = 0.0
            S[bp + 1, 1] = float("nan")                       # NaN block: dropped
            S[bp + 2, 2] = 1.0
            S[2 * bp:3 * bp, bq:2 * bq] = 0.0
            S[2 * bp, bq] = float("inf")                      # inf: kept
            S[3 * bp:4 * bp, 2 * bq:3 * bq] = 0.0
            S[3 * bp + 1, 2 * bq + 3] = 1e-40 if dt == torch.float32 else 1e-39  # subnormal: kept
            Sd = S.to(dt)
            ref = dense_to_bsr(Sd, bp, bq)
            key = f"d2b_{dt_name}_{bp}x{bq}"
            d2b[key] = dict(S=t2n(Sd), crow=t2n(ref.crow_indices()), col=t2n(ref.col_indices()),
                            values=t2n(ref.values()))
    # all-zero and all-live matrices
    Z = torch.zeros(32, 48)
    ref = dense_to_bsr(Z, 16, 16)
    d2b["d2b_f32_zero"] = dict(S=t2n(Z), crow=t2n(ref.crow_indices()), col=t2n(ref.col_indices()),
                               values=t2n(ref.values()))
    F = torch.randn(32, 48, generator=g)
    ref = dense_to_bsr(F, 16, 16)
    d2b["d2b_f32_full"] = dict(S=t2n(F), crow=t2n(ref.crow_indices()), col=t2n(ref.col_indices()),
                               values=t2n(ref.values()))
    np.savez_compressed(HERE / "dense_to_bsr.npz", **{f"{k}__{f}": v for k, d in d2b.items() for f, v in d.items()})
    manifest["cases"]["dense_to_bsr"] = sorted(d2b)

    # 4. cfg1-shaped layer through the reference CPU layer, T = 32 sampled tokens.
    spec = workloads.cfg1_layer(0)
    t = spec.tensors("cpu", torch.float32)
    x = workloads.tokens(32, spec.in_features, seed=5)
    S = spec.dense_S(t)
    layer = LRSLinear(t["A"], t["B"], dense_to_bsr(S, 16, 16), in_features=spec.in_features,
                      out_features=spec.out_features, bias=t["bias"], block_p=16, block_q=16)
    assert isinstance(layer, _LRSLinearLRBlockCPU)
    with torch.no_grad():
        y = layer(x)
    np.savez_compressed(HERE / "lrs_cfg1_T32.npz", y=t2n(y),
                        inputs_sha256=np.array(digest(t["A"], t["B"], t["bias"], t["values_pq"], spec.crow, spec.col, x)))
    manifest["cases"]["lrs_cfg1_T32"] = "reference _LRSLinearLRBlockCPU on cfg1 (seed 0), x = tokens(32, 512, seed=5)"

    # 5. bf16-valued weights, 32x32 blocks, evaluated by the fp32 CPU reference
    #    (the bf16 oracle: fp32 CPU path on fp32 copies of bf16 tensors).
    crow, col = workloads.bernoulli_structure(256 // 32, 512 // 32, 0.3, seed=21)
    spec = workloads.LayerSpec("b32", 256, 512, 64, 32, 32, crow, col, seed=22)
    t = spec.tensors("cpu", torch.bfloat16)
    x = workloads.tokens(16, 512, seed=23, dtype=torch.bfloat16)
    S = spec.dense_S(t).float()
    layer = LRSLinear(t["A"].float(), t["B"].float(), dense_to_bsr(S, 32, 32), in_features=512,
                      out_features=256, bias=None, block_p=32, block_q=32)
    with torch.no_grad():
        y = layer(x.float())
    np.savez_compressed(HERE / "lrs_b32_bf16vals.npz", y=t2n(y),
                        inputs_sha256=np.array(digest(t["A"], t["B"], t["values_pq"], spec.crow, spec.col, x)))
    manifest["cases"]["lrs_b32_bf16vals"] = "reference CPU layer on fp32 copies of bf16 tensors, 32x32 blocks"

    # 6. The reference bundle test's layer (tests/test_ssalaad.py:229-259 shapes):
    #    32x32 q_proj, rank 4, one 16x16 block, bias-free.
    g = torch.Generator().manual_seed(7)
    A, B = torch.randn(32, 4, generator=g) * 0.01, torch.randn(4, 32, generator=g) * 0.01
    S = torch.zeros(32, 32)
    S[:16, :16] = torch.randn(16, 16, generator=g) * 0.01
    x = torch.randn(4, 32, generator=g)
    layer = LRSLinear(A, B, dense_to_bsr(S, 16, 16), in_features=32, out_features=32, block_p=16, block_q=16)
    with torch.no_grad():
        y = layer(x)
    np.savez_compressed(HERE / "lrs_tiny_rank4.npz", A=t2n(A), B=t2n(B), S=t2n(S), x=t2n(x), y=t2n(y))
    manifest["cases"]["lrs_tiny_rank4"] = "reference CPU layer, 32x32, rank 4, one 16x16 block"

    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
