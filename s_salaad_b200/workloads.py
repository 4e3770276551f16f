"""Seeded synthetic S+LR layers for the five benchmark configurations.

No public dataset is involved: every input is generated here from a seed.
Block structure (crow/col) comes from numpy's PCG64 generator on the host;
values, factors, bias and activations come from torch generators (CPU for
parity cases, the target device for large benchmark cases).

Configurations (the reference publishes no benchmark; shapes follow LLaMA
projection sizes):

* cfg1  fp32, in=512, out=1376, 16x16 blocks, Bernoulli(0.5) block mask,
        values ~N(0, .02), A/B ~N(0, .02/sqrt(64)), r=64, bias ~N(0, .01),
        x [256, 512] ~N(0, 1).
* cfg2  bf16 LLaMA-60M-shaped model: 8 layers, hidden 512, 8 heads, SwiGLU
        FFN 1376, vocab 32000; all 7 projections per layer S+LR with 16x16
        blocks, Bernoulli(0.5), r=64, everything ~N(0, .02); ids [8, 256].
* cfg3  bf16 LLaMA-1B layer set: q,k,v,o 2048x2048, gate/up 5504x2048,
        down 2048x5504; 32x32 blocks, Bernoulli(0.3), r=256, ~N(0, .02);
        T in {1, 16, 128, 2048, 8192}.
* cfg4  bf16 LLaMA-7B layer set: 4096x4096 x4, 11008x4096 x2, 4096x11008;
        64x64 blocks, 20% of blocks with Zipf(1.1) skew over block-rows, r=512,
        T=4096.
* cfg5  bf16 8192x8192, 16x16 blocks (512x512 grid), r=32: a diagonal band of
        64 block-diagonals (-32 <= j - i < 32) sampled so it holds 4% of all
        blocks, plus off-band blocks at 1% of all blocks; T in {1, 32}.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np
import torch

LLAMA_1B = dict(hidden=2048, ffn=5504)
LLAMA_7B = dict(hidden=4096, ffn=11008)


def projection_shapes(hidden: int, ffn: int) -> list[tuple[str, int, int]]:
    """(name, out_features, in_features) of one LLaMA decoder layer."""
    return [("q_proj", hidden, hidden), ("k_proj", hidden, hidden), ("v_proj", hidden, hidden),
            ("o_proj", hidden, hidden), ("gate_proj", ffn, hidden), ("up_proj", ffn, hidden),
            ("down_proj", hidden, ffn)]


# ------------------------------------------------------------ structure --

def _crow_col_from_mask(mask: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    counts = mask.sum(axis=1).astype(np.int64)
    crow = np.concatenate([np.zeros(1, np.int64), np.cumsum(counts)])
    _, cols = np.nonzero(mask)
    return crow, cols.astype(np.int64)


def bernoulli_structure(nb: int, nbk: int, density: float, seed: int):
    rng = np.random.Generator(np.random.PCG64(seed))
    mask = rng.random((nb, nbk)) < density
    return _crow_col_from_mask(mask)


def zipf_counts(nb: int, nbk: int, density: float, s: float, rng) -> np.ndarray:
    """Blocks per block-row ∝ 1/rank^s over a random permutation of the rows,
    `density` of all blocks in total, each row capped at nbk (the excess is
    redistributed proportionally over uncapped rows until everything fits),
    rounded by largest remainder."""
    total = int(round(density * nb * nbk))
    ranks = np.empty(nb, np.int64)
    ranks[rng.permutation(nb)] = np.arange(1, nb + 1)
    w = 1.0 / ranks.astype(np.float64) ** s
    alloc = np.zeros(nb)
    capped = np.zeros(nb, bool)
    while True:
        free = ~capped
        rem = total - alloc[capped].sum()
        a = w[free] / w[free].sum() * rem
        over = a > nbk
        if not over.any():
            alloc[free] = a
            break
        idx = np.nonzero(free)[0][over]
        alloc[idx] = nbk
        capped[idx] = True
    base = np.floor(alloc).astype(np.int64)
    short = total - int(base.sum())
    frac = alloc - base
    order = np.lexsort((np.arange(nb), -frac))  # largest fraction first, ties by index
    for i in order:
        if short <= 0:
            break
        if base[i] < nbk:
            base[i] += 1
            short -= 1
    return base


def zipf_structure(nb: int, nbk: int, density: float, s: float, seed: int):
    rng = np.random.Generator(np.random.PCG64(seed))
    counts = zipf_counts(nb, nbk, density, s, rng)
    mask = np.zeros((nb, nbk), bool)
    for i in range(nb):
        if counts[i]:
            mask[i, rng.choice(nbk, size=int(counts[i]), replace=False)] = True
    return _crow_col_from_mask(mask)


def band_structure(nb: int, nbk: int, half: int, band_frac: float, off_frac: float, seed: int):
    """Band -half <= j - i < half holding band_frac of all blocks, plus
    off-band Bernoulli blocks holding off_frac of all blocks."""
    rng = np.random.Generator(np.random.PCG64(seed))
    i = np.arange(nb)[:, None]
    j = np.arange(nbk)[None, :]
    band = (j - i >= -half) & (j - i < half)
    n_all = nb * nbk
    p_band = min(1.0, band_frac * n_all / band.sum())
    p_off = min(1.0, off_frac * n_all / (~band).sum())
    u = rng.random((nb, nbk))
    mask = np.where(band, u < p_band, u < p_off)
    return _crow_col_from_mask(mask)


# --------------------------------------------------------------- layers --

@dataclass
class LayerSpec:
    name: str
    out_features: int
    in_features: int
    rank: int
    block_p: int
    block_q: int
    crow: np.ndarray
    col: np.ndarray
    seed: int
    value_std: float = 0.02
    lr_std: float = 0.02
    bias_std: float | None = None
    extra: dict = field(default_factory=dict)

    @property
    def nnz(self) -> int:
        return int(self.col.shape[0])

    @property
    def nb(self) -> int:
        return self.out_features // self.block_p

    def flops_per_token(self) -> int:
        return 2 * (self.nnz * self.block_p * self.block_q + self.rank * (self.out_features + self.in_features))

    def weight_bytes(self, elem: int) -> int:
        """Algorithmic bytes of the weights and indices (values, col, crow,
        active rows, A, B, bias)."""
        active = int(np.count_nonzero(np.diff(self.crow)))
        b = elem * self.nnz * self.block_p * self.block_q + 4 * self.nnz + 4 * (self.nb + 1) + 4 * active
        b += elem * self.rank * (self.out_features + self.in_features)
        if self.bias_std is not None:
            b += elem * self.out_features
        return b

    def tensors(self, device="cpu", dtype=torch.float32) -> dict:
        """Materialise the layer: A [N,r], B [r,K], bias [N] | None,
        values_pq [nnz,bp,bq] (artifact layout), S_values [nnz,bq,bp] (layer
        layout), int32 S_crow/S_col/S_active_rows, int64 crow/col."""
        dev = torch.device(device)
        g = torch.Generator(device=dev).manual_seed(self.seed)
        f = dict(device=dev, dtype=torch.float32, generator=g)
        vals = torch.randn(self.nnz, self.block_p, self.block_q, **f) * self.value_std
        A = torch.randn(self.out_features, self.rank, **f) * self.lr_std
        B = torch.randn(self.rank, self.in_features, **f) * self.lr_std
        bias = torch.randn(self.out_features, **f) * self.bias_std if self.bias_std is not None else None
        crow = torch.from_numpy(self.crow).to(dev)
        col = torch.from_numpy(self.col).to(dev)
        active = torch.from_numpy(np.nonzero(np.diff(self.crow))[0].astype(np.int32)).to(dev)
        out = dict(A=A.to(dtype), B=B.to(dtype), bias=None if bias is None else bias.to(dtype),
                   values_pq=vals.to(dtype), crow=crow, col=col)
        out["S_values"] = out["values_pq"].transpose(1, 2).contiguous()
        out["S_crow"] = crow.to(torch.int32)
        out["S_col"] = col.to(torch.int32)
        out["S_active_rows"] = active
        return out

    def dense_S(self, t: dict) -> torch.Tensor:
        """Dense S [N, K] from materialised tensors (for small cases)."""
        vals = t["values_pq"]
        S = torch.zeros(self.out_features, self.in_features, dtype=vals.dtype, device=vals.device)
        rows = np.repeat(np.arange(self.nb), np.diff(self.crow))
        for p, (i, j) in enumerate(zip(rows, self.col)):
            S[i * self.block_p:(i + 1) * self.block_p, j * self.block_q:(j + 1) * self.block_q] = vals[p]
        return S

    def structure_digest(self) -> str:
        h = hashlib.sha256()
        h.update(np.ascontiguousarray(self.crow, dtype=np.int64).tobytes())
        h.update(np.ascontiguousarray(self.col, dtype=np.int64).tobytes())
        return h.hexdigest()


def tokens(T: int, K: int, seed: int, device="cpu", dtype=torch.float32) -> torch.Tensor:
    g = torch.Generator(device=torch.device(device)).manual_seed(seed)
    return torch.randn(T, K, device=device, dtype=torch.float32, generator=g).to(dtype)


def cfg1_layer(seed: int = 0) -> LayerSpec:
    crow, col = bernoulli_structure(1376 // 16, 512 // 16, 0.5, seed)
    return LayerSpec("cfg1", 1376, 512, 64, 16, 16, crow, col, seed + 1000, 0.02, 0.02 / 8.0, 0.01)


def layer_set(cfg: str, seed: int = 0) -> list[LayerSpec]:
    """The projections of one decoder layer for cfg3/cfg4, or the single
    layer of cfg1/cfg5."""
    if cfg == "cfg1":
        return [cfg1_layer(seed)]
    if cfg == "cfg3":
        out = []
        for i, (name, n, k) in enumerate(projection_shapes(**LLAMA_1B)):
            crow, col = bernoulli_structure(n // 32, k // 32, 0.3, seed + i)
            out.append(LayerSpec(name, n, k, 256, 32, 32, crow, col, seed + 1000 + i))
        return out
    if cfg == "cfg4":
        out = []
        for i, (name, n, k) in enumerate(projection_shapes(**LLAMA_7B)):
            crow, col = zipf_structure(n // 64, k // 64, 0.2, 1.1, seed + i)
            out.append(LayerSpec(name, n, k, 512, 64, 64, crow, col, seed + 1000 + i))
        return out
    if cfg == "cfg5":
        crow, col = band_structure(512, 512, 32, 0.04, 0.01, seed)
        return [LayerSpec("band", 8192, 8192, 32, 16, 16, crow, col, seed + 1000)]
    if cfg == "cfg2":
        out = []
        for layer in range(8):
            for i, (name, n, k) in enumerate(projection_shapes(512, 1376)):
                s = seed + 100 * layer + i
                crow, col = bernoulli_structure(n // 16, k // 16, 0.5, s)
                out.append(LayerSpec(f"model.layers.{layer}.{'self_attn' if i < 4 else 'mlp'}.{name}",
                                     n, k, 64, 16, 16, crow, col, s + 1000))
        return out
    raise ValueError(f"unknown config {cfg!r}")


CFG_TOKENS = {"cfg1": [256], "cfg2": [2048], "cfg3": [1, 16, 128, 2048, 8192], "cfg4": [4096], "cfg5": [1, 32]}

LLAMA_60M = {
    "model_type": "llama", "hidden_size": 512, "intermediate_size": 1376, "num_hidden_layers": 8,
    "num_attention_heads": 8, "num_key_value_heads": 8, "vocab_size": 32000,
    "max_position_embeddings": 1024, "rms_norm_eps": 1e-6, "hidden_act": "silu",
    "tie_word_embeddings": False, "bos_token_id": 0, "eos_token_id": 1, "pad_token_id": None,
}


def compressed_bundle(path, *, n_layers: int = 8, seed: int = 0):
    """Write a synthetic cfg2 bundle: a randomly initialised LLaMA-60M-shaped
    model whose 7 × n_layers projections are S+LR (16×16 blocks, 50 % block
    density, rank 64, N(0, 0.02) weights as ``layer_set("cfg2")``), in the
    bundle format of ``save_artifact``.  Returns the dense weights
    ``{name: A·B + S}`` (fp32, CPU) for a reference model."""
    from .efficient.artifact import save_artifact
    from .efficient.model import build_model_from_config

    config = dict(LLAMA_60M, num_hidden_layers=n_layers)
    torch.manual_seed(seed)
    model = build_model_from_config(config, attn_implementation="sdpa")
    layers, dense = {}, {}
    for spec in layer_set("cfg2", seed=seed):
        if int(spec.name.split(".")[2]) >= n_layers:
            continue
        t = spec.tensors("cpu", torch.float32)
        S = torch.sparse_bsr_tensor(t["crow"], t["col"], t["values_pq"],
                                    size=(spec.out_features, spec.in_features))
        layers[spec.name] = {"A": t["A"], "B": t["B"], "S": S, "block_p": spec.block_p, "block_q": spec.block_q}
        dense[spec.name] = t["A"] @ t["B"] + S.to_dense()
    save_artifact(path, layers, {"mode": "synthetic"}, model=model, model_config=config)
    return dense
