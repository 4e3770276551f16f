"""BSR conversion on the GPU and the compressed-model bundle.

Mirrors ``ssalaad/efficient/artifact.py``:

* ``dense_to_bsr`` (reference :20-37): same name, arguments, ValueError text
  and result (a ``torch.sparse_bsr_tensor`` with int64 crow/col and blocks in
  row-major order), computed by the libslr_b200 kernels on the GPU (a CPU
  tensor is converted on the current CUDA device and the result returned on
  the CPU), bit-exact with the reference.
* ``encode_s_for_artifact``, ``save_artifact``, ``load_artifact`` (reference
  :64-118): the same bundle format (``format_version`` 1: ``layers``,
  ``base_state_dict``, ``model_config``, ``meta``), so bundles written by
  either side load in the other.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any

import torch

from .. import ops

# Fields of a model configuration kept in a bundle (the architecture and
# tokenizer, not the run that produced it); reference ssalaad/train/model.py:18-45.
MODEL_FIELDS = frozenset({
    "model_type", "architectures", "hidden_size", "intermediate_size", "hidden_act", "num_hidden_layers",
    "num_attention_heads", "num_key_value_heads", "head_dim", "vocab_size", "max_sequence_length",
    "max_position_embeddings", "rms_norm_eps", "rope_theta", "rope_scaling", "rope_parameters",
    "initializer_range", "tie_word_embeddings", "attention_bias", "attention_dropout", "mlp_bias",
    "bos_token_id", "eos_token_id", "pad_token_id", "tokenizer_id", "use_cache",
})


def dense_to_bsr(S: torch.Tensor, block_p: int, block_q: int) -> torch.Tensor:
    (n, m) = S.shape
    if n % block_p or m % block_q:
        raise ValueError(f"shape ({n}, {m}) not divisible by block ({block_p}, {block_q})")
    if S.is_cuda:
        crow, col, values = ops.dense_to_bsr_cuda(S, int(block_p), int(block_q))
        return torch.sparse_bsr_tensor(crow, col, values, size=(n, m))
    if not torch.cuda.is_available():
        raise RuntimeError("s_salaad_b200.dense_to_bsr runs on the GPU; no CUDA device is available.")
    crow, col, values = ops.dense_to_bsr_cuda(S.cuda(), int(block_p), int(block_q))
    return torch.sparse_bsr_tensor(crow.cpu(), col.cpu(), values.cpu(), size=(n, m))


def encode_s_for_artifact(S: torch.Tensor, *, block_p: int | None = None, block_q: int | None = None,
                          nm_n: int | None = None, nm_m: int | None = None) -> torch.Tensor:
    """S as a bundle stores it (reference artifact.py:64-75): BSR for a block
    shape other than 1×1, CSR for element-wise and N:M sparsity."""
    if block_p is not None and block_q is not None and (block_p, block_q) != (1, 1):
        return dense_to_bsr(S, int(block_p), int(block_q))
    return S.to_sparse_csr()


def export_model_config(config: dict) -> dict:
    """The architecture and tokenizer fields of a model configuration; a
    tokenizer given as a local path is dropped (reference ssalaad/train/model.py:63-69)."""
    result = {key: value for key, value in config.items() if key in MODEL_FIELDS}
    tokenizer = result.get("tokenizer_id", "")
    if tokenizer and (Path(tokenizer).is_absolute() or Path(tokenizer).exists()):
        result.pop("tokenizer_id")
    return result


def save_artifact(path: str | Path, layers: dict[str, dict[str, Any]], meta: dict[str, Any], *,
                  model: torch.nn.Module, model_config: dict) -> None:
    """Write compressed layers and every remaining model tensor as one bundle
    (reference artifact.py:78-105)."""
    allowed_meta = {"mode", "param_count", "p_tgt_million"}
    compressed_keys = {name + ".weight" for name in layers}
    base_state = {key: tensor.detach().cpu().clone() for key, tensor in model.state_dict().items()
                  if key not in compressed_keys}
    payload = {
        "format_version": 1,
        "layers": layers,
        "base_state_dict": base_state,
        "model_config": export_model_config(model_config),
        "meta": {key: value for key, value in meta.items() if key in allowed_meta},
    }
    destination = Path(path)
    destination.parent.mkdir(parents=True, exist_ok=True)
    torch.save(payload, destination)


def load_artifact(path: str | Path) -> dict[str, Any]:
    """Read a bundle; anything but a complete version-1 bundle raises
    ValueError with the reference's messages (reference artifact.py:108-118)."""
    payload = torch.load(path, map_location="cpu", weights_only=True)
    required = {"format_version", "layers", "base_state_dict", "model_config", "meta"}
    if not isinstance(payload, dict) or not required.issubset(payload):
        raise ValueError("Expected a complete model bundle produced by the compression entry point.")
    if payload["format_version"] != 1:
        raise ValueError("Unsupported model bundle version.")
    return payload


def module_buffers(S: torch.Tensor, block_p: int, block_q: int):
    """The layer buffers of ls_linear.py:86-97 straight from dense S:
    int32 crow/col, values ``[nnz, bq, bp]``, int32 active rows."""
    crow, col, values = ops.dense_to_bsr_cuda(S, int(block_p), int(block_q), transpose=True)
    active = (crow[1:] - crow[:-1]).nonzero(as_tuple=False).squeeze(-1)
    return crow.to(torch.int32), col.to(torch.int32), values, active.to(torch.int32)
