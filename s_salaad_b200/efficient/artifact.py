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


def _local_tokenizer(name: str) -> bool:
    """A tokenizer given as a file-system path (not portable with a bundle)."""
    path = Path(name)
    return path.is_absolute() or path.exists()


def export_model_config(config: dict) -> dict:
    """The architecture and tokenizer fields of a model configuration; a
    tokenizer given as a local path is dropped (reference
    ssalaad/train/model.py:63-69)."""
    exported = {}
    for key, value in config.items():
        if key not in MODEL_FIELDS:
            continue
        if key == "tokenizer_id" and value and _local_tokenizer(str(value)):
            continue
        exported[key] = value
    return exported


FORMAT_VERSION = 1
# Keys of a bundle (format version 1; the reference's save/load_artifact,
# ssalaad/efficient/artifact.py:78-118) and the meta entries it keeps.
_BUNDLE_KEYS = ("format_version", "layers", "base_state_dict", "model_config", "meta")
_META_KEYS = frozenset({"mode", "param_count", "p_tgt_million"})
_ERR_INCOMPLETE = "Expected a complete model bundle produced by the compression entry point."
_ERR_VERSION = "Unsupported model bundle version."


class _Bundle:
    """One compressed model on disk: the compressed layers (name -> factors
    and S), every other tensor of the model, its configuration and a few
    meta entries."""

    def __init__(self, layers: dict, base_state: dict, model_config: dict, meta: dict):
        self.layers = layers
        self.base_state = base_state
        self.model_config = model_config
        self.meta = meta

    @classmethod
    def from_model(cls, model: torch.nn.Module, layers: dict, meta: dict, model_config: dict) -> "_Bundle":
        # the weights of the compressed modules live in `layers`, not in the base state
        replaced = {f"{name}.weight" for name in layers}
        base = {}
        for key, tensor in model.state_dict().items():
            if key not in replaced:
                base[key] = tensor.detach().to("cpu", copy=True)
        kept_meta = {k: v for k, v in meta.items() if k in _META_KEYS}
        return cls(layers, base, export_model_config(model_config), kept_meta)

    def to_payload(self) -> dict:
        return dict(zip(_BUNDLE_KEYS, (FORMAT_VERSION, self.layers, self.base_state, self.model_config,
                                       self.meta)))

    @staticmethod
    def check_payload(payload: Any) -> dict:
        if not isinstance(payload, dict) or any(k not in payload for k in _BUNDLE_KEYS):
            raise ValueError(_ERR_INCOMPLETE)
        if payload["format_version"] != FORMAT_VERSION:
            raise ValueError(_ERR_VERSION)
        return payload


def save_artifact(path: str | Path, layers: dict[str, dict[str, Any]], meta: dict[str, Any], *,
                  model: torch.nn.Module, model_config: dict) -> None:
    """Write compressed layers and every remaining model tensor as one bundle
    in the reference's format (ssalaad/efficient/artifact.py:78-105)."""
    target = Path(path)
    target.parent.mkdir(parents=True, exist_ok=True)
    torch.save(_Bundle.from_model(model, layers, meta, model_config).to_payload(), target)


def load_artifact(path: str | Path) -> dict[str, Any]:
    """Read a bundle; anything but a complete version-1 bundle raises
    ValueError with the reference's messages (ssalaad/efficient/artifact.py:108-118)."""
    return _Bundle.check_payload(torch.load(path, map_location="cpu", weights_only=True))


def module_buffers(S: torch.Tensor, block_p: int, block_q: int):
    """The layer buffers of ls_linear.py:86-97 straight from dense S:
    int32 crow/col, values ``[nnz, bq, bp]``, int32 active rows."""
    crow, col, values = ops.dense_to_bsr_cuda(S, int(block_p), int(block_q), transpose=True)
    active = (crow[1:] - crow[:-1]).nonzero(as_tuple=False).squeeze(-1)
    return crow.to(torch.int32), col.to(torch.int32), values, active.to(torch.int32)
