"""A compressed model with the B200 layers swapped in.

Mirrors ``build_efficient_model`` (``ssalaad/efficient/model.py:11-63``) and
the model factory it uses (``ssalaad/train/model.py:14-17, 78-94``): the
bundle's base weights are loaded into a Hugging Face model built from its
configuration, and every compressed projection becomes an
:func:`~s_salaad_b200.efficient.LRSLinear`.  Same arguments, return value
``(model, model_config, meta)`` and errors; CUDA only (the reference's CPU
path stays the reference's).

On top of the reference, :func:`group_projections` (on by default) makes the
projections that read one input -- q/k/v of an attention block, gate/up of an
MLP -- one grouped call of the library (their ``x·Bᵀ`` products are one
launch); the outputs are bit-identical to separate calls.
"""
from __future__ import annotations

import torch
from torch import nn

from .. import ops
from .artifact import load_artifact
from .ls_linear import LRSLinear, _LRSLinearBase


def _model_classes() -> dict:
    from transformers import LlamaConfig, LlamaForCausalLM, Qwen3Config, Qwen3ForCausalLM

    return {"llama": (LlamaConfig, LlamaForCausalLM), "qwen3": (Qwen3Config, Qwen3ForCausalLM)}


def build_model_from_config(config: dict, *, attn_implementation: str | None = None, **overrides) -> nn.Module:
    """A randomly initialised model of the configured architecture
    (reference ssalaad/train/model.py:78-94)."""
    config = dict(config)
    if "max_sequence_length" in config and "max_position_embeddings" not in config:
        config["max_position_embeddings"] = config.pop("max_sequence_length")
    if config.get("pad_token_id") == -1:
        config["pad_token_id"] = None
    config["use_cache"] = False
    if attn_implementation is not None:
        config["attn_implementation"] = attn_implementation
    config.update({key: value for key, value in overrides.items() if value is not None})
    classes = _model_classes()
    model_type = config.get("model_type", "llama")
    if model_type not in classes:
        raise ValueError(f"Unsupported model type: {model_type}")
    config_cls, model_cls = classes[model_type]
    return model_cls(config_cls(**config))


class _ProjectionGroup:
    """Layers that read one input, computed together on the first call.

    The first member called with an input runs the grouped forward of all
    members; the others' outputs wait for their own call with the same tensor
    (same storage, version, shape), so a forward that calls q, k and v on one
    hidden state launches one ``x·Bᵀ`` GEMM (and, below 128 tokens, one
    combine) for the three.
    """

    def __init__(self, members: list[_LRSLinearBase]):
        self.members = members
        self._group: ops.LayerGroup | None = None
        self._keys: tuple | None = None
        self._pending: list[torch.Tensor | None] = [None] * len(members)
        self._input_key: tuple | None = None

    def _layer_group(self) -> ops.LayerGroup:
        descs = [m._layer_desc() for m in self.members]
        keys = tuple(d.key for d in descs)
        if self._group is None or self._keys != keys:
            self._group = ops.LayerGroup(descs)
            self._keys = keys
        return self._group

    def output(self, i: int, x: torch.Tensor) -> torch.Tensor:
        key = (x.data_ptr(), x._version, tuple(x.shape), x.dtype, x.device)
        if self._input_key == key and self._pending[i] is not None:
            y, self._pending[i] = self._pending[i], None
            return y
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        outs = self._layer_group().forward(x2)
        ys = [o.reshape(*x.shape[:-1], m.out_features) for o, m in zip(outs, self.members)]
        self._pending = [None if j == i else y for j, y in enumerate(ys)]
        self._input_key = key
        return ys[i]


_GROUPS = (("self_attn", ("q_proj", "k_proj", "v_proj")), ("mlp", ("gate_proj", "up_proj")))


def group_projections(model: nn.Module) -> int:
    """Link the q/k/v and gate/up projections of every decoder layer whose
    members are all B200 S+LR layers with one input width and dtype; returns
    the number of groups formed."""
    count = 0
    for module in model.modules():
        for block_name, names in _GROUPS:
            block = getattr(module, block_name, None)
            if block is None:
                continue
            members = [getattr(block, n, None) for n in names]
            if not all(isinstance(m, _LRSLinearBase) for m in members):
                continue
            if len({m.in_features for m in members}) != 1 or len({m.A.dtype for m in members}) != 1:
                continue
            group = _ProjectionGroup(members)
            for i, m in enumerate(members):
                m._group, m._group_index = group, i
            count += 1
    return count


def build_efficient_model(path, *, device="cuda", dtype=None, group: bool = True):
    """Load a complete compressed model (reference efficient/model.py:11-63)
    onto a CUDA device with the B200 kernels; returns (model, model_config, meta)."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("s_salaad_b200 runs compressed models on CUDA devices only.")
    dtype = dtype or torch.bfloat16
    payload = load_artifact(path)
    model = build_model_from_config(payload["model_config"], attn_implementation="sdpa")
    layers = payload["layers"]
    missing, unexpected = model.load_state_dict(payload["base_state_dict"], strict=False)
    expected = {name + ".weight" for name in layers}
    if set(missing) != expected or unexpected:
        raise ValueError("The bundle does not contain exactly the required model weights.")
    model.to(dtype=dtype)
    for name, data in layers.items():
        old = model.get_submodule(name)
        if not isinstance(old, (nn.Linear, nn.Embedding)):
            raise TypeError(f"Unsupported compressed module: {name}")
        if "W" in data:
            weight = data["W"]
        elif isinstance(old, nn.Embedding):
            weight = data["A"].float() @ data["B"].float() + data["S"].to_dense().float()
        else:
            new = LRSLinear(
                data["A"].to(device=device, dtype=dtype),
                data["B"].to(device=device, dtype=dtype),
                data["S"].to(device=device, dtype=dtype),
                in_features=old.in_features,
                out_features=old.out_features,
                bias=old.bias.detach().to(device=device, dtype=dtype) if old.bias is not None else None,
                block_p=data.get("block_p"),
                block_q=data.get("block_q"),
                nm_n=data.get("nm_n"),
                nm_m=data.get("nm_m"),
            )
            parent_name, _, attr = name.rpartition(".")
            parent = model.get_submodule(parent_name) if parent_name else model
            setattr(parent, attr, new)
            continue
        if weight.shape != old.weight.shape:
            raise ValueError(f"Weight shape mismatch: {name}")
        with torch.no_grad():
            old.weight.copy_(weight.to(dtype=dtype))
    model = model.to(device=device).eval()
    if group:
        group_projections(model)
    return model, payload["model_config"], payload["meta"]
