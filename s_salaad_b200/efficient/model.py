"""A compressed model with the B200 layers swapped in.

The counterpart of ``build_efficient_model`` (``ssalaad/efficient/model.py:11-63``)
and of the model factory it uses (``ssalaad/train/model.py:14-17, 78-94``): the
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


# Architectures a bundle may name (reference ssalaad/train/model.py:14-17).
_ARCHITECTURES = {"llama": "LlamaForCausalLM", "qwen3": "Qwen3ForCausalLM"}


def _config_kwargs(config: dict, attn_implementation: str | None, overrides: dict) -> dict:
    """Keyword arguments of the Hugging Face configuration class for a
    bundle's model configuration: the recipe name max_sequence_length stands
    for max_position_embeddings (unless that is given too), a pad id of -1
    means none, the model is built without a KV cache, and non-None
    overrides win."""
    has_positions = "max_position_embeddings" in config
    kwargs = {}
    for key, value in config.items():
        if key == "max_sequence_length" and not has_positions:
            key = "max_position_embeddings"
        if key == "pad_token_id" and value == -1:
            value = None
        kwargs[key] = value
    kwargs["use_cache"] = False
    if attn_implementation is not None:
        kwargs["attn_implementation"] = attn_implementation
    kwargs.update((k, v) for k, v in overrides.items() if v is not None)
    return kwargs


def build_model_from_config(config: dict, *, attn_implementation: str | None = None, **overrides) -> nn.Module:
    """A randomly initialised model of the configured architecture (the
    reference's factory, ssalaad/train/model.py:78-94: same arguments and
    ValueError for an unknown model type)."""
    import transformers

    kwargs = _config_kwargs(config, attn_implementation, overrides)
    model_type = kwargs.pop("model_type", "llama")
    if model_type not in _ARCHITECTURES:
        raise ValueError(f"Unsupported model type: {model_type}")
    hf_config = transformers.AutoConfig.for_model(model_type, **kwargs)
    return getattr(transformers, _ARCHITECTURES[model_type])(hf_config)


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
        # inference tensors keep no version counter; there the storage, shape
        # and the pending outputs being taken in member order identify the call
        version = -1 if x.is_inference() else x._version
        key = (x.data_ptr(), version, tuple(x.shape), x.dtype, x.device)
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


# Error texts of the reference loader (ssalaad/efficient/model.py:11-63), kept
# because callers match on them.
_ERR_WEIGHTS = "The bundle does not contain exactly the required model weights."


def _check_weight_coverage(model: nn.Module, base_state: dict, layers: dict) -> None:
    """The bundle's base tensors plus the compressed layers' weights must be
    exactly the model's state, each tensor from one place."""
    compressed = {f"{name}.weight" for name in layers}
    base = set(base_state)
    if set(model.state_dict()) != base | compressed or base & compressed:
        raise ValueError(_ERR_WEIGHTS)


def _dense_weight(module: nn.Module, data: dict) -> torch.Tensor | None:
    """The dense weight a compressed entry stands for when it is not served
    by an S+LR layer: an explicit W, or A·B + S materialised for an
    embedding; None for a linear layer (it becomes an LRSLinear)."""
    if "W" in data:
        return data["W"]
    if isinstance(module, nn.Embedding):
        return data["A"].float() @ data["B"].float() + data["S"].to_dense().float()
    return None


def _slr_layer(module: nn.Linear, data: dict, device, dtype) -> nn.Module:
    """The B200 S+LR layer replacing a compressed nn.Linear."""
    on = dict(device=device, dtype=dtype)
    bias = None if module.bias is None else module.bias.detach().to(**on)
    shape = {k: data.get(k) for k in ("block_p", "block_q", "nm_n", "nm_m")}
    return LRSLinear(data["A"].to(**on), data["B"].to(**on), data["S"].to(**on), in_features=module.in_features,
                     out_features=module.out_features, bias=bias, **shape)


def build_efficient_model(path, *, device="cuda", dtype=None, group: bool = True):
    """Load a complete compressed model (the reference's
    ssalaad/efficient/model.py:11-63: same bundle, return value
    (model, model_config, meta) and errors) onto a CUDA device with the B200
    kernels.  The loader first checks that the bundle covers the model
    exactly and that every compressed entry is a linear or embedding module,
    then loads the base tensors and installs each entry: an S+LR layer for a
    linear module, a dense weight for an explicit W or an embedding."""
    device = torch.device(device)
    if device.type != "cuda":
        raise ValueError("s_salaad_b200 runs compressed models on CUDA devices only.")
    dtype = dtype or torch.bfloat16
    bundle = load_artifact(path)
    model = build_model_from_config(bundle["model_config"], attn_implementation="sdpa")
    compressed = bundle["layers"]
    _check_weight_coverage(model, bundle["base_state_dict"], compressed)
    targets = {}
    for name in compressed:
        module = model.get_submodule(name)
        if not isinstance(module, (nn.Linear, nn.Embedding)):
            raise TypeError(f"Unsupported compressed module: {name}")
        targets[name] = module
    model.load_state_dict(bundle["base_state_dict"], strict=False)
    model.to(dtype=dtype)
    for name, module in targets.items():
        data = compressed[name]
        weight = _dense_weight(module, data)
        if weight is None:
            owner, _, attr = name.rpartition(".")
            setattr(model.get_submodule(owner) if owner else model, attr, _slr_layer(module, data, device, dtype))
        elif tuple(weight.shape) != tuple(module.weight.shape):
            raise ValueError(f"Weight shape mismatch: {name}")
        else:
            with torch.no_grad():
                module.weight.copy_(weight.to(dtype=dtype))
    model = model.to(device=device).eval()
    if group:
        group_projections(model)
    return model, bundle["model_config"], bundle["meta"]
