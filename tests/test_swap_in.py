"""The B200 layer swapped into the reference's own code, unchanged.

The reference package is imported from ``baseline/_ref`` (a plain
``pip install --target`` of the S-SALAAD project, kept out of the history);
without it these tests skip.  Nothing here reads the reference's source tree.

* CPU: a bundle written by this package loads with the reference's
  ``load_artifact`` and the other way round (format version 1,
  ssalaad/efficient/artifact.py:78-118), and both loaders reject the same
  malformed bundles.
* GPU: the reference's ``build_efficient_model``
  (ssalaad/efficient/model.py:11-63) builds the model with
  - Option B: its ``LRSLinear`` factory routing CUDA layers to the B200
    layer (the two-line change of ls_linear.py:263-266); the logits equal
    this package's loader bit for bit;
  - Option A: its own ``_LRSLinearLRBlockCUDA`` calling the in-place operator
    ``ssalaad::tilelang_bsr_addmm_inplace_dense_``, implemented by the B200
    kernel in a process that never imports the TileLang module; the logits
    match the dense-weight model as closely as a dense bf16 model does.
"""
from __future__ import annotations

import sys

import pytest
import torch

from conftest import REPO
from s_salaad_b200 import workloads

REF_DIR = REPO / "baseline" / "_ref"


@pytest.fixture(scope="module")
def ref():
    """The installed reference package's modules (skips without it)."""
    if not (REF_DIR / "ssalaad").is_dir():
        pytest.skip("reference package not installed in baseline/_ref")
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import ssalaad.efficient.artifact as artifact
    import ssalaad.efficient.ls_linear as ls_linear
    import ssalaad.efficient.model as model

    return {"artifact": artifact, "ls_linear": ls_linear, "model": model}


@pytest.fixture(scope="module")
def bundle(tmp_path_factory):
    path = tmp_path_factory.mktemp("swap") / "cfg2.pt"
    dense = workloads.compressed_bundle(path, n_layers=2)
    return path, dense


def _same_payload(a: dict, b: dict) -> None:
    assert a.keys() == b.keys() and a["format_version"] == b["format_version"] == 1
    assert a["model_config"] == b["model_config"] and a["meta"] == b["meta"]
    assert a["base_state_dict"].keys() == b["base_state_dict"].keys()
    for k, v in a["base_state_dict"].items():
        assert torch.equal(v, b["base_state_dict"][k]), k
    assert a["layers"].keys() == b["layers"].keys()
    for name, data in a["layers"].items():
        other = b["layers"][name]
        assert data.keys() == other.keys()
        for k, v in data.items():
            if isinstance(v, torch.Tensor):
                assert torch.equal(v.to_dense(), other[k].to_dense()), (name, k)
            else:
                assert v == other[k]


def test_bundles_cross_load(ref, bundle, tmp_path):
    from s_salaad_b200.efficient import load_artifact, save_artifact

    path, _ = bundle
    ours = load_artifact(path)
    theirs = ref["artifact"].load_artifact(path)  # written by this package, read by the reference
    _same_payload(ours, theirs)
    # written by the reference from the same model and layers, read by this package
    from s_salaad_b200.efficient import build_model_from_config

    model = build_model_from_config(ours["model_config"])
    model.load_state_dict(ours["base_state_dict"], strict=False)
    meta = {"mode": "synthetic", "not_kept": 1}
    ref["artifact"].save_artifact(tmp_path / "r.pt", ours["layers"], meta, model=model,
                                  model_config={**ours["model_config"], "run_name": "x"})
    save_artifact(tmp_path / "o.pt", ours["layers"], meta, model=model,
                  model_config={**ours["model_config"], "run_name": "x"})
    _same_payload(load_artifact(tmp_path / "r.pt"), ref["artifact"].load_artifact(tmp_path / "o.pt"))


@pytest.mark.parametrize("damage", ["drop_base", "extra_base", "overlap", "version", "partial"])
def test_loaders_reject_the_same_bundles(ref, bundle, tmp_path, damage):
    """Both loaders raise the same error class and text on the same damage
    (this package's checks run before any device work)."""
    from s_salaad_b200.efficient import load_artifact
    from s_salaad_b200.efficient.model import _check_weight_coverage, build_model_from_config

    path, _ = bundle
    p = load_artifact(path)
    base = dict(p["base_state_dict"])
    layers = dict(p["layers"])
    if damage == "drop_base":
        base.pop(next(iter(base)))
    elif damage == "extra_base":
        base["model.not_a_tensor_of_the_model"] = torch.zeros(1)
    elif damage == "overlap":
        name = next(iter(layers))  # a compressed weight also given as a base tensor
        base[name + ".weight"] = torch.zeros(layers[name]["A"].shape[0], layers[name]["B"].shape[1])
    bad = {**p, "base_state_dict": base, "layers": layers}
    if damage == "version":
        bad["format_version"] = 2
    if damage == "partial":
        bad.pop("meta")
    out = tmp_path / "bad.pt"
    torch.save(bad, out)
    with pytest.raises(ValueError) as theirs:
        ref["model"].build_efficient_model(out, device="cpu", dtype=torch.float32)
    with pytest.raises(ValueError) as ours:
        payload = load_artifact(out)
        model = build_model_from_config(payload["model_config"])
        _check_weight_coverage(model, payload["base_state_dict"], payload["layers"])
    assert str(ours.value) == str(theirs.value)


def _ids(device, vocab, batch=2, seq=96, seed=1):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randint(0, vocab, (batch, seq), generator=g).to(device)


@pytest.mark.gpu
def test_option_b_reference_loader_builds_b200_layers(cuda, ref, bundle, monkeypatch):
    from s_salaad_b200.efficient import build_efficient_model
    from s_salaad_b200.efficient.ls_linear import _LRSLinearBase, _LRSLinearLRBlockCUDA

    path, dense = bundle
    # ls_linear.py:263-266 routed to the B200 layer (same constructor, buffers and errors)
    monkeypatch.setattr(ref["ls_linear"], "_LRSLinearLRBlockCUDA", _LRSLinearLRBlockCUDA)
    model, config, meta = ref["model"].build_efficient_model(path, device="cuda")
    assert sum(isinstance(m, _LRSLinearBase) for m in model.modules()) == len(dense)
    ours, _, _ = build_efficient_model(path, device=cuda)
    ids = _ids(cuda, config["vocab_size"])
    with torch.no_grad():
        a = model(ids).logits
        b = ours(ids).logits
    assert torch.isfinite(a.float()).all()
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_option_a_reference_layer_on_b200_operator(cuda, ref, bundle, monkeypatch):
    import s_salaad_b200.cuda_sparse.addmm_inplace as shim
    from s_salaad_b200.cuda_sparse import register_reference_op

    path, dense = bundle
    # a process that never imports the TileLang module: the reference layer's
    # constructor finds get_tuned_config in the B200 shim, and the operator it
    # calls is the B200 kernel
    monkeypatch.setitem(sys.modules, "ssalaad.tilelang_sparse.addmm_inplace", shim)
    register_reference_op()
    model, config, _ = ref["model"].build_efficient_model(path, device="cuda")
    ref_cls = ref["ls_linear"]._LRSLinearLRBlockCUDA
    assert sum(isinstance(m, ref_cls) for m in model.modules()) == len(dense)
    payload = ref["artifact"].load_artifact(path)

    def dense_model(dtype):
        m = ref["model"].build_model_from_config(payload["model_config"], attn_implementation="sdpa")
        m.load_state_dict(payload["base_state_dict"], strict=False)
        with torch.no_grad():
            for name, W in dense.items():
                m.get_submodule(name).weight.copy_(W)
        return m.to(device=cuda, dtype=dtype).eval()

    ids = _ids(cuda, config["vocab_size"])
    with torch.no_grad():
        got = model(ids).logits.float()
        ref32 = dense_model(torch.float32)(ids).logits
        ref16 = dense_model(torch.bfloat16)(ids).logits.float()
    rel = lambda t: float((t - ref32).norm() / ref32.norm())  # noqa: E731
    assert rel(got) <= max(2.0 * rel(ref16), 1e-2), (rel(got), rel(ref16))
