"""B200 counterparts of ``ssalaad.efficient`` (the compressed-layer API)."""
from .artifact import (dense_to_bsr, encode_s_for_artifact, export_model_config, load_artifact, module_buffers,
                       save_artifact)
from .ls_linear import LRSLinear, _LRSLinearLR, _LRSLinearLRBlockBase, _LRSLinearLRBlockCUDA, _LRSLinearLRNM
from .model import build_efficient_model, build_model_from_config, group_projections

__all__ = ["LRSLinear", "build_efficient_model", "build_model_from_config", "dense_to_bsr",
           "encode_s_for_artifact", "export_model_config", "group_projections", "load_artifact",
           "module_buffers", "save_artifact", "_LRSLinearLR", "_LRSLinearLRBlockBase", "_LRSLinearLRBlockCUDA",
           "_LRSLinearLRNM"]
