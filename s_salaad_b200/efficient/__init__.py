"""B200 counterparts of ``ssalaad.efficient`` (the compressed-layer API)."""
from .artifact import dense_to_bsr, module_buffers
from .ls_linear import LRSLinear, _LRSLinearLR, _LRSLinearLRBlockBase, _LRSLinearLRBlockCUDA

__all__ = ["LRSLinear", "dense_to_bsr", "module_buffers", "_LRSLinearLR", "_LRSLinearLRBlockBase",
           "_LRSLinearLRBlockCUDA"]
