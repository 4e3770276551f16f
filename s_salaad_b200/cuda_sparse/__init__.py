"""The ``ssalaad::tilelang_bsr_addmm_inplace_dense_`` operator on B200 kernels."""
from .addmm_inplace import get_tuned_config, register_reference_op

__all__ = ["get_tuned_config", "register_reference_op"]
