"""Generation with a compressed model (counterpart of ``ssalaad.inference``)."""
from .generate import generate, generate_no_cache

__all__ = ["generate", "generate_no_cache"]
