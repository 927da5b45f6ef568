"""trit_b200: the greedy token loop of Trit's decoder language model
(CausalLm) on NVIDIA B200, behind the C ABI of include/trit_cuda.h."""
from .lm import CausalLm, Dense, Prefix, TritError, library, normal_row, synthesize  # noqa: F401
from . import presets  # noqa: F401

__all__ = ["CausalLm", "Dense", "Prefix", "TritError", "library", "synthesize", "normal_row", "presets"]
