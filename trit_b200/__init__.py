"""trit_b200: the greedy token loop of Trit's decoder language model
(CausalLm) on NVIDIA B200, behind the C ABI of include/trit_cuda.h."""
from .lm import CausalLm, Dense, Prefix, TritError, library  # noqa: F401

__all__ = ["CausalLm", "Dense", "Prefix", "TritError", "library"]
