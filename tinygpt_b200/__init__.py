"""tinygpt_b200 -- B200-native batched logits processing and sampling.

The product is the CUDA library libtgsample.so behind the C ABI in
include/tgsample.h; this package builds it, binds it with ctypes and offers a
host API with the reference sampler's parameter names (tinygpt_b200.sampler).
"""
from .sampler import Sampler, SpecVerifier, sample_next, row_params  # noqa: F401

__all__ = ["Sampler", "SpecVerifier", "sample_next", "row_params"]
