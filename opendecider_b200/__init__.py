"""OpenDecider's decision forward pass on NVIDIA B200 (sm_100a).

The hot path runs in libod_b200.so (hand-written CUDA kernels behind the C ABI of include/od_b200.h); this package
is the host side that mirrors the reference's Python seams: quant (Int8Tensor, Int8Linear and its `_fused` W8A8
slot), backbone (the int8 decoder, the left-padded state pass and the int8 KV cache), v3 (branched option rows and
the decision trunk), decider (requests -> probabilities), distributed (requests sharded over GPUs).
"""
from . import _lib  # noqa: F401

__all__ = ["_lib"]
