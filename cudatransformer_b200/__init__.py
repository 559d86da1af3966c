"""B200-native (sm_100a) flash attention for CudaTransformer's FlashAttentionLayer.

The compute path is ``libctfa_b200.so`` (hand-written tcgen05/TMA kernels,
C ABI in ``include/ctfa.h``); this package holds the host-side mirror of the
reference's operator interface and the multi-GPU drivers.
"""
from . import _lib
from .flash_attention_layer import FlashAttentionLayer
from .projection_layers import OutputProjectionLayer, QKVProjectionLayer

__all__ = ["FlashAttentionLayer", "QKVProjectionLayer", "OutputProjectionLayer", "_lib"]
