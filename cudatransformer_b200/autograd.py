"""PyTorch autograd binding of the attention path: `flash_attention(q, k, v)`
runs the forward and backward through libctfa_b200.so (tcgen05 kernels), so
the path can sit inside a PyTorch training step (BASELINE config 4 measures
it inside the NanoGPT architecture this way).  Inputs [B, H, T, D], CUDA,
fp32 / bf16 / fp16 / fp64; no CPU path."""
from __future__ import annotations

import torch

from .flash_attention_layer import FlashAttentionLayer


class FlashAttentionFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal: bool = False):
        B, H, T, D = q.shape
        layer = FlashAttentionLayer(D, H, causal=causal)
        o = layer.computeAttention(q.contiguous(), k.contiguous(), v.contiguous(), saveStates=True)
        ctx.layer = layer
        ctx.save_for_backward(q, k, v)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v = ctx.saved_tensors
        dq, dk, dv = ctx.layer.computeBackward(q.contiguous(), k.contiguous(), v.contiguous(), do.contiguous())
        ctx.layer.clearCache()
        return dq, dk, dv, None


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """softmax(q k^T / sqrt(D) [+ causal mask]) v with gradients for q, k, v."""
    return FlashAttentionFunction.apply(q, k, v, causal)
