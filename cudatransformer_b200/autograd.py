"""PyTorch autograd binding of the attention path: `flash_attention(q, k, v)`,
`qkv_projection(...)` and `out_projection(...)` run their forward and
backward through libctfa_b200.so (tcgen05 kernels), so the whole attention
layer (QKV projection -> attention -> output projection) can sit inside a
PyTorch training step (the NanoGPT step of BASELINE config 4 uses it this
way).  CUDA tensors, fp32 / bf16 / fp16 / fp64; no CPU path."""
from __future__ import annotations

import torch

from .flash_attention_layer import FlashAttentionLayer
from . import projection_layers as _proj


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


class QKVProjectionFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wq, bq, wk, bk, wv, bv, num_heads: int, head_dim: int):
        q, k, v = _proj.qkv_forward(x, wq, bq, wk, bk, wv, bv, num_heads, head_dim)
        ctx.save_for_backward(x, wq, wk, wv)
        ctx.bias_shapes = (bq is not None, bk is not None, bv is not None)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        x, wq, wk, wv = ctx.saved_tensors
        z = torch.zeros_like
        dwq, dwk, dwv = z(wq), z(wk), z(wv)
        hd = wq.shape[0]
        dbq, dbk, dbv = (torch.zeros(hd, dtype=wq.dtype, device=wq.device) if has else None
                         for has in ctx.bias_shapes)
        need_dx = ctx.needs_input_grad[0]
        dx = _proj.qkv_backward(x, dq, dk, dv, wq, wk, wv, dwq, dbq, dwk, dbk, dwv, dbv, want_dx=need_dx)
        if dx is not None:
            dx = dx.view(x.shape)
        return dx, dwq, dbq, dwk, dbk, dwv, dbv, None, None


class OutProjectionFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, wo, bo):
        y = _proj.out_proj_forward(a, wo, bo)
        ctx.save_for_backward(a, wo)
        ctx.has_bias = bo is not None
        return y

    @staticmethod
    def backward(ctx, dy):
        a, wo = ctx.saved_tensors
        dwo = torch.zeros_like(wo)
        dbo = torch.zeros(wo.shape[0], dtype=wo.dtype, device=wo.device) if ctx.has_bias else None
        da = _proj.out_proj_backward(a, dy, wo, dwo, dbo, want_da=ctx.needs_input_grad[0])
        return da, dwo, dbo


def qkv_projection(x, wq, bq, wk, bk, wv, bv, num_heads: int, head_dim: int):
    """q, k, v [B, H, T, D] = x [B, T, E] W^T + b with W [H*D, E] (row =
    output feature), with gradients for x, the weights and the biases."""
    return QKVProjectionFunction.apply(x, wq, bq, wk, bk, wv, bv, num_heads, head_dim)


def out_projection(a, wo, bo):
    """y [B, T, E] = a [B, H, T, D] (heads concatenated per row) Wo^T + bo
    with Wo [E, H*D], with gradients for a, Wo and bo."""
    return OutProjectionFunction.apply(a, wo, bo)
