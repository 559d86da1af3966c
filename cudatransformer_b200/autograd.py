"""PyTorch autograd binding of the library: `flash_attention(q, k, v)`,
`qkv_projection(...)`, `out_projection(...)`, `mlp(...)` (Linear -> ReLU ->
Linear) and `layer_norm(...)` run their forward and backward through
libctfa_b200.so (tcgen05 GEMMs, attention kernels, LayerNorm kernels), so a
whole transformer block can sit inside a PyTorch training step (the NanoGPT
step of BASELINE config 4 uses it this way).  CUDA tensors, fp32 / bf16 /
fp16 / fp64; no CPU path."""
from __future__ import annotations

import torch

from .flash_attention_layer import FlashAttentionLayer
from . import mlp_layers as _mlp
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


class MLPFunction(torch.autograd.Function):
    """y = relu(x W1^T + b1) W2^T + b2 (the reference's MLPLayer: Linear,
    ReLU, Linear).  The ReLU runs in the first GEMM's epilogue; its backward
    runs in the second GEMM's input-gradient epilogue."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2):
        h = _mlp.linear_forward(x, w1, b1, relu=True)
        y = _mlp.linear_forward(h, w2, b2)
        ctx.save_for_backward(x, w1, h, w2)
        ctx.has_bias = (b1 is not None, b2 is not None)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w1, h, w2 = ctx.saved_tensors
        dw1, dw2 = torch.zeros_like(w1), torch.zeros_like(w2)
        db1 = torch.zeros(w1.shape[0], dtype=w1.dtype, device=w1.device) if ctx.has_bias[0] else None
        db2 = torch.zeros(w2.shape[0], dtype=w2.dtype, device=w2.device) if ctx.has_bias[1] else None
        dpre = _mlp.linear_backward(h, dy, w2, dx_mask=h, dw=dw2, db=db2)
        dx = _mlp.linear_backward(x, dpre, w1, dw=dw1, db=db1, want_dx=ctx.needs_input_grad[0])
        return dx, dw1, db1, dw2, db2


class LayerNormFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps: float = 1e-5):
        y, mean, rstd = _mlp.layernorm_forward(x, w, b, eps)
        ctx.save_for_backward(x, w, mean, rstd)
        ctx.eps = eps
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, mean, rstd = ctx.saved_tensors
        dw, db = torch.zeros_like(w), torch.zeros_like(w)
        dx = _mlp.layernorm_backward(x, dy, w, mean, rstd, dw, db, ctx.eps)
        return dx, dw, db, None


def mlp(x, w1, b1, w2, b2):
    """relu(x W1^T + b1) W2^T + b2 with W [out, in], gradients for all inputs."""
    return MLPFunction.apply(x, w1, b1, w2, b2)


def layer_norm(x, w, b, eps: float = 1e-5):
    """LayerNorm over the last dimension (biased variance), gradients for x, w, b."""
    return LayerNormFunction.apply(x, w, b, eps)
