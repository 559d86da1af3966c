"""Functional wrappers of the Linear / LayerNorm entry points of libctfa_b200.so
(ctfa_linear_* / ctfa_layernorm_* in include/ctfa.h), the block's layers
around the attention in the reference's TransformerBlockLayer
(cuda_transformer/TransformerBlockLayer.cu:60-66: LayerNorm -> attention ->
LayerNorm -> Linear, ReLU, Linear).

Semantics follow the reference kernels: Linear y = x W^T + b with W [out, in]
(linear_kernels.cu:52-77), parameter gradients ADDED into the given buffers
(linearBackwardWB's atomicAdd, :159, :167), dx overwritten; LayerNorm with
biased variance and eps (layer_norm_kernels.cu), dw / db added
(:131-133).  Torch CUDA tensors, contiguous; no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib
from .flash_attention_layer import _stream_handle
from .projection_layers import _code, _contig, _p


def linear_forward(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, relu: bool = False) -> torch.Tensor:
    """y [..., N] = x [..., K] W^T + b (then max(., 0) when relu)."""
    x = _contig(x)
    K = x.shape[-1]
    M = x.numel() // K
    N = w.shape[0]
    y = torch.empty(*x.shape[:-1], N, dtype=x.dtype, device=x.device)
    lib = _lib.load()
    _lib.check(lib.ctfa_linear_forward(_p(x), _p(_contig(w)), _p(b), _p(y), M, K, N, int(relu), _code(x),
                                       _stream_handle(x.device)), "ctfa_linear_forward")
    return y


def linear_backward(x: torch.Tensor | None, dy: torch.Tensor, w: torch.Tensor, dx_mask: torch.Tensor | None = None,
                    dw: torch.Tensor | None = None, db: torch.Tensor | None = None, want_dx: bool = True):
    """dx (zeroed where dx_mask <= 0, when given) and, when dw / db are given,
    the parameter gradients added into them."""
    dy = _contig(dy)
    N = dy.shape[-1]
    M = dy.numel() // N
    K = w.shape[1]
    dx = torch.empty(*dy.shape[:-1], K, dtype=dy.dtype, device=dy.device) if want_dx else None
    lib = _lib.load()
    _lib.check(lib.ctfa_linear_backward(_p(None if x is None else _contig(x)), _p(dy), _p(_contig(w)),
                                        _p(None if dx_mask is None else _contig(dx_mask)), _p(dw), _p(db), _p(dx),
                                        M, K, N, _code(dy), _stream_handle(dy.device)), "ctfa_linear_backward")
    return dx


def layernorm_forward(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5):
    """y, mean (fp32 [M]), rstd (fp32 [M])."""
    x = _contig(x)
    E = x.shape[-1]
    M = x.numel() // E
    y = torch.empty_like(x)
    mean = torch.empty(M, dtype=torch.float32, device=x.device)
    rstd = torch.empty(M, dtype=torch.float32, device=x.device)
    lib = _lib.load()
    _lib.check(lib.ctfa_layernorm_forward(_p(x), _p(_contig(w)), _p(_contig(b)), _p(y), _p(mean), _p(rstd), M, E,
                                          float(eps), _code(x), _stream_handle(x.device)), "ctfa_layernorm_forward")
    return y, mean, rstd


def layernorm_backward(x: torch.Tensor, dy: torch.Tensor, w: torch.Tensor, mean: torch.Tensor | None,
                       rstd: torch.Tensor | None, dw: torch.Tensor | None = None, db: torch.Tensor | None = None,
                       eps: float = 1e-5) -> torch.Tensor:
    """dx; dw / db (when given) get sum dy * x_hat / sum dy added.  mean /
    rstd None: recomputed from x (with eps)."""
    x, dy = _contig(x), _contig(dy)
    E = x.shape[-1]
    M = x.numel() // E
    dx = torch.empty_like(x)
    lib = _lib.load()
    _lib.check(lib.ctfa_layernorm_backward(_p(x), _p(dy), _p(_contig(w)), _p(mean), _p(rstd), _p(dx), _p(dw), _p(db),
                                           M, E, float(eps), _code(x), _stream_handle(x.device)),
               "ctfa_layernorm_backward")
    return dx
