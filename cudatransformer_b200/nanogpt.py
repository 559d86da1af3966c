"""The reference's NanoGPT training step with every block
on this library: LayerNorm, QKV projection, attention, output projection and
the ReLU MLP run as libctfa_b200.so kernels (autograd.py); the embeddings,
unembedding (vocab 65), softmax, loss and optimizer are PyTorch ops
(plumbing).

Architecture and optimiser follow the reference (cuda_transformer/):
  * forward, NanoGPT.cu:80-94: token + position embedding -> blocks ->
    unembedding x U^T (Embedding.cu:360-376) -> softmax;
  * block, TransformerBlockLayer.cu:60-66: LayerNorm -> attention ->
    LayerNorm -> Linear, ReLU, Linear, with no residual connections;
  * LayerNorm eps 1e-5 with biased variance (layer_norm_kernels.cu:34-90);
    Linear y = x W^T + b, W [out, in] (LinearLayer.cu:13,111);
  * attention weights read row = output feature (attention_qkv_kernels.cu:92,
    attention_proj_kernels.cu:83);
  * loss, loss_kernels.cu:150-189: mean of -log p[target] over all tokens, on
    the softmax probabilities;
  * Adam, adam_kernels.cu:44-52 and AdamOptimizer.cu:74-96: the bias-corrected
    moments are stored back, and the step counter advances twice per step.
Parameter names are those of the reference's NanoGPT.getParameters().
"""
from __future__ import annotations

import numpy as np
import torch

from .autograd import flash_attention, layer_norm, mlp, out_projection, qkv_projection


def parameter_shapes(layers: int, heads: int, head_dim: int, vocab: int, seq_len: int, mlp: int) -> dict:
    E = heads * head_dim
    shapes = {"tokenEmbedding": (vocab, E), "positionEmbedding": (seq_len, E), "unEmbedding": (vocab, E)}
    for i in range(layers):
        for n in ("firstNorm", "secondNorm"):
            shapes[f"layer_{i}.{n}.weights"] = (E,)
            shapes[f"layer_{i}.{n}.biases"] = (E,)
        for n in ("query", "key", "value", "output"):
            shapes[f"layer_{i}.attention.{n}.weights"] = (E, E)
            shapes[f"layer_{i}.attention.{n}.biases"] = (E,)
        shapes[f"layer_{i}.mlp.layer_0.weights"] = (mlp, E)
        shapes[f"layer_{i}.mlp.layer_0.biases"] = (mlp,)
        shapes[f"layer_{i}.mlp.layer_2.weights"] = (E, mlp)
        shapes[f"layer_{i}.mlp.layer_2.biases"] = (E,)
    return shapes


def init_parameters(shapes: dict, seed: int, std: float = 0.02) -> dict:
    """N(0, std) weights, LayerNorm scales 1, biases 0 (float32 numpy)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name in sorted(shapes):
        if name.endswith("Norm.weights"):
            out[name] = np.ones(shapes[name], dtype=np.float32)
        elif name.endswith("biases"):
            out[name] = np.zeros(shapes[name], dtype=np.float32)
        else:
            out[name] = (rng.standard_normal(shapes[name]) * std).astype(np.float32)
    return out


def forward(params: dict, ids: torch.Tensor, layers: int, heads: int, head_dim: int, causal: bool) -> torch.Tensor:
    """Softmax probabilities [B, T, vocab]."""
    B, T = ids.shape
    x = params["tokenEmbedding"][ids] + params["positionEmbedding"][:T].unsqueeze(0)
    for i in range(layers):
        p = lambda n: params[f"layer_{i}.{n}"]
        h = layer_norm(x, p("firstNorm.weights"), p("firstNorm.biases"), 1e-5)
        q, k, v = qkv_projection(h, p("attention.query.weights"), p("attention.query.biases"),
                                 p("attention.key.weights"), p("attention.key.biases"),
                                 p("attention.value.weights"), p("attention.value.biases"), heads, head_dim)
        a = out_projection(flash_attention(q, k, v, causal), p("attention.output.weights"),
                           p("attention.output.biases"))
        h2 = layer_norm(a, p("secondNorm.weights"), p("secondNorm.biases"), 1e-5)
        x = mlp(h2, p("mlp.layer_0.weights"), p("mlp.layer_0.biases"), p("mlp.layer_2.weights"),
                p("mlp.layer_2.biases"))
    return torch.softmax(x @ params["unEmbedding"].T, -1)


def loss_from_probs(probs: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    return -torch.log(probs.gather(-1, target.unsqueeze(-1)).squeeze(-1)).mean()


class ReferenceAdam:
    """Adam as the reference implements it: m and v are stored back already
    bias-corrected, and the step counter advances twice per step."""

    def __init__(self, params: dict, lr: float = 3e-4, b1: float = 0.9, b2: float = 0.999, eps: float = 1e-8):
        self.params, self.lr, self.b1, self.b2, self.eps = params, lr, b1, b2, eps
        self.m = {k: torch.zeros_like(v) for k, v in params.items()}
        self.v = {k: torch.zeros_like(v) for k, v in params.items()}
        self.t = 0

    @torch.no_grad()
    def step(self, grads: dict) -> None:
        """One update of every parameter, as multi-tensor (foreach) ops: a
        handful of launches for all parameters instead of several per
        parameter."""
        self.t += 1
        c1, c2 = 1 - self.b1 ** self.t, 1 - self.b2 ** self.t
        keys = list(self.params)
        ps = [self.params[k] for k in keys]
        gs = [grads[k] for k in keys]
        ms = [self.m[k] for k in keys]
        vs = [self.v[k] for k in keys]
        torch._foreach_mul_(ms, self.b1)
        torch._foreach_add_(ms, gs, alpha=1 - self.b1)
        torch._foreach_div_(ms, c1)
        torch._foreach_mul_(vs, self.b2)
        torch._foreach_addcmul_(vs, gs, gs, value=1 - self.b2)
        torch._foreach_div_(vs, c2)
        den = torch._foreach_sqrt(vs)
        torch._foreach_add_(den, self.eps)
        torch._foreach_addcdiv_(ps, ms, den, value=-self.lr)
        self.t += 1


def train_step(params: dict, opt: ReferenceAdam, ids: torch.Tensor, target: torch.Tensor, layers: int, heads: int,
               head_dim: int, causal: bool) -> torch.Tensor:
    """One step: forward, loss, backward, Adam update.  Returns the loss
    (device tensor, before the update)."""
    for p in params.values():
        p.grad = None
    loss = loss_from_probs(forward(params, ids, layers, heads, head_dim, causal), target)
    loss.backward()
    opt.step({k: p.grad for k, p in params.items()})
    return loss.detach()
