"""TEST / MEASUREMENT INFRASTRUCTURE ONLY: a PyTorch fp64 restatement of the
reference's NanoGPT training step, used to check the
loss curve of the reference model running with this repository's attention.

Restated from the reference sources (no code copied):

* forward, cuda_transformer/NanoGPT.cu:80-94: token + position embedding ->
  TransformerLayer -> UnEmbedding (x U^T, no bias, Embedding.cu:360-376) ->
  Softmax (temperature 1);
* block, TransformerBlockLayer.cu:60-66: LayerNorm -> Attention -> LayerNorm
  -> MLP (Linear, ReLU, Linear), with NO residual connections;
* LayerNorm, layer_norm_kernels.cu:34-90: biased variance, eps 1e-5, affine;
* Linear, LinearLayer.cu:13,111: y = x W^T + b, W [out, in];
* attention: q/k/v = x W^T + b, the weight buffer read as [H*D, in] (row =
  output feature, attention_qkv_kernels.cu:92-95; getParameters labels it
  [in, H*D], AttentionLayer.cu:342, which only matters when in != H*D),
  heads split as [B, T, H, D] -> [B, H, T, D]; softmax(q k^T / sqrt(D)) v
  (non-causal, as the reference's kernel; causal optional); output
  projection a W_o^T + b_o, W_o read as [in, H*D] (attention_proj_kernels.cu:83);
* loss, loss_kernels.cu:150-189: mean over all B*T tokens of -log p[target],
  taken on the softmax *probabilities*;
* Adam, adam_kernels.cu:44-52 and AdamOptimizer.cu:74-96: the bias-corrected
  moments are stored back into m and v, and the step counter advances twice
  per step (t = 1, 3, 5, ...).
"""
from __future__ import annotations

import math

import numpy as np
import torch


def layer_norm(x, w, b, eps=1e-5):
    mean = x.mean(-1, keepdim=True)
    var = ((x - mean) ** 2).mean(-1, keepdim=True)
    return (x - mean) / torch.sqrt(var + eps) * w + b


def project(x, w, b):
    """x W^T + b with the weight buffer read row = output feature, whatever
    shape label it carries (the reference's projection kernels index it as
    [out, in])."""
    return x @ w.reshape(-1, x.shape[-1]).T + b


def attention_f64(q, k, v, causal: bool):
    s = (q @ k.transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if causal:
        T = q.shape[-2]
        s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    return torch.softmax(s, -1) @ v


def forward(params: dict, ids: torch.Tensor, num_layers: int, num_heads: int, head_dim: int, causal: bool,
            attention=attention_f64):
    """Softmax probabilities [B, T, V] of the reference architecture.
    `attention(q, k, v, causal)` on [B, H, T, D] (tests swap in the library)."""
    B, T = ids.shape
    x = params["tokenEmbedding"][ids] + params["positionEmbedding"][:T].unsqueeze(0)
    for i in range(num_layers):
        p = lambda name: params[f"layer_{i}.{name}"]
        h = layer_norm(x, p("firstNorm.weights"), p("firstNorm.biases"))
        split = lambda t: t.view(B, T, num_heads, head_dim).transpose(1, 2).contiguous()
        q = split(project(h, p("attention.query.weights"), p("attention.query.biases")))
        k = split(project(h, p("attention.key.weights"), p("attention.key.biases")))
        v = split(project(h, p("attention.value.weights"), p("attention.value.biases")))
        o = attention(q, k, v, causal).transpose(1, 2).reshape(B, T, num_heads * head_dim)
        a = project(o, p("attention.output.weights"), p("attention.output.biases"))
        h2 = layer_norm(a, p("secondNorm.weights"), p("secondNorm.biases"))
        m = torch.relu(h2 @ p("mlp.layer_0.weights").T + p("mlp.layer_0.biases"))
        x = m @ p("mlp.layer_2.weights").T + p("mlp.layer_2.biases")
    logits = x @ params["unEmbedding"].T
    return torch.softmax(logits, -1)


def loss_from_probs(probs, target):
    return -torch.log(probs.gather(-1, target.unsqueeze(-1)).squeeze(-1)).mean()


class ReferenceAdam:
    """The reference's Adam, including its stored bias-corrected moments and
    its double step-counter increment."""

    def __init__(self, params: dict, lr=3e-4, b1=0.9, b2=0.999, eps=1e-8):
        self.params, self.lr, self.b1, self.b2, self.eps = params, lr, b1, b2, eps
        self.m = {k: torch.zeros_like(v) for k, v in params.items()}
        self.v = {k: torch.zeros_like(v) for k, v in params.items()}
        self.t = 0

    @torch.no_grad()
    def step(self, grads: dict):
        self.t += 1
        for k, p in self.params.items():
            g = grads[k]
            m = (self.m[k] * self.b1 + g * (1 - self.b1)) / (1 - self.b1 ** self.t)
            v = (self.v[k] * self.b2 + g * g * (1 - self.b2)) / (1 - self.b2 ** self.t)
            p -= self.lr * m / (torch.sqrt(v) + self.eps)
            self.m[k], self.v[k] = m, v
        self.t += 1


def train(params_np: dict, batches, num_layers, num_heads, head_dim, causal=False, lr=3e-4,
          dtype=torch.float64, device="cpu", attention=attention_f64):
    """Run len(batches) reference training steps; returns the loss before each
    update.  batches: list of (ids [B, T], target [B, T]) int arrays."""
    params = {k: torch.tensor(np.asarray(v), dtype=dtype, device=device).requires_grad_() for k, v in params_np.items()}
    opt = ReferenceAdam(params, lr=lr)
    losses = []
    for ids, target in batches:
        ids_t = torch.as_tensor(np.asarray(ids), dtype=torch.long, device=device)
        tgt_t = torch.as_tensor(np.asarray(target), dtype=torch.long, device=device)
        for p in params.values():
            p.grad = None
        loss = loss_from_probs(forward(params, ids_t, num_layers, num_heads, head_dim, causal, attention), tgt_t)
        loss.backward()
        losses.append(float(loss.detach()))
        opt.step({k: p.grad for k, p in params.items()})
    return losses
