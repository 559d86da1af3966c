"""Shared helpers for the GPU parity tests: run the library on seeded inputs
and compute the fp64 oracle on the same (dtype-rounded) inputs."""
from __future__ import annotations

import numpy as np
import torch

from cudatransformer_b200 import FlashAttentionLayer
from oracle import oracle as orc

TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "f64": torch.float64}
# max|x - x64| / max|x64| per output tensor (spec: 2e-3 fp32 I/O via tf32, 1e-2 bf16)
TOL = {"f32": 2e-3, "bf16": 1e-2, "f16": 1e-2, "f64": 1e-9}


def to_device(x: np.ndarray, kind: str, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).to(device=device, dtype=TORCH[kind]).contiguous()


def to_numpy(t: torch.Tensor) -> np.ndarray:
    return t.detach().to(torch.float64).cpu().numpy()


def run_library(q, k, v, do, kind: str, causal: bool, device, backward: bool = True, keep_torch: bool = False):
    """Forward (+ backward) through FlashAttentionLayer; float64 numpy results
    (or the device tensors themselves with keep_torch=True)."""
    B, H, T, D = q.shape
    layer = FlashAttentionLayer(D, H, causal=causal)
    tq, tk, tv = (to_device(x, kind, device) for x in (q, k, v))
    conv = (lambda t: t) if keep_torch else to_numpy
    o = layer.computeAttention(tq, tk, tv, saveStates=backward)
    out = {"o": conv(o)}
    if backward:
        out["lse"] = layer.cachedLSE if keep_torch else layer.cachedLSE.cpu().numpy().astype(np.float64)
        dq, dk, dv = layer.computeBackward(tq, tk, tv, to_device(do, kind, device))
        out.update(dq=conv(dq), dk=conv(dk), dv=conv(dv))
        layer.clearCache()
    torch.cuda.synchronize(device)
    return out


def oracle_for(q, k, v, do, kind: str, causal: bool, backward: bool = True):
    """fp64 attention on the inputs rounded to the I/O type."""
    q, k, v, do = (orc.round_to(x, kind) for x in (q, k, v, do))
    o, lse = orc.attention_f64(q, k, v, causal)
    out = {"o": o, "lse": lse}
    if backward:
        dq, dk, dv = orc.attention_backward_f64(q, k, v, do, causal)
        out.update(dq=dq, dk=dk, dv=dv)
    return out


# Denominator floor of the error metric.  Some exact gradients vanish (T = 1:
# a single key gives dS = 0, so dq = dk = 0 up to rounding); dividing rounding
# noise by max|ref| ~ 1e-17 measures nothing.  Inputs here are O(1), so a
# floor of 1e-3 only matters in such degenerate cases.
DEN_FLOOR = 1e-3


def errors(ours: dict, ref: dict) -> dict:
    out = {}
    for name in ours:
        if name in ref:
            r = np.asarray(ref[name], dtype=np.float64)
            x = np.asarray(ours[name], dtype=np.float64)
            out[name] = float(np.abs(x - r).max() / max(np.abs(r).max(), DEN_FLOOR))
    return out


def attention_f64_device(q, k, v, do, causal: bool, chunk: int = 16):
    """Exact float64 attention forward and backward on the GPU (torch fp64
    matmuls, `chunk` (batch, head) problems at a time): the same math as
    oracle.attention_f64 / attention_backward_f64 (softmax(q k^T / sqrt(D)),
    dS = P (dP - rowsum(O dO)), dq = dS k / sqrt(D), dk = dS^T q / sqrt(D),
    dv = P^T dO), for full-size checks the CPU oracle would take minutes on.
    q, k, v, do: device tensors [B, H, T, D] already rounded to the I/O type.
    Returns float64 device tensors o, lse, dq, dk, dv."""
    B, H, T, D = q.shape
    f = lambda t: t.reshape(B * H, T, D).to(torch.float64)
    qq, kk, vv, dd = f(q), f(k), f(v), f(do)
    outs = {n: torch.empty((B * H, T, D), dtype=torch.float64, device=q.device) for n in ("o", "dq", "dk", "dv")}
    lse = torch.empty((B * H, T), dtype=torch.float64, device=q.device)
    scale = 1.0 / np.sqrt(D)
    mask = torch.triu(torch.ones(T, T, dtype=torch.bool, device=q.device), diagonal=1) if causal else None
    for a in range(0, B * H, chunk):
        sl = slice(a, min(a + chunk, B * H))
        s = torch.matmul(qq[sl], kk[sl].transpose(1, 2)) * scale
        if mask is not None:
            s.masked_fill_(mask, float("-inf"))
        m = s.amax(dim=-1, keepdim=True)
        p = torch.exp(s - m)
        l = p.sum(dim=-1, keepdim=True)
        p /= l
        del s
        o = torch.matmul(p, vv[sl])
        lse[sl] = (m + torch.log(l))[..., 0]
        outs["o"][sl] = o
        outs["dv"][sl] = torch.matmul(p.transpose(1, 2), dd[sl])
        dp = torch.matmul(dd[sl], vv[sl].transpose(1, 2))
        delta = (o * dd[sl]).sum(dim=-1, keepdim=True)
        ds = p * (dp - delta)
        del dp, p
        outs["dq"][sl] = torch.matmul(ds, kk[sl]) * scale
        outs["dk"][sl] = torch.matmul(ds.transpose(1, 2), qq[sl]) * scale
        del ds
    res = {n: t.reshape(B, H, T, D) for n, t in outs.items()}
    res["lse"] = lse.reshape(B, H, T)
    return res


def per_head_errors(ours: dict, ref: dict) -> dict:
    """max|x - x64| / max|x64| for every (batch, head) slice and output, on the
    device; returns {name: float64 tensor [B, H]}."""
    out = {}
    for name in ("o", "dq", "dk", "dv"):
        x = ours[name].to(torch.float64)
        r = ref[name]
        num = (x - r).abs().amax(dim=(-2, -1))
        den = r.abs().amax(dim=(-2, -1)).clamp_min(DEN_FLOOR)
        out[name] = num / den
    return out
