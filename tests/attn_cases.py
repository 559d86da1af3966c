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
