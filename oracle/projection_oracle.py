"""TEST INFRASTRUCTURE ONLY: float64 numpy restatement of the reference's QKV
projection and output projection (the steps either side of the attention in
AttentionLayer), the checker for libctfa_b200.so's ctfa_qkv_* /
ctfa_out_proj_* entry points.  Never imported by the product path.

Restated from the reference kernels (cuda_transformer/), no code copied:

* getQKVmatrices, attention_qkv_kernels.cu:51-122: for row r = b*T + t and
  column c = h*D + d, Q[b,h,t,d] = sum_i x[r, i] * Wq[c*E + i] + bq[c]
  (the weight buffer is read row = output feature, :92-95); same for K, V.
* qkvBackwardWB, attention_qkv_kernels.cu:164-241: dWq[c*E + i] +=
  sum_r dQ[b,h,t,d] x[r, i]; dbq[c] += sum_r dQ[b,h,t,d] (atomic adds into
  the layer's gradient buffers: accumulation across calls).
* qkvBackward, attention_qkv_kernels.cu:283-362: dx[r, i] = sum_c
  (dQ Wq + dK Wk + dV Wv)[r, c-major] (atomic adds into a fresh zero tensor).
* attentionProj, attention_proj_kernels.cu:48-98: y[r, o] = sum_c
  a[b,h,t,d] Wo[o*HD + c] + bo[o].
* projBackwardWB, attention_proj_kernels.cu:148-199: dWo[o*HD + c] +=
  sum_r dy[r, o] a[b,h,t,d]; dbo[o] += sum_r dy[r, o].
* projBackward, attention_proj_kernels.cu:240-288: da[b,h,t,d] =
  sum_o dy[r, o] Wo[o*HD + c].

Pinning: tests/test_gpu_reference.py runs the reference's own
QKVProjectionLayer / OutputProjectionLayer (compiled from the reference tree
into oracle/_ref/libctref.so) on the same inputs and compares them with this
restatement; tests/test_projection_oracle.py checks the backward formulas
against finite differences of the forward.
"""
from __future__ import annotations

import numpy as np


def _heads(m: np.ndarray, B: int, T: int, H: int, D: int) -> np.ndarray:
    """[B*T, H*D] rows -> [B, H, T, D]."""
    return m.reshape(B, T, H, D).transpose(0, 2, 1, 3)


def _rows(t: np.ndarray) -> np.ndarray:
    """[B, H, T, D] -> [B*T, H*D] rows (heads concatenated per row)."""
    B, H, T, D = t.shape
    return t.transpose(0, 2, 1, 3).reshape(B * T, H * D)


def qkv_forward(x, wq, bq, wk, bk, wv, bv, H: int, D: int):
    """x [B, T, E]; w* [H*D, E]; b* [H*D] or None -> q, k, v [B, H, T, D]."""
    x = np.asarray(x, np.float64)
    B, T, E = x.shape
    xr = x.reshape(B * T, E)
    out = []
    for w, b in ((wq, bq), (wk, bk), (wv, bv)):
        y = xr @ np.asarray(w, np.float64).reshape(H * D, E).T
        if b is not None:
            y = y + np.asarray(b, np.float64)
        out.append(_heads(y, B, T, H, D))
    return out


def qkv_backward(x, dq, dk, dv, wq, wk, wv):
    """-> dx [B, T, E], (dWq, dWk, dWv) [H*D, E], (dbq, dbk, dbv) [H*D]
    (the increments the reference adds to its gradient buffers)."""
    x = np.asarray(x, np.float64)
    B, T, E = x.shape
    xr = x.reshape(B * T, E)
    dx = np.zeros((B * T, E))
    dws, dbs = [], []
    for g, w in ((dq, wq), (dk, wk), (dv, wv)):
        gr = _rows(np.asarray(g, np.float64))
        W = np.asarray(w, np.float64).reshape(gr.shape[1], E)
        dx += gr @ W
        dws.append(gr.T @ xr)
        dbs.append(gr.sum(0))
    return dx.reshape(B, T, E), dws, dbs


def out_proj_forward(a, wo, bo):
    """a [B, H, T, D]; wo [E, H*D]; bo [E] or None -> y [B, T, E]."""
    a = np.asarray(a, np.float64)
    B, H, T, D = a.shape
    W = np.asarray(wo, np.float64)
    E = W.size // (H * D)
    y = _rows(a) @ W.reshape(E, H * D).T
    if bo is not None:
        y = y + np.asarray(bo, np.float64)
    return y.reshape(B, T, E)


def out_proj_backward(a, dy, wo):
    """-> da [B, H, T, D], dWo [E, H*D], dbo [E]."""
    a = np.asarray(a, np.float64)
    B, H, T, D = a.shape
    dyr = np.asarray(dy, np.float64).reshape(B * T, -1)
    E = dyr.shape[1]
    W = np.asarray(wo, np.float64).reshape(E, H * D)
    da = _heads(dyr @ W, B, T, H, D)
    return da, dyr.T @ _rows(a), dyr.sum(0)


def reference_bias_grad(g_rows) -> np.ndarray:
    """What the reference's bias-gradient code actually accumulates: only rows
    r = 0, 32, 64, ... of the [B*T, N] gradient.  In qkvBackwardWB
    (attention_qkv_kernels.cu:233-237) the bias sum runs only in the thread
    with inputIdx == 0 and reads its own tile column threadIdx.x = 0, i.e. row
    tile + 0 of each 32-row tile; projBackwardWB
    (attention_proj_kernels.cu:188, :195-197) sums per thread column but adds
    only the inputDimIdx == 0 thread's partial (rows tile + 0) to the
    gradient.  BLOCKDIM = 32 (ModuleLayer.cu:6).  The true bias gradient sums
    every row; tests use this emulation to confirm the reference's behaviour
    on the GPU, not as a target."""
    g = np.asarray(g_rows, np.float64)
    return g[::32].sum(0)


def max_rel_err(x, ref) -> float:
    """max |x - ref| / max |ref| (norm-wise relative error)."""
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(x - ref).max() / (den if den > 0 else 1.0))
