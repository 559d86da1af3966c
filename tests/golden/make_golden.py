"""Generates tests/golden/attention_golden.npz (run once here; committed).

The reference's only attention test checks its output against
torch.nn.functional.scaled_dot_product_attention (test_flash_attention.py:43-52),
so that function -- on CPU, in float64, with autograd for the gradients --
is the independent implementation the oracle is pinned against.

Inputs are not stored: they are regenerated from the seed with
oracle.make_inputs (numpy default_rng), which is reproducible everywhere.

Cases
  small_{nc,c}   B=1 H=2 T=48  D=64  seed 11 (T not a multiple of 32)   full tensors
  cfg1_{nc,c}    B=2 H=4 T=128 D=64  seed 0  (BASELINE config 1)       1024 sampled
                                                                      elements + sums
Outputs per case: o, lse, dq, dk, dv (float64).

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle.oracle import make_inputs  # noqa: E402

CASES = {
    "small": dict(B=1, H=2, T=48, D=64, seed=11, sample=False),
    "cfg1": dict(B=2, H=4, T=128, D=64, seed=0, sample=True),
}
N_SAMPLE = 1024


def torch_reference(q, k, v, do, causal):
    tq, tk, tv = (torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v))
    o = F.scaled_dot_product_attention(tq, tk, tv, is_causal=causal)
    o.backward(torch.tensor(do, dtype=torch.float64))
    D = q.shape[-1]
    s = (tq.detach() @ tk.detach().transpose(-1, -2)) / np.sqrt(D)
    if causal:
        T = q.shape[-2]
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool), 1), float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    return {
        "o": o.detach().numpy(),
        "lse": lse.numpy(),
        "dq": tq.grad.numpy(),
        "dk": tk.grad.numpy(),
        "dv": tv.grad.numpy(),
    }


def main():
    out = {}
    for name, c in CASES.items():
        q, k, v, do = make_inputs(c["B"], c["H"], c["T"], c["D"], c["seed"])
        for causal in (False, True):
            key = f"{name}_{'c' if causal else 'nc'}"
            ref = torch_reference(q, k, v, do, causal)
            for t, arr in ref.items():
                if c["sample"]:
                    rng = np.random.default_rng(1234)
                    idx = rng.choice(arr.size, size=min(N_SAMPLE, arr.size), replace=False)
                    out[f"{key}/{t}/idx"] = idx.astype(np.int64)
                    out[f"{key}/{t}/val"] = arr.reshape(-1)[idx]
                    out[f"{key}/{t}/sum"] = np.array(arr.sum())
                    out[f"{key}/{t}/sumsq"] = np.array((arr * arr).sum())
                else:
                    out[f"{key}/{t}"] = arr
    dst = Path(__file__).resolve().parent / "attention_golden.npz"
    np.savez_compressed(dst, **out)
    print(dst, dst.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
