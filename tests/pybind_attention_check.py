"""The check of the reference's test_flash_attention.py (lines 14-52), run
through the reference's own pybind module `cuda_transformer` built by
oracle/Makefile (target `pybind`) over this repository's drop-ins.

    python tests/pybind_attention_check.py <module dir> N [N ...]

Imports `FloatTensor, FloatModule, AttentionFloat, FloatAttentionLayer` from
the module in <module dir> exactly as the reference's test does, sets the
four weight matrices (torch.randn(E, E) / sqrt(E), B=8, E=1024, H=16, D=64),
runs `attention(FloatTensor.fromNumpy(X))` for each N and compares the output
with the test's own PyTorch computation (X W^T per head through
F.scaled_dot_product_attention, non-causal, then W_o) on the GPU, in fp32 as
the test does (TF32 matmuls off, torch's default) and in fp64.  The matplotlib
timing part of the reference test is not run.  Prints one JSON line per N.

Run as a child process by tests/test_gpu_pybind.py: the module's pybind types
register globally, so each build of it gets a fresh interpreter.
"""
import json
import math
import sys

sys.path.insert(0, sys.argv[1])

import numpy as np  # noqa: E402
import torch  # noqa: E402
from torch.nn import functional as F  # noqa: E402

from cuda_transformer import AttentionFloat, FloatAttentionLayer, FloatModule, FloatTensor  # noqa: E402,F401

torch.backends.cuda.matmul.allow_tf32 = False
torch.backends.cudnn.allow_tf32 = False

B, E, H, D = 8, 1024, 16, 64
torch.manual_seed(0)
attention = AttentionFloat(input_dim=E, num_heads=H, head_dim=D)
Wq = torch.randn(E, E).cuda() / math.sqrt(E)
Wk = torch.randn(E, E).cuda() / math.sqrt(E)
Wv = torch.randn(E, E).cuda() / math.sqrt(E)
Wo = torch.randn(E, E).cuda() / math.sqrt(E)
attention.setQueryWeights(FloatTensor.fromNumpy(Wq.cpu().numpy()))
attention.setKeyWeights(FloatTensor.fromNumpy(Wk.cpu().numpy()))
attention.setValueWeights(FloatTensor.fromNumpy(Wv.cpu().numpy()))
attention.setOutputWeights(FloatTensor.fromNumpy(Wo.cpu().numpy()))


def torch_attention(X, wq, wk, wv, wo):
    """test_flash_attention.py:35-42, in the dtype of its arguments."""
    Q, K, V = X @ wq.T, X @ wk.T, X @ wv.T
    C = torch.zeros_like(Q)
    for b in range(0, E, D):
        C[:, :, b:b + D] = F.scaled_dot_product_attention(Q[:, :, b:b + D], K[:, :, b:b + D], V[:, :, b:b + D],
                                                          attn_mask=None, dropout_p=0.0, is_causal=False)
    return C @ wo.T


for N in (int(a) for a in sys.argv[2:]):
    X = torch.randn(B, N, E).cuda()
    out = attention(FloatTensor.fromNumpy(X.cpu().numpy())).numpy()
    O32 = torch_attention(X, Wq, Wk, Wv, Wo).cpu().numpy()
    O64 = torch_attention(*(t.double() for t in (X, Wq, Wk, Wv, Wo))).cpu().numpy()
    print(json.dumps({
        "N": N,
        "allclose_atol_1e-4": bool(np.allclose(O32, out, atol=1e-4)),
        "max_abs_vs_fp32": float(np.abs(out.astype(np.float64) - O32).max()),
        "max_abs_vs_fp64": float(np.abs(out - O64).max()),
        "max_rel_vs_fp64": float(np.abs(out - O64).max() / np.abs(O64).max()),
        "torch_fp32_max_rel_vs_fp64": float(np.abs(O32 - O64).max() / np.abs(O64).max()),
        "max_abs_fp64": float(np.abs(O64).max()),
    }), flush=True)
