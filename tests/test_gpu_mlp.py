"""GPU: the block's MLP Linear layers and LayerNorm on the library
(ctfa_linear_* on the projection GEMM, fused ReLU; ctfa_layernorm_*) against
float64 restatements of the reference kernels (linear_kernels.cu,
relu_kernels.cu, layer_norm_kernels.cu; oracle/nanogpt_oracle.layer_norm).

Tolerances (max |x - x64| / max |x64|): 2e-3 fp32 (tf32 GEMMs), 1e-2 bf16,
1e-5 for fp32 LayerNorm (no tensor cores), 1e-10 double.  Parameter
gradients must ADD into pre-filled buffers, as the reference's atomics do."""
import numpy as np
import pytest
import torch

from oracle import nanogpt_oracle as nano
from oracle import projection_oracle as po

pytestmark = pytest.mark.gpu

GEMM_TOL = {torch.float32: 2e-3, torch.bfloat16: 1e-2, torch.float64: 1e-10}


def _np(t):
    return t.detach().double().cpu().numpy()


def _check(got, want, tol, what):
    err = po.max_rel_err(_np(got) if torch.is_tensor(got) else got, want)
    assert err < tol, f"{what}: max rel err {err:.2e} >= {tol:.0e}"


# (M, K, N): config-4 MLP (K=384 -> N=1536 and back), ragged M, K/N not
# multiples of 128 bytes (SIMT path), one row
LIN_SHAPES = [(1000, 384, 1536), (777, 1536, 384), (300, 100, 72), (1, 64, 64)]


@pytest.mark.parametrize("shape", LIN_SHAPES)
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("relu", [False, True])
def test_linear_matches_restatement(cuda_device, shape, dt, relu):
    from cudatransformer_b200 import mlp_layers as ml

    M, K, N = shape
    if dt == torch.float64 and M * K * N > 2e7:
        pytest.skip("SIMT double checked on the small shapes")
    rng = np.random.default_rng(M + K + N)
    mk = lambda *s, scale=1.0: torch.tensor(rng.standard_normal(s) * scale).to(dt).to(cuda_device)
    x, w, b, dy = mk(M, K), mk(N, K, scale=K ** -0.5), mk(N, scale=0.1), mk(M, N)
    mask = mk(M, K)  # sign pattern for the fused ReLU backward
    tol = GEMM_TOL[dt]
    y = ml.linear_forward(x, w, b, relu=relu)
    ry = _np(x) @ _np(w).T + _np(b)
    if relu:
        ry = np.maximum(ry, 0)
    _check(y, ry, tol, "y")
    pre_w, pre_b = mk(N, K), mk(N)
    dw, db = pre_w.clone(), pre_b.clone()
    dx = ml.linear_backward(x, dy, w, dx_mask=mask, dw=dw, db=db)
    rdx = (_np(dy) @ _np(w)) * (_np(mask) > 0)
    _check(dx, rdx, tol, "dx (masked)")
    loose = tol * 4 if dt == torch.bfloat16 else tol
    _check(dw.double() - pre_w.double(), _np(dy).T @ _np(x), loose, "dw increment")
    _check(db.double() - pre_b.double(), _np(dy).sum(0), loose, "db increment")
    torch.cuda.synchronize()


# (40, 3000), (4, 12000), (3, 30000): rows wider than 1024 -- column sums in
# shared memory, in opt-in shared memory, and straight into global memory
@pytest.mark.parametrize("ME", [(777, 384), (64, 1000), (5, 33), (40, 3000), (4, 12000), (3, 30000)])
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float64])
def test_layernorm_matches_restatement(cuda_device, ME, dt):
    from cudatransformer_b200 import mlp_layers as ml

    M, E = ME
    rng = np.random.default_rng(M * E)
    mk = lambda *s, scale=1.0, shift=0.0: torch.tensor(rng.standard_normal(s) * scale + shift).to(dt).to(cuda_device)
    x, w, b, dy = mk(M, E, scale=2.0, shift=0.5), mk(E, scale=0.5, shift=1.0), mk(E, scale=0.1), mk(M, E)
    tol = {torch.float32: 1e-5, torch.bfloat16: 1e-2, torch.float64: 1e-10}[dt]
    y, mean, rstd = ml.layernorm_forward(x, w, b, 1e-5)
    tx, tw, tb = (torch.tensor(_np(t), requires_grad=True) for t in (x, w, b))
    ry = nano.layer_norm(tx, tw, tb, 1e-5)
    ry.backward(torch.tensor(_np(dy)))
    _check(y, ry.detach().numpy(), tol, "y")
    pre = mk(E), mk(E)
    dw, db = pre[0].clone(), pre[1].clone()
    dx = ml.layernorm_backward(x, dy, w, mean, rstd, dw, db)
    dx2 = ml.layernorm_backward(x, dy, w, None, None)  # statistics recomputed
    _check(dx2, tx.grad.numpy(), tol * (4 if dt == torch.float32 else 1), "dx (recomputed statistics)")
    _check(dx, tx.grad.numpy(), tol * (4 if dt == torch.float32 else 1), "dx")
    loose = tol * 4 if dt == torch.bfloat16 else max(tol, 1e-5)
    _check(dw.double() - pre[0].double(), tw.grad.numpy(), loose, "dw increment")
    _check(db.double() - pre[1].double(), tb.grad.numpy(), loose, "db increment")


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_block_layers_under_autograd(cuda_device, dt):
    """layer_norm -> mlp under autograd against float64 autograd of the same
    composition (two tf32 / bf16 GEMMs in a row: 5e-3 / 2e-2).  The float64
    side applies the ReLU pattern of the library's own forward: a hidden unit
    within rounding of zero may switch sides between precisions, which moves
    its gradient by O(1) and is not an error of either."""
    from cudatransformer_b200 import mlp_layers as ml
    from cudatransformer_b200.autograd import layer_norm, mlp

    M, E, F = 512, 384, 1536
    rng = np.random.default_rng(3)
    mk = lambda *s, scale=1.0: torch.tensor(rng.standard_normal(s) * scale).to(dt).to(cuda_device)
    leaves = [mk(M, E), mk(E, scale=0.2) + 1, mk(E, scale=0.1), mk(F, E, scale=E ** -0.5), mk(F, scale=0.1),
              mk(E, F, scale=F ** -0.5), mk(E, scale=0.1)]
    leaves = [t.clone().requires_grad_() for t in leaves]
    dy = mk(M, E)
    y = mlp(layer_norm(leaves[0], leaves[1], leaves[2]), *leaves[3:])
    y.backward(dy)
    with torch.no_grad():
        hid = ml.linear_forward(layer_norm(leaves[0], leaves[1], leaves[2]), leaves[3], leaves[4], relu=True)
    keep = torch.tensor(_np(hid) > 0)
    ref = [torch.tensor(_np(t), requires_grad=True) for t in leaves]
    h = nano.layer_norm(ref[0], ref[1], ref[2])
    ry = ((h @ ref[3].T + ref[4]) * keep) @ ref[5].T + ref[6]
    ry.backward(torch.tensor(_np(dy)))
    tol = 5e-3 if dt == torch.float32 else 2e-2
    _check(y, ry.detach().numpy(), tol, "y")
    for got, want, n in zip(leaves, ref, ("x", "ln_w", "ln_b", "w1", "b1", "w2", "b2")):
        _check(got.grad, want.grad.numpy(), tol, f"grad {n}")
