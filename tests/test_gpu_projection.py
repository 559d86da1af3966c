"""GPU: the projection GEMMs (ctfa_qkv_forward / ctfa_qkv_backward /
ctfa_out_proj_forward / ctfa_out_proj_backward, tcgen05 kernels
proj_gemm_sm100 and the SIMT kernels for double and odd shapes) against the
float64 restatement of the reference kernels (oracle/projection_oracle.py).

Tolerance (max |x - x64| / max |x64| per output): 2e-3 for fp32 I/O (tf32
tensor cores), 1e-2 for bf16 / fp16, 1e-10 for double.  Weight and bias
gradients must ACCUMULATE into the buffers (pre-filled here with known values),
as the reference's atomic kernels do."""
import numpy as np
import pytest
import torch

from oracle import projection_oracle as po

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 2e-3, torch.bfloat16: 1e-2, torch.float16: 1e-2, torch.float64: 1e-10}

# (B, T, E, H, D): config-4 block shape; ragged T with H*D % 128 = 64; D = 128;
# E not a multiple of 128 (fp32: tensor cores, 16-bit: SIMT since E*2 % 16 != 0);
# one sequence shorter than a tile; one-token sequences
SHAPES = [(2, 256, 384, 6, 64), (3, 200, 192, 3, 64), (2, 77, 256, 2, 128), (1, 130, 100, 2, 64), (2, 9, 64, 1, 64),
          (1, 1, 384, 6, 64), (3, 1, 128, 2, 128)]


def _inputs(B, T, E, H, D, dt, dev, seed):
    rng = np.random.default_rng(seed)
    mk = lambda *s, scale=1.0: torch.tensor(rng.standard_normal(s) * scale).to(dt).to(dev)
    x = mk(B, T, E)
    w = [mk(H * D, E, scale=E ** -0.5) for _ in range(3)]
    b = [mk(H * D, scale=0.1) for _ in range(3)]
    g = [mk(B, H, T, D) for _ in range(3)]
    a = mk(B, H, T, D)
    wo = mk(E, H * D, scale=(H * D) ** -0.5)
    bo = mk(E, scale=0.1)
    dy = mk(B, T, E)
    return x, w, b, g, a, wo, bo, dy


def _np(t):
    return t.detach().double().cpu().numpy()


def _check(got, want, tol, what):
    err = po.max_rel_err(_np(got), want)
    assert err < tol, f"{what}: max rel err {err:.2e} >= {tol:.0e}"


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16, torch.float64])
def test_projections_match_oracle(cuda_device, shape, dt):
    from cudatransformer_b200 import projection_layers as pl

    B, T, E, H, D = shape
    if dt == torch.float64 and B * T * E > 40000:
        pytest.skip("SIMT double path checked on the small shapes")
    x, w, b, g, a, wo, bo, dy = _inputs(B, T, E, H, D, dt, cuda_device, seed=hash(shape) % 1000)
    tol = TOL[dt]

    q, k, v = pl.qkv_forward(x, w[0], b[0], w[1], b[1], w[2], b[2], H, D)
    ref = po.qkv_forward(_np(x), *(_np(t) for t in (w[0], b[0], w[1], b[1], w[2], b[2])), H, D)
    for got, want, n in zip((q, k, v), ref, "qkv"):
        _check(got, want, tol, f"qkv_forward {n}")

    # gradients accumulate into pre-filled buffers
    rng = np.random.default_rng(3)
    pre_w = [torch.tensor(rng.standard_normal((H * D, E))).to(dt).to(cuda_device) for _ in range(3)]
    pre_b = [torch.tensor(rng.standard_normal(H * D)).to(dt).to(cuda_device) for _ in range(3)]
    dws = [p.clone() for p in pre_w]
    dbs = [p.clone() for p in pre_b]
    dx = pl.qkv_backward(x, g[0], g[1], g[2], w[0], w[1], w[2], dws[0], dbs[0], dws[1], dbs[1], dws[2], dbs[2])
    rdx, rdw, rdb = po.qkv_backward(_np(x), *(_np(t) for t in g), *(_np(t) for t in w))
    _check(dx, rdx, tol, "qkv_backward dx")
    for i in range(3):
        _check(dws[i].double() - pre_w[i].double(), rdw[i], tol * 4 if dt != torch.float32 and dt != torch.float64 else tol,
               f"qkv_backward dW[{i}]")
        _check(dbs[i].double() - pre_b[i].double(), rdb[i], tol * 4 if dt != torch.float32 and dt != torch.float64 else tol,
               f"qkv_backward db[{i}]")

    y = pl.out_proj_forward(a, wo, bo)
    _check(y, po.out_proj_forward(_np(a), _np(wo), _np(bo)), tol, "out_proj_forward")
    pre_wo = torch.tensor(rng.standard_normal((E, H * D))).to(dt).to(cuda_device)
    pre_bo = torch.tensor(rng.standard_normal(E)).to(dt).to(cuda_device)
    dwo, dbo = pre_wo.clone(), pre_bo.clone()
    da = pl.out_proj_backward(a, dy, wo, dwo, dbo)
    rda, rdwo, rdbo = po.out_proj_backward(_np(a), _np(dy), _np(wo))
    _check(da, rda, tol, "out_proj_backward da")
    loose = tol * 4 if dt in (torch.bfloat16, torch.float16) else tol
    _check(dwo.double() - pre_wo.double(), rdwo, loose, "out_proj_backward dWo")
    _check(dbo.double() - pre_bo.double(), rdbo, loose, "out_proj_backward dbo")
    torch.cuda.synchronize()


def test_partial_backward_requests(cuda_device):
    """dx only (no parameter gradients) and parameter gradients only (no dx)
    give the same numbers as the full call; a null bias-gradient pointer alone
    is allowed."""
    from cudatransformer_b200 import projection_layers as pl

    B, T, E, H, D = 2, 150, 256, 4, 64
    x, w, b, g, a, wo, bo, dy = _inputs(B, T, E, H, D, torch.float32, cuda_device, seed=7)
    dx_only = pl.qkv_backward(x, g[0], g[1], g[2], w[0], w[1], w[2])
    dws = [torch.zeros_like(t) for t in w]
    none_dx = pl.qkv_backward(x, g[0], g[1], g[2], w[0], w[1], w[2], dws[0], None, dws[1], None, dws[2], None,
                              want_dx=False)
    assert none_dx is None
    rdx, rdw, _ = po.qkv_backward(_np(x), *(_np(t) for t in g), *(_np(t) for t in w))
    _check(dx_only, rdx, 2e-3, "dx only")
    for i in range(3):
        _check(dws[i], rdw[i], 2e-3, f"dW[{i}] without dx / db")
    da_only = pl.out_proj_backward(a, dy, wo)
    _check(da_only, po.out_proj_backward(_np(a), _np(dy), _np(wo))[0], 2e-3, "da only")


def test_layer_mirrors_accumulate_like_the_reference(cuda_device):
    """QKVProjectionLayer / OutputProjectionLayer: two backward calls add
    twice the gradient (the reference's atomicAdd accumulation,
    attention_qkv_kernels.cu:230-238, attention_proj_kernels.cu:193-198)."""
    from cudatransformer_b200 import OutputProjectionLayer, QKVProjectionLayer

    B, T, E, H, D = 2, 64, 128, 2, 64
    x, w, b, g, a, wo, bo, dy = _inputs(B, T, E, H, D, torch.float32, cuda_device, seed=9)
    qkv = QKVProjectionLayer(E, H, D, device=cuda_device)
    for name, t in zip(("weightsQuery", "weightsKey", "weightsValue", "biasesQuery", "biasesKey", "biasesValue"),
                       (*w, *b)):
        getattr(qkv, name).copy_(t)
    outs = qkv.computeQKV(x)
    ref = po.qkv_forward(_np(x), *(_np(t) for t in (w[0], b[0], w[1], b[1], w[2], b[2])), H, D)
    for got, want in zip(outs, ref):
        _check(got, want, 2e-3, "computeQKV")
    qkv.computeBackward(x, *g)
    dx = qkv.computeBackward(x, *g)
    rdx, rdw, rdb = po.qkv_backward(_np(x), *(_np(t) for t in g), *(_np(t) for t in w))
    _check(dx, rdx, 2e-3, "computeBackward dx")
    _check(qkv.weightsQueryGrad, 2 * rdw[0], 2e-3, "weightsQueryGrad after two calls")
    _check(qkv.biasesValueGrad, 2 * rdb[2], 2e-3, "biasesValueGrad after two calls")
    c = qkv.clone()
    assert torch.equal(c.weightsKey, qkv.weightsKey) and c.weightsKeyGrad is None

    op = OutputProjectionLayer(E, D, H, device=cuda_device)
    op.weightsProj.copy_(wo)
    op.biasesProj.copy_(bo)
    _check(op.forward(a), po.out_proj_forward(_np(a), _np(wo), _np(bo)), 2e-3, "OutputProjectionLayer.forward")
    op.backward(a, dy)
    da = op.backward(a, dy)
    rda, rdwo, rdbo = po.out_proj_backward(_np(a), _np(dy), _np(wo))
    _check(da, rda, 2e-3, "OutputProjectionLayer.backward")
    _check(op.weightsProjGrad, 2 * rdwo, 2e-3, "weightsProjGrad after two calls")
    _check(op.biasesProjGrad, 2 * rdbo, 2e-3, "biasesProjGrad after two calls")


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_autograd_projection_gradients(cuda_device, dt):
    """qkv_projection -> flash_attention -> out_projection under autograd
    against float64 torch autograd of the same composition."""
    from cudatransformer_b200.autograd import flash_attention, out_projection, qkv_projection

    B, T, E, H, D = 2, 192, 256, 4, 64
    x, w, b, g, a, wo, bo, dy = _inputs(B, T, E, H, D, dt, cuda_device, seed=13)
    leaves = [t.clone().requires_grad_() for t in (x, w[0], b[0], w[1], b[1], w[2], b[2], wo, bo)]
    q, k, v = qkv_projection(*leaves[:7], H, D)
    y = out_projection(flash_attention(q, k, v, True), leaves[7], leaves[8])
    y.backward(dy)
    ref = [t.detach().double().clone().requires_grad_() for t in leaves]
    rx, rwq, rbq, rwk, rbk, rwv, rbv, rwo, rbo = ref
    split = lambda t: t.view(B, T, H, D).transpose(1, 2)
    rq, rk, rv = (split(rx @ W.T + bb) for W, bb in ((rwq, rbq), (rwk, rbk), (rwv, rbv)))
    s = (rq @ rk.transpose(-1, -2)) / D ** 0.5
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=s.device).triu(1), float("-inf"))
    ro = torch.softmax(s, -1) @ rv
    ry = ro.transpose(1, 2).reshape(B, T, H * D) @ rwo.T + rbo
    ry.backward(dy.double())
    # three tf32 (bf16) stages in a row -> 5e-3 (2e-2); per-kernel bounds are
    # checked above.  The exact gradient of the key bias is zero (a constant
    # added to every key shifts each score row by q.b, which the softmax
    # ignores), so bk is checked against the scale of the query-bias gradient.
    tol = 5e-3 if dt == torch.float32 else 2e-2
    _check(y, ry.detach().cpu().numpy(), tol, "y")
    for got, want, n in zip(leaves, ref, ("x", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo")):
        if n == "bk":
            scale = rbq.grad.abs().max().item()
            assert got.grad.double().abs().max().item() < tol * scale, "grad bk not ~0"
            continue
        _check(got.grad, want.grad.cpu().numpy(), tol, f"grad {n}")
