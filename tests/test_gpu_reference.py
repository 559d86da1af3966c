"""GPU: the reference's own CUDA FlashAttentionLayer (compiled from its sources
into oracle/_ref/libctref.so by oracle/Makefile) against the oracle and
against libctfa_b200.so, on the same seeded inputs.

* reference O and dQ == exact attention (non-causal, T % 32 == 0);
* reference dK / dV == the float64 emulation of its kernels (which is not the
  gradient: flash_attention.cu:310-321), confirming the divergence on the GPU;
* libctfa O and dQ == reference O and dQ within the fp32 tolerance.
"""
import numpy as np
import pytest
import torch

from attn_cases import TOL, run_library, to_device, to_numpy
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

REF = orc.load_reference_cuda()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref/libctref.so not built (needs the reference tree)")


def run_reference(q, k, v, do, device):
    B, H, T, D = q.shape
    tq, tk, tv, tdo = (to_device(x, "f32", device) for x in (q, k, v, do))
    o, dq, dk, dv = (torch.empty_like(tq) for _ in range(4))
    rc = REF.ctref_forward_backward(0, tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tdo.data_ptr(), o.data_ptr(),
                                    dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, H, T, D)
    assert rc == 0, f"reference CUDA returned {rc}"
    return {n: to_numpy(t) for n, t in dict(o=o, dq=dq, dk=dk, dv=dv).items()}


@needs_ref
@pytest.mark.parametrize("shape", [(2, 4, 128, 64), (1, 3, 256, 64)])
def test_reference_cuda_matches_oracle_and_emulation(cuda_device, shape):
    B, H, T, D = shape
    q, k, v, do = orc.make_inputs(B, H, T, D, seed=0)
    q, k, v, do = (orc.round_to(x, "f32") for x in (q, k, v, do))
    ref = run_reference(q, k, v, do, cuda_device)
    o, _ = orc.attention_f64(q, k, v, False)
    dq, dk, dv = orc.attention_backward_f64(q, k, v, do, False)
    emu = orc.reference_emulation(q, k, v, do)
    assert orc.max_rel_err(ref["o"], o) < 1e-5
    assert orc.max_rel_err(ref["dq"], dq) < 1e-4
    assert orc.max_rel_err(ref["dk"], emu["dk"]) < 1e-4
    assert orc.max_rel_err(ref["dv"], emu["dv"]) < 1e-4
    assert orc.max_rel_err(ref["dk"], dk) > 0.3  # the reference's dK is not the gradient


@needs_ref
def test_library_matches_reference_cuda_on_o_and_dq(cuda_device):
    q, k, v, do = orc.make_inputs(2, 4, 128, 64, seed=0)
    ref = run_reference(q, k, v, do, cuda_device)
    ours = run_library(q, k, v, do, "f32", False, cuda_device)
    assert orc.max_rel_err(ours["o"], ref["o"]) < TOL["f32"]
    assert orc.max_rel_err(ours["dq"], ref["dq"]) < TOL["f32"]


@needs_ref
def test_reference_projection_layers_match_oracle_and_library(cuda_device):
    """The reference's own QKVProjectionLayer / OutputProjectionLayer (fp32
    SIMT kernels) == the float64 restatement (pins its weight orientation and
    accumulation) -- except its bias gradients, which sum only every 32nd row
    (confirmed here against po.reference_bias_grad); libctfa_b200.so's tcgen05
    projections == the reference within the fp32 tolerance, and its bias
    gradients == the true gradient."""
    import ctypes

    from cudatransformer_b200 import projection_layers as pl
    from oracle import projection_oracle as po

    if not hasattr(REF, "ctref_qkv_projection"):
        pytest.skip("libctref.so predates the projection entry points; rebuild with make -C oracle ref")
    B, T, E, H, D = 2, 96, 192, 2, 64  # E != H*D: a transposed weight read would show
    rng = np.random.default_rng(21)
    mk = lambda *s, scale=1.0: torch.tensor(rng.standard_normal(s) * scale, dtype=torch.float32, device=cuda_device)
    x = mk(B, T, E)
    w = [mk(H * D, E, scale=E ** -0.5) for _ in range(3)]
    b = [mk(H * D, scale=0.1) for _ in range(3)]
    g = [mk(B, H, T, D) for _ in range(3)]
    a, wo, bo, dy = mk(B, H, T, D), mk(E, H * D, scale=(H * D) ** -0.5), mk(E, scale=0.1), mk(B, T, E)
    P3 = ctypes.c_void_p * 3
    ptrs = lambda ts: P3(*(t.data_ptr() for t in ts))
    out = [torch.empty(B, H, T, D, device=cuda_device) for _ in range(3)]
    dx = torch.empty(B, T, E, device=cuda_device)
    dw = [torch.empty(H * D, E, device=cuda_device) for _ in range(3)]
    db = [torch.empty(H * D, device=cuda_device) for _ in range(3)]
    rc = REF.ctref_qkv_projection(x.data_ptr(), ptrs(w), ptrs(b), ptrs(out), ptrs(g), dx.data_ptr(), ptrs(dw),
                                  ptrs(db), B, T, E, H, D)
    assert rc == 0
    y = torch.empty(B, T, E, device=cuda_device)
    da, dwo, dbo = torch.empty(B, H, T, D, device=cuda_device), torch.empty(E, H * D, device=cuda_device), torch.empty(
        E, device=cuda_device)
    rc = REF.ctref_out_projection(a.data_ptr(), wo.data_ptr(), bo.data_ptr(), y.data_ptr(), dy.data_ptr(),
                                  da.data_ptr(), dwo.data_ptr(), dbo.data_ptr(), B, T, E, H, D)
    assert rc == 0
    n = lambda t: t.double().cpu().numpy()
    oq = po.qkv_forward(n(x), n(w[0]), n(b[0]), n(w[1]), n(b[1]), n(w[2]), n(b[2]), H, D)
    odx, odw, odb = po.qkv_backward(n(x), *(n(t) for t in g), *(n(t) for t in w))
    oy = po.out_proj_forward(n(a), n(wo), n(bo))
    oda, odwo, odbo = po.out_proj_backward(n(a), n(dy), n(wo))
    # reference (fp32 SIMT) vs the restatement, except its bias gradients,
    # which sum only every 32nd row (po.reference_bias_grad)
    errs = {}
    for name, got, want in [*zip(("q", "k", "v"), out, oq), ("dx", dx, odx), *zip(("dwq", "dwk", "dwv"), dw, odw),
                            ("y", y, oy), ("da", da, oda), ("dwo", dwo, odwo)]:
        errs[name] = po.max_rel_err(n(got), want)
    rows = lambda t: n(t).transpose(0, 2, 1, 3).reshape(B * T, H * D)  # [B,H,T,D] -> [B*T, H*D]
    for name, got, gt in zip(("dbq", "dbk", "dbv"), db, g):
        errs[name + " (every 32nd row)"] = po.max_rel_err(n(got), po.reference_bias_grad(rows(gt)))
    errs["dbo (every 32nd row)"] = po.max_rel_err(n(dbo), po.reference_bias_grad(n(dy).reshape(B * T, E)))
    bad = {k: v for k, v in errs.items() if not v < 1e-5}
    assert not bad, f"reference vs restatement: {bad}"
    # the reference's bias gradients are not the gradient (differ by O(1))
    assert po.max_rel_err(n(db[0]), odb[0]) > 0.1 and po.max_rel_err(n(dbo), odbo) > 0.1
    # library (tf32 tensor cores) vs the reference
    lq = pl.qkv_forward(x, w[0], b[0], w[1], b[1], w[2], b[2], H, D)
    ldw = [torch.zeros_like(t) for t in w]
    ldb = [torch.zeros_like(t) for t in b]
    ldx = pl.qkv_backward(x, *g, *w, ldw[0], ldb[0], ldw[1], ldb[1], ldw[2], ldb[2])
    ly = pl.out_proj_forward(a, wo, bo)
    ldwo, ldbo = torch.zeros_like(wo), torch.zeros_like(bo)
    lda = pl.out_proj_backward(a, dy, wo, ldwo, ldbo)
    for got, want in [*zip(lq, out), (ldx, dx), *zip(ldw, dw), (ly, y), (lda, da), (ldwo, dwo)]:
        assert po.max_rel_err(n(got), n(want)) < TOL["f32"]
    # bias gradients: ours are the true gradient (the restatement)
    for got, want in [*zip(ldb, odb), (ldbo, odbo)]:
        assert po.max_rel_err(n(got), want) < TOL["f32"]


@needs_ref
def test_reference_linear_and_layernorm_match_restatement_and_library(cuda_device):
    """The reference's own LinearLayer<float> and LayerNormLayer<float>
    (compiled from its sources) == the float64 restatements (y = x W^T + b,
    dW/db accumulated from zero, dx; LayerNorm with eps 1e-5), and the
    library's ctfa_linear_* / ctfa_layernorm_* == the reference within the
    fp32 tolerances (2e-3 tf32 GEMMs, 1e-5 LayerNorm)."""
    from cudatransformer_b200 import mlp_layers as ml
    from oracle import nanogpt_oracle as nano
    from oracle import projection_oracle as po

    if not hasattr(REF, "ctref_linear"):
        pytest.skip("libctref.so predates the Linear / LayerNorm entry points; rebuild with make -C oracle ref")
    M, K, N = 300, 384, 256
    rng = np.random.default_rng(31)
    mk = lambda *s, scale=1.0, shift=0.0: torch.tensor(rng.standard_normal(s) * scale + shift, dtype=torch.float32,
                                                       device=cuda_device)
    x, w, b, dy = mk(M, K), mk(N, K, scale=K ** -0.5), mk(N, scale=0.1), mk(M, N)
    y, dx, dw, db = (torch.empty(M, N, device=cuda_device), torch.empty(M, K, device=cuda_device),
                     torch.empty(N, K, device=cuda_device), torch.empty(N, device=cuda_device))
    P = lambda t: t.data_ptr()
    assert REF.ctref_linear(P(x), P(w), P(b), P(y), P(dy), P(dx), P(dw), P(db), M, K, N) == 0
    n = lambda t: t.detach().double().cpu().numpy()
    want = {"y": n(x) @ n(w).T + n(b), "dx": n(dy) @ n(w), "dw": n(dy).T @ n(x), "db": n(dy).sum(0)}
    for name, got in (("y", y), ("dx", dx), ("dw", dw), ("db", db)):
        assert po.max_rel_err(n(got), want[name]) < 1e-5, name
    ly = ml.linear_forward(x, w, b)
    ldw, ldb = torch.zeros_like(w), torch.zeros_like(b)
    ldx = ml.linear_backward(x, dy, w, dw=ldw, db=ldb)
    for got, ref in ((ly, y), (ldx, dx), (ldw, dw), (ldb, db)):
        assert po.max_rel_err(n(got), n(ref)) < TOL["f32"]

    E = 384
    xl, gl, bl, dyl = mk(M, E, scale=2.0, shift=0.5), mk(E, scale=0.5, shift=1.0), mk(E, scale=0.1), mk(M, E)
    yl, dxl, dgl, dbl = (torch.empty(M, E, device=cuda_device), torch.empty(M, E, device=cuda_device),
                         torch.empty(E, device=cuda_device), torch.empty(E, device=cuda_device))
    assert REF.ctref_layernorm(P(xl), P(gl), P(bl), P(yl), P(dyl), P(dxl), P(dgl), P(dbl), M, E) == 0
    tx, tg, tb = (torch.tensor(n(t), requires_grad=True) for t in (xl, gl, bl))
    ry = nano.layer_norm(tx, tg, tb, 1e-5)
    ry.backward(torch.tensor(n(dyl)))
    for got, want in ((yl, ry.detach().numpy()), (dxl, tx.grad.numpy()), (dgl, tg.grad.numpy()),
                      (dbl, tb.grad.numpy())):
        assert po.max_rel_err(n(got), want) < 1e-5
    my, mean, rstd = ml.layernorm_forward(xl, gl, bl)
    mg, mb = torch.zeros_like(gl), torch.zeros_like(bl)
    mdx = ml.layernorm_backward(xl, dyl, gl, mean, rstd, mg, mb)
    for got, ref in ((my, yl), (mdx, dxl), (mg, dgl), (mb, dbl)):
        assert po.max_rel_err(n(got), n(ref)) < 1e-5
