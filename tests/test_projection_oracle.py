"""CPU: the float64 projection restatement (oracle/projection_oracle.py).

* Its forward equals a literal loop over the reference kernels' index
  expressions (getQKVmatrices, attention_qkv_kernels.cu:87-121; attentionProj,
  attention_proj_kernels.cu:66-97), on a tiny case with E != H*D so that a
  transposed weight read would show.
* Its backward equals finite differences of its forward (every gradient the
  reference's backward kernels produce: dx, dW, db, da, dWo, dbo).
"""
import numpy as np

from oracle import projection_oracle as po


def _case(seed=0, B=2, T=3, E=5, H=2, D=3):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, T, E))
    w = [rng.standard_normal((H * D, E)) for _ in range(3)]
    b = [rng.standard_normal(H * D) for _ in range(3)]
    a = rng.standard_normal((B, H, T, D))
    wo = rng.standard_normal((E, H * D))
    bo = rng.standard_normal(E)
    return x, w, b, a, wo, bo


def test_forward_matches_reference_index_loops():
    B, T, E, H, D = 2, 3, 5, 2, 3
    x, w, b, a, wo, bo = _case(B=B, T=T, E=E, H=H, D=D)
    q, k, v = po.qkv_forward(x, w[0], b[0], w[1], b[1], w[2], b[2], H, D)
    xf = x.reshape(-1)
    for which, got in enumerate((q, k, v)):
        wf = w[which].reshape(-1)
        for row in range(B * T):
            for col in range(H * D):
                acc = sum(xf[row * E + kk] * wf[col * E + kk] for kk in range(E))  # weightIdx = col*E + k
                bi, si, hi, di = row // T, row % T, col // D, col % D
                assert abs(got[bi, hi, si, di] - (acc + b[which][col])) < 1e-12
    y = po.out_proj_forward(a, wo, bo)
    af, wof = a.reshape(-1), wo.reshape(-1)
    for row in range(B * T):
        for col in range(E):
            acc = 0.0
            for c in range(H * D):
                bi, si, hi, di = row // T, row % T, c // D, c % D
                acc += af[((bi * H + hi) * T + si) * D + di] * wof[col * H * D + c]
            assert abs(y.reshape(B * T, E)[row, col] - (acc + bo[col])) < 1e-12


def _fd(f, arr, seed_dir, eps=1e-6):
    """Directional derivative of scalar f along a random direction of arr."""
    d = np.random.default_rng(seed_dir).standard_normal(arr.shape)
    p, m = arr + eps * d, arr - eps * d
    return (f(p) - f(m)) / (2 * eps), d


def test_backward_matches_finite_differences():
    B, T, E, H, D = 2, 3, 5, 2, 3
    x, w, b, a, wo, bo = _case(seed=1, B=B, T=T, E=E, H=H, D=D)
    rng = np.random.default_rng(2)
    gq, gk, gv = (rng.standard_normal((B, H, T, D)) for _ in range(3))
    gy = rng.standard_normal((B, T, E))

    def loss_qkv(x_, w_, b_):
        q, k, v = po.qkv_forward(x_, w_[0], b_[0], w_[1], b_[1], w_[2], b_[2], H, D)
        return float((q * gq).sum() + (k * gk).sum() + (v * gv).sum())

    dx, dws, dbs = po.qkv_backward(x, gq, gk, gv, w[0], w[1], w[2])
    fd, d = _fd(lambda t: loss_qkv(t, w, b), x, 3)
    assert abs(fd - (dx * d).sum()) < 1e-6
    for i in range(3):
        fd, d = _fd(lambda t: loss_qkv(x, [t if j == i else w[j] for j in range(3)], b), w[i], 4 + i)
        assert abs(fd - (dws[i] * d).sum()) < 1e-6
        fd, d = _fd(lambda t: loss_qkv(x, w, [t if j == i else b[j] for j in range(3)]), b[i], 7 + i)
        assert abs(fd - (dbs[i] * d).sum()) < 1e-6

    loss_out = lambda a_, wo_, bo_: float((po.out_proj_forward(a_, wo_, bo_) * gy).sum())
    da, dwo, dbo = po.out_proj_backward(a, gy, wo)
    for arr, grad, f, s in ((a, da, lambda t: loss_out(t, wo, bo), 10), (wo, dwo, lambda t: loss_out(a, t, bo), 11),
                            (bo, dbo, lambda t: loss_out(a, wo, t), 12)):
        fd, d = _fd(f, arr, s)
        assert abs(fd - (grad * d).sum()) < 1e-6
