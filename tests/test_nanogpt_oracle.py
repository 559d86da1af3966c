"""CPU: the NanoGPT restatement used for BASELINE config 4 follows the
reference's optimizer quirks (AdamOptimizer.cu:74-96, adam_kernels.cu:44-52):
the step counter advances twice per step and the stored moments are the
bias-corrected ones."""
import math

import torch

from oracle import nanogpt_oracle as nano


def test_reference_adam_quirks():
    p = {"w": torch.tensor([1.0], dtype=torch.float64)}
    opt = nano.ReferenceAdam(p, lr=0.1, b1=0.9, b2=0.999, eps=0.0)
    g = torch.tensor([2.0], dtype=torch.float64)
    opt.step({"w": g})
    assert opt.t == 2
    # t = 1 inside the update: m = g, v = g^2 after bias correction
    assert math.isclose(float(opt.m["w"]), 2.0) and math.isclose(float(opt.v["w"]), 4.0)
    assert math.isclose(float(p["w"]), 1.0 - 0.1)
    opt.step({"w": g})
    assert opt.t == 4
    m = (2.0 * 0.9 + 2.0 * 0.1) / (1 - 0.9 ** 3)  # second update uses t = 3
    assert math.isclose(float(opt.m["w"]), m)


def test_forward_is_a_distribution():
    torch.manual_seed(0)
    E, H, D, V, T = 8, 2, 4, 5, 6
    params = {"tokenEmbedding": torch.randn(V, E), "positionEmbedding": torch.randn(T, E),
              "unEmbedding": torch.randn(V, E)}
    for n in ("firstNorm", "secondNorm"):
        params[f"layer_0.{n}.weights"], params[f"layer_0.{n}.biases"] = torch.ones(E), torch.zeros(E)
    for n in ("query", "key", "value", "output"):
        params[f"layer_0.attention.{n}.weights"], params[f"layer_0.attention.{n}.biases"] = torch.randn(E, E), torch.zeros(E)
    params["layer_0.mlp.layer_0.weights"], params["layer_0.mlp.layer_0.biases"] = torch.randn(16, E), torch.zeros(16)
    params["layer_0.mlp.layer_2.weights"], params["layer_0.mlp.layer_2.biases"] = torch.randn(E, 16), torch.zeros(E)
    ids = torch.randint(0, V, (3, T))
    for causal in (False, True):
        p = nano.forward(params, ids, 1, H, D, causal)
        assert p.shape == (3, T, V)
        assert torch.allclose(p.sum(-1), torch.ones(3, T))


def test_package_adam_equals_the_restated_reference_adam():
    """cudatransformer_b200.nanogpt.ReferenceAdam (multi-tensor ops) makes the
    same updates as the restatement of the reference's Adam
    (adam_kernels.cu:44-52, AdamOptimizer.cu:74-96), bit for bit in float64."""
    import torch

    from cudatransformer_b200.nanogpt import ReferenceAdam as PackageAdam
    from oracle.nanogpt_oracle import ReferenceAdam

    g = torch.Generator().manual_seed(0)
    p1 = {k: torch.randn(5, 7, generator=g, dtype=torch.float64) for k in "abc"}
    p2 = {k: v.clone() for k, v in p1.items()}
    a, r = PackageAdam(p1, lr=1e-2), ReferenceAdam(p2, lr=1e-2)
    for _ in range(4):
        grads = {k: torch.randn(5, 7, generator=g, dtype=torch.float64) for k in "abc"}
        a.step(grads)
        r.step(grads)
    assert all(torch.equal(p1[k], p2[k]) for k in "abc")
    assert a.t == r.t == 8
