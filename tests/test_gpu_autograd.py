"""GPU: the PyTorch autograd binding (cudatransformer_b200.autograd) gives the
fp64 oracle's outputs and q/k/v gradients through loss.backward(), at the
dtype tolerances, causal and non-causal; and the NanoGPT restatement used for
BASELINE config 4 trains identically (3 steps) with it in place of the fp64
attention."""
import numpy as np
import pytest
import torch

from attn_cases import TOL
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_autograd_matches_oracle(cuda_device, kind, causal):
    from cudatransformer_b200.autograd import flash_attention

    B, H, T, D = 2, 3, 200, 64
    q, k, v, do = orc.make_inputs(B, H, T, D, seed=11)
    q, k, v, do = (orc.round_to(x, kind) for x in (q, k, v, do))
    dt = torch.float32 if kind == "f32" else torch.bfloat16
    tq, tk, tv = (torch.tensor(x, device=cuda_device).to(dt).requires_grad_() for x in (q, k, v))
    o = flash_attention(tq, tk, tv, causal)
    o.backward(torch.tensor(do, device=cuda_device).to(dt))
    o_ref, _ = orc.attention_f64(q, k, v, causal)
    dq, dk, dv = orc.attention_backward_f64(q, k, v, do, causal)
    for got, want in ((o, o_ref), (tq.grad, dq), (tk.grad, dk), (tv.grad, dv)):
        assert orc.max_rel_err(got.float().detach().cpu().numpy(), want) < TOL[kind]


def test_nanogpt_restatement_trains_the_same_with_our_attention(cuda_device):
    """Three reference-Adam steps of a 2-layer NanoGPT restatement: fp64
    attention vs this repository's attention (fp32 I/O) in an otherwise fp64
    model; the losses agree to 1e-4."""
    from cudatransformer_b200.autograd import flash_attention
    from oracle import nanogpt_oracle as nano

    rng = np.random.default_rng(5)
    L, H, D, V, T, B = 2, 2, 64, 65, 128, 4
    E = H * D
    shapes = {"tokenEmbedding": (V, E), "positionEmbedding": (T, E), "unEmbedding": (V, E)}
    for i in range(L):
        for n in ("firstNorm", "secondNorm"):
            shapes[f"layer_{i}.{n}.weights"], shapes[f"layer_{i}.{n}.biases"] = (E,), (E,)
        for n in ("query", "key", "value", "output"):
            shapes[f"layer_{i}.attention.{n}.weights"], shapes[f"layer_{i}.attention.{n}.biases"] = (E, E), (E,)
        shapes[f"layer_{i}.mlp.layer_0.weights"], shapes[f"layer_{i}.mlp.layer_0.biases"] = (4 * E, E), (4 * E,)
        shapes[f"layer_{i}.mlp.layer_2.weights"], shapes[f"layer_{i}.mlp.layer_2.biases"] = (E, 4 * E), (E,)
    init = {k: (np.ones(s) if k.endswith("Norm.weights") else np.zeros(s) if k.endswith("biases")
                else rng.standard_normal(s) * 0.02).astype(np.float32) for k, s in shapes.items()}
    data = []
    for _ in range(3):
        ids = rng.integers(0, V, size=(B, T + 1))
        data.append((ids[:, :-1], ids[:, 1:]))
    ref = nano.train(init, data, L, H, D, device=str(cuda_device))
    lib = lambda q, k, v, causal: flash_attention(q.float(), k.float(), v.float(), causal).double()
    ours = nano.train(init, data, L, H, D, device=str(cuda_device), attention=lib)
    assert max(abs(a - b) for a, b in zip(ours, ref)) < 1e-4


@pytest.mark.parametrize("causal", [False, True])
def test_package_nanogpt_step_tracks_the_fp64_restatement(cuda_device, causal):
    """cudatransformer_b200.nanogpt (fp32; QKV projection, attention and
    output projection on the library's tf32 kernels, the rest PyTorch fp32)
    against the fp64 restatement: same weights, tokens and reference Adam,
    four steps; every loss within 2e-3."""
    from cudatransformer_b200 import nanogpt as model
    from oracle import nanogpt_oracle as nano

    L, H, D, V, T, B = 2, 2, 64, 65, 128, 4
    init = model.init_parameters(model.parameter_shapes(L, H, D, V, T, 4 * H * D), seed=8)
    rng = np.random.default_rng(9)
    data = []
    for _ in range(4):
        ids = rng.integers(0, V, size=(B, T + 1))
        data.append((ids[:, :-1], ids[:, 1:]))
    ref = nano.train(init, data, L, H, D, causal=causal, device=str(cuda_device))
    params = {k: torch.tensor(v, device=cuda_device).requires_grad_() for k, v in init.items()}
    opt = model.ReferenceAdam(params)
    ours = []
    for ids, tgt in data:
        ids_t = torch.as_tensor(ids, device=cuda_device)
        tgt_t = torch.as_tensor(tgt, device=cuda_device)
        ours.append(float(model.train_step(params, opt, ids_t, tgt_t, L, H, D, causal)))
    assert max(abs(a - b) for a, b in zip(ours, ref)) < 2e-3, (ours, ref)
