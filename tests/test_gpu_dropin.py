"""GPU: the drop-ins.  The reference's own AttentionLayer<float> (QKV
projection -> FlashAttentionLayer -> output projection, compiled unmodified
from the reference tree by oracle/Makefile) runs with
cudatransformer_b200/{QKVProjectionLayer,FlashAttentionLayer,
OutputProjectionLayer}.cu in place of the reference's layers.  Same check as
the reference's test_flash_attention.py:43-52 (forward against
scaled-dot-product attention of X W^T per head, then W_o) against an fp64
restatement, causal and non-causal, at 5e-3 (max|x - x64| / max|x64|): three
tf32 stages in a row, each held to 2e-3 by its own tests.  And: with
device-resident inputs, building the layer, its forward and its teardown
issue no device-wide synchronisation (stream-ordered allocation).
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as orc

pytestmark = pytest.mark.gpu

LIB = orc.HERE / "_ref" / "libct_dropin.so"
needs_lib = pytest.mark.skipif(not LIB.exists(), reason="oracle/_ref/libct_dropin.so not built (needs the reference tree)")


def reference_fp64(x, wq, wk, wv, wo, H, causal):
    B, N, E = x.shape
    D = E // H
    q, k, v = (x @ w.T for w in (wq, wk, wv))
    split = lambda t: t.reshape(B, N, H, D).transpose(0, 2, 1, 3)
    o, _ = orc.attention_f64(split(q), split(k), split(v), causal)
    return o.transpose(0, 2, 1, 3).reshape(B, N, E) @ wo.T


@needs_lib
@pytest.mark.parametrize("B,N,E,H", [(2, 128, 256, 4), (2, 256, 256, 4), (1, 192, 512, 4)])
@pytest.mark.parametrize("causal", [False, True])
def test_reference_attention_layer_with_dropin(cuda_device, B, N, E, H, causal):
    lib = ctypes.CDLL(str(LIB))
    fp = ctypes.POINTER(ctypes.c_float)
    I = ctypes.c_int
    lib.dropin_attention_forward.argtypes = [fp] * 6 + [I] * 5
    lib.dropin_attention_forward.restype = I
    rng = np.random.default_rng(N + E)
    x = rng.standard_normal((B, N, E)).astype(np.float32)
    ws = [(rng.standard_normal((E, E)) / np.sqrt(E)).astype(np.float32) for _ in range(4)]
    out = np.empty((B, N, E), dtype=np.float32)
    ptr = lambda a: a.ctypes.data_as(fp)
    rc = lib.dropin_attention_forward(ptr(x), *(ptr(w) for w in ws), ptr(out), B, N, E, H, int(causal))
    assert rc == 0
    ref = reference_fp64(x.astype(np.float64), *(w.astype(np.float64) for w in ws), H, causal)
    assert orc.max_rel_err(out, ref) < 5e-3


@needs_lib
def test_dropins_do_not_synchronise(cuda_device):
    """A ~50 ms sleep kernel on the default stream is still running when the
    device-resident AttentionLayer forward (construction, forward, teardown)
    returns: nothing in it waited for the device.  The result is then checked
    as above."""
    import torch

    lib = ctypes.CDLL(str(LIB))
    V, I = ctypes.c_void_p, ctypes.c_int
    lib.dropin_attention_forward_device.argtypes = [V] * 6 + [I] * 5
    lib.dropin_attention_forward_device.restype = I
    B, N, E, H = 2, 256, 256, 4
    rng = np.random.default_rng(77)
    x = rng.standard_normal((B, N, E)).astype(np.float32)
    ws = [(rng.standard_normal((E, E)) / np.sqrt(E)).astype(np.float32) for _ in range(4)]
    tx = torch.tensor(x, device=cuda_device)
    tws = [torch.tensor(w, device=cuda_device) for w in ws]
    ty = torch.empty(B, N, E, device=cuda_device)
    stream = torch.cuda.default_stream(cuda_device)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(100_000_000)  # ~50 ms at 1.9 GHz
        rc = lib.dropin_attention_forward_device(tx.data_ptr(), *(t.data_ptr() for t in tws), ty.data_ptr(),
                                                 B, N, E, H, 1)
        still_running = not stream.query()
    torch.cuda.synchronize()
    assert rc == 0
    assert still_running, "the drop-in layer waited for the device"
    ref = reference_fp64(x.astype(np.float64), *(w.astype(np.float64) for w in ws), H, True)
    assert orc.max_rel_err(ty.cpu().numpy(), ref) < 5e-3


def _block_names(E, mlp_dim):
    """getParameters() names and shapes of the reference's
    TransformerBlockLayer (TransformerBlockLayer.cu getParameters; MLP
    sub-layers prefixed layer_<i>, MLPLayer.cu:108-117)."""
    out = {"firstNorm.weights": (E,), "firstNorm.biases": (E,)}
    for p in ("query", "key", "value"):
        out[f"attention.{p}.weights"] = (E, E)
        out[f"attention.{p}.biases"] = (E,)
    out["attention.output.weights"] = (E, E)
    out["attention.output.biases"] = (E,)
    out.update({"secondNorm.weights": (E,), "secondNorm.biases": (E,),
                "mlp.layer_0.weights": (mlp_dim, E), "mlp.layer_0.biases": (mlp_dim,),
                "mlp.layer_2.weights": (E, mlp_dim), "mlp.layer_2.biases": (E,)})
    return out


def block_fp64(x, params, H, causal, relu_mask):
    """fp64 restatement of TransformerBlockLayer::forward
    (TransformerBlockLayer.cu:60-66: LayerNorm -> attention -> LayerNorm ->
    Linear, ReLU, Linear; no residual), on torch tensors under autograd.  The
    ReLU keeps the units `relu_mask` marks (the pattern of the library's own
    forward: a unit within rounding of zero may switch sides between
    precisions, which moves its gradient by O(1) and is an error of neither)."""
    import torch
    from oracle import nanogpt_oracle as nano

    B, N, E = x.shape
    D = E // H
    p = params
    h = nano.layer_norm(x, p["firstNorm.weights"], p["firstNorm.biases"])
    heads = lambda t: t.reshape(B, N, H, D).transpose(1, 2)
    q, k, v = (heads(nano.project(h, p[f"attention.{n}.weights"], p[f"attention.{n}.biases"]))
               for n in ("query", "key", "value"))
    o = nano.attention_f64(q, k, v, causal).transpose(1, 2).reshape(B, N, E)
    a = nano.project(o, p["attention.output.weights"], p["attention.output.biases"])
    h2 = nano.layer_norm(a, p["secondNorm.weights"], p["secondNorm.biases"])
    m = nano.project(h2, p["mlp.layer_0.weights"], p["mlp.layer_0.biases"]) * relu_mask
    return nano.project(m, p["mlp.layer_2.weights"], p["mlp.layer_2.biases"])


BLOCK_LIB = orc.HERE / "_ref" / "libct_dropin_block.so"


def _block_inputs(B, N, E, mlp_dim):
    rng = np.random.default_rng(B * N + E + mlp_dim)
    shapes = _block_names(E, mlp_dim)
    params = {}
    for name, shp in shapes.items():
        if name.endswith("Norm.weights"):
            params[name] = (1.0 + 0.2 * rng.standard_normal(shp)).astype(np.float32)
        elif name.endswith("biases"):
            params[name] = (0.1 * rng.standard_normal(shp)).astype(np.float32)
        else:
            params[name] = (rng.standard_normal(shp) / np.sqrt(shp[1])).astype(np.float32)
    x = rng.standard_normal((B, N, E)).astype(np.float32)
    dy = rng.standard_normal((B, N, E)).astype(np.float32)
    return params, x, dy


def _run_block(path, params, x, dy, H, mlp_dim, causal):
    """dropin_block_step of the harness at `path`: (rc, message, y, dx,
    hidden, grads, held) -- held: the parameters the block held after its
    setParameters(params)."""
    lib = ctypes.CDLL(str(path))
    fp = ctypes.POINTER(ctypes.c_float)
    I = ctypes.c_int
    lib.dropin_block_step.argtypes = [fp] * 4 + [I] * 7 + [ctypes.POINTER(ctypes.c_char_p),
                                                           ctypes.POINTER(fp), ctypes.POINTER(fp),
                                                           ctypes.POINTER(ctypes.c_longlong), fp]
    lib.dropin_block_step.restype = I
    lib.dropin_last_error.restype = ctypes.c_char_p
    B, N, E = x.shape
    y, dx = np.empty_like(x), np.empty_like(x)
    hidden = np.empty((B, N, mlp_dim), dtype=np.float32)
    names = list(params)
    held = {k: v.copy() for k, v in params.items()}
    grads = {n: np.empty_like(params[n]) for n in names}
    ptr = lambda a: a.ctypes.data_as(fp)
    n = len(names)
    rc = lib.dropin_block_step(ptr(x), ptr(dy), ptr(y), ptr(dx), B, N, E, H, mlp_dim, int(causal), n,
                               (ctypes.c_char_p * n)(*(s.encode() for s in names)),
                               (fp * n)(*(ptr(held[s]) for s in names)), (fp * n)(*(ptr(grads[s]) for s in names)),
                               (ctypes.c_longlong * n)(*(params[s].size for s in names)), ptr(hidden))
    return rc, lib.dropin_last_error().decode(), y, dx, hidden, grads, held


@pytest.mark.skipif(not BLOCK_LIB.exists(), reason="oracle/_ref/libct_dropin_block.so not built (needs the reference tree)")
@pytest.mark.parametrize("B,N,E,H,mlp_dim,causal", [(2, 128, 256, 4, 512, True), (1, 192, 256, 4, 256, False)])
def test_reference_transformer_block_with_dropins(cuda_device, B, N, E, H, mlp_dim, causal):
    """The reference's TransformerBlockLayer<float> forward + backward with
    every sub-layer it builds from a drop-in (LayerNorm, the F3-fixed
    AttentionLayer over the projection and flash-attention drop-ins, the MLP's
    Linear layers; the ReLU is the reference's): y, dx and all 16 parameter
    gradients against fp64 autograd of the same block, at 1e-2
    (max|x - x64| / max|x64|; about seven tf32 GEMM / attention stages in a
    row, each held to 2e-3 by its own tests).  The key-bias gradient is zero
    in exact arithmetic (softmax is shift invariant), so it is held to the
    query-bias gradient's scale.  getGradients() must list the LayerNorm
    gradients, which the reference's LayerNorm lacks.

    The block's setParameters() keeps every parameter given except the
    second LayerNorm's, which stay at their initial scale 1 / shift 0: it
    strips 12 characters from the 11-character prefix "secondNorm."
    (TransformerBlockLayer.cu:159).  The fp64 side uses the parameters the
    block held."""
    import torch

    params, x, dy = _block_inputs(B, N, E, mlp_dim)
    rc, msg, y, dx, hidden, grads, held = _run_block(BLOCK_LIB, params, x, dy, H, mlp_dim, causal)
    assert rc != -2, "getGradients() lacks a parameter getParameters() lists"
    assert rc == 0, msg
    for name in params:
        if name.startswith("secondNorm."):
            assert np.array_equal(held[name], np.full_like(params[name], name.endswith("weights")))
        else:
            assert np.array_equal(held[name], params[name]), name

    tp = {k: torch.tensor(v, dtype=torch.float64, requires_grad=True) for k, v in held.items()}
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    ty = block_fp64(tx, tp, H, causal, torch.tensor(hidden > 0))
    ty.backward(torch.tensor(dy, dtype=torch.float64))
    tol = 1e-2
    errs = {"y": orc.max_rel_err(y, ty.detach().numpy()), "dx": orc.max_rel_err(dx, tx.grad.numpy())}
    for name in params:
        ref = tp[name].grad.numpy()
        if name == "attention.key.biases":
            errs[name] = np.abs(grads[name] - ref).max() / np.abs(tp["attention.query.biases"].grad.numpy()).max()
        else:
            errs[name] = orc.max_rel_err(grads[name], ref)
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, bad


@needs_lib
def test_reference_attention_layer_backward_stops_at_released_output(cuda_device):
    """F3 in place: the same block with the reference's own AttentionLayer
    (libct_dropin.so) runs its forward, and its backward hands the output
    projection the attention output that AttentionLayer::forward released
    (AttentionLayer.cu:88-100, :136).  The output-projection drop-in rejects
    the empty tensor on the host, before any launch (the reference's own
    layer divides by its zero sequence length, OutputProjectionLayer.cu:76-77)."""
    params, x, dy = _block_inputs(1, 128, 256, 256)
    rc, msg, *_ = _run_block(LIB, params, x, dy, 4, 256, True)
    assert rc == -1
    assert "OutputProjectionLayer" in msg, msg


@needs_lib
def test_flash_dropin_step_config2(cuda_device):
    """The C++ FlashAttentionLayer<float> drop-in at BASELINE config 2 (B=8
    H=12 T=1024 D=64, causal), driven the way the reference's AttentionLayer
    drives it (computeAttention with saveStates, computeBackward, clearCache):
    its backward reuses the forward's tf32-rounded q, k, v, so its gradients
    are bitwise those of the Python mirror (which does the same), and its step
    costs at most 6 % more than the bare C-ABI calls (measured 3 %: the
    drop-in adds stream-ordered allocations and one small kernel for the
    reference's max / denominator caches; its cached output shares the
    returned tensor's buffer)."""
    import torch

    from cudatransformer_b200 import FlashAttentionLayer, _lib

    lib = ctypes.CDLL(str(LIB))
    V, I = ctypes.c_void_p, ctypes.c_int
    lib.dropin_flash_step_f32.argtypes = [V] * 8 + [I] * 6 + [ctypes.POINTER(ctypes.c_float)]
    lib.dropin_flash_step_f32.restype = I
    B, H, T, D = 8, 12, 1024, 64
    g = torch.Generator(device=cuda_device).manual_seed(21)
    q, k, v = (torch.randn(B, H, T, D, device=cuda_device, generator=g) * 0.5 for _ in range(3))
    do = torch.randn(B, H, T, D, device=cuda_device, generator=g)
    outs = [torch.empty_like(q) for _ in range(4)]
    ms = ctypes.c_float(0.0)
    rc = lib.dropin_flash_step_f32(*(t.data_ptr() for t in (q, k, v, do, *outs)), B, H, T, D, 1, 20,
                                   ctypes.byref(ms))
    assert rc == 0
    layer = FlashAttentionLayer(D, H, causal=True)
    o = layer.computeAttention(q, k, v, saveStates=True)
    grads = layer.computeBackward(q, k, v, do)
    torch.cuda.synchronize()
    for name, a, b in zip(("o", "dq", "dk", "dv"), outs, [o, *grads]):
        assert torch.equal(a, b), name

    # the bare C-ABI step (forward, backward on the forward's rounded copies)
    code = _lib.CTFA_DTYPE_F32
    clib = _lib.load()
    lse = torch.empty(B, H, T, device=cuda_device)
    fws = torch.empty(clib.ctfa_forward_workspace_bytes(B, H, T, D, code), dtype=torch.uint8, device=cuda_device)
    qb, kb, vb = _lib.rounded_copies(fws, B, H, T, D)
    bws = torch.empty(clib.ctfa_backward_workspace_bytes(B, H, T, D, _lib.CTFA_DTYPE_TF32), dtype=torch.uint8,
                      device=cuda_device)
    st = torch.cuda.current_stream().cuda_stream
    x = [torch.empty_like(q) for _ in range(4)]

    def bare():
        _lib.check(clib.ctfa_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), x[0].data_ptr(), lse.data_ptr(),
                                     B, H, T, D, code, 1, fws.data_ptr(), fws.numel(), st), "fwd")
        _lib.check(clib.ctfa_backward(qb, kb, vb, x[0].data_ptr(), do.data_ptr(), lse.data_ptr(), x[1].data_ptr(),
                                      x[2].data_ptr(), x[3].data_ptr(), bws.data_ptr(), bws.numel(), B, H, T, D,
                                      _lib.CTFA_DTYPE_TF32, 1, st), "bwd")

    bare()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_ev.record()
    for _ in range(20):
        bare()
    e_ev.record()
    torch.cuda.synchronize()
    bare_ms = s_ev.elapsed_time(e_ev) / 20
    print(f"config-2 step: drop-in {ms.value:.4f} ms, bare C ABI {bare_ms:.4f} ms, ratio {ms.value / bare_ms:.3f}")
    assert ms.value < 1.06 * bare_ms, (ms.value, bare_ms)
