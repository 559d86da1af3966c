"""GPU parity: libctfa_b200.so (through the FlashAttentionLayer mirror and the
C ABI) against the fp64 oracle on the same seeded, dtype-rounded inputs.

Tolerance (max|x - x64| / max|x64| per output): 2e-3 for fp32 I/O (tf32 MMA),
1e-2 for bf16 / fp16, 1e-9 for fp64 (SIMT).
"""
import numpy as np
import pytest
import torch

from attn_cases import TOL, attention_f64_device, errors, oracle_for, per_head_errors, run_library
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TC_SHAPES = [  # (B, H, T, D): tensor-core head dims; T covers partial tiles and T < one tile
    (1, 2, 1, 64),
    (1, 2, 48, 64),
    (2, 3, 128, 64),
    (1, 2, 130, 64),
    (2, 2, 300, 128),
    (1, 3, 513, 64),
    (1, 2, 256, 128),
]


@pytest.mark.parametrize("kind", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("shape", TC_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_tensor_core_forward_backward(cuda_device, kind, causal, shape):
    B, H, T, D = shape
    q, k, v, do = orc.make_inputs(B, H, T, D, seed=100 + T + D)
    ours = run_library(q, k, v, do, kind, causal, cuda_device)
    ref = oracle_for(q, k, v, do, kind, causal)
    err = errors(ours, ref)
    for name, e in err.items():
        assert e < TOL[kind], (name, e, err)
    # lse is fp32 in every mode
    assert np.abs(ours["lse"] - ref["lse"]).max() < 1e-3 * max(1.0, np.abs(ref["lse"]).max())


@pytest.mark.parametrize("kind,D", [("f64", 64), ("f64", 128), ("f32", 32), ("bf16", 80), ("f32", 128)])
@pytest.mark.parametrize("causal", [False, True])
def test_simt_paths(cuda_device, kind, D, causal):
    """fp64 and head dims off the tensor-core path run the SIMT kernels (fp32
    D=128 backward too: it does not fit the tensor-core backward's smem)."""
    B, H, T = 1, 2, 70
    q, k, v, do = orc.make_inputs(B, H, T, D, seed=7 + D)
    ours = run_library(q, k, v, do, kind, causal, cuda_device)
    ref = oracle_for(q, k, v, do, kind, causal)
    tol = TOL[kind] if kind != "f32" else 1e-4  # SIMT fp32 does not round to tf32
    if kind == "f32" and D == 128:
        tol = TOL["f32"]  # the fp32 D=128 forward is tensor-core (tf32)
    for name, e in errors(ours, ref).items():
        assert e < (max(tol, 1e-6) if name == "lse" else tol), (name, e)  # lse is fp32 in every mode


@pytest.mark.parametrize("causal", [False, True])
def test_config1_against_golden(cuda_device, golden, causal):
    """BASELINE config 1 (fp32, B=2 H=4 T=128 D=64, seed 0) vs the torch-SDPA
    golden fixture."""
    q, k, v, do = orc.make_inputs(2, 4, 128, 64, seed=0)
    ours = run_library(q, k, v, do, "f32", causal, cuda_device)
    key = f"cfg1_{'c' if causal else 'nc'}"
    for name in ("o", "dq", "dk", "dv"):
        idx = golden[f"{key}/{name}/idx"]
        val = golden[f"{key}/{name}/val"]
        flat = ours[name].reshape(-1)
        assert orc.max_rel_err(flat[idx], val) < TOL["f32"], name
        s = float(golden[f"{key}/{name}/sumsq"])
        assert abs((flat * flat).sum() / s - 1) < 1e-2, name


def _full_check(ours, q, k, v, do, kind, causal, pinned_heads):
    """Every (batch, head) problem of a full-size configuration against an
    fp64 restatement run on the GPU (attn_cases.attention_f64_device); that
    restatement is first pinned to the CPU oracle on `pinned_heads`.  The
    persistent backward kernels hand (key tile, head) and (query tile, head)
    items to CTAs heavy-first, so a scheduling or indexing fault could hit any
    head: all of them are compared, for o, lse, dq, dk and dv."""
    dev = ours["o"].device
    rq, rk, rv, rdo = (orc.round_to(x, kind) for x in (q, k, v, do))
    ref = attention_f64_device(*(torch.from_numpy(x).to(dev) for x in (rq, rk, rv, rdo)), causal)
    for b, h in pinned_heads:
        sl = (slice(b, b + 1), slice(h, h + 1))
        cpu = oracle_for(q[sl], k[sl], v[sl], do[sl], kind, causal)
        for name in ("o", "lse", "dq", "dk", "dv"):
            got = ref[name][sl].cpu().numpy()
            assert np.abs(got - cpu[name]).max() <= 1e-9 * max(1.0, np.abs(cpu[name]).max()), (b, h, name)
    errs = per_head_errors(ours, ref)
    for name, e in errs.items():
        worst = float(e.max())
        bh = divmod(int(e.argmax()), e.shape[1])
        assert worst < TOL[kind], (name, worst, "worst (batch, head)", bh)
    lse_err = (ours["lse"].to(torch.float64) - ref["lse"]).abs().max().item()
    assert lse_err < 1e-3 * max(1.0, ref["lse"].abs().max().item()), lse_err


def test_config2_gpt2_small_shape(cuda_device):
    """causal, fp32 I/O, B=8 H=12 T=1024 D=64, q/k/v ~ 0.5 N(0,1), seed 1:
    all 96 (batch, head) problems."""
    q, k, v, do = orc.make_inputs(8, 12, 1024, 64, seed=1, qkv_scale=0.5)
    ours = run_library(q, k, v, do, "f32", True, cuda_device, keep_torch=True)
    _full_check(ours, q, k, v, do, "f32", True, [(0, 0), (3, 7), (7, 11)])


def test_config3_bf16_d128(cuda_device):
    """causal, bf16 I/O, B=16 H=16 T=2048 D=128, dO ~ N(0, 0.1^2), seed 2:
    all 256 (batch, head) problems."""
    q, k, v, do = orc.make_inputs(16, 16, 2048, 128, seed=2, do_scale=0.1)
    ours = run_library(q, k, v, do, "bf16", True, cuda_device, keep_torch=True)
    _full_check(ours, q, k, v, do, "bf16", True, [(0, 0), (15, 15)])


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_many_heads_multi_wave(cuda_device, kind):
    """More (key tile, head) items than SMs, with ragged T, so that every
    persistent CTA walks several items of different lengths (a multi-wave
    schedule), causal and not; every head checked against the fp64 oracle."""
    B, H, T, D = 3, 40, 333, 64
    q, k, v, do = orc.make_inputs(B, H, T, D, seed=31)
    for causal in (True, False):
        ours = run_library(q, k, v, do, kind, causal, cuda_device, keep_torch=True)
        _full_check(ours, q, k, v, do, kind, causal, [(0, 0), (2, 39)])


@pytest.mark.parametrize("kind,shape", [("f32", (5, 15, 2048, 64)), ("bf16", (1, 36, 4096, 128))])
def test_head_chunked_order_with_a_partial_last_chunk(cuda_device, kind, shape):
    """Heads whose streamed operands exceed 64 MiB together are walked in
    chunks of 16 MiB worth of heads (fp32 D=64 T=2048: 16 heads of 1 MiB, 75
    heads = four chunks and one of 11; bf16 D=128 T=4096: 8 heads of 2 MiB, 36
    heads = four chunks and one of 4), and the persistent backward kernels
    claim those items dynamically: every head checked, causal and not."""
    B, H, T, D = shape
    q, k, v, do = orc.make_inputs(B, H, T, D, seed=41, do_scale=0.1)
    for causal in (True, False):
        ours = run_library(q, k, v, do, kind, causal, cuda_device, keep_torch=True)
        _full_check(ours, q, k, v, do, kind, causal, [(0, 0), (B - 1, H - 1)])


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_deterministic(cuda_device, kind):
    """No atomics anywhere: two runs are bitwise identical."""
    q, k, v, do = orc.make_inputs(2, 4, 384, 64, seed=5)
    a = run_library(q, k, v, do, kind, True, cuda_device)
    b = run_library(q, k, v, do, kind, True, cuda_device)
    for name in a:
        assert np.array_equal(a[name], b[name]), name


def test_outputs_do_not_write_past_their_rows(cuda_device, ctfa):
    """Canary words around o/dq/dk/dv survive forward + backward (T not a tile multiple)."""
    from cudatransformer_b200 import _lib

    B, H, T, D = 1, 2, 200, 128
    n = B * H * T * D
    pad = 4096
    q, k, v, do = (torch.randn(B, H, T, D, device=cuda_device, dtype=torch.bfloat16) for _ in range(4))
    bufs = {name: torch.full((n + 2 * pad,), 7.0, device=cuda_device, dtype=torch.bfloat16)
            for name in ("o", "dq", "dk", "dv")}
    views = {name: buf[pad:pad + n] for name, buf in bufs.items()}
    lse = torch.empty(B * H * T, device=cuda_device, dtype=torch.float32)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(ctfa.ctfa_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), views["o"].data_ptr(), lse.data_ptr(),
                                 B, H, T, D, _lib.CTFA_DTYPE_BF16, 1, None, 0, st), "fwd")
    ws = torch.empty(ctfa.ctfa_backward_workspace_bytes(B, H, T, D, _lib.CTFA_DTYPE_BF16), dtype=torch.uint8,
                     device=cuda_device)
    _lib.check(ctfa.ctfa_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), views["o"].data_ptr(), do.data_ptr(),
                                  lse.data_ptr(), views["dq"].data_ptr(), views["dk"].data_ptr(),
                                  views["dv"].data_ptr(), ws.data_ptr(), ws.numel(), B, H, T, D,
                                  _lib.CTFA_DTYPE_BF16, 1, st), "bwd")
    _lib.check(ctfa.ctfa_check_device_error(st), "device")
    for name, buf in bufs.items():
        assert bool((buf[:pad] == 7.0).all()) and bool((buf[pad + n:] == 7.0).all()), name


def test_layer_cache_semantics(cuda_device):
    """saveStates caches lse in cachedMaxScores and ones in cachedDenominators
    (so exp(s - max)/denom is still the softmax); backward without a cache
    recomputes the forward (FlashAttentionLayer.cu:114-127)."""
    from cudatransformer_b200 import FlashAttentionLayer

    q, k, v, do = (torch.randn(1, 2, 96, 64, device=cuda_device) for _ in range(4))
    layer = FlashAttentionLayer(64, 2, causal=True)
    o = layer.computeAttention(q, k, v, saveStates=True)
    assert layer.cachedBatchSize == 1 and layer.cachedSequenceLength == 96
    assert torch.equal(layer.cachedOutput, o) and layer.cachedOutput.data_ptr() != o.data_ptr()
    assert torch.allclose(layer.cachedMaxScores, layer.cachedLSE) and bool((layer.cachedDenominators == 1).all())
    g_cached = layer.computeBackward(q, k, v, do)
    layer.clearCache()
    assert layer.cachedOutput is None and layer.cachedMaxScores is None
    g_recomputed = layer.computeBackward(q, k, v, do)
    for a, b in zip(g_cached, g_recomputed):
        assert torch.equal(a, b)


def test_fp32_backward_reuses_forward_rounding(cuda_device, ctfa):
    """The layer hands the forward's tf32-rounded q/k/v to the backward as
    CTFA_DTYPE_TF32; results are bitwise those of a plain fp32 backward."""
    from cudatransformer_b200 import FlashAttentionLayer, _lib

    q, k, v, do = (torch.randn(2, 3, 200, 64, device=cuda_device) for _ in range(4))
    layer = FlashAttentionLayer(64, 3, causal=True)
    layer.computeAttention(q, k, v, saveStates=True)
    assert layer._cachedRounded is not None
    reused = layer.computeBackward(q, k, v, do)
    o, lse = layer.cachedOutput, layer.cachedLSE
    B, H, T, D = q.shape
    ws = torch.empty(ctfa.ctfa_backward_workspace_bytes(B, H, T, D, _lib.CTFA_DTYPE_F32), dtype=torch.uint8,
                     device=cuda_device)
    plain = [torch.empty_like(q) for _ in range(3)]
    _lib.check(ctfa.ctfa_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                  lse.data_ptr(), *(t.data_ptr() for t in plain), ws.data_ptr(), ws.numel(),
                                  B, H, T, D, _lib.CTFA_DTYPE_F32, 1, torch.cuda.current_stream().cuda_stream),
               "ctfa_backward")
    for a, b in zip(reused, plain):
        assert torch.equal(a, b)
    q.add_(0)  # bumps the version counter: the cache no longer matches
    layer.computeBackward(q, k, v, do)


@pytest.mark.parametrize("T,D,causal", [(700, 64, True), (700, 64, False), (513, 128, True), (1024, 64, True)])
def test_fp32_forward_writes_exact_rounded_copies(cuda_device, ctfa, T, D, causal):
    """The fp32 forward rounds q/k/v to tf32 inside the kernel and stores the
    rounded tiles (Q by every CTA, each K/V tile by one designated CTA) into
    its workspace for the backward: every element must equal the
    round-to-nearest-away tf32 value of the input, with no tile missing."""
    from cudatransformer_b200 import _lib

    B, H = 2, 3
    q, k, v = (torch.randn(B, H, T, D, device=cuda_device) for _ in range(3))
    o = torch.empty_like(q)
    lse = torch.empty(B, H, T, device=cuda_device)
    n = ctfa.ctfa_forward_workspace_bytes(B, H, T, D, _lib.CTFA_DTYPE_F32)
    ws = torch.full((n,), 0x7F, dtype=torch.uint8, device=cuda_device)  # NaN-like poison
    _lib.check(ctfa.ctfa_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, H, T, D,
                                 _lib.CTFA_DTYPE_F32, int(causal), ws.data_ptr(), n,
                                 torch.cuda.current_stream().cuda_stream), "ctfa_forward")
    torch.cuda.synchronize()
    a = (B * H * T * D * 4 + 255) // 256 * 256
    for i, x in enumerate((q, k, v)):
        got = ws[i * a:i * a + x.numel() * 4].view(torch.int32).view(B, H, T, D)
        want = (x.contiguous().view(torch.int32) + 0x1000) & ~0x1FFF
        assert torch.equal(got, want), f"rounded copy {i} differs"
