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
