"""GPU: ctfa_backward_noalloc, the backward entry point that allocates nothing.

Callers that cannot allocate device memory while they run (a host that has
handed all device memory to its own pool, or one that cannot take the
synchronisation cudaMalloc may imply) use it; its scratch is a static device
array inside the library.  The kernels are deterministic, so it must give
bitwise the same gradients as ctfa_backward with a caller workspace, on
repeated calls (the array keeps the previous call's contents), on the
tensor-core and the SIMT paths (fp32 at head dim 128 takes the SIMT backward,
which keeps its delta rows in the same array), causal and not; it must not
change the device's free memory; and it must refuse problems whose scratch
would not fit.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest
import torch

from attn_cases import TOL
from cudatransformer_b200 import _lib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

# name -> (dtype, (B, H, T, D), causal)
CASES = {
    "bf16": ("bf16", (2, 4, 300, 128), 1),
    "f32": ("f32", (1, 3, 200, 64), 1),
    "f16": ("f16", (1, 2, 130, 64), 1),
    "f32_noncausal": ("f32", (1, 2, 257, 64), 0),
    "f32_d128_simt": ("f32", (1, 2, 140, 128), 1),
}
TORCH = {"bf16": torch.bfloat16, "f32": torch.float32, "f16": torch.float16}
CODE = {"bf16": _lib.CTFA_DTYPE_BF16, "f32": _lib.CTFA_DTYPE_F32, "f16": _lib.CTFA_DTYPE_F16}


def _inputs(shape, kind, device):
    q, k, v, do = orc.make_inputs(*shape, seed=77)
    return [torch.from_numpy(x).to(device, TORCH[kind]).contiguous() for x in (q, k, v, do)]


@pytest.mark.parametrize("case", sorted(CASES))
def test_noalloc_backward_matches_workspace_backward(cuda_device, ctfa, case):
    kind, (B, H, T, D), causal = CASES[case]
    code = CODE[kind]
    q, k, v, do = _inputs((B, H, T, D), kind, cuda_device)
    st = torch.cuda.current_stream().cuda_stream
    o = torch.empty_like(q)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=cuda_device)
    fws_n = ctfa.ctfa_forward_workspace_bytes(B, H, T, D, code)
    fws = torch.empty(max(fws_n, 256), dtype=torch.uint8, device=cuda_device)
    _lib.check(ctfa.ctfa_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, H, T,
                                 D, code, causal, fws.data_ptr(), fws.numel(), st), "ctfa_forward")
    # the existing entry point, with a caller-provided workspace
    ws = torch.empty(ctfa.ctfa_backward_workspace_bytes(B, H, T, D, code), dtype=torch.uint8, device=cuda_device)
    want = [torch.empty_like(q) for _ in range(3)]
    _lib.check(ctfa.ctfa_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                  lse.data_ptr(), *(t.data_ptr() for t in want), ws.data_ptr(), ws.numel(),
                                  B, H, T, D, code, causal, st), "ctfa_backward")
    # two calls in a row of the entry point that allocates nothing
    got = [[torch.full_like(q, float("nan")) for _ in range(3)] for _ in range(2)]
    torch.cuda.synchronize()
    for call in range(2):
        if call == 1:  # after the first call's set-up, the device's free memory must not move
            free_before = torch.cuda.mem_get_info()[0]
        _lib.check(ctfa.ctfa_backward_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                                              do.data_ptr(), lse.data_ptr(), *(t.data_ptr() for t in got[call]),
                                              B, H, T, D, code, causal, st), f"ctfa_backward_noalloc call {call}")
        _lib.check(ctfa.ctfa_check_device_error(st), f"ctfa_backward_noalloc call {call} (device)")
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free_before, "ctfa_backward_noalloc changed free device memory"
    for call in range(2):
        for name, g, w in zip(("dq", "dk", "dv"), got[call], want):
            assert torch.equal(g, w), (case, call, name, orc.max_rel_err(g.double().cpu().numpy(),
                                                                        w.double().cpu().numpy()))
    # and both equal the fp64 oracle within the usual tolerance
    qn, kn, vn, don = (t.double().cpu().numpy() for t in (q, k, v, do))
    ref = orc.attention_backward_f64(qn, kn, vn, don, bool(causal))
    for name, g, r in zip(("dq", "dk", "dv"), got[1], ref):
        assert orc.max_rel_err(g.double().cpu().numpy(), r) < TOL[kind], (case, name)


def test_noalloc_backward_rejects_problems_above_the_static_scratch(ctfa):
    # fp32, D=64: scratch = delta + 4 rounded operand copies, far above 32 MiB here
    B, H, T, D = 8, 12, 4096, 64
    need = ctfa.ctfa_backward_workspace_bytes(B, H, T, D, _lib.CTFA_DTYPE_F32)
    assert need > _lib.CTFA_NOALLOC_SCRATCH_BYTES
    fake = 4096  # never dereferenced: the size check fails first
    status = ctfa.ctfa_backward_noalloc(*([fake] * 9), B, H, T, D, _lib.CTFA_DTYPE_F32, 1, None)
    assert status == _lib.CTFA_ERR_WORKSPACE
    assert "static scratch" in _lib.last_error()
