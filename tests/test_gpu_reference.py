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
