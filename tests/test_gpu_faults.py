"""GPU: the bounded-wait path.  A kernel that waits on an mbarrier nothing
arrives on gives up after the limit, records CTFA_ERR_DEVICE_TIMEOUT in the
device error word and exits; the context stays usable.  No trap, no fault,
no unbounded spin."""
import numpy as np
import pytest
import torch

from attn_cases import TOL, errors, oracle_for, run_library
from cudatransformer_b200 import _lib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_survives(cuda_device, ctfa):
    st = torch.cuda.current_stream().cuda_stream
    assert ctfa.ctfa_check_device_error(st) == _lib.CTFA_OK
    status = ctfa.ctfa_selftest_wait_timeout(2_000_000, st)  # 2 ms limit
    assert status == _lib.CTFA_ERR_DEVICE_TIMEOUT, _lib.last_error()
    assert "site 100" in _lib.last_error()
    # the error word was cleared and the context still runs attention correctly
    assert ctfa.ctfa_check_device_error(st) == _lib.CTFA_OK
    q, k, v, do = orc.make_inputs(1, 2, 128, 64, seed=3)
    ours = run_library(q, k, v, do, "bf16", True, cuda_device)
    for name, e in errors(ours, oracle_for(q, k, v, do, "bf16", True)).items():
        assert e < TOL["bf16"], name


def test_layer_rejects_bad_inputs_before_launch(cuda_device):
    from cudatransformer_b200 import FlashAttentionLayer

    layer = FlashAttentionLayer(64, 2)
    q = torch.randn(1, 2, 16, 64, device=cuda_device)
    with pytest.raises(RuntimeError):
        layer.computeAttention(q, q, q[:, :, :8].contiguous())
    with pytest.raises(RuntimeError):
        layer.computeAttention(q.transpose(2, 3), q, q)
    with pytest.raises(RuntimeError):
        FlashAttentionLayer(64, 3).computeAttention(q, q, q)
    big = FlashAttentionLayer(300, 1)
    x = torch.randn(1, 1, 4, 300, device=cuda_device)
    with pytest.raises(_lib.CtfaError) as ei:
        big.computeAttention(x, x, x)
    assert ei.value.status == _lib.CTFA_ERR_UNSUPPORTED


def test_misaligned_tensor_core_input_is_rejected(cuda_device, ctfa):
    B, H, T, D = 1, 1, 32, 64
    buf = torch.zeros(B * H * T * D + 8, device=cuda_device, dtype=torch.bfloat16)
    x = buf[1:1 + B * H * T * D]  # 2-byte offset
    o = torch.empty(B * H * T * D, device=cuda_device, dtype=torch.bfloat16)
    st = torch.cuda.current_stream().cuda_stream
    assert ctfa.ctfa_forward(x.data_ptr(), x.data_ptr(), x.data_ptr(), o.data_ptr(), None, B, H, T, D,
                             _lib.CTFA_DTYPE_BF16, 0, None, 0, st) == _lib.CTFA_ERR_MISALIGNED
