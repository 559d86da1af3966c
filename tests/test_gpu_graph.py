"""GPU: the attention entry points inside a captured CUDA graph.

ctfa_forward and ctfa_backward launch their kernels with programmatic stream
serialization (each kernel may start while its predecessor on the stream
finishes and waits for it before touching memory).  Captured into a CUDA
graph those launches become programmatic graph edges; this checks that a
captured forward + backward, replayed twice, gives bitwise the same outputs
as the same calls run eagerly (the kernels are deterministic).
"""
import pytest
import torch

from cudatransformer_b200 import _lib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TORCH = {"f32": torch.float32, "bf16": torch.bfloat16}
CODE = {"f32": _lib.CTFA_DTYPE_F32, "bf16": _lib.CTFA_DTYPE_BF16}


@pytest.mark.parametrize("kind,shape", [("f32", (2, 3, 300, 64)), ("bf16", (1, 4, 513, 128))])
def test_forward_backward_replayed_from_a_cuda_graph(cuda_device, ctfa, kind, shape):
    B, H, T, D = shape
    code = CODE[kind]
    q, k, v, do = (torch.from_numpy(x).to(cuda_device, TORCH[kind]).contiguous()
                   for x in orc.make_inputs(B, H, T, D, seed=123))
    fws = torch.empty(max(ctfa.ctfa_forward_workspace_bytes(B, H, T, D, code), 256), dtype=torch.uint8,
                      device=cuda_device)
    bws = torch.empty(ctfa.ctfa_backward_workspace_bytes(B, H, T, D, code), dtype=torch.uint8, device=cuda_device)

    def outputs():
        o, dq, dk, dv = (torch.empty_like(q) for _ in range(4))
        lse = torch.empty((B, H, T), dtype=torch.float32, device=cuda_device)
        return o, lse, dq, dk, dv

    def run(bufs, stream):
        o, lse, dq, dk, dv = bufs
        _lib.check(ctfa.ctfa_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), B, H, T,
                                     D, code, 1, fws.data_ptr(), fws.numel(), stream), "ctfa_forward")
        _lib.check(ctfa.ctfa_backward(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                      lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), bws.data_ptr(),
                                      bws.numel(), B, H, T, D, code, 1, stream), "ctfa_backward")

    eager = outputs()
    run(eager, torch.cuda.current_stream().cuda_stream)  # also the first-call set-up, outside any capture
    torch.cuda.synchronize()
    _lib.check(ctfa.ctfa_check_device_error(None), "eager (device)")

    captured = outputs()
    side = torch.cuda.Stream(cuda_device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        run(captured, side.cuda_stream)
    for replay in range(2):
        for t in captured:
            t.fill_(float("nan"))
        graph.replay()
        torch.cuda.synchronize()
        _lib.check(ctfa.ctfa_check_device_error(None), f"replay {replay} (device)")
        for name, a, b in zip(("o", "lse", "dq", "dk", "dv"), captured, eager):
            assert torch.equal(a, b), (kind, replay, name)
    del graph
