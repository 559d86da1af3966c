"""GPU: two attention problems in flight at once on two streams.

The persistent backward kernels take their work items from counters that
live in the caller's workspace (zeroed by the delta pass of the same call),
and the forward keeps no state between launches, so two calls on different
streams with separate workspaces must not interfere.  This runs two problems
forward + backward interleaved on two streams (several rounds, so that their
kernels overlap on the device) and checks every output bitwise against the
same calls run one after the other on one stream (the kernels are
deterministic).
"""
import pytest
import torch

from cudatransformer_b200 import _lib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TORCH = {"f32": torch.float32, "bf16": torch.bfloat16}
CODE = {"f32": _lib.CTFA_DTYPE_F32, "bf16": _lib.CTFA_DTYPE_BF16}


class Problem:
    def __init__(self, ctfa, dev, kind, shape, seed):
        self.lib, self.kind = ctfa, kind
        self.B, self.H, self.T, self.D = shape
        self.code = CODE[kind]
        self.q, self.k, self.v, self.do = (torch.from_numpy(x).to(dev, TORCH[kind]).contiguous()
                                           for x in orc.make_inputs(*shape, seed=seed))
        n = ctfa.ctfa_forward_workspace_bytes(*shape, self.code)
        self.fws = torch.empty(max(n, 256), dtype=torch.uint8, device=dev)
        self.bws = torch.empty(ctfa.ctfa_backward_workspace_bytes(*shape, self.code), dtype=torch.uint8,
                               device=dev)
        self.out = [torch.empty_like(self.q) for _ in range(4)]
        self.lse = torch.empty((self.B, self.H, self.T), dtype=torch.float32, device=dev)

    def run(self, stream):
        o, dq, dk, dv = self.out
        dims = (self.B, self.H, self.T, self.D, self.code, 1)
        _lib.check(self.lib.ctfa_forward(self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), o.data_ptr(),
                                         self.lse.data_ptr(), *dims, self.fws.data_ptr(), self.fws.numel(), stream),
                   "ctfa_forward")
        _lib.check(self.lib.ctfa_backward(self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), o.data_ptr(),
                                          self.do.data_ptr(), self.lse.data_ptr(), dq.data_ptr(), dk.data_ptr(),
                                          dv.data_ptr(), self.bws.data_ptr(), self.bws.numel(), *dims, stream),
                   "ctfa_backward")

    def results(self):
        return [t.clone() for t in self.out] + [self.lse.clone()]


@pytest.mark.parametrize("kind", ["f32", "bf16"])
def test_two_streams_with_separate_workspaces(cuda_device, ctfa, kind):
    # more (tile, head) items than SMs in each, so both persistent grids are
    # busy claiming items while the other stream's kernels run
    a = Problem(ctfa, cuda_device, kind, (2, 40, 520, 64), seed=71)
    b = Problem(ctfa, cuda_device, kind, (1, 36, 1030, 64), seed=72)
    main = torch.cuda.current_stream(cuda_device)
    a.run(main.cuda_stream)
    b.run(main.cuda_stream)
    torch.cuda.synchronize(cuda_device)
    _lib.check(ctfa.ctfa_check_device_error(None), "serial (device)")
    ref_a, ref_b = a.results(), b.results()

    s1, s2 = torch.cuda.Stream(cuda_device), torch.cuda.Stream(cuda_device)
    for rnd in range(4):
        for t in a.out + b.out:
            t.fill_(float("nan"))
        torch.cuda.synchronize(cuda_device)
        a.run(s1.cuda_stream)
        b.run(s2.cuda_stream)
        torch.cuda.synchronize(cuda_device)
        _lib.check(ctfa.ctfa_check_device_error(None), f"round {rnd} (device)")
        for name, x, y in zip(("o", "dq", "dk", "dv", "lse"), a.results(), ref_a):
            assert torch.equal(x, y), (kind, rnd, "a", name)
        for name, x, y in zip(("o", "dq", "dk", "dv", "lse"), b.results(), ref_b):
            assert torch.equal(x, y), (kind, rnd, "b", name)
