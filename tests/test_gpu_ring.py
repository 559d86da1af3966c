"""GPU: ring (sequence-parallel) attention.

* single GPU: the ring schedule for G virtual ranks run on one device through
  the block entry points (ctfa_forward_block / ctfa_merge_blocks /
  ctfa_backward_block / ctfa_convert_f32), against fp64 full attention;
* two or more GPUs: the real ring (one process per GPU, NCCL send/recv of K/V
  and dK/dV), gathered and checked the same way.  Skipped with one GPU.
Tolerance: bf16 I/O, max|x - x64| / max|x64| < 1e-2.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cudatransformer_b200 import ring_attention as ra
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _reference(q, k, v, do):
    q, k, v, do = (orc.round_to(x, "bf16") for x in (q, k, v, do))
    o, lse = orc.attention_f64(q, k, v, True)
    dq, dk, dv = orc.attention_backward_f64(q, k, v, do, True)
    return dict(o=o, lse=lse, dq=dq, dk=dk, dv=dv)


@pytest.mark.parametrize("world,T,D", [(2, 512, 128), (4, 1024, 64), (3, 768, 128)])
def test_emulated_ring_block_kernels(cuda_device, world, T, D):
    q, k, v, do = orc.make_inputs(1, 2, T, D, seed=31 + world)
    tq, tk, tv, tdo = (torch.from_numpy(x).to(cuda_device, torch.bfloat16) for x in (q, k, v, do))
    o, lse, dq, dk, dv = ra.ring_attention_emulated(tq, tk, tv, tdo, world)
    torch.cuda.synchronize()
    ref = _reference(q, k, v, do)
    got = dict(o=o, dq=dq, dk=dk, dv=dv)
    for name, x in got.items():
        assert orc.max_rel_err(x.double().cpu().numpy(), ref[name]) < 1e-2, name
    assert np.abs(lse.cpu().numpy() - ref["lse"]).max() < 1e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, T, D, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        q, k, v, do = orc.make_inputs(1, 2, T, D, seed=57)
        loc = [ra.shard_zigzag(torch.from_numpy(x), world, rank).to(f"cuda:{rank}", torch.bfloat16)
               for x in (q, k, v, do)]
        ring = ra.RingAttention()
        o, lse = ring.forward(loc[0], loc[1], loc[2])
        dq, dk, dv = ring.backward(loc[0], loc[1], loc[2], o, lse, loc[3])
        torch.cuda.synchronize()
        out_q.put((rank, [t.double().cpu().numpy() for t in (o, dq, dk, dv)]))
    finally:
        dist.destroy_process_group()


def test_nccl_ring_across_gpus():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    world = min(n, 4)
    T, D = 1024, 128
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, T, D, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(out_q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = {name: ra.unshard_zigzag([torch.from_numpy(results[r][i]) for r in range(world)]).numpy()
           for i, name in enumerate(("o", "dq", "dk", "dv"))}
    ref = _reference(*orc.make_inputs(1, 2, T, D, seed=57))
    for name, x in got.items():
        assert orc.max_rel_err(x, ref[name]) < 1e-2, name
