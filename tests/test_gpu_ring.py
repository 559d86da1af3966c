"""GPU: ring (sequence-parallel) attention.

* single GPU: the ring schedule for G virtual ranks run on one device through
  the block entry points (ctfa_forward_block_merge / ctfa_backward_block /
  ctfa_convert_f32), against fp64 full attention; and the epilogue merge
  against the separate block forward + ctfa_merge_blocks;
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


@pytest.mark.parametrize("D", [64, 128])
def test_epilogue_merge_matches_separate_merge(cuda_device, D):
    """ctfa_forward_block_merge (merge in the kernel's epilogue) against
    ctfa_forward_block + ctfa_merge_blocks on the same blocks: a first block
    (init), a full block and a causal diagonal block folded into the same
    rows, plus rows of a query tile whose causal diagonal leaves early rows
    with few keys."""
    ops = ra.CudaBlockOps()
    B, H, C = 2, 3, 320
    q, k, v, _ = orc.make_inputs(B, H, 3 * C, D, seed=90 + D)
    tq, tk, tv = (torch.from_numpy(x).to(cuda_device, torch.bfloat16) for x in (q, k, v))
    rows = 3 * C
    runs = {}
    for mode in ("fused", "separate"):
        o_acc = torch.zeros((B, H, rows, D), dtype=torch.float32, device=cuda_device)
        lse_acc = torch.full((B, H, rows), float("-inf"), dtype=torch.float32, device=cuda_device)
        o_blk, lse_blk = torch.empty_like(o_acc), torch.empty_like(lse_acc)
        # rows [2C, 3C) see key blocks [0, C) (init), [C, 2C) (full) and [2C, 3C) (causal diagonal)
        for i, (k0, causal) in enumerate([(0, False), (C, False), (2 * C, True)]):
            if mode == "fused":
                ops.forward_merge(tq, tk, tv, o_acc, lse_acc, 2 * C, k0, C, causal, i == 0)
            else:
                ops.forward_block(tq, tk, tv, o_blk, lse_blk, 2 * C, k0, C, causal)
                ops.merge(o_acc, lse_acc, o_blk, lse_blk, 2 * C, C, i == 0)
        torch.cuda.synchronize()
        runs[mode] = (o_acc[:, :, 2 * C:].cpu(), lse_acc[:, :, 2 * C:].cpu())
    (of, lf), (os_, ls_) = runs["fused"], runs["separate"]
    assert torch.allclose(of, os_, rtol=1e-5, atol=1e-6), (of - os_).abs().max()
    assert torch.allclose(lf, ls_, rtol=1e-6, atol=1e-5), (lf - ls_).abs().max()
    # and both are the attention of rows [2C, 3C) over keys [0, 3C) (causal on the last block)
    qq, kk, vv = (orc.round_to(x, "bf16") for x in (q, k, v))
    o_ref, lse_ref = orc.attention_f64(qq, kk, vv, True)
    assert orc.max_rel_err(of.double().numpy(), o_ref[:, :, 2 * C:]) < 1e-2
    assert np.abs(lf.numpy() - lse_ref[:, :, 2 * C:]).max() < 1e-2


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
