"""CPU, multi-process: the ring-attention schedule (zig-zag partition, block
plan, logsumexp merge, K/V rotation and dK/dV forwarding through
torch.distributed send/recv) on gloo ranks, with the exact float64 block
compute of tests/ring_cpu_ops.py, against full-sequence attention."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cudatransformer_b200 import ring_attention as ra
from oracle import oracle as orc

B, H, T, D = 1, 2, 48, 16


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from ring_cpu_ops import CpuBlockOps

        q, k, v, do = (torch.from_numpy(x) for x in orc.make_inputs(B, H, T, D, seed=9))
        loc = [ra.shard_zigzag(x, world, rank) for x in (q, k, v, do)]
        ring = ra.RingAttention(ops=CpuBlockOps())
        o, lse = ring.forward(loc[0], loc[1], loc[2])
        dq, dk, dv = ring.backward(loc[0], loc[1], loc[2], o, lse, loc[3])
        out_q.put((rank, [t.numpy() for t in (o, lse.double(), dq, dk, dv)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_ring_schedule_on_gloo_ranks(world):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(out_q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    parts = [[torch.from_numpy(results[r][i]) for r in range(world)] for i in range(5)]
    o, dq, dk, dv = (ra.unshard_zigzag(parts[i]).numpy() for i in (0, 2, 3, 4))
    lse = ra.unshard_zigzag([x.unsqueeze(-1) for x in parts[1]])[..., 0].numpy()
    q, k, v, do = orc.make_inputs(B, H, T, D, seed=9)
    ro, rlse = orc.attention_f64(q, k, v, True)
    rdq, rdk, rdv = orc.attention_backward_f64(q, k, v, do, True)
    for name, x, r in (("o", o, ro), ("lse", lse, rlse), ("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
        assert orc.max_rel_err(x, r) < 1e-5, name


def test_block_plan_covers_the_causal_triangle_once():
    for world in (1, 2, 3, 4, 8):
        seen = set()
        work = []
        for r in range(world):
            per_rank = 0
            for step in range(world):
                src = (r - step) % world
                qi, ki = ra.zigzag_chunks(world, r), ra.zigzag_chunks(world, src)
                for a, b, causal in ra.block_plan(world, r, step):
                    pair = (qi[a], ki[b])
                    assert pair not in seen
                    assert causal == (pair[0] == pair[1])
                    seen.add(pair)
                    per_rank += 0.5 if causal else 1.0
            work.append(per_rank)
        n = 2 * world
        assert seen == {(a, b) for a in range(n) for b in range(n) if b <= a}
        assert max(work) == min(work)  # zig-zag balances the causal work


def test_emulated_ring_on_cpu_matches_full_attention():
    from ring_cpu_ops import CpuBlockOps

    q, k, v, do = (torch.from_numpy(x) for x in orc.make_inputs(1, 2, 64, 16, seed=4))
    o, lse, dq, dk, dv = ra.ring_attention_emulated(q, k, v, do, world=4, ops=CpuBlockOps())
    ro, rlse = orc.attention_f64(q.numpy(), k.numpy(), v.numpy(), True)
    grads = orc.attention_backward_f64(q.numpy(), k.numpy(), v.numpy(), do.numpy(), True)
    assert orc.max_rel_err(o.numpy(), ro) < 1e-6
    assert orc.max_rel_err(lse.numpy(), rlse) < 1e-6
    for x, r in zip((dq, dk, dv), grads):
        assert orc.max_rel_err(x.numpy(), r) < 1e-6
