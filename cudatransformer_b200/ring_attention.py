"""Sequence-parallel ("ring") causal attention across torch.distributed ranks.

No counterpart in the reference, which runs one device and streams one
sequence's keys through shared memory (flash_attention.cu:97).  This is the
long-context path (sequence sharded over G GPUs, K/V blocks exchanged with
NCCL send/recv over NVLink while each rank computes on the block it holds).

Partition (zig-zag, balances the causal triangle): the sequence of length T
is cut into 2G chunks of C = T / (2G) rows; rank r holds chunks r and 2G-1-r
of q, k, v, o and their gradients as local tensors [B, H, 2C, D] (local rows
[0, C) = chunk r, [C, 2C) = chunk 2G-1-r).

Forward, step s = 0..G-1: rank r holds the k/v of rank src = (r - s) mod G.
For each local query chunk a and held key chunk b (global chunk ids): b < a
is a full block, b == a the causal diagonal, b > a is skipped.  Each block's
normalised output and logsumexp are folded into fp32 accumulators with a
logsumexp-weighted merge, done in the block kernel's epilogue
(ctfa_forward_block_merge: no per-block partial goes through HBM).  The next
k/v block is sent/received (one batched NCCL send+recv) while the current one
is computed.

Backward: the same schedule; dq accumulates locally, dK/dV contributions for
the held block accumulate in a fresh buffer, are added to the partial sums
received from the previous rank and sent on; after G steps every rank has
received the complete dK/dV of its own chunks.  Posting order per neighbour
pair is identical on both sides (k/v at the start of steps 0..G-2, dK/dV at
the end of steps 0..G-1), so NCCL matches every message.

The per-block compute is an injected ``ops`` object: ``CudaBlockOps`` calls
the tcgen05 kernels through the C ABI (ctfa_forward_block_merge,
ctfa_backward_block, ctfa_convert_f32); tests plug in a CPU implementation to
check the schedule on gloo ranks.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib


# ---------------------------------------------------------------------------
# partition helpers
# ---------------------------------------------------------------------------
def zigzag_chunks(world: int, rank: int) -> tuple[int, int]:
    return rank, 2 * world - 1 - rank


def shard_zigzag(x: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    """[B, H, T, D] (or [B, H, T]) -> this rank's [B, H, 2C, ...] local rows."""
    T = x.shape[2]
    assert T % (2 * world) == 0, "sequence length must split into 2*world chunks"
    C = T // (2 * world)
    a, b = zigzag_chunks(world, rank)
    return torch.cat([x[:, :, a * C:(a + 1) * C], x[:, :, b * C:(b + 1) * C]], dim=2).contiguous()


def unshard_zigzag(parts: list[torch.Tensor]) -> torch.Tensor:
    """Inverse of shard_zigzag given every rank's local tensor (rank order)."""
    world = len(parts)
    C = parts[0].shape[2] // 2
    chunks = [None] * (2 * world)
    for r, x in enumerate(parts):
        a, b = zigzag_chunks(world, r)
        chunks[a] = x[:, :, :C]
        chunks[b] = x[:, :, C:]
    return torch.cat(chunks, dim=2)


def block_plan(world: int, rank: int, step: int):
    """(local q chunk, local kv chunk, causal) blocks computed at `step`."""
    src = (rank - step) % world
    q_ids = zigzag_chunks(world, rank)
    kv_ids = zigzag_chunks(world, src)
    plan = []
    for a_loc, ga in enumerate(q_ids):
        for b_loc, gb in enumerate(kv_ids):
            if gb <= ga:
                plan.append((a_loc, b_loc, gb == ga))
    return plan


# ---------------------------------------------------------------------------
# per-block compute on the tensor cores (C ABI)
# ---------------------------------------------------------------------------
_CODES = {torch.bfloat16: _lib.CTFA_DTYPE_BF16, torch.float16: _lib.CTFA_DTYPE_F16}


class CudaBlockOps:
    """Block compute through libctfa_b200.so (bf16 / fp16, head dim 64 / 128)."""

    def __init__(self):
        self.lib = _lib.load()
        self._ws = None  # backward block workspace, kept across blocks and calls

    @staticmethod
    def _stream(t):
        return torch.cuda.current_stream(t.device).cuda_stream

    def forward_block(self, q, k, v, o_blk, lse_blk, q_row0, k_row0, n, causal):
        B, H, rows, D = q.shape
        _lib.check(self.lib.ctfa_forward_block(q.data_ptr(), k.data_ptr(), v.data_ptr(), o_blk.data_ptr(),
                                               lse_blk.data_ptr(), B, H, D, _CODES[q.dtype], rows, q_row0, n,
                                               k.shape[2], k_row0, n, int(causal), 0, self._stream(q)),
                   "ctfa_forward_block")

    def forward_merge(self, q, k, v, o_acc, lse_acc, q_row0, k_row0, n, causal, init):
        """Block forward folded into the running (o_acc, lse_acc) rows in the
        kernel's epilogue (init: the rows' first block, overwritten)."""
        B, H, rows, D = q.shape
        _lib.check(self.lib.ctfa_forward_block_merge(q.data_ptr(), k.data_ptr(), v.data_ptr(), o_acc.data_ptr(),
                                                     lse_acc.data_ptr(), B, H, D, _CODES[q.dtype], rows, q_row0, n,
                                                     k.shape[2], k_row0, n, int(causal), 0, int(init),
                                                     self._stream(q)), "ctfa_forward_block_merge")

    def merge(self, o_acc, lse_acc, o_blk, lse_blk, row0, n, init):
        B, H, rows, D = o_acc.shape
        _lib.check(self.lib.ctfa_merge_blocks(o_acc.data_ptr(), lse_acc.data_ptr(), o_blk.data_ptr(),
                                              lse_blk.data_ptr(), B, H, D, rows, row0, n, int(init),
                                              self._stream(o_acc)), "ctfa_merge_blocks")

    def finalize(self, o_acc, dtype):
        out = torch.empty(o_acc.shape, dtype=dtype, device=o_acc.device)
        _lib.check(self.lib.ctfa_convert_f32(o_acc.data_ptr(), out.data_ptr(), _CODES[dtype], o_acc.numel(),
                                             self._stream(o_acc)), "ctfa_convert_f32")
        return out

    def backward_block(self, q, k, v, o, do, lse, dq_acc, dk_acc, dv_acc, q_row0, k_row0, n, causal):
        B, H, rows, D = q.shape
        code = _CODES[q.dtype]
        ws_bytes = max(self.lib.ctfa_backward_block_workspace_bytes(B, H, n, D, code), 256)
        if self._ws is None or self._ws.device != q.device or self._ws.numel() < ws_bytes:
            self._ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
        ws = self._ws  # stream-ordered reuse: the blocks run one after another on one stream
        _lib.check(self.lib.ctfa_backward_block(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(),
                                                lse.data_ptr(), dq_acc.data_ptr(), dk_acc.data_ptr(), dv_acc.data_ptr(),
                                                ws.data_ptr(), ws.numel(), B, H, D, code, rows, q_row0, n,
                                                k.shape[2], k_row0, n, int(causal), 0, self._stream(q)),
                   "ctfa_backward_block")


# ---------------------------------------------------------------------------
# the ring
# ---------------------------------------------------------------------------
class RingAttention:
    """Causal attention over a zig-zag sharded sequence.

    forward(q, k, v) -> (o, lse) and backward(q, k, v, o, lse, do) -> (dq, dk, dv)
    on this rank's local [B, H, 2C, D] tensors.
    """

    def __init__(self, group=None, ops=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.next = dist.get_global_rank(group, (self.rank + 1) % self.world) if group is not None else (
            self.rank + 1) % self.world
        self.prev = dist.get_global_rank(group, (self.rank - 1) % self.world) if group is not None else (
            self.rank - 1) % self.world
        self.ops = ops if ops is not None else CudaBlockOps()

    def _exchange(self, send, recv):
        if self.world == 1:
            return []
        ops = [dist.P2POp(dist.isend, send, self.next, self.group),
               dist.P2POp(dist.irecv, recv, self.prev, self.group)]
        return dist.batch_isend_irecv(ops)

    def forward(self, q, k, v):
        B, H, rows, D = q.shape
        C = rows // 2
        o_acc = torch.zeros((B, H, rows, D), dtype=torch.float32, device=q.device)
        lse_acc = torch.full((B, H, rows), float("-inf"), dtype=torch.float32, device=q.device)
        kv = torch.stack([k, v])
        kv_next = torch.empty_like(kv)
        seen = [False, False]
        for step in range(self.world):
            reqs = self._exchange(kv, kv_next) if step + 1 < self.world else []
            for a_loc, b_loc, causal in block_plan(self.world, self.rank, step):
                self.ops.forward_merge(q, kv[0], kv[1], o_acc, lse_acc, a_loc * C, b_loc * C, C, causal,
                                       not seen[a_loc])
                seen[a_loc] = True
            for r in reqs:
                r.wait()
            kv, kv_next = kv_next, kv
        return self.ops.finalize(o_acc, q.dtype), lse_acc

    def backward(self, q, k, v, o, lse, do):
        B, H, rows, D = q.shape
        C = rows // 2
        dq_acc = torch.zeros((B, H, rows, D), dtype=torch.float32, device=q.device)
        kv = torch.stack([k, v])
        kv_next = torch.empty_like(kv)
        dkv_out = [torch.empty((2, B, H, rows, D), dtype=torch.float32, device=q.device) for _ in range(2)]
        dkv_in = torch.empty((2, B, H, rows, D), dtype=torch.float32, device=q.device)
        dkv_reqs = []
        for step in range(self.world):
            kv_reqs = self._exchange(kv, kv_next) if step + 1 < self.world else []
            local = dkv_out[step % 2]
            local.zero_()
            for a_loc, b_loc, causal in block_plan(self.world, self.rank, step):
                self.ops.backward_block(q, kv[0], kv[1], o, do, lse, dq_acc, local[0], local[1],
                                        a_loc * C, b_loc * C, C, causal)
            if step > 0:
                for r in dkv_reqs:
                    r.wait()
                local += dkv_in
            dkv_reqs = self._exchange(local, dkv_in)
            for r in kv_reqs:
                r.wait()
            kv, kv_next = kv_next, kv
        for r in dkv_reqs:
            r.wait()
        if self.world == 1:
            dkv_in = dkv_out[0]
        dq = self.ops.finalize(dq_acc, q.dtype)
        dk = self.ops.finalize(dkv_in[0].contiguous(), q.dtype)
        dv = self.ops.finalize(dkv_in[1].contiguous(), q.dtype)
        return dq, dk, dv


def ring_attention_emulated(q, k, v, do, world: int, ops=None):
    """The ring schedule for `world` virtual ranks on one device (no
    communication): every block each rank would compute, merged the same way.
    q, k, v, do: full [B, H, T, D].  Returns full (o, lse, dq, dk, dv)."""
    ops = ops if ops is not None else CudaBlockOps()
    B, H, T, D = q.shape
    C = T // (2 * world)
    loc = [[shard_zigzag(x, world, r) for r in range(world)] for x in (q, k, v, do)]
    qs, ks, vs, dos = loc
    outs, lses = [], []
    for r in range(world):
        o_acc = torch.zeros((B, H, 2 * C, D), dtype=torch.float32, device=q.device)
        lse_acc = torch.full((B, H, 2 * C), float("-inf"), dtype=torch.float32, device=q.device)
        seen = [False, False]
        for step in range(world):
            src = (r - step) % world
            for a_loc, b_loc, causal in block_plan(world, r, step):
                ops.forward_merge(qs[r], ks[src], vs[src], o_acc, lse_acc, a_loc * C, b_loc * C, C, causal,
                                  not seen[a_loc])
                seen[a_loc] = True
        outs.append(ops.finalize(o_acc, q.dtype))
        lses.append(lse_acc)
    dq_acc = [torch.zeros((B, H, 2 * C, D), dtype=torch.float32, device=q.device) for _ in range(world)]
    dk_acc = [torch.zeros_like(dq_acc[0]) for _ in range(world)]
    dv_acc = [torch.zeros_like(dq_acc[0]) for _ in range(world)]
    for r in range(world):
        for step in range(world):
            src = (r - step) % world
            for a_loc, b_loc, causal in block_plan(world, r, step):
                ops.backward_block(qs[r], ks[src], vs[src], outs[r], dos[r], lses[r], dq_acc[r], dk_acc[src],
                                   dv_acc[src], a_loc * C, b_loc * C, C, causal)
    fin = lambda accs: unshard_zigzag([ops.finalize(a, q.dtype) for a in accs])
    lse_full = unshard_zigzag([x.unsqueeze(-1) for x in lses])[..., 0]
    return unshard_zigzag(outs), lse_full, fin(dq_acc), fin(dk_acc), fin(dv_acc)
