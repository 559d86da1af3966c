"""CPU (float64 torch) block compute for the ring-attention schedule tests.
Same contract as cudatransformer_b200.ring_attention.CudaBlockOps; the math
is the exact attention of oracle/oracle.py restricted to one block."""
import math

import torch


def _mask(n, causal, device):
    if not causal:
        return None
    return torch.triu(torch.ones(n, n, dtype=torch.bool, device=device), 1)


class CpuBlockOps:
    def forward_block(self, q, k, v, o_blk, lse_blk, q_row0, k_row0, n, causal):
        D = q.shape[-1]
        qb = q[:, :, q_row0:q_row0 + n].double()
        kb = k[:, :, k_row0:k_row0 + n].double()
        vb = v[:, :, k_row0:k_row0 + n].double()
        s = qb @ kb.transpose(-1, -2) / math.sqrt(D)
        m = _mask(n, causal, q.device)
        if m is not None:
            s = s.masked_fill(m, float("-inf"))
        lse = torch.logsumexp(s, dim=-1)
        o_blk[:, :, q_row0:q_row0 + n] = (torch.exp(s - lse[..., None]) @ vb).to(o_blk.dtype)
        lse_blk[:, :, q_row0:q_row0 + n] = lse.to(lse_blk.dtype)

    def forward_merge(self, q, k, v, o_acc, lse_acc, q_row0, k_row0, n, causal, init):
        o_blk, lse_blk = torch.empty_like(o_acc), torch.empty_like(lse_acc)
        self.forward_block(q, k, v, o_blk, lse_blk, q_row0, k_row0, n, causal)
        self.merge(o_acc, lse_acc, o_blk, lse_blk, q_row0, n, init)

    def merge(self, o_acc, lse_acc, o_blk, lse_blk, row0, n, init):
        sl = slice(row0, row0 + n)
        if init:
            o_acc[:, :, sl] = o_blk[:, :, sl]
            lse_acc[:, :, sl] = lse_blk[:, :, sl]
            return
        l1, l2 = lse_acc[:, :, sl], lse_blk[:, :, sl]
        lse = torch.logaddexp(l1, l2)
        o_acc[:, :, sl] = o_acc[:, :, sl] * torch.exp(l1 - lse)[..., None] + o_blk[:, :, sl] * torch.exp(l2 - lse)[..., None]
        lse_acc[:, :, sl] = lse

    def finalize(self, o_acc, dtype):
        return o_acc.to(dtype)

    def backward_block(self, q, k, v, o, do, lse, dq_acc, dk_acc, dv_acc, q_row0, k_row0, n, causal):
        D = q.shape[-1]
        qs, ks = slice(q_row0, q_row0 + n), slice(k_row0, k_row0 + n)
        qb, kb, vb = q[:, :, qs].double(), k[:, :, ks].double(), v[:, :, ks].double()
        ob, dob, lb = o[:, :, qs].double(), do[:, :, qs].double(), lse[:, :, qs].double()
        scale = 1.0 / math.sqrt(D)
        s = qb @ kb.transpose(-1, -2) * scale
        m = _mask(n, causal, q.device)
        p = torch.exp(s - lb[..., None])
        if m is not None:
            p = p.masked_fill(m, 0.0)
        delta = (ob * dob).sum(-1, keepdim=True)
        ds = p * (dob @ vb.transpose(-1, -2) - delta) * scale
        dq_acc[:, :, qs] += (ds @ kb).to(dq_acc.dtype)
        dk_acc[:, :, ks] += (ds.transpose(-1, -2) @ qb).to(dk_acc.dtype)
        dv_acc[:, :, ks] += (p.transpose(-1, -2) @ dob).to(dv_acc.dtype)
