"""CPU restatement of the expert-parallel steps - TEST INFRASTRUCTURE ONLY.

Same contract and byte layout as the CUDA path (include/b200moe.h,
b200moe_ep_dispatch / b200moe_layer_packed / b200moe_ep_combine), so the rank
orchestration of trials_b200.ep.ExpertParallelMoE can run on CPU gloo ranks
in tests. The layer math is oracle.moe_oracle.moe_layer.
"""
from __future__ import annotations

import numpy as np
import torch

from . import moe_oracle as orc


def target(table, slots: int, num_experts: int, src_rank: int, expert: int, t: int, j: int, topk: int) -> int:
    """Physical slot of routed slot (t, j) (the dispatch's replica choice,
    include/b200moe.h): the replica on the sending rank if there is one,
    else replica (t*topk + j) mod n; table None = expert e in slot e."""
    if expert < 0 or expert >= num_experts:
        return -1
    if table is None:
        return expert
    n = int(table[expert][0])
    reps = [int(p) for p in table[expert][1:1 + n]]
    for p in reps:
        if p // slots == src_rank:
            return p
    return reps[(t * topk + j) % n]


def row_bytes(H: int, topk: int) -> int:
    n = H + (H // 128) * 4 + 8 * topk
    return (n + 15) // 16 * 16


class OracleEPOps:
    """Drop-in for trials_b200.ep.CudaEPOps on CPU tensors."""

    def row_bytes(self, H, topk):
        return row_bytes(H, topk)

    def quant(self, hidden, q, s):
        qq, ss = orc.per_token_group_quant_fp8(hidden)
        q.copy_(qq)
        s.copy_(ss)

    def dispatch(self, q, s, topk_ids, topk_weights, num_experts, G, rows_per_rank, send, pos, tok_of, counts, err,
                 rank=0, placement=None):
        M, H = q.shape
        topk = topk_ids.shape[1]
        table, slots = None, num_experts // G
        if placement is not None:
            table, slots = placement[0].cpu().numpy(), placement[1].slots
        rb = row_bytes(H, topk)
        buf = send.view(G * rows_per_rank, rb)
        ids = topk_ids.numpy()
        phys = np.array([[target(table, slots, num_experts, rank, int(ids[t, j]), t, j, topk) for j in range(topk)]
                         for t in range(M)], dtype=np.int64).reshape(M, topk)
        owner = np.where(phys >= 0, phys // slots, -1)
        pos_np = np.full((M, G), -1, dtype=np.int32)
        for d in range(G):
            need = np.nonzero((owner == d).any(axis=1))[0]
            n = min(len(need), rows_per_rank)
            counts[d] = n
            for r in range(rows_per_rank):
                row = buf[d * rows_per_rank + r]
                meta = row[H + (H // 128) * 4:].view(torch.int32)
                if r >= n:
                    meta[:topk] = -1
                    meta[topk:2 * topk] = 0
                    continue
                t = int(need[r])
                pos_np[t, d] = r
                tok_of[d * rows_per_rank + r] = t
                row[:H] = q[t].view(torch.uint8)
                row[H:H + (H // 128) * 4] = s[t].contiguous().view(torch.uint8)
                mine = owner[t] == d
                local = np.where(mine, phys[t] - d * slots, -1).astype(np.int32)
                wts = np.where(mine, topk_weights[t].numpy(), 0.0).astype(np.float32)
                meta[:topk] = torch.from_numpy(local)
                meta[topk:2 * topk] = torch.from_numpy(wts).view(torch.int32)
        pos.copy_(torch.from_numpy(pos_np.reshape(-1)))

    def workspace_bytes(self, R, H, I, E_local, topk):
        return 256

    def layer_packed(self, rows, R, H, I, E_local, topk, w13, w13_scale, w2, w2_scale, out, ws, num_ranks=1):
        rb = row_bytes(H, topk)
        buf = rows.view(R, rb)
        q = buf[:, :H].contiguous().view(torch.float8_e4m3fn)
        s = buf[:, H:H + (H // 128) * 4].contiguous().view(torch.float32)
        meta = buf[:, H + (H // 128) * 4:H + (H // 128) * 4 + 8 * topk].contiguous().view(torch.int32)
        ids = meta[:, :topk].contiguous()
        w = meta[:, topk:].contiguous().view(torch.float32)
        hidden = torch.zeros(R, H, dtype=torch.bfloat16)
        res = orc.moe_layer(hidden, w13, w13_scale, w2, w2_scale, w, ids, a1=(q, s))
        out.copy_(res)

    def combine(self, returned, pos, M, H, G, rows_per_rank, out):
        p = pos.view(M, G)
        acc = torch.zeros(M, H, dtype=torch.float32)
        for d in range(G):
            for t in range(M):
                r = int(p[t, d])
                if r >= 0:
                    acc[t] += returned[d * rows_per_rank + r].float()
        out.copy_(acc.to(torch.bfloat16))
