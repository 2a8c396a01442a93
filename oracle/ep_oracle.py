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

    def dispatch(self, q, s, topk_ids, topk_weights, num_experts, G, rows_per_rank, send, pos, tok_of, counts, err):
        M, H = q.shape
        topk = topk_ids.shape[1]
        per = num_experts // G
        rb = row_bytes(H, topk)
        buf = send.view(G * rows_per_rank, rb)
        ids = topk_ids.numpy()
        owner = np.where((ids >= 0) & (ids < num_experts), ids // per, -1)
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
                local = np.where(mine, ids[t] - d * per, -1).astype(np.int32)
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
