"""CPU oracle for the FP8 128x128 block-scaled MoE layer - TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU, the reference algorithm of the hot path so
that tests can check the CUDA kernels against it. Nothing in the product
package imports it; only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline use it.

Parity pin: tests/test_oracle_golden.py checks every function here against
fixtures produced by running the reference's own code (its Triton kernels in
the Triton CPU interpreter and its torch helpers) with
tests/golden/make_golden.py.

Functions follow these reference sources (paths inside the reference repo):
  * per_token_group_quant_fp8  - phase5_orchestrator.py:26-32
  * per_block_quant_fp8        - phase5_orchestrator.py:35-41
  * moe_align_block_size       - ordering of build_routing_from_topk
                                 (phase5_orchestrator.py:51-57, stable argsort
                                 of flat ids) with the per-expert block padding,
                                 sentinel and capacity of sglang's
                                 moe_align_block_size as used at
                                 sglang_integration/aiter.py:113-123
  * blockscaled_gemm           - aiter_module/moe_decode_megakernel.py:71-81
  * silu_mul_interleaved       - sglang_integration/aiter.py:145-148,
                                 phase5_orchestrator.py:44-48
  * moe_layer                  - sglang_integration/aiter.py:74-177 (quantise
                                 -> GEMM1 -> SiLU*up -> quantise -> GEMM2 ->
                                 weighted unpermute and top-k sum)

Rounding modes of moe_layer:
  * "exact": the rounding points of the CUDA kernels - fp32 GEMM results go
    straight into SiLU*up, inter is re-quantised from fp32, the weighted
    rows are summed in fp32 and rounded to bf16 once.
  * "reference": the rounding points of the reference orchestrator - GEMM1 and
    GEMM2 outputs rounded to bf16, SiLU and the product in bf16, router weight
    applied as a bf16 product (aiter.py:138-177).
"""
from __future__ import annotations

import numpy as np
import torch

FP8_MAX = 448.0
GROUP = 128


# ----------------------------------------------------------------------------
# Quantisation
# ----------------------------------------------------------------------------
# Both quantisers run on the CPU whatever the input device: torch's CUDA kernels
# evaluate "tensor / python scalar" as a multiplication by the reciprocal, which
# is not the IEEE division the reference's formula (evaluated on the CPU) uses,
# and a one-ulp change of a scale flips fp8 roundings.
def per_token_group_quant_fp8(x: torch.Tensor, gk: int = GROUP):
    """(M, K) -> (q e4m3 (M, K), s fp32 (M, K/gk)). phase5_orchestrator.py:26-32."""
    dev = x.device
    x = x.cpu()
    M, K = x.shape
    xg = x.reshape(M, K // gk, gk)
    amax = xg.abs().amax(dim=-1).float()
    scale = (amax / FP8_MAX).clamp(min=1e-12)
    q = (xg.float() / scale.unsqueeze(-1)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).reshape(M, K)
    return q.to(dev), scale.to(dev)


def per_block_quant_fp8(w: torch.Tensor, bn: int = GROUP, bk: int = GROUP):
    """(E, N, K) -> (q e4m3, s fp32 (E, N/bn, K/bk)). phase5_orchestrator.py:35-41."""
    dev = w.device
    w = w.cpu()
    E, N, K = w.shape
    wg = w.reshape(E, N // bn, bn, K // bk, bk)
    amax = wg.abs().amax(dim=(2, 4)).float()
    scale = (amax / FP8_MAX).clamp(min=1e-12)
    q = (wg.float() / scale.unsqueeze(2).unsqueeze(4)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q.reshape(E, N, K).to(dev), scale.to(dev)


def dequant_rows(q: torch.Tensor, s: torch.Tensor, dtype=torch.float64):
    """1x128 dequantisation of (M, K) with scales (M, K/128)."""
    M, K = q.shape
    return (q.to(dtype).reshape(M, K // GROUP, GROUP) * s.to(dtype).unsqueeze(-1)).reshape(M, K)


def dequant_blocks(q: torch.Tensor, s: torch.Tensor, dtype=torch.float64):
    """128x128 dequantisation of (..., N, K) with scales (..., N/128, K/128)."""
    N, K = q.shape[-2:]
    lead = q.shape[:-2]
    qq = q.to(dtype).reshape(*lead, N // GROUP, GROUP, K // GROUP, GROUP)
    return (qq * s.to(dtype).unsqueeze(-1).unsqueeze(-3)).reshape(*lead, N, K)


# ----------------------------------------------------------------------------
# Routing
# ----------------------------------------------------------------------------
def align_capacity_rows(numel: int, num_experts: int, block_m: int) -> int:
    return numel + (num_experts + 1) * (block_m - 1)


def map_ids(topk_ids: np.ndarray, num_experts: int, expert_map=None, num_local: int | None = None):
    """Flat ids -> weight index or -1 (dropped); also returns a bad-id flag."""
    ids = np.asarray(topk_ids, dtype=np.int64).reshape(-1)
    bad = ((ids < -1) | (ids >= num_experts)).any()
    valid = (ids >= 0) & (ids < num_experts)
    out = np.full(ids.shape, -1, dtype=np.int64)
    if expert_map is None:
        out[valid] = ids[valid]
    else:
        em = np.asarray(expert_map, dtype=np.int64)
        m = np.where(valid, em[np.clip(ids, 0, num_experts - 1)], -1)
        E = num_local if num_local is not None else int(em.max()) + 1
        bad = bad or ((m >= E).any())
        m[m >= E] = -1
        out = m
    return out, bool(bad)


def moe_align_block_size(topk_ids, block_m: int, num_experts: int, expert_map=None, num_local=None):
    """Reference-format routing.

    Returns (sorted_token_ids (cap,), expert_ids (cap_blocks,), ntp) as int32
    numpy arrays / int. Flat ids ascending inside each expert; experts in id
    order; each padded to a multiple of block_m with sentinel M*topk; blocks
    past ntp/block_m have expert id -1.
    """
    ids = np.asarray(topk_ids)
    numel = ids.size
    E = num_local if expert_map is not None else num_experts
    mapped, _ = map_ids(ids, num_experts, expert_map, num_local)
    cap = align_capacity_rows(numel, E, block_m)
    cap_blocks = -(-cap // block_m)
    sorted_ids = np.full(cap, numel, dtype=np.int32)
    expert_ids = np.full(cap_blocks, -1, dtype=np.int32)
    keep = np.nonzero(mapped >= 0)[0]
    order = keep[np.argsort(mapped[keep], kind="stable")]
    counts = np.bincount(mapped[keep], minlength=E) if keep.size else np.zeros(E, dtype=np.int64)
    padded = -(-counts // block_m) * block_m
    base = np.concatenate([[0], np.cumsum(padded)])
    pos = 0
    for e in range(E):
        c = int(counts[e])
        sorted_ids[base[e]:base[e] + c] = order[pos:pos + c]
        expert_ids[base[e] // block_m: base[e + 1] // block_m] = e
        pos += c
    return sorted_ids, expert_ids, int(base[E])


def route_chunks(topk_ids, num_experts: int, tile_tokens: int, expert_map=None, num_local=None):
    """The GEMM work list: align with block 16, then each expert's rows cut into
    ceil(rows / tile_tokens) nearly equal chunks (multiples of 16)."""
    sorted_ids, expert_ids, ntp = moe_align_block_size(topk_ids, 16, num_experts, expert_map, num_local)
    E = num_local if expert_map is not None else num_experts
    chunks = []
    blocks_per_expert = np.bincount(expert_ids[expert_ids >= 0], minlength=E)
    row = 0
    for e in range(E):
        nb = int(blocks_per_expert[e])
        if nb == 0:
            continue
        P = nb * 16
        nc = -(-P // tile_tokens)
        per, extra = divmod(nb, nc)
        for c in range(nc):
            r = (per + (1 if c < extra else 0)) * 16
            chunks.append((e, row, r))
            row += r
    return sorted_ids, ntp, np.array(chunks, dtype=np.int32).reshape(-1, 3)


# ----------------------------------------------------------------------------
# GEMM and activation
# ----------------------------------------------------------------------------
def blockscaled_gemm(a_q, a_s, w_q, w_s, dtype=torch.float64):
    """C = sum_kb (A_kb W_kb^T) * a_s[:, kb] * w_s[n/128, kb]
    (aiter_module/moe_decode_megakernel.py:71-81). Exact fp8 products and
    a wide accumulator make this equal to dequantise-then-matmul."""
    return dequant_rows(a_q, a_s, dtype) @ dequant_blocks(w_q, w_s, dtype).T


def silu_mul_interleaved(c: torch.Tensor):
    """inter[:, j] = silu(c[:, 2j]) * c[:, 2j+1] (gate/up interleaved)."""
    gate, up = c[:, 0::2], c[:, 1::2]
    return torch.nn.functional.silu(gate) * up


def _bf16(x):
    return x.to(torch.bfloat16)


def bf16_truncate(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 by dropping the low 16 bits (round toward zero): the cast
    the Triton CPU interpreter applies for acc.to(tl.bfloat16), which the
    golden fixtures were produced with. GPUs round to nearest even."""
    i = x.float().contiguous().view(torch.int32)
    return (i & ~0xFFFF).view(torch.float32).to(torch.bfloat16)


def moe_layer(hidden, w13_q, w13_s, w2_q, w2_s, topk_weights, topk_ids, *, rounding: str = "exact",
              expert_map=None, num_local=None, stage2_a_by_token: bool = False, dtype=torch.float64,
              return_stages: bool = False, gemm_cast=_bf16, a1=None):
    """Full layer on the CPU (or any torch device), expert by expert.

    gemm_cast: fp32 -> bf16 cast of the GEMM outputs in "reference" rounding
    (bf16_truncate reproduces the Triton CPU interpreter).
    a1=(q, s) gives the 1x128-quantised activations directly (hidden is then
    only used for its shape and device).
    stage2_a_by_token=True plants the reference's historic A_BY_SORTED bug
    (stage-2 activations read by token index instead of by routed row,
    MBR/phase13_findings.md:21-25); used only to show the parity gate rejects it.
    """
    assert rounding in ("exact", "reference")
    M, H = hidden.shape
    topk = topk_ids.shape[1]
    E_ids = w13_q.shape[0] if expert_map is None else len(expert_map)
    mapped, _ = map_ids(topk_ids.cpu().numpy(), E_ids, expert_map, num_local)
    a1_q, a1_s = per_token_group_quant_fp8(hidden) if a1 is None else a1
    flat_w = topk_weights.reshape(-1)
    out = torch.zeros(M * topk, H, dtype=torch.float32, device=hidden.device)
    stages = {"gemm1": {}, "inter": {}, "a2": {}, "gemm2": {}}
    inter_by_pair = {}
    for e in np.unique(mapped[mapped >= 0]):
        pairs = np.nonzero(mapped == e)[0]
        toks = torch.as_tensor(pairs // topk, device=hidden.device)
        g1 = blockscaled_gemm(a1_q[toks], a1_s[toks], w13_q[e], w13_s[e], dtype)
        if rounding == "reference":
            g1 = gemm_cast(g1)
            inter = _bf16(torch.nn.functional.silu(g1[:, 0::2]) * g1[:, 1::2])
        else:
            inter = silu_mul_interleaved(g1.float())
        a2_q, a2_s = per_token_group_quant_fp8(inter)
        for i, pr in enumerate(pairs):
            inter_by_pair[int(pr)] = (a2_q[i], a2_s[i])
        stages["gemm1"][int(e)] = g1
        stages["inter"][int(e)] = inter
        stages["a2"][int(e)] = (a2_q, a2_s)
    if stage2_a_by_token:
        sorted_ref = moe_align_block_size(topk_ids.cpu().numpy(), 128, E_ids, expert_map, num_local)[0]
    for e in np.unique(mapped[mapped >= 0]):
        pairs = np.nonzero(mapped == e)[0]
        if stage2_a_by_token:
            # Wrong rows, as in the bug: the sorted activation matrix is read at row
            # index t = f // topk (the token) instead of at the routed row of f.
            zero = (torch.zeros_like(a1_q[0, :w2_q.shape[2]]), torch.zeros_like(a1_s[0, :w2_q.shape[2] // GROUP]))
            rows = []
            for pr in pairs:
                src = int(sorted_ref[int(pr) // topk])
                rows.append(inter_by_pair.get(src, zero) if src < M * topk else zero)
        else:
            rows = [inter_by_pair[int(pr)] for pr in pairs]
        a2_q = torch.stack([r[0] for r in rows])
        a2_s = torch.stack([r[1] for r in rows])
        g2 = blockscaled_gemm(a2_q, a2_s, w2_q[e], w2_s[e], dtype)
        wts = flat_w[torch.as_tensor(pairs, device=hidden.device)]
        if rounding == "reference":
            g2 = gemm_cast(g2)
            weighted = (g2 * _bf16(wts).unsqueeze(1)).float()
        else:
            weighted = (g2.float() * wts.float().unsqueeze(1))
        stages["gemm2"][int(e)] = g2
        out[torch.as_tensor(pairs, device=hidden.device)] = weighted
    res = out.view(M, topk, H).sum(dim=1).to(torch.bfloat16)
    if return_stages:
        return res, stages
    return res


def moe_layer_fp32_unquantized_act(hidden, w13_q, w13_s, w2_q, w2_s, topk_weights, topk_ids):
    """fp32 layer on dequantised weights without activation quantisation: the
    per-token loop of MBR/phase13_decode_revalidate.py:23-32 evaluated expert by
    expert, with fp8 weights dequantised to fp32."""
    M, H = hidden.shape
    topk = topk_ids.shape[1]
    ids = topk_ids.reshape(-1).cpu().numpy()
    out = torch.zeros(M * topk, H, dtype=torch.float32)
    hf = hidden.float()
    for e in np.unique(ids[ids >= 0]):
        pairs = np.nonzero(ids == e)[0]
        x = hf[torch.as_tensor(pairs // topk)]
        w13 = dequant_blocks(w13_q[e], w13_s[e], torch.float32)
        w2 = dequant_blocks(w2_q[e], w2_s[e], torch.float32)
        inter = silu_mul_interleaved(x @ w13.T)
        out[torch.as_tensor(pairs)] = (inter @ w2.T) * topk_weights.reshape(-1)[torch.as_tensor(pairs)].float()[:, None]
    return out.view(M, topk, H).sum(1).to(torch.bfloat16)


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a = a.double().cpu()
    b = b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


# ----------------------------------------------------------------------------
# Router
# ----------------------------------------------------------------------------
def router_topk(logits, topk: int, scoring: str = "softmax", correction_bias=None, renormalize: bool = True,
                scaling: float = 1.0):
    """float64 restatement of the router (GLM sigmoid routing,
    measure_xcd_imbalance.py:50-55; softmax top-k of the tiny configuration).
    Returns (weights (M, k) f64, ids (M, k) int64, margin (M,) f64): ids in
    descending selection value, ties -> lower id; margin = relative gap between
    the k-th and (k+1)-th selection values (tiny margins are ambiguous in fp32)."""
    x = np.asarray(logits, dtype=np.float64)
    M, E = x.shape
    if scoring == "softmax":
        p = np.exp(x - x.max(axis=1, keepdims=True))
        p /= p.sum(axis=1, keepdims=True)
        sel = x
    else:
        p = 1.0 / (1.0 + np.exp(-x))
        sel = p + (np.asarray(correction_bias, dtype=np.float64)[None, :] if correction_bias is not None else 0.0)
    order = np.lexsort((np.broadcast_to(np.arange(E), (M, E)), -sel), axis=1)
    ids = order[:, :topk]
    w = np.take_along_axis(p, ids, axis=1)
    if renormalize:
        w = w / w.sum(axis=1, keepdims=True)
    w = w * scaling
    srt = np.take_along_axis(sel, order, axis=1)
    if topk < E:
        margin = np.abs(srt[:, topk - 1] - srt[:, topk]) / np.maximum(np.abs(srt[:, topk - 1]), 1e-30)
    else:
        margin = np.full(M, np.inf)
    return w, ids, margin
