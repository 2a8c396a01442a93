"""Seeded synthetic MoE layers with the reference's benchmark shapes.

The reference measures on synthetic data only (random router, N(0, 0.02)
weights, random activations; e.g. MBR/phase13_decode_revalidate.py:35-50), so
these generators stand in for its inputs. Draw order from one torch.Generator:
router logits, w13, w2, hidden.

Configurations (name -> shape):
  tiny    M=16, H=256,  I=128,  E=8,   top-2, softmax router   (CPU-runnable)
  glm     M=64, H=6144, I=2048, E=256, top-8, sigmoid router   (decode)
  any other M with the glm layer via make_layer(..., M=...).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, Optional

import torch


@dataclass(frozen=True)
class LayerShape:
    M: int
    H: int
    I: int
    E: int
    topk: int
    scoring: str = "sigmoid"   # router: "softmax" or "sigmoid", then top-k and renormalise
    hot_experts: int = 0       # skewed router: +hot_bias on the logits of experts [0, hot_experts)
    hot_bias: float = 2.0


TINY = LayerShape(M=16, H=256, I=128, E=8, topk=2, scoring="softmax")
GLM_DECODE = LayerShape(M=64, H=6144, I=2048, E=256, topk=8, scoring="sigmoid")


def glm(M: int, hot_experts: int = 0) -> LayerShape:
    return LayerShape(M=M, H=6144, I=2048, E=256, topk=8, scoring="sigmoid", hot_experts=hot_experts)


@dataclass
class Layer:
    shape: LayerShape
    hidden: torch.Tensor          # (M, H) bf16
    topk_weights: torch.Tensor    # (M, topk) f32
    topk_ids: torch.Tensor        # (M, topk) int32
    w13: torch.Tensor             # (E, 2I, H) e4m3
    w13_scale: torch.Tensor       # (E, 2I/128, H/128) f32
    w2: torch.Tensor              # (E, H, I) e4m3
    w2_scale: torch.Tensor        # (E, H/128, I/128) f32
    extra: dict = field(default_factory=dict)


def make_router(logits: torch.Tensor, topk: int, scoring: str):
    scores = torch.softmax(logits.float(), dim=-1) if scoring == "softmax" else torch.sigmoid(logits.float())
    w, ids = torch.topk(scores, topk, dim=-1)
    w = w / w.sum(dim=-1, keepdim=True)
    return w.float().contiguous(), ids.to(torch.int32).contiguous()


def make_layer(shape: LayerShape, quant_fn: Callable, seed: int = 0, device="cpu",
               keep_bf16_weights: bool = False, weight_chunk: int = 16) -> Layer:
    """Builds one layer. quant_fn(w_bf16 (e, N, K)) -> (q e4m3, s f32) quantises
    weights 128x128 (the library's per_block_quant_fp8 on a GPU). Weights are drawn
    `weight_chunk` experts at a time so that only fp8 copies stay resident."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    s = shape
    logits = torch.randn(s.M, s.E, generator=g, device=dev)
    if s.hot_experts:
        logits[:, : s.hot_experts] += s.hot_bias
    topk_w, topk_ids = make_router(logits, s.topk, s.scoring)

    def draw(N, K):
        qs, ss, raws = [], [], []
        for e0 in range(0, s.E, weight_chunk):
            n = min(weight_chunk, s.E - e0)
            w = (torch.randn(n, N, K, generator=g, device=dev) * 0.02).to(torch.bfloat16)
            q, sc = quant_fn(w)
            qs.append(q)
            ss.append(sc)
            if keep_bf16_weights:
                raws.append(w)
        return torch.cat(qs), torch.cat(ss), (torch.cat(raws) if keep_bf16_weights else None)

    w13, w13_s, w13_raw = draw(2 * s.I, s.H)
    w2, w2_s, w2_raw = draw(s.H, s.I)
    hidden = torch.randn(s.M, s.H, generator=g, device=dev).to(torch.bfloat16)
    layer = Layer(s, hidden, topk_w, topk_ids, w13, w13_s, w2, w2_s)
    if keep_bf16_weights:
        layer.extra["w13_bf16"] = w13_raw
        layer.extra["w2_bf16"] = w2_raw
    return layer


def active_experts(topk_ids: torch.Tensor, num_experts: int) -> int:
    ids = topk_ids.reshape(-1)
    ids = ids[(ids >= 0) & (ids < num_experts)]
    return int(torch.unique(ids).numel())


def weight_bytes_per_expert(H: int, I: int) -> int:
    """fp8 bytes of w13 + w2 for one expert."""
    return 2 * I * H + H * I


def scale_bytes_per_expert(H: int, I: int) -> int:
    return 4 * ((2 * I // 128) * (H // 128) + (H // 128) * (I // 128))
