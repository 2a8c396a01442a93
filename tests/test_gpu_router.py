"""Router kernel (b200moe_router_topk) against the float64 oracle router."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from trials_b200 import moe, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]

AMBIGUOUS = 1e-5  # relative gap at the k-th position below which fp32 may order differently


@pytest.mark.parametrize("M,E,k,scoring,bias,dtype,scale", [
    (16, 8, 2, "softmax", False, torch.float32, 1.0),
    (300, 256, 8, "sigmoid", False, torch.float32, 1.0),
    (300, 256, 8, "sigmoid", True, torch.float32, 2.5),
    (129, 1024, 16, "softmax", False, torch.float32, 1.0),
    (77, 60, 4, "sigmoid", True, torch.bfloat16, 1.0),
    (5, 256, 8, "softmax", False, torch.bfloat16, 1.0),
])
def test_router_matches_oracle(cuda_device, M, E, k, scoring, bias, dtype, scale):
    g = torch.Generator().manual_seed(M * E + k)
    logits = (torch.randn(M, E, generator=g) * 2).to(dtype)
    b = (torch.randn(E, generator=g) * 0.1) if bias else None
    w, ids = moe.select_experts(logits.to(cuda_device), k, scoring, None if b is None else b.to(cuda_device),
                                renormalize=True, routed_scaling_factor=scale)
    rw, rids, margin = orc.router_topk(logits.float().numpy(), k, scoring, None if b is None else b.numpy(),
                                       True, scale)
    ids = ids.cpu().numpy()
    w = w.cpu().numpy()
    clear = margin > AMBIGUOUS
    assert clear.mean() > 0.95
    assert np.array_equal(ids[clear], rids[clear])
    assert np.allclose(w[clear], rw[clear], rtol=2e-5, atol=1e-7)
    # every row is a set of k distinct valid experts
    assert all(len(set(r)) == k for r in ids) and ids.min() >= 0 and ids.max() < E


def test_router_feeds_the_layer(cuda_device):
    """select_experts reproduces the synthetic generator's router (torch
    sigmoid + topk + renormalise) for the GLM-shaped router."""
    g = torch.Generator(device=cuda_device).manual_seed(0)
    logits = torch.randn(64, 256, generator=g, device=cuda_device)
    tw_ref, ids_ref = synth.make_router(logits, 8, "sigmoid")
    tw, ids = moe.select_experts(logits, 8, "sigmoid")
    assert torch.equal(ids, ids_ref)
    assert torch.allclose(tw, tw_ref, rtol=1e-5, atol=1e-7)


# Routing from router logits (router inside routing's first launch): every
# output equals select_experts followed by route(), bit for bit, on the
# one-launch path (below 16,384 routed slots: the last router CTA routes) and
# the multi-CTA path (from 16,384: each CTA routes the tokens it counts).
@pytest.mark.parametrize("M,E,k,scoring,bias,dtype,scale,tile", [
    (1, 256, 8, "sigmoid", False, torch.bfloat16, 1.0, 32),
    (64, 256, 8, "sigmoid", True, torch.float32, 2.5, 32),
    (16, 8, 2, "softmax", False, torch.float32, 1.0, 16),
    (1000, 256, 8, "sigmoid", False, torch.float32, 1.0, 64),
    (300, 1024, 16, "softmax", False, torch.float32, 1.0, 32),
    (2047, 256, 8, "softmax", False, torch.float32, 1.0, 128),
    (2048, 256, 8, "sigmoid", True, torch.bfloat16, 1.0, 128),
    (8192, 256, 8, "sigmoid", True, torch.float32, 2.5, 128),
    (5000, 96, 6, "sigmoid", False, torch.float32, 1.0, 128),
])
def test_route_logits_equals_router_then_route(cuda_device, M, E, k, scoring, bias, dtype, scale, tile):
    from trials_b200 import stages

    g = torch.Generator().manual_seed(M + E + k)
    logits = (torch.randn(M, E, generator=g) * 2).to(dtype).to(cuda_device)
    b = (torch.randn(E, generator=g) * 0.1).to(cuda_device) if bias else None
    w_ref, ids_ref = moe.select_experts(logits, k, scoring, b, renormalize=True, routed_scaling_factor=scale)
    r_ref = stages.route(ids_ref, E, tile)
    for _ in range(2):  # the router's CTA counter is left at zero for the next call
        r, w, ids = stages.route_logits(logits, k, tile, scoring, b, True, scale)
        assert torch.equal(ids, ids_ref) and torch.equal(w, w_ref)
        assert torch.equal(r.counts, r_ref.counts)
        n = int(r.counts[0].item())
        for f in ("chunk_expert", "chunk_row0", "chunk_rows"):
            assert torch.equal(getattr(r, f)[:n], getattr(r_ref, f)[:n]), f
        assert torch.equal(r.sorted_ids, r_ref.sorted_ids)
        assert torch.equal(r.slot_pos, r_ref.slot_pos)
        assert torch.equal(r.chunk_ready, torch.zeros_like(r.chunk_ready))
        assert moe.read_device_error(r.err) == 0


def test_route_logits_with_expert_map(cuda_device):
    from trials_b200 import stages

    M, E, k = 333, 64, 4
    g = torch.Generator().manual_seed(11)
    logits = torch.randn(M, E, generator=g).to(cuda_device)
    emap = torch.full((E,), -1, dtype=torch.int32)
    local = torch.arange(0, E, 3)
    emap[local] = torch.arange(len(local), dtype=torch.int32)
    w_ref, ids_ref = moe.select_experts(logits, k, "sigmoid")
    r_ref = stages.route(ids_ref, E, 32, expert_map=emap.to(cuda_device), num_local_experts=len(local))
    r, w, ids = stages.route_logits(logits, k, 32, "sigmoid", expert_map=emap, num_local_experts=len(local))
    assert torch.equal(ids, ids_ref) and torch.equal(w, w_ref)
    assert torch.equal(r.sorted_ids, r_ref.sorted_ids) and torch.equal(r.slot_pos, r_ref.slot_pos)
    assert torch.equal(r.counts, r_ref.counts)


@pytest.mark.parametrize("shape", [synth.TINY, synth.LayerShape(M=96, H=512, I=256, E=16, topk=4),
                                   synth.glm(64)], ids=["tiny", "small", "glm64"])
def test_layer_from_logits_equals_router_then_layer(cuda_device, shape):
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=21, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    bias = torch.randn(shape.E, generator=g, device=cuda_device) * 0.05 if shape.scoring == "sigmoid" else None
    for M in (shape.M, max(1, shape.M // 3), shape.M):  # several calls on the same cached workspace
        logits = torch.randn(M, shape.E, generator=g, device=cuda_device)
        hidden = torch.randn(M, shape.H, generator=g, device=cuda_device).to(torch.bfloat16)
        w_ref, ids_ref = moe.select_experts(logits, shape.topk, shape.scoring, bias, routed_scaling_factor=2.5)
        ref = moe.moe_decode_megakernel_full(hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, w_ref, ids_ref)
        out, w, ids = moe.moe_layer_from_logits(hidden, logits, L.w13, L.w13_scale, L.w2, L.w2_scale, shape.topk,
                                                shape.scoring, bias, routed_scaling_factor=2.5)
        assert torch.equal(ids, ids_ref) and torch.equal(w, w_ref)
        assert torch.equal(out, ref)
    assert moe.read_device_error(moe.layer_error_word(cuda_device)) == 0


def test_layer_from_logits_matches_oracle(cuda_device):
    """The CPU oracle's router (float64) and layer on the tiny configuration."""
    L = synth.make_layer(synth.TINY, orc.per_block_quant_fp8, seed=8)
    g = torch.Generator().manual_seed(8)
    logits = torch.randn(L.shape.M, L.shape.E, generator=g)
    dev = cuda_device
    out, w, ids = moe.moe_layer_from_logits(L.hidden.to(dev), logits.to(dev), L.w13.to(dev), L.w13_scale.to(dev),
                                            L.w2.to(dev), L.w2_scale.to(dev), L.shape.topk, "softmax")
    rw, rids, margin = orc.router_topk(logits.numpy(), L.shape.topk, "softmax")
    assert (margin > AMBIGUOUS).all()
    assert np.array_equal(ids.cpu().numpy(), rids)
    ref = orc.moe_layer(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, torch.as_tensor(rw, dtype=torch.float32),
                        torch.as_tensor(rids, dtype=torch.int32))
    assert orc.rel_l2(out, ref) < 5e-3
