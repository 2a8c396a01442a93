"""Public layer calls with non-contiguous inputs: the copies the host code
makes must live until the kernels have read them (same bits as contiguous
inputs)."""
import pytest
import torch

from trials_b200 import moe, stages, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]


def _strided(t):
    """The same values in a non-contiguous layout (last two dims swapped in memory)."""
    return t.transpose(-1, -2).contiguous().transpose(-1, -2)


def test_non_contiguous_scales_and_hidden(cuda_device):
    shape = synth.LayerShape(M=48, H=512, I=256, E=16, topk=4, scoring="sigmoid")
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=12, device=cuda_device)
    ref = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights, L.topk_ids)
    s13, s2 = _strided(L.w13_scale), _strided(L.w2_scale)
    assert not s13.is_contiguous() and not s2.is_contiguous()
    out = moe.moe_decode_megakernel_full(L.hidden, L.w13, s13, L.w2, s2, L.topk_weights, L.topk_ids)
    assert torch.equal(out, ref)
    out = moe.fused_moe(L.hidden, L.w13, L.w2, L.topk_weights, L.topk_ids, w1_scale=s13, w2_scale=s2)
    assert torch.equal(out, ref)
    # the layer from router logits, with a non-contiguous hidden too
    logits = torch.randn(shape.M, shape.E, device=cuda_device)
    h_nc = torch.cat([L.hidden, L.hidden], dim=1)[:, : shape.H]
    assert not h_nc.is_contiguous()
    out2, w, ids = moe.moe_layer_from_logits(h_nc, logits, L.w13, s13, L.w2, s2, shape.topk, "sigmoid")
    ref2 = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, w, ids)
    assert torch.equal(out2, ref2)
    # staged calls
    r = stages.route(L.topk_ids, shape.E, 32)
    a1, a1s = stages.gather_quant(L.hidden, shape.topk, r)
    a2, a2s = stages.gemm1_silu(a1, a1s, L.w13, s13, r)
    b2, b2s = stages.gemm1_silu(a1, a1s, L.w13, L.w13_scale, r)
    assert torch.equal(a2, b2) and torch.equal(a2s, b2s)
    p1 = stages.gemm2_combine(a2, a2s, L.w2, s2, r, L.topk_weights)
    p2 = stages.gemm2_combine(a2, a2s, L.w2, L.w2_scale, r, L.topk_weights)
    assert torch.equal(p1, p2)
