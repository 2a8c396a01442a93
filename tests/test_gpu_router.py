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
