"""The layer has no host synchronisation, so it can be captured in a CUDA graph
and replayed on new inputs written into the captured buffers."""
import pytest
import torch

from trials_b200 import moe, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(300)]


def test_layer_replays_from_a_cuda_graph(cuda_device):
    shape = synth.LayerShape(M=48, H=512, I=256, E=16, topk=4, scoring="sigmoid")
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=0, device=cuda_device)
    other = synth.make_layer(shape, moe.per_block_quant_fp8, seed=1, device=cuda_device)
    h, tw, ids = L.hidden.clone(), L.topk_weights.clone(), L.topk_ids.clone()
    args = (L.w13, L.w13_scale, L.w2, L.w2_scale)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        moe.moe_decode_megakernel_full(h, args[0], args[1], args[2], args[3], tw, ids)  # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = moe.moe_decode_megakernel_full(h, args[0], args[1], args[2], args[3], tw, ids)
    for src in (L, other, L):
        h.copy_(src.hidden)
        tw.copy_(src.topk_weights)
        ids.copy_(src.topk_ids)
        g.replay()
        torch.cuda.synchronize()
        eager = moe.moe_decode_megakernel_full(src.hidden, *args[:2], *args[2:], src.topk_weights, src.topk_ids)
        assert torch.equal(out, eager)
