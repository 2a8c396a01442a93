"""GPU tests of the expert-parallel kernels and the pre-quantised layer entry.

The G ranks of an expert-parallel layer are simulated in one process on one
GPU: each rank's dispatch buffer is built by b200moe_ep_dispatch, the
all-to-all is a re-slicing of those buffers, every rank runs
b200moe_layer_packed on what it received with its own experts, and
b200moe_ep_combine adds the returned rows. The result must match the
single-GPU layer over all experts (only the bf16 rounding of each rank's
partial sum differs) and the dispatch bytes must match the oracle's layout.
"""
import pytest
import torch

from oracle import ep_oracle
from oracle import moe_oracle as orc
from trials_b200 import ep, moe, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]

EP_TOL = 1e-2     # bf16 partial sums per rank
SHAPE = synth.LayerShape(M=40, H=512, I=256, E=16, topk=4, scoring="sigmoid")


def _tokens(shape, seed, M, dev):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(M, shape.E, generator=g)
    tw, ids = synth.make_router(logits, shape.topk, shape.scoring)
    hidden = torch.randn(M, shape.H, generator=g).to(torch.bfloat16)
    return hidden.to(dev), tw.to(dev), ids.to(dev)


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_ep_kernels_simulated_ranks_match_single_gpu_layer(cuda_device, G):
    dev = cuda_device
    L = synth.make_layer(SHAPE, orc.per_block_quant_fp8, seed=0)
    W = {k: getattr(L, k).to(dev) for k in ["w13", "w13_scale", "w2", "w2_scale"]}
    cap = SHAPE.M
    ops = ep.CudaEPOps()
    H, topk = SHAPE.H, SHAPE.topk
    rb = ops.row_bytes(H, topk)
    assert rb == ep_oracle.row_bytes(H, topk)
    toks, sends, poss = [], [], []
    for r in range(G):
        M = cap - 3 * r
        hidden, tw, ids = _tokens(SHAPE, 10 + r, M, dev)
        q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=dev)
        s = torch.empty(M, H // 128, dtype=torch.float32, device=dev)
        ops.quant(hidden, q, s)
        send = torch.zeros(G * cap * rb, dtype=torch.uint8, device=dev)
        pos = torch.empty(M * G, dtype=torch.int32, device=dev)
        tok_of = torch.empty(G * cap, dtype=torch.int32, device=dev)
        counts = torch.empty(G, dtype=torch.int32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        ops.dispatch(q, s, ids, tw, SHAPE.E, G, cap, send, pos, tok_of, counts, err)
        # the oracle builds the same bytes (used rows entirely, ids/weights of unused rows)
        o_send = torch.zeros(G * cap * rb, dtype=torch.uint8)
        o_pos = torch.empty(M * G, dtype=torch.int32)
        o_tok = torch.empty(G * cap, dtype=torch.int32)
        o_cnt = torch.empty(G, dtype=torch.int32)
        ep_oracle.OracleEPOps().dispatch(q.cpu(), s.cpu(), ids.cpu(), tw.cpu(), SHAPE.E, G, cap, o_send, o_pos,
                                         o_tok, o_cnt, None)
        assert torch.equal(counts.cpu(), o_cnt) and torch.equal(pos.cpu(), o_pos)
        got = send.cpu().view(G * cap, rb)
        ref = o_send.view(G * cap, rb)
        for d in range(G):
            n = int(o_cnt[d])
            blk = slice(d * cap, d * cap + n)
            assert torch.equal(got[blk], ref[blk])
            meta = slice(H + (H // 128) * 4, rb)
            assert torch.equal(got[d * cap + n:(d + 1) * cap, meta], ref[d * cap + n:(d + 1) * cap, meta])
        assert int(err.item()) == 0
        toks.append((hidden, tw, ids))
        sends.append(send.view(G, cap * rb))
        poss.append(pos)
    # all-to-all: rank d receives block d of every rank's send buffer
    per = SHAPE.E // G
    local_outs = []
    for d in range(G):
        recv = torch.cat([sends[r][d] for r in range(G)]).contiguous()
        R = G * cap
        out_d = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
        ws = torch.zeros(max(ops.workspace_bytes(R, H, SHAPE.I, per, topk), 256), dtype=torch.uint8, device=dev)
        sl = slice(d * per, (d + 1) * per)
        ops.layer_packed(recv, R, H, SHAPE.I, per, topk, W["w13"][sl].contiguous(), W["w13_scale"][sl].contiguous(),
                         W["w2"][sl].contiguous(), W["w2_scale"][sl].contiguous(), out_d, ws)
        assert moe.read_device_error(ws[:4].view(torch.int32)) == 0
        local_outs.append(out_d.view(G, cap, H))
    for r in range(G):
        hidden, tw, ids = toks[r]
        M = hidden.shape[0]
        returned = torch.cat([local_outs[d][r] for d in range(G)]).contiguous()
        out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
        ops.combine(returned, poss[r], M, H, G, cap, out)
        single = moe.moe_decode_megakernel_full(hidden, W["w13"], W["w13_scale"], W["w2"], W["w2_scale"], tw, ids)
        ref = orc.moe_layer(hidden.cpu(), L.w13, L.w13_scale, L.w2, L.w2_scale, tw.cpu(), ids.cpu())
        assert orc.rel_l2(out, single) < EP_TOL
        assert orc.rel_l2(out, ref) < EP_TOL


def test_prequantised_input_is_bit_identical(cuda_device):
    L = synth.make_layer(SHAPE, orc.per_block_quant_fp8, seed=4)
    g = {k: getattr(L, k).to(cuda_device) for k in ["hidden", "topk_weights", "topk_ids", "w13", "w13_scale", "w2",
                                                     "w2_scale"]}
    ref = moe.moe_decode_megakernel_full(g["hidden"], g["w13"], g["w13_scale"], g["w2"], g["w2_scale"],
                                         g["topk_weights"], g["topk_ids"])
    q, s = moe.per_token_group_quant_fp8(g["hidden"])
    out = moe.moe_decode_megakernel_full(q, g["w13"], g["w13_scale"], g["w2"], g["w2_scale"], g["topk_weights"],
                                         g["topk_ids"], a1_scale=s)
    assert torch.equal(out, ref)
    out2 = moe.fused_moe(q, g["w13"], g["w2"], g["topk_weights"], g["topk_ids"], w1_scale=g["w13_scale"],
                         w2_scale=g["w2_scale"], a1_scale=s)
    assert torch.equal(out2, ref)
    with pytest.raises(NotImplementedError):
        moe.moe_decode_megakernel_full(q, g["w13"], g["w13_scale"], g["w2"], g["w2_scale"], g["topk_weights"],
                                       g["topk_ids"], a1_scale=torch.ones(q.shape[0], device=cuda_device))
