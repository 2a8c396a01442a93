"""GPU parity: every CUDA kernel against the oracle on the same seeded inputs.

Integer/byte work (routing, quantisation) must match bit for bit. The GEMM
stages and the layer are floating point: fp8 products are exact and both sides
accumulate in at least fp32, so they are compared by relative L2 error with
the tolerances written next to each check (the layer gate is the north-star
bound 2e-2; measured values are far below it).
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from trials_b200 import moe, stages, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(900)]

LAYER_GATE = 2e-2     # rel-L2 bound of the layer vs the fp32-dequantised oracle
EXACT_TOL = 5e-3      # same rounding points as the oracle: only accumulation order differs


def _u8(t):
    return t.contiguous().view(torch.uint8).cpu()


def _gen(seed):
    return torch.Generator().manual_seed(seed)


# ----------------------------------------------------------------------------
# quantisation (bit-exact)
# ----------------------------------------------------------------------------
@pytest.mark.parametrize("M,K", [(1, 128), (16, 256), (64, 6144), (37, 2048), (300, 384)])
def test_quant_1x128_bit_exact(cuda_device, M, K):
    x = (torch.randn(M, K, generator=_gen(M * K)) * 3).to(torch.bfloat16)
    x[0, :7] = 0  # a partially zero group
    if M > 2:
        x[2, 128:256] = 0  # an all-zero group: scale clamps to 1e-12
    q, s = moe.per_token_group_quant_fp8(x.to(cuda_device))
    rq, rs = orc.per_token_group_quant_fp8(x)
    assert torch.equal(_u8(q), _u8(rq))
    assert torch.equal(s.cpu(), rs)


def test_block_quant_bit_exact(cuda_device):
    w = (torch.randn(3, 256, 384, generator=_gen(7)) * 0.02).to(torch.bfloat16)
    w[1, :128, :128] = 0
    q, s = moe.per_block_quant_fp8(w.to(cuda_device))
    rq, rs = orc.per_block_quant_fp8(w)
    assert torch.equal(_u8(q), _u8(rq))
    assert torch.equal(s.cpu(), rs)


# ----------------------------------------------------------------------------
# routing (bit-exact)
# ----------------------------------------------------------------------------
def _ids(M, E, topk, seed, skew=0, minus_one=0.0):
    logits = torch.randn(M, E, generator=_gen(seed))
    if skew:
        logits[:, :skew] += 2.0
    ids = torch.topk(logits, topk, dim=-1).indices.to(torch.int32)
    if minus_one:
        drop = torch.rand(M, topk, generator=_gen(seed + 1)) < minus_one
        ids[drop] = -1
    return ids


ALIGN_CASES = [
    # M, topk, E, BM, skew, minus_one
    (16, 2, 8, 128, 0, 0.0),
    (64, 8, 256, 128, 0, 0.0),
    (64, 8, 256, 16, 0, 0.0),
    (1024, 8, 256, 128, 16, 0.0),
    (8192, 8, 256, 128, 0, 0.0),
    (3, 2, 8, 64, 0, 0.0),
    (1, 1, 1, 16, 0, 0.0),
    (200, 4, 64, 32, 0, 0.3),
    (0, 8, 256, 128, 0, 0.0),
]


@pytest.mark.parametrize("M,topk,E,BM,skew,minus_one", ALIGN_CASES)
def test_align_bit_exact(cuda_device, M, topk, E, BM, skew, minus_one):
    ids = _ids(M, E, topk, seed=M + E, skew=skew, minus_one=minus_one) if M else torch.zeros(0, topk, dtype=torch.int32)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    s, e, n = moe.moe_align_block_size(ids.to(cuda_device), BM, E, err_word=err)
    rs, re_, rn = orc.moe_align_block_size(ids.numpy(), BM, E)
    assert int(n.item()) == rn
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(e.cpu().numpy(), re_)
    assert int(err.item()) == 0


def test_align_expert_map_and_bad_ids(cuda_device):
    M, topk, E = 100, 4, 32
    ids = _ids(M, E, topk, seed=3)
    ids[5, 1] = 77      # out of range -> dropped + error bit
    ids[6, 0] = -5      # negative other than -1 -> dropped + error bit
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[8:16] = torch.arange(8, dtype=torch.int32)  # this rank owns experts 8..15
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    s, e, n = moe.moe_align_block_size(ids.to(cuda_device), 16, E, expert_map=emap.to(cuda_device),
                                       num_local_experts=8, err_word=err)
    rs, re_, rn = orc.moe_align_block_size(ids.numpy(), 16, E, expert_map=emap.numpy(), num_local=8)
    assert int(n.item()) == rn
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(e.cpu().numpy(), re_)
    assert int(err.item()) & 1


@pytest.mark.parametrize("M,E,topk,tile", [(16, 8, 2, 32), (64, 256, 8, 32), (1024, 256, 8, 64),
                                           (1024, 256, 8, 128), (512, 256, 8, 16)])
def test_route_chunks_exact(cuda_device, M, E, topk, tile):
    ids = _ids(M, E, topk, seed=M, skew=16 if M == 1024 else 0)
    r = stages.route(ids.to(cuda_device), E, tile)
    rs, rn, chunks = orc.route_chunks(ids.numpy(), E, tile)
    nc = int(r.counts[0].item())
    assert int(r.counts[1].item()) == rn
    assert nc == len(chunks)
    got_sorted = r.sorted_ids.cpu().numpy()
    assert np.array_equal(got_sorted[:rn], rs[:rn])
    assert (got_sorted[rn:] == M * topk).all() and (rs[rn:] == M * topk).all()
    got = np.stack([r.chunk_expert[:nc].cpu().numpy(), r.chunk_row0[:nc].cpu().numpy(),
                    r.chunk_rows[:nc].cpu().numpy()], 1)
    assert np.array_equal(got, chunks)


def _same_routing(a, b):
    nc = int(a.counts[0].item())
    for name in ("sorted_ids", "counts", "slot_pos", "err"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    for name in ("chunk_expert", "chunk_row0", "chunk_rows"):  # defined up to n_chunks
        assert torch.equal(getattr(a, name)[:nc], getattr(b, name)[:nc]), name


@pytest.mark.parametrize("M,E,topk,tile,skew,minus_one", [(4096, 256, 8, 128, 0, 0.0), (8192, 256, 8, 128, 16, 0.0),
                                                        (3000, 64, 8, 64, 0, 0.2), (2048, 1024, 8, 32, 0, 0.0)])
def test_route_on_several_ctas_equals_one_cta(cuda_device, M, E, topk, tile, skew, minus_one):
    """From 16,384 routed slots routing runs on several CTAs; the result is the
    one-CTA kernel's and the oracle's, slot positions included."""
    from trials_b200 import _lib

    assert _lib.lib().b200moe_route_scratch_ints(M * topk, E) > 0
    ids = _ids(M, E, topk, seed=M + 7, skew=skew, minus_one=minus_one)
    multi = stages.route(ids.to(cuda_device), E, tile)
    one = stages.route(ids.to(cuda_device), E, tile, multi_cta=False)
    _same_routing(multi, one)
    assert int(multi.err.item()) == 0
    rs, rn, chunks = orc.route_chunks(ids.numpy(), E, tile)
    assert int(multi.counts[1].item()) == rn
    assert np.array_equal(multi.sorted_ids.cpu().numpy()[:rn], rs[:rn])
    pos = multi.slot_pos.cpu().numpy()
    flat = ids.numpy().reshape(-1)
    routed = flat >= 0
    assert (pos[~routed] == -1).all()
    assert np.array_equal(multi.sorted_ids.cpu().numpy()[pos[routed]], np.nonzero(routed)[0])


def test_route_on_several_ctas_expert_map_and_bad_ids(cuda_device):
    M, E, topk = 4096, 64, 8
    ids = _ids(M, E, topk, seed=11)
    ids[5, 1] = 77
    ids[4000, 0] = -5
    emap = torch.full((E,), -1, dtype=torch.int32)
    emap[8:24] = torch.arange(16, dtype=torch.int32)
    multi = stages.route(ids.to(cuda_device), E, 128, expert_map=emap.to(cuda_device), num_local_experts=16)
    one = stages.route(ids.to(cuda_device), E, 128, expert_map=emap.to(cuda_device), num_local_experts=16,
                       multi_cta=False)
    _same_routing(multi, one)
    assert int(multi.err.item()) & 1


# ----------------------------------------------------------------------------
# GEMM stages
# ----------------------------------------------------------------------------
def _tiny_layer(dev, shape=synth.TINY, seed=0):
    L = synth.make_layer(shape, orc.per_block_quant_fp8, seed=seed)
    return L, {k: getattr(L, k).to(dev) for k in ["hidden", "topk_weights", "topk_ids", "w13", "w13_scale", "w2",
                                                   "w2_scale"]}


SMALL = synth.LayerShape(M=96, H=512, I=256, E=16, topk=4, scoring="sigmoid")


@pytest.mark.parametrize("shape,tile", [(synth.TINY, 32), (SMALL, 32), (SMALL, 64), (SMALL, 128), (SMALL, 16),
                                        (SMALL, 256), (synth.TINY, 256)])
def test_gather_and_gemm_stages(cuda_device, shape, tile):
    L, g = _tiny_layer(cuda_device, shape)
    topk = shape.topk
    r = stages.route(g["topk_ids"], shape.E, tile)
    a1_q, a1_sT = stages.gather_quant(g["hidden"], topk, r)
    torch.cuda.synchronize()
    n_rows = int(r.counts[1].item())
    sorted_ids = r.sorted_ids[:n_rows].cpu().numpy()
    valid = sorted_ids < shape.M * topk
    # gather + quantise: bit-exact routed rows (padding rows are not written)
    hq, hs = orc.per_token_group_quant_fp8(L.hidden)
    tok = torch.as_tensor(sorted_ids[valid] // topk, dtype=torch.long)
    assert torch.equal(_u8(a1_q[:n_rows][torch.as_tensor(valid)]), _u8(hq[tok]))
    assert torch.equal(a1_sT[:, :n_rows].T.cpu()[torch.as_tensor(valid)], hs[tok])

    # stage 1 vs oracle (fp32 gate/up -> SiLU*up -> 1x128 requant)
    a2_q, a2_sT = stages.gemm1_silu(a1_q, a1_sT, g["w13"], g["w13_scale"], r)
    torch.cuda.synchronize()
    experts = L.topk_ids.reshape(-1).numpy()[sorted_ids[valid]]
    g1 = torch.cat([orc.blockscaled_gemm(hq[t:t + 1], hs[t:t + 1], L.w13[e], L.w13_scale[e])
                    for t, e in zip(tok.tolist(), experts)])
    inter = orc.silu_mul_interleaved(g1.float())
    rq, rsc = orc.per_token_group_quant_fp8(inter)
    got_q = a2_q[:n_rows][torch.as_tensor(valid)].cpu()
    got_s = a2_sT[:, :n_rows].T.cpu()[torch.as_tensor(valid)]
    same = (_u8(got_q) == _u8(rq)).float().mean().item()
    assert same > 0.995, f"fp8 inter bytes equal: {same:.4f}"
    assert orc.rel_l2(orc.dequant_rows(got_q, got_s), orc.dequant_rows(rq, rsc)) < EXACT_TOL
    assert torch.allclose(got_s, rsc, rtol=1e-5, atol=0)

    # stage 2 vs oracle given the GPU's own stage-1 output (fp32 accumulation only)
    pair = stages.gemm2_combine(a2_q, a2_sT, g["w2"], g["w2_scale"], r, g["topk_weights"])
    torch.cuda.synchronize()
    g2 = torch.cat([orc.blockscaled_gemm(got_q[i:i + 1], got_s[i:i + 1], L.w2[e], L.w2_scale[e])
                    for i, e in enumerate(experts)])
    w = L.topk_weights.reshape(-1)[torch.as_tensor(sorted_ids[valid], dtype=torch.long)].double()
    ref_pair = g2 * w[:, None]
    if r.sorted_rows:
        got_pair = pair.cpu()[:n_rows][torch.as_tensor(valid)]
    else:
        got_pair = pair.cpu()[torch.as_tensor(sorted_ids[valid], dtype=torch.long)]
    # fp32 accumulation, then one bf16 rounding of each weighted row
    assert orc.rel_l2(got_pair, ref_pair) < 4e-3
    assert orc.rel_l2(got_pair, ref_pair.float().to(torch.bfloat16)) < 1e-3

    # slot positions: the inverse of the routed part of sorted_ids
    pos = r.slot_pos.cpu().numpy()
    assert (pos[sorted_ids[valid]] == np.nonzero(valid)[0]).all()
    assert np.count_nonzero(pos >= 0) == int(valid.sum())

    # top-k reduce: slot rows gathered by position, summed in slot order
    out = stages.combine_reduce(pair, r, shape.M, topk)
    by_slot = torch.zeros(shape.M * topk, shape.H, dtype=torch.float32)
    by_slot[torch.as_tensor(sorted_ids[valid], dtype=torch.long)] = got_pair.float()
    ref_out = by_slot.view(shape.M, topk, shape.H).sum(1).to(torch.bfloat16)
    assert orc.rel_l2(out, ref_out) < 1e-2 ** 2
    assert int(r.err.item()) == 0


@pytest.mark.parametrize("shape,tile,grid", [(synth.TINY, 32, 0), (SMALL, 16, 0), (SMALL, 32, 0), (SMALL, 64, 0),
                                             (SMALL, 32, 5), (SMALL, 64, 37), (SMALL, 32, 148)])
def test_one_launch_layer_bit_identical(cuda_device, shape, tile, grid):
    """Gather + quantise, both GEMM stages and the top-k reduce in one launch
    (phases ordered by device counters) equal the separate stages bit for bit."""
    L, g = _tiny_layer(cuda_device, shape, seed=4)
    r = stages.route(g["topk_ids"], shape.E, tile)
    a1_q, a1_sT = stages.gather_quant(g["hidden"], shape.topk, r)
    _, _, pair = stages.experts(a1_q, a1_sT, g["w13"], g["w13_scale"], g["w2"], g["w2_scale"], r, g["topk_weights"])
    ref = stages.combine_reduce(pair, r, shape.M, shape.topk)
    r2 = stages.route(g["topk_ids"], shape.E, tile)  # fresh counters
    out = stages.experts_fused(g["hidden"], g["w13"], g["w13_scale"], g["w2"], g["w2_scale"], r2, g["topk_weights"],
                               grid_ctas=grid)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert int(r2.err.item()) == 0
    nc = int(r2.counts[0].item())
    assert (r2.chunk_ready[:nc] == 2 * shape.I // 256).all()


@pytest.mark.parametrize("M,tile", [(16, 32), (300, 64), (600, 128)])
def test_gather_rows_equals_gather_quant(cuda_device, M, tile):
    """Quantising in the gather and copying rows quantised beforehand give the
    same routed rows and scales (per-slot warps at M=16 and 300, per-token
    fan-out at 600)."""
    shape = synth.LayerShape(M=M, H=512, I=256, E=16, topk=4, scoring="sigmoid")
    L, g = _tiny_layer(cuda_device, shape, seed=3)
    r = stages.route(g["topk_ids"], shape.E, tile)
    a_q, a_sT = stages.gather_quant(g["hidden"], shape.topk, r)
    tq, ts = moe.per_token_group_quant_fp8(g["hidden"])
    b_q, b_sT = stages.gather_rows(tq, ts, shape.topk, r)
    torch.cuda.synchronize()
    n_rows = int(r.counts[1].item())
    valid = torch.as_tensor(r.sorted_ids[:n_rows].cpu().numpy() < M * shape.topk)
    assert torch.equal(_u8(a_q[:n_rows][valid]), _u8(b_q[:n_rows][valid]))
    assert torch.equal(a_sT[:, :n_rows].T.cpu()[valid], b_sT[:, :n_rows].T.cpu()[valid])


@pytest.mark.parametrize("M,topk,minus_one", [(16, 4, 0.0), (600, 4, 0.0), (700, 8, 0.2), (300, 8, 0.0)])
def test_gathered_rows_are_token_quant_at_slot_rows(cuda_device, M, topk, minus_one):
    """Both gathers (one warp per slot below 2,048 routed pairs, one per token
    storing to all its slots from there on) put token t's 1x128 quantisation
    at every routed slot's sorted row."""
    E = 16
    ids = _ids(M, E, topk, seed=M + topk, minus_one=minus_one)
    g = torch.Generator().manual_seed(M)
    hidden = torch.randn(M, 512, generator=g).to(torch.bfloat16).to(cuda_device)
    r = stages.route(ids.to(cuda_device), E, 64)
    a_q, a_sT = stages.gather_quant(hidden, topk, r)
    tq, ts = moe.per_token_group_quant_fp8(hidden)
    b_q, b_sT = stages.gather_rows(tq, ts, topk, r)
    torch.cuda.synchronize()
    pos = r.slot_pos.cpu().long()
    routed = pos >= 0
    assert bool(routed.any())
    tok = torch.arange(M * topk)[routed] // topk
    want_q, want_s = _u8(tq)[tok], ts.cpu()[tok]
    for q, sT in ((a_q, a_sT), (b_q, b_sT)):
        assert torch.equal(_u8(q)[pos[routed]], want_q)
        assert torch.equal(sT.cpu().T[pos[routed]], want_s)


@pytest.mark.parametrize("grid,tile", [(1, 32), (5, 32), (37, 32), (1, 128), (7, 128), (3, 64), (2, 256),
                                       (6, 256)])
def test_schedule_invariance_bit_exact(cuda_device, grid, tile):
    """Any persistent grid gives bit-identical results (the reference's MODE 0/1
    equivalence check, phase3_blockscale.py:150-164)."""
    L, g = _tiny_layer(cuda_device, SMALL, seed=1)
    r = stages.route(g["topk_ids"], SMALL.E, tile)
    a1_q, a1_sT = stages.gather_quant(g["hidden"], SMALL.topk, r)
    ref_q, ref_s = stages.gemm1_silu(a1_q, a1_sT, g["w13"], g["w13_scale"], r, grid_ctas=0)
    q, s = stages.gemm1_silu(a1_q, a1_sT, g["w13"], g["w13_scale"], r, grid_ctas=grid)
    # bit patterns (rows of padding tokens may hold NaN from unwritten inputs)
    assert torch.equal(_u8(q), _u8(ref_q)) and torch.equal(s.view(torch.int32), ref_s.view(torch.int32))
    p0 = stages.gemm2_combine(ref_q, ref_s, g["w2"], g["w2_scale"], r, g["topk_weights"], grid_ctas=0)
    p1 = stages.gemm2_combine(ref_q, ref_s, g["w2"], g["w2_scale"], r, g["topk_weights"], grid_ctas=grid)
    assert torch.equal(p0, p1)


@pytest.mark.parametrize("shape,tile,grid", [(synth.TINY, 32, 0), (SMALL, 16, 0), (SMALL, 32, 0), (SMALL, 64, 0),
                                             (SMALL, 32, 1), (SMALL, 32, 5), (SMALL, 64, 37), (SMALL, 32, 148),
                                             (SMALL, 128, 0), (SMALL, 128, 1), (SMALL, 128, 7)])
def test_fused_experts_bit_identical_to_split(cuda_device, shape, tile, grid):
    """Both GEMM stages in one launch (stage-2 units wait per chunk on the
    stage-1 units) give exactly the two-launch results, for any grid."""
    L, g = _tiny_layer(cuda_device, shape, seed=2)
    r = stages.route(g["topk_ids"], shape.E, tile)
    a1_q, a1_sT = stages.gather_quant(g["hidden"], shape.topk, r)
    q1, s1 = stages.gemm1_silu(a1_q, a1_sT, g["w13"], g["w13_scale"], r)
    p1 = stages.gemm2_combine(q1, s1, g["w2"], g["w2_scale"], r, g["topk_weights"])
    q2, s2, p2 = stages.experts(a1_q, a1_sT, g["w13"], g["w13_scale"], g["w2"], g["w2_scale"], r,
                                g["topk_weights"], grid_ctas=grid)
    torch.cuda.synchronize()
    assert torch.equal(_u8(q1), _u8(q2)) and torch.equal(s1.view(torch.int32), s2.view(torch.int32))
    assert torch.equal(p1, p2)
    assert int(r.err.item()) == 0
    if tile <= 64:
        nc = int(r.counts[0].item())
        assert (r.chunk_ready[:nc] == 2 * shape.I // 256).all()


# ----------------------------------------------------------------------------
# full layer
# ----------------------------------------------------------------------------
def _layer_out(g):
    return moe.moe_decode_megakernel_full(g["hidden"], g["w13"], g["w13_scale"], g["w2"], g["w2_scale"],
                                          g["topk_weights"], g["topk_ids"])


@pytest.mark.parametrize("shape", [synth.TINY, SMALL])
def test_layer_small_vs_oracle(cuda_device, shape):
    L, g = _tiny_layer(cuda_device, shape)
    out = _layer_out(g)
    ref = orc.moe_layer(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights, L.topk_ids)
    assert orc.rel_l2(out, ref) < EXACT_TOL
    out2 = _layer_out(g)
    assert torch.equal(out, out2), "layer must be deterministic"
    assert int(moe.read_device_error(moe.layer_error_word(cuda_device))) == 0


def test_layer_tiny_vs_reference_golden(cuda_device):
    """End to end against the reference orchestrator's own output (golden)."""
    from pathlib import Path

    z = np.load(Path(__file__).resolve().parent / "golden" / "tiny_seed0.npz")
    _, g = _tiny_layer(cuda_device)
    out = _layer_out(g)
    ref = torch.from_numpy(z["out"]).view(torch.bfloat16)
    assert orc.rel_l2(out, ref) < LAYER_GATE


@pytest.mark.parametrize("M,hot", [(64, 0), (256, 0), (1024, 16), (2048, 0)])
def test_layer_glm_shapes_vs_oracle(cuda_device, M, hot):
    shape = synth.glm(M, hot)
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=0, device=cuda_device)
    out = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights,
                                         L.topk_ids)
    ref = orc.moe_layer(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights, L.topk_ids)
    err = orc.rel_l2(out, ref)
    assert err < EXACT_TOL, err
    ref_r = orc.moe_layer(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights, L.topk_ids,
                          rounding="reference")
    assert orc.rel_l2(out, ref_r) < LAYER_GATE
    bad = orc.moe_layer(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights, L.topk_ids,
                        stage2_a_by_token=True)
    assert orc.rel_l2(out, bad) > 0.5, "the gate must reject the A_BY_SORTED failure"
    assert int(moe.read_device_error(moe.layer_error_word(cuda_device))) == 0


def test_fused_moe_expert_mask_matches_oracle(cuda_device):
    L, g = _tiny_layer(cuda_device, SMALL, seed=2)
    mask = torch.zeros(SMALL.E, dtype=torch.int32)
    mask[4:12] = 1
    out = moe.fused_moe(g["hidden"], g["w13"][4:12].contiguous(), g["w2"][4:12].contiguous(), g["topk_weights"],
                        g["topk_ids"], w1_scale=g["w13_scale"][4:12].contiguous(),
                        w2_scale=g["w2_scale"][4:12].contiguous(), expert_mask=mask.to(cuda_device))
    emap = moe.expert_map_from_mask(mask)
    ref = orc.moe_layer(L.hidden, L.w13[4:12], L.w13_scale[4:12], L.w2[4:12], L.w2_scale[4:12], L.topk_weights,
                        L.topk_ids, expert_map=emap.numpy(), num_local=8)
    assert orc.rel_l2(out, ref) < EXACT_TOL


def test_empty_batch_and_bad_ids(cuda_device):
    _, g = _tiny_layer(cuda_device)
    empty = moe.fused_moe(g["hidden"][:0], g["w13"], g["w2"], g["topk_weights"][:0], g["topk_ids"][:0],
                          w1_scale=g["w13_scale"], w2_scale=g["w2_scale"])
    assert empty.shape == (0, synth.TINY.H)
    ids = g["topk_ids"].clone()
    ids[0, 0] = 99
    moe.read_device_error(moe.layer_error_word(cuda_device), clear=True)
    moe.moe_decode_megakernel_full(g["hidden"], g["w13"], g["w13_scale"], g["w2"], g["w2_scale"],
                                   g["topk_weights"], ids)
    assert moe.read_device_error(moe.layer_error_word(cuda_device), clear=True) & 1


def test_bounded_wait_reports_timeout_and_context_survives(cuda_device):
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    stages.selftest_wait_timeout(err, timeout_us=20000)
    torch.cuda.synchronize()
    assert int(err.item()) & 2
    # the context is still usable
    x = torch.randn(4, 256, device=cuda_device).to(torch.bfloat16)
    q, s = moe.per_token_group_quant_fp8(x)
    rq, rs = orc.per_token_group_quant_fp8(x.cpu())
    assert torch.equal(_u8(q), _u8(rq))


def test_layer_glm_prefill_cta_pairs_vs_oracle(cuda_device):
    """M=8192: 256 routed rows per expert, served by the CTA-pair kernel."""
    shape = synth.glm(8192)
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=0, device=cuda_device)
    out = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights,
                                         L.topk_ids)
    ref = orc.moe_layer(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights, L.topk_ids)
    assert orc.rel_l2(out, ref) < EXACT_TOL
    assert int(moe.read_device_error(moe.layer_error_word(cuda_device))) == 0
