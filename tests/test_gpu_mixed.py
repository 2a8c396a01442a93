"""Mixed work lists: in a skewed decode batch the experts with more than 128
padded rows (hot experts) are routed into a second work list and computed by
the token-major stages in the same layer call, the others by the swap-AB
launch (b200moe_route_mixed, b200moe_experts_heavy; what b200moe_layer does
by itself)."""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from trials_b200 import _lib, moe, stages, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]

SKEW = synth.LayerShape(M=400, H=512, I=256, E=64, topk=4, scoring="sigmoid", hot_experts=4)


def _ids(M, E, topk, hot, seed):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(M, E, generator=g)
    logits[:, :hot] += 2.0
    return synth.make_router(logits, topk, "sigmoid")


@pytest.mark.parametrize("M,E,topk,hot,tile", [(400, 64, 4, 4, 32), (1024, 256, 8, 16, 64), (700, 32, 8, 2, 64),
                                               (300, 64, 4, 0, 32)])
def test_route_mixed_layout(cuda_device, M, E, topk, hot, tile):
    tw, ids = _ids(M, E, topk, hot, seed=M + E)
    r, heavy, counts = stages.route_mixed(ids.to(cuda_device), E, tile)
    c = counts.cpu().numpy()
    n_light, rows, n_heavy, row0 = (int(x) for x in c)
    flat = ids.reshape(-1).numpy()
    per = np.bincount(flat, minlength=E)
    pad = (per + 15) // 16 * 16
    hv = pad > 128
    assert rows == pad.sum() and row0 == pad[~hv].sum()
    assert (n_heavy > 0) == bool(hv.any())
    sorted_ids = r.sorted_ids.cpu().numpy()
    slot_pos = r.slot_pos.cpu().numpy()
    # every routed slot exactly once, at its slot_pos, in its expert's row range
    assert (sorted_ids[slot_pos] == np.arange(M * topk)).all()
    assert (sorted_ids[rows:] == M * topk).all()
    base = np.zeros(E, dtype=np.int64)
    base[~hv] = np.concatenate([[0], np.cumsum(pad[~hv])[:-1]]) if (~hv).any() else []
    if hv.any():
        base[hv] = row0 + np.concatenate([[0], np.cumsum(pad[hv])[:-1]])
    for f, e in enumerate(flat):
        assert base[e] <= slot_pos[f] < base[e] + per[e]
    # stable order inside an expert
    for e in range(E):
        seg = sorted_ids[base[e]:base[e] + per[e]]
        assert (np.diff(seg) > 0).all() and (flat[seg] == e).all()
    # the two chunk lists cover each expert's padded rows in order, in tiles of <= tile / <= 128 rows
    for lst, n, lim, sel in ((r, n_light, tile, ~hv), (heavy, n_heavy, 128, hv)):
        ce = (lst.chunk_expert if lst is r else lst["chunk_expert"]).cpu().numpy()[:n]
        c0 = (lst.chunk_row0 if lst is r else lst["chunk_row0"]).cpu().numpy()[:n]
        cr = (lst.chunk_rows if lst is r else lst["chunk_rows"]).cpu().numpy()[:n]
        assert (cr <= lim).all() and (cr % 16 == 0).all() and (cr > 0).all()
        for e in np.nonzero(sel & (per > 0))[0]:
            m = ce == e
            assert cr[m].sum() == pad[e] and c0[m].min() == base[e]
        assert set(ce.tolist()) == set(np.nonzero(sel & (per > 0))[0].tolist())
    assert int(heavy["counters"][0].item()) == 0 and int(heavy["counters"][1].item()) == 0
    assert moe.read_device_error(r.err) == 0


def test_layer_with_heavy_experts_matches_oracle(cuda_device):
    """A decode batch where 4 hot experts exceed 128 rows: the layer (swap-AB
    tiles for the others, token-major stages for the hot ones) against the
    oracle, and the staged pipeline against the layer bit for bit."""
    L = synth.make_layer(SKEW, moe.per_block_quant_fp8, seed=31, device=cuda_device)
    E, topk = SKEW.E, SKEW.topk
    lib = _lib.lib()
    pipe = stages.LayerPipeline(SKEW.M, SKEW.H, SKEW.I, E, topk, cuda_device)
    assert pipe.tile <= 64 and pipe.heavy_rows == 128 == lib.b200moe_heavy_rows(SKEW.M, topk, pipe.tile)
    out = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights, L.topk_ids)
    staged = pipe.run(L.hidden, L.topk_ids, L.topk_weights, L.w13, L.w13_scale, L.w2, L.w2_scale)
    torch.cuda.synchronize()
    assert int(pipe.counts[2].item()) > 0, "the skewed batch must have heavy experts"
    assert torch.equal(staged, out)
    ref = orc.moe_layer(L.hidden.cpu(), L.w13.cpu(), L.w13_scale.cpu(), L.w2.cpu(), L.w2_scale.cpu(),
                        L.topk_weights.cpu(), L.topk_ids.cpu())
    assert orc.rel_l2(out, ref) < 5e-3
    assert moe.read_device_error(pipe.err) == 0
    assert moe.read_device_error(moe.layer_error_word(cuda_device)) == 0


def test_mixed_without_heavy_experts_equals_single_list(cuda_device):
    """No expert above 128 rows: the heavy list is empty and the result is the
    one-list layer's bit for bit."""
    shape = synth.LayerShape(M=256, H=512, I=256, E=64, topk=4, scoring="sigmoid")
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=32, device=cuda_device)
    mixed = stages.LayerPipeline(shape.M, shape.H, shape.I, shape.E, shape.topk, cuda_device)
    single = stages.LayerPipeline(shape.M, shape.H, shape.I, shape.E, shape.topk, cuda_device, split=True)
    assert mixed.heavy_rows == 128 and single.heavy_rows == 0
    a = mixed.run(L.hidden, L.topk_ids, L.topk_weights, L.w13, L.w13_scale, L.w2, L.w2_scale).clone()
    b = single.run(L.hidden, L.topk_ids, L.topk_weights, L.w13, L.w13_scale, L.w2, L.w2_scale)
    torch.cuda.synchronize()
    assert int(mixed.counts[2].item()) == 0
    assert torch.equal(a, b)
