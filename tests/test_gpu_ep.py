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
                         W["w2"][sl].contiguous(), W["w2_scale"][sl].contiguous(), out_d, ws, num_ranks=G)
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


def _rank_weights(W, G, placement=None):
    """Each rank's (w13, w13_scale, w2, w2_scale): an even split, or the
    placement's slots."""
    keys = ["w13", "w13_scale", "w2", "w2_scale"]
    if placement is None:
        per = SHAPE.E // G
        return [[W[k][d * per:(d + 1) * per].contiguous() for k in keys] for d in range(G)]
    return [[ep.place_experts(W[k], placement, d) for k in keys] for d in range(G)]


def _all_to_all_form(G, cap, toks, W, dev, placement=None, check_bytes=False):
    """Outputs of the all-to-all form (dispatch buffers re-sliced in place of
    the exchange) for G simulated ranks' tokens; with check_bytes, every
    rank's dispatch buffer is compared with the oracle's."""
    ops = ep.CudaEPOps()
    H, I, topk = SHAPE.H, SHAPE.I, SHAPE.topk
    rb = ops.row_bytes(H, topk)
    table = None if placement is None else torch.as_tensor(placement.table(), device=dev)
    E_local = SHAPE.E // G if placement is None else placement.slots
    sends, poss = [], []
    for r, (hidden, tw, ids) in enumerate(toks):
        M = hidden.shape[0]
        q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=dev)
        s = torch.empty(M, H // 128, dtype=torch.float32, device=dev)
        ops.quant(hidden, q, s)
        send = torch.zeros(G * cap * rb, dtype=torch.uint8, device=dev)
        pos = torch.empty(M * G, dtype=torch.int32, device=dev)
        counts = torch.empty(G, dtype=torch.int32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        pl_arg = None if placement is None else (table, placement)
        ops.dispatch(q, s, ids, tw, SHAPE.E, G, cap, send, pos, torch.empty(G * cap, dtype=torch.int32, device=dev),
                     counts, err, rank=r, placement=pl_arg)
        if check_bytes:
            o_send = torch.zeros(G * cap * rb, dtype=torch.uint8)
            o_pos = torch.empty(M * G, dtype=torch.int32)
            o_cnt = torch.empty(G, dtype=torch.int32)
            ep_oracle.OracleEPOps().dispatch(q.cpu(), s.cpu(), ids.cpu(), tw.cpu(), SHAPE.E, G, cap, o_send, o_pos,
                                             torch.empty(G * cap, dtype=torch.int32), o_cnt, None, rank=r,
                                             placement=None if placement is None else (table.cpu(), placement))
            assert torch.equal(counts.cpu(), o_cnt) and torch.equal(pos.cpu(), o_pos)
            got, ref = send.cpu().view(G * cap, rb), o_send.view(G * cap, rb)
            for d in range(G):
                n = int(o_cnt[d])
                assert torch.equal(got[d * cap:d * cap + n], ref[d * cap:d * cap + n]), (r, d)
            assert moe.read_device_error(err) == 0
        sends.append(send.view(G, cap * rb))
        poss.append(pos)
    local = []
    weights = _rank_weights(W, G, placement)
    for d in range(G):
        recv = torch.cat([sends[r][d] for r in range(G)]).contiguous()
        out_d = torch.empty(G * cap, H, dtype=torch.bfloat16, device=dev)
        ws = torch.zeros(max(ops.workspace_bytes(G * cap, H, I, E_local, topk), 256), dtype=torch.uint8, device=dev)
        ops.layer_packed(recv, G * cap, H, I, E_local, topk, *weights[d], out_d, ws, num_ranks=G)
        local.append(out_d.view(G, cap, H))
    outs = []
    for r, (hidden, _, _) in enumerate(toks):
        M = hidden.shape[0]
        out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
        ops.combine(torch.cat([local[d][r] for d in range(G)]).contiguous(), poss[r], M, H, G, cap, out)
        outs.append(out)
    return outs


@pytest.mark.parametrize("G", [1, 2, 4, 8])
def test_peer_exchange_simulated_ranks_bit_identical_to_all_to_all(cuda_device, G):
    """The G ranks' exchange buffers live in one process on one GPU. Every
    kernel of a call is launched after the kernels whose flags it waits for
    (all dispatches, then all layers, then all combines), so no wait depends
    on a later launch. Three calls exercise both buffer parities; the pack
    quantises the bf16 rows itself in calls 1 and 3 and copies rows quantised
    beforehand in call 2."""
    import ctypes

    from trials_b200 import _lib

    dev = cuda_device
    L = synth.make_layer(SHAPE, orc.per_block_quant_fp8, seed=1)
    W = {k: getattr(L, k).to(dev) for k in ["w13", "w13_scale", "w2", "w2_scale"]}
    lib = _lib.lib()
    H, I, topk, cap, per = SHAPE.H, SHAPE.I, SHAPE.topk, SHAPE.M, SHAPE.E // G
    nbytes = lib.b200moe_ep_peer_bytes(cap, H, topk, G)
    bases = []
    for _ in range(G):
        b = ctypes.c_void_p()
        h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        _lib.check(lib.b200moe_ep_peer_alloc(nbytes, ctypes.byref(b), h), "ep_peer_alloc")
        bases.append(b.value)
    table = torch.tensor(bases, dtype=torch.int64, device=dev)
    ops = ep.CudaEPOps()
    R = G * cap
    ws = [torch.zeros(max(ops.workspace_bytes(R, H, I, per, topk), 256), dtype=torch.uint8, device=dev)
          for _ in range(G)]
    rank_w = _rank_weights(W, G)
    st = torch.cuda.current_stream(dev).cuda_stream
    try:
        for epoch in (1, 2, 3):
            toks = [_tokens(SHAPE, 100 * epoch + r, cap - 3 * r - epoch, dev) for r in range(G)]
            state = []
            for r, (hidden, tw, ids) in enumerate(toks):
                M = hidden.shape[0]
                q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=dev)
                s = torch.empty(M, H // 128, dtype=torch.float32, device=dev)
                ops.quant(hidden, q, s)
                pos = torch.empty(M * G, dtype=torch.int32, device=dev)
                tok_of = torch.empty(R, dtype=torch.int32, device=dev)
                counts = torch.empty(G, dtype=torch.int32, device=dev)
                err = torch.zeros(1, dtype=torch.int32, device=dev)
                quantise_in_pack = epoch != 2
                _lib.check(lib.b200moe_ep_dispatch_peer(
                    hidden.data_ptr() if quantise_in_pack else None, None if quantise_in_pack else q.data_ptr(),
                    None if quantise_in_pack else s.data_ptr(), ids.data_ptr(), tw.data_ptr(), M, H, topk, SHAPE.E,
                    G, r, None, 0, 0, cap,
                    table.data_ptr(), bases[r], epoch, pos.data_ptr(), tok_of.data_ptr(), counts.data_ptr(),
                    err.data_ptr(), st), "dispatch_peer")
                state.append((pos, err))
            for d in range(G):
                w13, w13s, w2, w2s = rank_w[d]
                _lib.check(lib.b200moe_layer_packed_peer(
                    bases[d], table.data_ptr(), G, d, cap, epoch, H, I, per, topk, w13.data_ptr(), w13s.data_ptr(),
                    w2.data_ptr(), w2s.data_ptr(), ws[d].data_ptr(), ws[d].numel(), st), "layer_packed_peer")
            outs = []
            for r, (hidden, _, _) in enumerate(toks):
                M = hidden.shape[0]
                out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
                pos, err = state[r]
                _lib.check(lib.b200moe_ep_combine_peer(bases[r], pos.data_ptr(), M, H, topk, G, cap, epoch,
                                                       out.data_ptr(), err.data_ptr(), st), "combine_peer")
                outs.append(out)
            ref = _all_to_all_form(G, cap, toks, W, dev)
            for r in range(G):
                assert moe.read_device_error(state[r][1]) == 0
                assert moe.read_device_error(ws[r][:4].view(torch.int32)) == 0
                assert torch.equal(outs[r], ref[r]), (epoch, r)
    finally:
        torch.cuda.synchronize(dev)
        for b in bases:
            lib.b200moe_ep_peer_free(b)


def test_expert_parallel_module_peer_exchange_one_rank(cuda_device):
    """ExpertParallelMoE with the peer exchange and no process group (G = 1)
    equals the single-GPU layer bit for bit on repeated calls."""
    dev = cuda_device
    L = synth.make_layer(SHAPE, orc.per_block_quant_fp8, seed=2)
    W = {k: getattr(L, k).to(dev) for k in ["w13", "w13_scale", "w2", "w2_scale"]}
    model = ep.ExpertParallelMoE(W["w13"], W["w13_scale"], W["w2"], W["w2_scale"], num_experts=SHAPE.E,
                                 rows_per_rank=SHAPE.M)
    assert model.exchange == "peer"
    try:
        for call in range(3):
            hidden, tw, ids = _tokens(SHAPE, 200 + call, SHAPE.M - call, dev)
            out = model(hidden, tw, ids)
            single = moe.moe_decode_megakernel_full(hidden, W["w13"], W["w13_scale"], W["w2"], W["w2_scale"], tw,
                                                    ids)
            assert orc.rel_l2(out, single) < EP_TOL
            assert model.device_errors() == 0
    finally:
        model.close()


def test_peer_waits_end_with_timeout_when_a_rank_never_dispatches(cuda_device):
    """Two ranks' exchange buffers in one process; rank 1 never runs. Rank 0's
    layer waits for rank 1's dispatch flag and its combine for rank 1's
    combine flag: with a 20 ms limit both calls must return, each set
    B200MOE_DEVERR_TIMEOUT in its error word, the whole sequence must take
    about two limits (not the 10 s default), and the context must stay usable."""
    import time

    from trials_b200 import _lib

    dev = cuda_device
    lib = _lib.lib()
    G, rank, cap = 2, 0, 8
    H, I, topk, per = SHAPE.H, SHAPE.I, SHAPE.topk, SHAPE.E // 2
    L = synth.make_layer(SHAPE, orc.per_block_quant_fp8, seed=3)
    W = {k: getattr(L, k)[:per].contiguous().to(dev) for k in ["w13", "w13_scale", "w2", "w2_scale"]}
    nbytes = lib.b200moe_ep_peer_bytes(cap, H, topk, G)
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(G)]  # zeroed receive areas
    table = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    ws = torch.zeros(max(lib.b200moe_layer_packed_workspace_size(G * cap, H, I, per, topk), 256), dtype=torch.uint8,
                     device=dev)
    hidden, tw, ids = _tokens(SHAPE, 7, cap, dev)
    pos = torch.empty(cap * G, dtype=torch.int32, device=dev)
    tok_of = torch.empty(G * cap, dtype=torch.int32, device=dev)
    counts = torch.empty(G, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    out = torch.empty(cap, H, dtype=torch.bfloat16, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    limit_us = 20_000
    previous = lib.b200moe_ep_peer_wait_limit_us(limit_us)
    try:
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        _lib.check(lib.b200moe_ep_dispatch_peer(
            hidden.data_ptr(), None, None, ids.data_ptr(), tw.data_ptr(), cap, H, topk, SHAPE.E, G, rank, None, 0, 0,
            cap, table.data_ptr(), bufs[rank].data_ptr(), 1, pos.data_ptr(), tok_of.data_ptr(), counts.data_ptr(),
            err.data_ptr(), st), "dispatch_peer")
        _lib.check(lib.b200moe_layer_packed_peer(
            bufs[rank].data_ptr(), table.data_ptr(), G, rank, cap, 1, H, I, per, topk, W["w13"].data_ptr(),
            W["w13_scale"].data_ptr(), W["w2"].data_ptr(), W["w2_scale"].data_ptr(), ws.data_ptr(), ws.numel(), st),
            "layer_packed_peer")
        _lib.check(lib.b200moe_ep_combine_peer(bufs[rank].data_ptr(), pos.data_ptr(), cap, H, topk, G, cap, 1,
                                               out.data_ptr(), err.data_ptr(), st), "combine_peer")
        torch.cuda.synchronize(dev)
        wall = time.perf_counter() - t0
    finally:
        lib.b200moe_ep_peer_wait_limit_us(previous)
    assert moe.read_device_error(ws[:4].view(torch.int32)) & _lib.DEVERR_TIMEOUT   # the layer's dispatch wait
    assert moe.read_device_error(err) & _lib.DEVERR_TIMEOUT                        # the combine's wait
    assert 2 * limit_us * 1e-6 <= wall < 2.0, wall
    # the context still runs work
    x = torch.arange(1024, device=dev, dtype=torch.float32)
    assert float(x.sum().item()) == 1023 * 1024 / 2


def _skewed_tokens(G, cap, dev, hot=4, seed=300):
    toks = []
    for r in range(G):
        g = torch.Generator().manual_seed(seed + r)
        logits = torch.randn(cap - 2 * r, SHAPE.E, generator=g)
        logits[:, :hot] += 2.0
        tw, ids = synth.make_router(logits, SHAPE.topk, SHAPE.scoring)
        hidden = torch.randn(cap - 2 * r, SHAPE.H, generator=g).to(torch.bfloat16)
        toks.append((hidden.to(dev), tw.to(dev), ids.to(dev)))
    return toks


def _peer_call(lib, G, cap, bases, table_ptr, ws, toks, weights, epoch, dev, placement=None):
    """One call of the peer exchange for G simulated ranks in one process:
    every dispatch, then every layer, then every combine (no wait depends on a
    later launch)."""
    from trials_b200 import _lib

    H, I, topk = SHAPE.H, SHAPE.I, SHAPE.topk
    st = torch.cuda.current_stream(dev).cuda_stream
    ptable = None if placement is None else torch.as_tensor(placement.table(), device=dev)
    E_local = SHAPE.E // G if placement is None else placement.slots
    state = []
    for r, (hidden, tw, ids) in enumerate(toks):
        M = hidden.shape[0]
        pos = torch.empty(M * G, dtype=torch.int32, device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        # named (not temporaries): a tensor whose data_ptr() alone is passed would
        # be freed, and its memory handed to the next allocation, before the kernels run
        tok_of = torch.empty(G * cap, dtype=torch.int32, device=dev)
        counts = torch.empty(G, dtype=torch.int32, device=dev)
        _lib.check(lib.b200moe_ep_dispatch_peer(
            hidden.data_ptr(), None, None, ids.data_ptr(), tw.data_ptr(), M, H, topk, SHAPE.E, G, r,
            None if ptable is None else ptable.data_ptr(), 0 if placement is None else placement.max_replicas,
            0 if placement is None else placement.slots, cap, table_ptr, bases[r], epoch, pos.data_ptr(),
            tok_of.data_ptr(), counts.data_ptr(), err.data_ptr(), st), "dispatch_peer")
        state.append((pos, err, tok_of, counts))
    for d in range(G):
        w13, w13s, w2, w2s = weights[d]
        _lib.check(lib.b200moe_layer_packed_peer(bases[d], table_ptr, G, d, cap, epoch, H, I, E_local, topk,
                                                 w13.data_ptr(), w13s.data_ptr(), w2.data_ptr(), w2s.data_ptr(),
                                                 ws[d].data_ptr(), ws[d].numel(), st), "layer_packed_peer")
    outs = []
    for r, (hidden, _, _) in enumerate(toks):
        out = torch.empty(hidden.shape[0], H, dtype=torch.bfloat16, device=dev)
        pos, err = state[r][:2]
        _lib.check(lib.b200moe_ep_combine_peer(bases[r], pos.data_ptr(), hidden.shape[0], H, topk, G, cap, epoch,
                                               out.data_ptr(), err.data_ptr(), st), "combine_peer")
        outs.append((out, err))
    torch.cuda.synchronize(dev)
    for r in range(G):
        assert moe.read_device_error(outs[r][1]) == 0
        assert moe.read_device_error(ws[r][:4].view(torch.int32)) == 0
    return [o for o, _ in outs]


@pytest.mark.parametrize("G", [2, 4, 8])
def test_replicated_hot_experts_both_exchange_forms(cuda_device, G):
    """A skewed router (experts 0-3 hot) with eplb_placement's replicas (two
    spare slots per rank): the dispatch bytes equal the oracle's replica
    choice, the peer exchange equals the all-to-all form bit for bit over two
    calls (both buffer parities), and both equal the single-GPU layer up to
    the bf16 rounding of each rank's partial sum."""
    from trials_b200 import _lib

    dev = cuda_device
    L = synth.make_layer(SHAPE, orc.per_block_quant_fp8, seed=6)
    W = {k: getattr(L, k).to(dev) for k in ["w13", "w13_scale", "w2", "w2_scale"]}
    cap = SHAPE.M
    lib = _lib.lib()
    H, I, topk = SHAPE.H, SHAPE.I, SHAPE.topk
    toks0 = _skewed_tokens(G, cap, dev)
    load = sum(torch.bincount(ids.reshape(-1).cpu(), minlength=SHAPE.E) for _, _, ids in toks0)
    pl = ep.eplb_placement(load.numpy(), G, SHAPE.E // G + 2)
    assert pl.max_replicas > 1
    weights = _rank_weights(W, G, pl)
    nbytes = lib.b200moe_ep_peer_bytes(cap, H, topk, G)
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(G)]
    bases = [b.data_ptr() for b in bufs]
    table = torch.tensor(bases, dtype=torch.int64, device=dev)
    R = G * cap
    ws = [torch.zeros(max(lib.b200moe_layer_packed_workspace_size(R, H, I, pl.slots, topk), 256), dtype=torch.uint8,
                      device=dev) for _ in range(G)]
    for epoch in (1, 2):
        toks = toks0 if epoch == 1 else _skewed_tokens(G, cap, dev, seed=400)
        ref = _all_to_all_form(G, cap, toks, W, dev, placement=pl, check_bytes=(epoch == 1))
        outs = _peer_call(lib, G, cap, bases, table.data_ptr(), ws, toks, weights, epoch, dev, placement=pl)
        for r, (hidden, tw, ids) in enumerate(toks):
            assert torch.equal(outs[r], ref[r]), (epoch, r)
            single = moe.moe_decode_megakernel_full(hidden, W["w13"], W["w13_scale"], W["w2"], W["w2_scale"], tw, ids)
            assert orc.rel_l2(outs[r], single) < EP_TOL
    torch.cuda.synchronize(dev)


@pytest.mark.parametrize("M,G", [(40, 2), (40, 8), (256, 4), (300, 2), (200, 8)])
def test_peer_dispatch_plan_matches_all_to_all_form(cuda_device, M, G):
    """The peer dispatch (the pack quantising the bf16 rows on its way into
    the destinations' receive areas) leaves the same plan outputs (pos,
    counts, tok_of of the used rows) and the same row bytes in every
    destination's receive area as the all-to-all form's dispatch, with dropped
    (-1) and out-of-range ids among them."""
    from trials_b200 import _lib

    dev = cuda_device
    lib = _lib.lib()
    H, topk, E, cap = 512, 4, 16, M
    rank = G - 1
    rb = lib.b200moe_ep_row_bytes(H, topk)
    g = torch.Generator(device=dev).manual_seed(M * 10 + G)
    hidden = torch.randn(M, H, generator=g, device=dev).to(torch.bfloat16)
    tw, ids = synth.make_router(torch.randn(M, E, generator=g, device=dev), topk, "sigmoid")
    ids[::5, 1] = -1
    ids[3, 0] = E + 2  # out of range: dropped and reported
    st = torch.cuda.current_stream(dev).cuda_stream
    z = lambda n, v=0: torch.full((n,), v, dtype=torch.int32, device=dev)  # noqa: E731
    # the all-to-all form (plan launch + pack into the send buffer)
    q = torch.empty(M, H, dtype=torch.float8_e4m3fn, device=dev)
    s = torch.empty(M, H // 128, dtype=torch.float32, device=dev)
    ep.CudaEPOps().quant(hidden, q, s)
    send = torch.zeros(G * cap * rb, dtype=torch.uint8, device=dev)
    pos_a, tok_a, cnt_a, err_a = z(M * G), z(G * cap, -7), z(G), z(1)
    _lib.check(lib.b200moe_ep_dispatch(q.data_ptr(), s.data_ptr(), ids.data_ptr(), tw.data_ptr(), M, H, topk, E, G,
                                       rank, None, 0, 0, cap, send.data_ptr(), pos_a.data_ptr(), tok_a.data_ptr(),
                                       cnt_a.data_ptr(), err_a.data_ptr(), st), "dispatch")
    # the peer form, G exchange buffers in this process, epoch 1
    nbytes = lib.b200moe_ep_peer_bytes(cap, H, topk, G)
    bufs = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(G)]
    table = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device=dev)
    pos_p, tok_p, cnt_p, err_p = z(M * G), z(G * cap, -7), z(G), z(1)
    _lib.check(lib.b200moe_ep_dispatch_peer(hidden.data_ptr(), None, None, ids.data_ptr(), tw.data_ptr(), M, H, topk,
                                            E, G, rank, None, 0, 0, cap, table.data_ptr(), bufs[rank].data_ptr(), 1,
                                            pos_p.data_ptr(), tok_p.data_ptr(), cnt_p.data_ptr(), err_p.data_ptr(),
                                            st), "dispatch_peer")
    torch.cuda.synchronize(dev)
    assert torch.equal(pos_a, pos_p) and torch.equal(cnt_a, cnt_p)
    recv_bytes = (G * cap * rb + 255) // 256 * 256
    off = 1024 + recv_bytes  # receive area of epoch 1 (odd parity)
    rows_a = send.view(G, cap, rb)
    for d in range(G):
        n = int(cnt_a[d].item())
        assert torch.equal(tok_a[d * cap:d * cap + n], tok_p[d * cap:d * cap + n])
        area = bufs[d][off + rank * cap * rb: off + (rank + 1) * cap * rb].view(cap, rb)
        assert torch.equal(area[:n], rows_a[d, :n]), d
        # rows past the count carry no expert (ids -1)
        meta = area[n:, H + (H // 128) * 4: H + (H // 128) * 4 + 4 * topk].contiguous().view(torch.int32)
        assert bool((meta == -1).all())
        assert int(bufs[d][rank * 4:rank * 4 + 4].view(torch.int32).item()) == 1  # this rank's dispatch flag
    assert moe.read_device_error(err_a) == moe.read_device_error(err_p) != 0
