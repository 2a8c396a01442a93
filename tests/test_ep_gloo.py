"""Expert-parallel orchestration on CPU gloo ranks (world size 2 and 4).

trials_b200.ep.ExpertParallelMoE runs its real rank logic - buffer sizing,
packed-row layout, the two equal-split all-to-alls, combine - with the
rank-local steps supplied by oracle.ep_oracle (the CPU restatement of the CUDA
kernels' contract). Each rank's output is checked against the single-process
oracle layer over all experts. A second test makes one rank fail before the
exchange and checks that the other rank gets an error from the short
process-group timeout instead of waiting forever.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

SHAPE_KW = dict(M=24, H=256, I=128, E=8, topk=2, scoring="softmax")
TOL = 1e-2  # bf16 rounding of each rank's partial sum before the cross-rank add


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(shape, rank, M):
    from trials_b200 import synth

    g = torch.Generator().manual_seed(100 + rank)
    logits = torch.randn(M, shape.E, generator=g)
    tw, ids = synth.make_router(logits, shape.topk, shape.scoring)
    hidden = torch.randn(M, shape.H, generator=g).to(torch.bfloat16)
    return hidden, tw, ids


def _worker(rank, world, port, results, fail_rank, eplb=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    from oracle import ep_oracle
    from oracle import moe_oracle as orc
    from trials_b200 import ep, synth

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=8))
    try:
        shape = synth.LayerShape(**SHAPE_KW)
        L = synth.make_layer(shape, orc.per_block_quant_fp8, seed=0)
        M = shape.M - 7 * rank  # ranks bring different token counts
        hidden, tw, ids = _tokens(shape, rank, M)
        if eplb:
            # every rank derives the same placement from the load of all ranks' tokens
            load = sum(torch.bincount(_tokens(shape, r, shape.M - 7 * r)[2].reshape(-1), minlength=shape.E)
                       for r in range(world))
            pl = ep.eplb_placement(load.numpy(), world, shape.E // world + 1)
            w = [ep.place_experts(t, pl, rank) for t in (L.w13, L.w13_scale, L.w2, L.w2_scale)]
        else:
            pl = None
            w = [ep.shard_experts(t, rank, world) for t in (L.w13, L.w13_scale, L.w2, L.w2_scale)]
        model = ep.ExpertParallelMoE(*w, num_experts=shape.E, rows_per_rank=shape.M, ops=ep_oracle.OracleEPOps(),
                                     device="cpu", placement=pl)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the exchange")
        out = model(hidden, tw, ids)
        out2 = model(hidden, tw, ids)  # buffers are reused across calls
        ref = orc.moe_layer(hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, tw, ids)
        results.put((rank, "ok", orc.rel_l2(out, ref), bool(torch.equal(out, out2))))
    except Exception as exc:  # reported to the parent, which decides
        results.put((rank, "error", repr(exc)[:200], False))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1, timeout=120, eplb=False):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results, fail_rank, eplb)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, status, val, same = results.get(timeout=timeout)
        out[rank] = (status, val, same)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("eplb", [False, True], ids=["split", "replicated"])
@pytest.mark.parametrize("world", [2, 4])
def test_expert_parallel_matches_single_process_layer(world, eplb):
    """eplb=True: hot experts replicated (one spare slot per rank) by
    eplb_placement; the result is the same layer."""
    res = _run(world, eplb=eplb)
    for rank in range(world):
        status, err, same = res[rank]
        assert status == "ok", res[rank]
        assert err < TOL, (rank, err)
        assert same, "two calls must give the same output"


def test_rank_failure_surfaces_as_error_not_hang():
    res = _run(2, fail_rank=1)
    assert res[1][0] == "error" and "injected" in res[1][1]
    assert res[0][0] == "error", "the surviving rank must see an error from the collective"
