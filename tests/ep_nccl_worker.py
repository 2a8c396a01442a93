"""One rank of the multi-GPU expert-parallel check (launched by torchrun from
tests/test_gpu_ep_nccl.py). Every rank builds the same global layer from the
same seed, keeps its experts, runs its own tokens through ExpertParallelMoE
with both exchanges (NCCL all-to-alls, and the kernels' own stores into the
other GPUs' memory) and compares with the single-GPU layer over all experts;
the two exchanges must agree bit for bit, over several calls (both buffer
parities of the peer exchange). A second pass does the same with a skewed
router and hot experts replicated over the ranks (eplb_placement). Rank 0
prints EP_NCCL_OK when every rank passes."""
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from oracle import moe_oracle as orc  # noqa: E402
from trials_b200 import ep, moe, synth  # noqa: E402

TOL = 1e-2


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    shape = synth.LayerShape(M=48, H=512, I=256, E=16, topk=4, scoring="sigmoid")
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=0, device=dev)

    def tokens(r, call, hot):
        g = torch.Generator().manual_seed(100 + 10 * call + r + 1000 * hot)
        M = shape.M - 5 * r - call
        logits = torch.randn(M, shape.E, generator=g)
        logits[:, :hot] += 2.0
        tw, ids = synth.make_router(logits, shape.topk, shape.scoring)
        hidden = torch.randn(M, shape.H, generator=g).to(torch.bfloat16).to(dev)
        return hidden, tw.to(dev), ids.to(dev)

    worst_rel, mismatch, dev_err = 0.0, 0.0, 0
    for hot in (0, 4):
        if hot:  # every rank derives the same placement from all ranks' first batch
            load = sum(torch.bincount(tokens(r, 0, hot)[2].reshape(-1).cpu(), minlength=shape.E)
                       for r in range(world))
            pl = ep.eplb_placement(load.numpy(), world, shape.E // world + 1)
            w = [ep.place_experts(t, pl, rank) for t in (L.w13, L.w13_scale, L.w2, L.w2_scale)]
        else:
            pl = None
            w = [ep.shard_experts(t, rank, world) for t in (L.w13, L.w13_scale, L.w2, L.w2_scale)]
        models = {x: ep.ExpertParallelMoE(*w, num_experts=shape.E, rows_per_rank=shape.M, exchange=x, placement=pl)
                  for x in ("nccl", "peer")}
        for call in range(3):
            hidden, tw, ids = tokens(rank, call, hot)
            out = {x: m(hidden, tw, ids) for x, m in models.items()}
            ref = moe.moe_decode_megakernel_full(hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, tw, ids)
            worst_rel = max(worst_rel, orc.rel_l2(out["nccl"], ref), orc.rel_l2(out["peer"], ref))
            mismatch = max(mismatch, 0.0 if torch.equal(out["nccl"], out["peer"]) else 1.0)
            dev_err |= models["nccl"].device_errors() | models["peer"].device_errors()
        models["peer"].close()
    err = torch.tensor([worst_rel, mismatch, float(dev_err)], device=dev, dtype=torch.float64)
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    if rank == 0:
        ok = err[0].item() < TOL and err[1].item() == 0 and err[2].item() == 0
        print(("EP_NCCL_OK" if ok else "EP_NCCL_FAIL") + f" world={world} max_rel={err[0].item():.3e} "
              f"peer_vs_nccl_mismatch={err[1].item():.0f} device_errors={err[2].item():.0f}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
