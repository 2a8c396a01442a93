"""One rank of the NCCL expert-parallel check (launched by torchrun from
tests/test_gpu_ep_nccl.py). Every rank builds the same global layer from the
same seed, keeps its experts, runs its own tokens through ExpertParallelMoE
and compares with the single-GPU layer over all experts. Rank 0 prints
EP_NCCL_OK when every rank is within tolerance."""
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
    model = ep.ExpertParallelMoE(ep.shard_experts(L.w13, rank, world), ep.shard_experts(L.w13_scale, rank, world),
                                 ep.shard_experts(L.w2, rank, world), ep.shard_experts(L.w2_scale, rank, world),
                                 num_experts=shape.E, rows_per_rank=shape.M)
    g = torch.Generator().manual_seed(100 + rank)
    M = shape.M - 5 * rank
    tw, ids = synth.make_router(torch.randn(M, shape.E, generator=g), shape.topk, shape.scoring)
    hidden = torch.randn(M, shape.H, generator=g).to(torch.bfloat16).to(dev)
    tw, ids = tw.to(dev), ids.to(dev)
    out = model(hidden, tw, ids)
    out2 = model(hidden, tw, ids)
    ref = moe.moe_decode_megakernel_full(hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, tw, ids)
    err = torch.tensor([orc.rel_l2(out, ref), 0.0 if torch.equal(out, out2) else 1.0, float(model.device_errors())],
                       device=dev, dtype=torch.float64)
    dist.all_reduce(err, op=dist.ReduceOp.MAX)
    if rank == 0:
        ok = err[0].item() < TOL and err[1].item() == 0 and err[2].item() == 0
        print(("EP_NCCL_OK" if ok else "EP_NCCL_FAIL") + f" world={world} max_rel={err[0].item():.3e} "
              f"nondeterministic={err[1].item():.0f} device_errors={err[2].item():.0f}", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
