"""Generates the golden fixtures that pin the oracle to the reference.

Runs the reference's OWN code on the CPU, in this container (the reference is
not needed at test time; only the .npz files it writes are):
  * its Triton kernels (aiter_module/moe_decode_megakernel.py and
    aiter_module/moe_decode_megakernel_fused.py) under TRITON_INTERPRET=1;
  * its torch helpers per_token_group_quant_fp8, per_block_quant_fp8,
    silu_gate_up and build_routing_from_topk (phase5_orchestrator.py:26-66),
    compiled from the source text because the module imports aiter at load;
  * its full orchestrator _moe_decode_megakernel_full
    (sglang_integration/aiter.py:74-177), compiled from the source text with
    its imports pointed at: the reference Triton module above, the reference
    torch quantiser above (standing in for sglang's per_token_group_quant_fp8,
    the same formula), and moe_align_block_size restated by the oracle (sglang's
    CUDA op is not vendored in the reference).
The tiny shape needs the orchestrator's BLOCK_N set to 32: the reference's
N-split grid uses (N/8)//BLOCK_N programs per slice, which is 0 for N=256 at 128
(aiter_module/moe_decode_megakernel.py:107-110).

Usage:  python tests/golden/make_golden.py --reference <reference checkout>
        (or TRIALS_REFERENCE=<reference checkout> python tests/golden/make_golden.py)
"""
from __future__ import annotations

import argparse
import ast
import hashlib
import os
import sys
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import moe_oracle as orc  # noqa: E402
from trials_b200 import synth  # noqa: E402


def load_functions(path: Path, names: list[str], glb: dict) -> dict:
    """Compiles only the named top-level functions of a source file."""
    tree = ast.parse(path.read_text())
    keep = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in names]
    missing = set(names) - {n.name for n in keep}
    if missing:
        raise RuntimeError(f"{path}: functions not found: {missing}")
    mod = ast.Module(body=keep, type_ignores=[])
    exec(compile(mod, str(path), "exec"), glb)
    return glb


def sha(t: torch.Tensor) -> str:
    t = t.contiguous().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    elif t.dtype == torch.float8_e4m3fn:
        t = t.view(torch.uint8)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()[:16]


def u8(t):
    return t.contiguous().view(torch.uint8).numpy()


def bf(t):
    return t.contiguous().to(torch.bfloat16).view(torch.int16).numpy()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TRIALS_REFERENCE"),
                    help="the reference checkout (default: $TRIALS_REFERENCE)")
    args = ap.parse_args(argv)
    if not args.reference:
        ap.error("give the reference checkout with --reference or TRIALS_REFERENCE")
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "aiter_module"))
    import moe_decode_megakernel as mk  # reference Triton kernel
    import moe_decode_megakernel_fused as mkf  # reference fused Triton kernel

    p5 = load_functions(ref / "phase5_orchestrator.py",
                        ["per_token_group_quant_fp8", "per_block_quant_fp8", "silu_gate_up",
                         "build_routing_from_topk"],
                        {"torch": torch, "BLOCK_M": 64})

    shape = synth.TINY
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(shape.M, shape.E, generator=g)
    topk_w, topk_ids = synth.make_router(logits, shape.topk, shape.scoring)
    w13_bf = (torch.randn(shape.E, 2 * shape.I, shape.H, generator=g) * 0.02).to(torch.bfloat16)
    w2_bf = (torch.randn(shape.E, shape.H, shape.I, generator=g) * 0.02).to(torch.bfloat16)
    hidden = torch.randn(shape.M, shape.H, generator=g).to(torch.bfloat16)
    # Same draws as synth.make_layer (one expert chunk covers all 8 experts).
    w13, w13_s = p5["per_block_quant_fp8"](w13_bf)
    w2, w2_s = p5["per_block_quant_fp8"](w2_bf)

    # ---- reference orchestrator with recording stubs
    rec = {}

    def align_stub(topk_ids_t, bm, E):
        s, e, n = orc.moe_align_block_size(topk_ids_t.numpy(), bm, E)
        rec["align"] = (s.copy(), e.copy(), n)
        # The reference launcher runs expert_ids.shape[0] (capacity) blocks
        # (aiter_module/moe_decode_megakernel.py:104-110), so its last block reads
        # sorted ids up to blocks*bm, past the sglang allocation. Pad that slack
        # with the sentinel so the interpreter reads defined memory.
        s = np.concatenate([s, np.full(e.size * bm - s.size, topk_ids_t.numel(), dtype=np.int32)])
        # The launcher also takes its block count from expert_ids.shape[0], and in
        # stage 2 its row mask passes every row (nvt = rows(a) * topk), so the
        # capacity-tail blocks would read a2 and write gemm2 past npm*BM rows.
        # Hand it the valid blocks only; tail blocks produce no valid rows.
        e = e[: n // bm].copy()
        return torch.from_numpy(s), torch.from_numpy(e), torch.tensor([n], dtype=torch.int32)

    def quant_stub(x, gk):
        q, s = p5["per_token_group_quant_fp8"](x, gk)
        rec.setdefault("quant", []).append((x.clone(), q.clone(), s.clone()))
        return q, s

    def stage_stub(*a, **kw):
        mk.moe_decode_megakernel_stage1(*a, **kw)
        rec.setdefault("stage", []).append(a[6].clone())

    def install(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        sys.modules[name] = m

    for name in ["sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.moe",
                 "sglang.srt.layers.moe.moe_runner", "sglang.srt.layers.moe.moe_runner.triton_utils",
                 "sglang.kernels", "sglang.kernels.ops", "sglang.kernels.ops.quantization",
                 "aiter", "aiter.ops", "aiter.ops.triton", "aiter.ops.triton._triton_kernels",
                 "aiter.ops.triton._triton_kernels.moe"]:
        install(name)
    install("sglang.srt.layers.moe.moe_runner.triton_utils.moe_align_block_size", moe_align_block_size=align_stub)
    install("sglang.kernels.ops.quantization.fp8_kernel", per_token_group_quant_fp8=quant_stub)
    install("aiter.ops.triton._triton_kernels.moe.moe_decode_megakernel", moe_decode_megakernel_stage1=stage_stub)

    glb = {"torch": torch, "Optional": __import__("typing").Optional,
           "_MOE_DECODE_MEGA_BLOCK_M": 128, "_MOE_DECODE_MEGA_BLOCK_N": 32, "_MOE_DECODE_MEGA_BLOCK_K": 128}
    load_functions(ref / "sglang_integration" / "aiter.py", ["_moe_decode_megakernel_full"], glb)
    out = glb["_moe_decode_megakernel_full"](hidden, w13, w13_s, w2, w2_s, topk_w, topk_ids)

    sorted128, eids128, ntp128 = rec["align"]
    T = shape.M * shape.topk
    valid = np.nonzero(sorted128 < T)[0]
    flat_order = sorted128[valid]
    (_, a1_q, a1_s), (inter_in, a2_q, a2_s) = rec["quant"]
    gemm1, gemm2 = rec["stage"]

    # ---- reference fused kernels (stage-1 SiLU, stage-2 atomic unpermute), BM=128, BN=32
    st, ei = torch.from_numpy(sorted128), torch.from_numpy(eids128[: ntp128 // 128].copy())
    inter_f = torch.zeros(ntp128, shape.I, dtype=torch.bfloat16)
    mkf.moe_decode_megakernel_stage1_fused(a1_q, w13, a1_s, w13_s, st, ei, inter_f, shape.topk,
                                           block_m=128, block_n=32, block_k=128, fused_silu=True)
    a2f_q, a2f_s = p5["per_token_group_quant_fp8"](inter_f, 128)
    # The fused stage-2 launcher takes nvt = rows(a) * topk with a in sorted
    # order (npm*BM rows), not M * topk (moe_decode_megakernel_fused.py:150-153),
    # so padding rows (sentinel M*topk) pass the mask: they read
    # topk_weights[M*topk] and atomically add into out_final row M. One slack
    # output row and one zero weight keep those accesses in bounds here.
    out_f = torch.zeros(shape.M + 1, shape.H, dtype=torch.float32)
    tw_pad = torch.cat([topk_w.reshape(-1), torch.zeros(1)])
    mkf.moe_decode_megakernel_stage2_fused(a2f_q, w2, a2f_s, w2_s, st, ei, out_f, tw_pad,
                                           shape.topk, block_m=128, block_n=32, block_k=128)
    out_f = out_f[: shape.M]

    # ---- reference routing helper (stable order, no per-expert padding)
    sorted_tok, _, _ = p5["build_routing_from_topk"](topk_ids, "cpu")

    fixture = {
        "sha_w13_bf16": sha(w13_bf), "sha_w2_bf16": sha(w2_bf), "sha_hidden": sha(hidden),
        "sha_topk_ids": sha(topk_ids), "sha_topk_w": sha(topk_w),
        "topk_ids": topk_ids.numpy(), "topk_w": topk_w.numpy(),
        "sha_w13_q": sha(w13), "w13_s": w13_s.numpy(), "sha_w2_q": sha(w2), "w2_s": w2_s.numpy(),
        "a1_q": u8(a1_q), "a1_s": a1_s.numpy(),
        "align128_sorted": sorted128, "align128_eids": eids128, "align128_ntp": np.int64(ntp128),
        "build_routing_order": sorted_tok.numpy()[: T],
        "valid_pos": valid, "flat_order": flat_order,
        "gemm1_valid": bf(gemm1[valid]), "inter_valid": bf(inter_in[valid]),
        "a2_q_valid": u8(a2_q[valid]), "a2_s_valid": a2_s[valid].numpy(),
        "gemm2_valid": bf(gemm2[valid]), "out": bf(out),
        "fused_inter_valid": bf(inter_f[valid]), "fused_out": out_f.numpy(),
    }
    dst = Path(__file__).resolve().parent / "tiny_seed0.npz"
    np.savez_compressed(dst, **{k: np.asarray(v) for k, v in fixture.items()})
    print(f"wrote {dst} ({dst.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
