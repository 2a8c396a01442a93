"""Stage-level calls of the layer (route -> gather/quantise -> GEMM1+SiLU ->
GEMM2+combine -> top-k reduce, or the two GEMM stages as one launch) on
explicit torch buffers.

These mirror the reference's kernel launchers (moe_decode_megakernel_stage1,
..._stage1_fused with fused_silu, ..._stage2_fused:
aiter_module/moe_decode_megakernel.py:88-123,
aiter_module/moe_decode_megakernel_fused.py:125-157) on the library's own
expert-sorted row layout (each expert padded to 16 rows).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from .moe import FP8, _ptr, _require_cuda, _stream


@dataclass
class Routing:
    tile_tokens: int
    rows_cap: int
    chunks_cap: int
    sorted_ids: torch.Tensor    # (rows_cap,) int32
    chunk_expert: torch.Tensor  # (chunks_cap,) int32
    chunk_row0: torch.Tensor
    chunk_rows: torch.Tensor
    counts: torch.Tensor        # [n_chunks, num_rows] int32
    err: torch.Tensor           # (1,) int32
    chunk_ready: torch.Tensor   # (chunks_cap + 2,) int32, zeroed by route for experts()
    slot_pos: torch.Tensor      # (M*topk,) int32: sorted row of each flat slot, -1 if dropped

    @property
    def n_chunks(self):
        return self.counts[0:1]

    @property
    def num_rows(self):
        return self.counts[1:2]

    def a_s_ld(self) -> int:
        return (self.rows_cap + 256 + 63) // 64 * 64

    @property
    def sorted_rows(self) -> int:
        """Stage-2 output layout: 1 = row p (sorted, token-major tiles), 0 = row of the slot."""
        return 1 if self.tile_tokens > 64 else 0

    def pair_rows(self, M: int, topk: int) -> int:
        return self.rows_cap if self.sorted_rows else M * topk


def route(topk_ids: torch.Tensor, num_experts: int, tile_tokens: int, expert_map: Optional[torch.Tensor] = None,
          num_local_experts: Optional[int] = None, err: Optional[torch.Tensor] = None,
          multi_cta: bool = True) -> Routing:
    """Routing into expert-sorted rows and the GEMM work list. multi_cta=False
    keeps large batches on the one-CTA kernel (the two give the same result)."""
    dev = _require_cuda(topk_ids)
    ids = topk_ids.to(torch.int32).contiguous()
    M, topk = ids.shape
    E = num_local_experts if expert_map is not None else num_experts
    L = _lib.lib()
    rows_cap = L.b200moe_route_capacity_rows(M * topk, E)
    chunks_cap = L.b200moe_route_capacity_chunks(M * topk, E, tile_tokens)
    z = lambda n: torch.empty(max(n, 1), dtype=torch.int32, device=dev)  # noqa: E731
    r = Routing(tile_tokens, rows_cap, chunks_cap, z(rows_cap), z(chunks_cap), z(chunks_cap), z(chunks_cap),
                torch.zeros(2, dtype=torch.int32, device=dev),
                err if err is not None else torch.zeros(1, dtype=torch.int32, device=dev), z(chunks_cap + 2), z(M * topk))
    if expert_map is not None:
        expert_map = expert_map.to(device=dev, dtype=torch.int32).contiguous()
    ns = L.b200moe_route_scratch_ints(M * topk, E) if multi_cta else 0
    scratch = torch.empty(ns, dtype=torch.int32, device=dev) if ns > 0 else None
    _lib.check(L.b200moe_route(_ptr(ids), M, topk, num_experts, _ptr(expert_map), E, tile_tokens,
                               _ptr(r.sorted_ids), rows_cap, _ptr(r.chunk_expert), _ptr(r.chunk_row0),
                               _ptr(r.chunk_rows), chunks_cap, _ptr(r.n_chunks), _ptr(r.num_rows), _ptr(r.slot_pos),
                               _ptr(r.chunk_ready), _ptr(scratch), ns, _ptr(r.err), _stream(dev)), "route")
    return r


def route_logits(logits: torch.Tensor, top_k: int, tile_tokens: int, scoring_func: str = "sigmoid",
                 correction_bias: Optional[torch.Tensor] = None, renormalize: bool = True,
                 routed_scaling_factor: float = 1.0, expert_map: Optional[torch.Tensor] = None,
                 num_local_experts: Optional[int] = None, err: Optional[torch.Tensor] = None):
    """Router + routing (b200moe_route_logits) -> (Routing, topk_weights (M, k)
    f32, topk_ids (M, k) int32), equal to select_experts followed by route()."""
    dev = _require_cuda(logits)
    logits = logits.contiguous()
    M, E_router = logits.shape
    E = num_local_experts if expert_map is not None else E_router
    L = _lib.lib()
    numel = M * top_k
    rows_cap = L.b200moe_route_capacity_rows(numel, E)
    chunks_cap = L.b200moe_route_capacity_chunks(numel, E, tile_tokens)
    z = lambda n: torch.empty(max(n, 1), dtype=torch.int32, device=dev)  # noqa: E731
    r = Routing(tile_tokens, rows_cap, chunks_cap, z(rows_cap), z(chunks_cap), z(chunks_cap), z(chunks_cap),
                torch.zeros(2, dtype=torch.int32, device=dev),
                err if err is not None else torch.zeros(1, dtype=torch.int32, device=dev), z(chunks_cap + 2), z(numel))
    tw = torch.empty(M, top_k, dtype=torch.float32, device=dev)
    ids = torch.empty(M, top_k, dtype=torch.int32, device=dev)
    if expert_map is not None:
        expert_map = expert_map.to(device=dev, dtype=torch.int32).contiguous()
    ns = L.b200moe_route_logits_scratch_ints(numel, E)
    scratch = torch.zeros(ns, dtype=torch.int32, device=dev)
    bias = None if correction_bias is None else correction_bias.to(device=dev, dtype=torch.float32).contiguous()
    scoring = {"softmax": 0, "sigmoid": 1}[scoring_func]
    _lib.check(L.b200moe_route_logits(_ptr(logits), int(logits.dtype == torch.bfloat16), M, E_router, top_k, scoring,
                                      _ptr(bias), int(renormalize), float(routed_scaling_factor), _ptr(tw), _ptr(ids),
                                      _ptr(expert_map), E, tile_tokens, _ptr(r.sorted_ids), rows_cap,
                                      _ptr(r.chunk_expert), _ptr(r.chunk_row0), _ptr(r.chunk_rows), chunks_cap,
                                      _ptr(r.n_chunks), _ptr(r.num_rows), _ptr(r.slot_pos), _ptr(r.chunk_ready),
                                      _ptr(scratch), ns, _ptr(r.err), _stream(dev)), "route_logits")
    return r, tw, ids


def route_mixed(topk_ids: torch.Tensor, num_experts: int, tile_tokens: int, heavy_rows: int = 128):
    """Mixed work lists (b200moe_route_mixed) -> (Routing of the light list,
    heavy list dict {chunk_expert, chunk_row0, chunk_rows, counters, cap},
    counts (4,) = [light chunks, rows, heavy chunks, first heavy row])."""
    dev = _require_cuda(topk_ids)
    ids = topk_ids.to(torch.int32).contiguous()
    M, topk = ids.shape
    L = _lib.lib()
    rows_cap = L.b200moe_route_capacity_rows(M * topk, num_experts)
    chunks_cap = L.b200moe_route_capacity_chunks(M * topk, num_experts, tile_tokens)
    cap2 = L.b200moe_route_capacity_chunks(M * topk, num_experts, 128)
    z = lambda n: torch.full((max(n, 1),), -7, dtype=torch.int32, device=dev)  # noqa: E731
    counts = torch.zeros(4, dtype=torch.int32, device=dev)
    r = Routing(tile_tokens, rows_cap, chunks_cap, z(rows_cap), z(chunks_cap), z(chunks_cap), z(chunks_cap),
                counts[:2], torch.zeros(1, dtype=torch.int32, device=dev), z(chunks_cap + 2), z(M * topk))
    heavy = {"chunk_expert": z(cap2), "chunk_row0": z(cap2), "chunk_rows": z(cap2), "counters": z(2), "cap": cap2}
    _lib.check(L.b200moe_route_mixed(_ptr(ids), M, topk, num_experts, None, num_experts, tile_tokens, heavy_rows,
                                     _ptr(r.sorted_ids), rows_cap, _ptr(r.chunk_expert), _ptr(r.chunk_row0),
                                     _ptr(r.chunk_rows), chunks_cap, _ptr(heavy["chunk_expert"]),
                                     _ptr(heavy["chunk_row0"]), _ptr(heavy["chunk_rows"]), cap2, _ptr(counts),
                                     _ptr(r.slot_pos), _ptr(r.chunk_ready), _ptr(heavy["counters"]), _ptr(r.err),
                                     _stream(dev)), "route_mixed")
    return r, heavy, counts


def gather_quant(hidden: torch.Tensor, topk: int, r: Routing):
    """-> (a_q (rows_cap, H) e4m3, a_sT (H/128, ld) f32) in sorted row order."""
    dev = _require_cuda(hidden)
    hidden = hidden.contiguous()
    M, H = hidden.shape
    ld = r.a_s_ld()
    a_q = torch.empty(r.rows_cap, H, dtype=FP8, device=dev)
    a_sT = torch.empty(H // 128, ld, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().b200moe_gather_quant(_ptr(hidden), M, H, topk, _ptr(r.slot_pos), r.rows_cap, _ptr(a_q),
                                               _ptr(a_sT), ld, _stream(dev)), "gather_quant")
    return a_q, a_sT


def gather_rows(xq: torch.Tensor, xs: torch.Tensor, topk: int, r: Routing):
    """Already quantised token rows (xq (M, H) e4m3, xs (M, H/128) f32) ->
    (a_q (rows_cap, H), a_sT (H/128, ld)) in sorted row order."""
    dev = _require_cuda(xq, xs)
    M, H = xq.shape
    xq, xs = xq.contiguous(), xs.contiguous()
    ld = r.a_s_ld()
    a_q = torch.empty(r.rows_cap, H, dtype=FP8, device=dev)
    a_sT = torch.empty(H // 128, ld, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().b200moe_gather_rows(_ptr(xq), _ptr(xs), H, xs.shape[1], M, H, topk, _ptr(r.slot_pos),
                                              r.rows_cap, _ptr(a_q), _ptr(a_sT), ld, _stream(dev)), "gather_rows")
    return a_q, a_sT


def gemm1_silu(a1_q, a1_sT, w13, w13_scale, r: Routing, grid_ctas: int = 0):
    """-> (a2_q (rows_cap, I) e4m3, a2_sT (I/128, ld) f32)."""
    dev = _require_cuda(a1_q, w13)
    E, N2, H = w13.shape
    I = N2 // 2
    ld = r.a_s_ld()
    a2_q = torch.zeros(r.rows_cap, I, dtype=FP8, device=dev)
    a2_sT = torch.zeros(I // 128, ld, dtype=torch.float32, device=dev)
    w13_scale = w13_scale.contiguous()  # held until the call returns (the kernel reads it later)
    _lib.check(_lib.lib().b200moe_gemm1_silu(
        _ptr(a1_q), _ptr(a1_sT), ld, r.rows_cap, _ptr(w13), _ptr(w13_scale), E, H, I,
        _ptr(r.chunk_expert), _ptr(r.chunk_row0), _ptr(r.chunk_rows), _ptr(r.n_chunks), r.chunks_cap,
        r.tile_tokens, _ptr(a2_q), _ptr(a2_sT), _ptr(r.err), grid_ctas, _stream(dev)), "gemm1_silu")
    return a2_q, a2_sT


def gemm2_combine(a2_q, a2_sT, w2, w2_scale, r: Routing, topk_weights: torch.Tensor, grid_ctas: int = 0,
                  out_pair: Optional[torch.Tensor] = None):
    """-> out_pair bf16 rows of H: row p = sorted row p for token-major tiles (rows_cap
    rows), else row f = slot (M*topk rows). Dropped slots untouched; padding rows
    untouched, except inside a chunk of 128-token tiles (written as zeros)."""
    dev = _require_cuda(a2_q, w2)
    E, H, I = w2.shape
    M, topk = topk_weights.shape
    tw = topk_weights.to(torch.float32).contiguous()
    if out_pair is None:
        out_pair = torch.zeros(r.pair_rows(M, topk), H, dtype=torch.bfloat16, device=dev)
    w2_scale = w2_scale.contiguous()
    _lib.check(_lib.lib().b200moe_gemm2_combine(
        _ptr(a2_q), _ptr(a2_sT), r.a_s_ld(), r.rows_cap, _ptr(w2), _ptr(w2_scale), E, H, I,
        _ptr(r.chunk_expert), _ptr(r.chunk_row0), _ptr(r.chunk_rows), _ptr(r.n_chunks), r.chunks_cap,
        r.tile_tokens, _ptr(r.sorted_ids), _ptr(tw), M, topk, _ptr(out_pair), _ptr(r.err), grid_ctas,
        _stream(dev)), "gemm2_combine")
    return out_pair


def experts(a1_q, a1_sT, w13, w13_scale, w2, w2_scale, r: Routing, topk_weights: torch.Tensor,
            grid_ctas: int = 0, out_pair: Optional[torch.Tensor] = None):
    """Both GEMM stages in one launch -> (a2_q, a2_sT, out_pair), the same
    values as gemm1_silu followed by gemm2_combine. Needs the chunk_ready
    counters as zeroed by route() for this routing."""
    dev = _require_cuda(a1_q, w13, w2)
    E, N2, H = w13.shape
    I = N2 // 2
    M, topk = topk_weights.shape
    ld = r.a_s_ld()
    a2_q = torch.zeros(r.rows_cap, I, dtype=FP8, device=dev)
    a2_sT = torch.zeros(I // 128, ld, dtype=torch.float32, device=dev)
    tw = topk_weights.to(torch.float32).contiguous()
    if out_pair is None:
        out_pair = torch.zeros(r.pair_rows(M, topk), H, dtype=torch.bfloat16, device=dev)
    w13_scale, w2_scale = w13_scale.contiguous(), w2_scale.contiguous()
    _lib.check(_lib.lib().b200moe_experts(
        _ptr(a1_q), _ptr(a1_sT), ld, r.rows_cap, _ptr(w13), _ptr(w13_scale), _ptr(w2),
        _ptr(w2_scale), E, H, I, _ptr(r.chunk_expert), _ptr(r.chunk_row0), _ptr(r.chunk_rows),
        _ptr(r.n_chunks), r.chunks_cap, _ptr(r.chunk_ready), r.tile_tokens, _ptr(a2_q), _ptr(a2_sT),
        _ptr(r.sorted_ids), _ptr(tw), M, topk, _ptr(out_pair), _ptr(r.err), grid_ctas, _stream(dev)), "experts")
    return a2_q, a2_sT, out_pair


def experts_fused(hidden, w13, w13_scale, w2, w2_scale, r: Routing, topk_weights: torch.Tensor,
                  grid_ctas: int = 0) -> torch.Tensor:
    """Gather + quantise, both GEMM stages and the top-k reduce in one launch
    (tiles of 16..64 tokens) -> out (M, H) bf16, the same values as
    gather_quant, experts and combine_reduce. Needs the counters zeroed by
    route() for this routing."""
    dev = _require_cuda(hidden, w13, w2)
    hidden = hidden.contiguous()
    E, N2, H = w13.shape
    I = N2 // 2
    M, topk = topk_weights.shape
    ld = r.a_s_ld()
    a1_q = torch.empty(r.rows_cap, H, dtype=FP8, device=dev)
    a1_sT = torch.empty(H // 128, ld, dtype=torch.float32, device=dev)
    a2_q = torch.zeros(r.rows_cap, I, dtype=FP8, device=dev)
    a2_sT = torch.zeros(I // 128, ld, dtype=torch.float32, device=dev)
    out_pair = torch.zeros(M * topk, H, dtype=torch.bfloat16, device=dev)
    out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    tw = topk_weights.to(torch.float32).contiguous()
    w13_scale, w2_scale = w13_scale.contiguous(), w2_scale.contiguous()
    _lib.check(_lib.lib().b200moe_experts_fused(
        _ptr(hidden), M, topk, _ptr(r.slot_pos), _ptr(a1_q), _ptr(a1_sT), ld, r.rows_cap, _ptr(w13),
        _ptr(w13_scale), _ptr(w2), _ptr(w2_scale), E, H, I, _ptr(r.chunk_expert),
        _ptr(r.chunk_row0), _ptr(r.chunk_rows), _ptr(r.n_chunks), r.chunks_cap, _ptr(r.chunk_ready), r.tile_tokens,
        _ptr(a2_q), _ptr(a2_sT), _ptr(r.sorted_ids), _ptr(tw), _ptr(out_pair), _ptr(out), _ptr(r.err), grid_ctas,
        _stream(dev)), "experts_fused")
    return out


def combine_reduce(out_pair: torch.Tensor, r: Routing, M: int, topk: int) -> torch.Tensor:
    """out[t] = bf16(sum over the routed slots j of the slot's stage-2 row)."""
    dev = _require_cuda(out_pair)
    H = out_pair.shape[1]
    out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.lib().b200moe_combine_reduce(_ptr(out_pair), _ptr(r.slot_pos), r.sorted_rows, M, topk, H,
                                                 _ptr(out), _stream(dev)), "combine_reduce")
    return out


def selftest_wait_timeout(err: torch.Tensor, timeout_us: int = 20000) -> None:
    dev = _require_cuda(err)
    _lib.check(_lib.lib().b200moe_selftest_wait_timeout(_ptr(err), timeout_us, _stream(dev)), "selftest")


# From this many routed pairs on, the gather quantises each token once and
# stores it to all its slot rows (the same rule as the C layer, capi.cu); below
# it the one-launch layer is eligible.
FAN_OUT_MIN_PAIRS = 2048


def pick_tile_tokens(numel: int, num_local_experts: int) -> int:
    """Token columns per GEMM unit; the same rule as the C layer (capi.cu)."""
    avg = numel / max(num_local_experts, 1)
    if avg <= 26.0:
        return 32
    if avg <= 48.0:
        return 64
    return 128


class LayerPipeline:
    """The launches of the layer on preallocated buffers, with optional CUDA
    events between stages (used by the benchmark to time each kernel on the
    launching stream). Same kernels and order as b200moe_layer: where
    b200moe_layer runs the whole layer as one launch (small batches, see
    b200moe_set_layer_launch) the pipeline calls it (one stage, "layer");
    otherwise route, gather_quant, experts (both GEMM stages in one launch),
    combine_reduce; with split=True the GEMM stages run as two launches."""

    WHOLE_STAGES = ("layer",)  # routing, gather, both GEMM stages and the reduce in one launch
    LAYER_STAGES = ("route", "layer")  # everything after routing in one launch (b200moe_experts_fused)
    FUSED_STAGES = ("route", "gather_quant", "experts", "combine_reduce")
    SPLIT_STAGES = ("route", "gather_quant", "gemm1_silu", "gemm2_combine", "combine_reduce")

    def __init__(self, M: int, H: int, I: int, num_experts: int, topk: int, device, tile_tokens: int = 0,
                 expert_map: Optional[torch.Tensor] = None, num_local_experts: Optional[int] = None,
                 split: bool = False, one_launch: Optional[bool] = None, router: Optional[dict] = None,
                 whole: Optional[bool] = None):
        """router: {"scoring_func", "correction_bias", "renormalize",
        "routed_scaling_factor"} to run the layer from router logits
        (run_from_logits: the router inside routing's first launch).
        whole: None = the whole-layer launch where b200moe_layer uses it,
        False = separate launches."""
        self.M, self.H, self.I, self.topk = M, H, I, topk
        self.num_experts = num_experts
        self.E = num_local_experts if expert_map is not None else num_experts
        self.expert_map = None if expert_map is None else expert_map.to(device=device, dtype=torch.int32).contiguous()
        self.device = torch.device(device)
        L = _lib.lib()
        numel = M * topk
        self.tile = tile_tokens or pick_tile_tokens(numel, self.E)
        self.rows_cap = L.b200moe_route_capacity_rows(numel, self.E)
        self.chunks_cap = L.b200moe_route_capacity_chunks(numel, self.E, self.tile)
        self.ld = (self.rows_cap + 256 + 63) // 64 * 64
        z = lambda n: torch.zeros(max(n, 1), dtype=torch.int32, device=device)  # noqa: E731
        self.sorted_ids, self.ce, self.cr0, self.crows = z(self.rows_cap), z(self.chunks_cap), z(self.chunks_cap), \
            z(self.chunks_cap)
        self.ready = z(self.chunks_cap + 2)
        self.slot_pos = z(numel)
        self.rscratch_ints = L.b200moe_route_scratch_ints(numel, self.E)
        self.rscratch = z(self.rscratch_ints)
        self.split = split
        # One launch after routing (b200moe_experts_fused) on request: measured
        # equal at 64 tokens and 24 us slower at 128 than the three launches.
        eligible = (not split) and self.tile <= 64 and M * topk < FAN_OUT_MIN_PAIRS
        self.one_launch = bool(one_launch) and eligible
        self.whole = (not split and not self.one_launch and whole is not False and
                      L.b200moe_layer_launches(M, H, I, num_experts, self.E, topk) == 1)
        self.stages = self.SPLIT_STAGES if split else (
            self.WHOLE_STAGES if self.whole else (self.LAYER_STAGES if self.one_launch else self.FUSED_STAGES))
        self.counts = z(2)
        self.err = z(1)
        self.a1 = torch.zeros(self.rows_cap, H, dtype=FP8, device=device)
        self.a1s = torch.zeros(H // 128, self.ld, dtype=torch.float32, device=device)
        self.a2 = torch.zeros(self.rows_cap, I, dtype=FP8, device=device)
        self.a2s = torch.zeros(I // 128, self.ld, dtype=torch.float32, device=device)
        self.sorted_rows = 1 if self.tile > 64 else 0
        self.pair = torch.zeros(max(self.rows_cap if self.sorted_rows else numel, 1), H, dtype=torch.bfloat16,
                                device=device)
        # Mixed work lists (the C layer's rule): a skewed decode batch's heavy
        # experts go through the token-major stages in the same step.
        self.heavy_rows = 0 if (split or self.one_launch or self.whole) else L.b200moe_heavy_rows(M, topk, self.tile)
        if self.heavy_rows:
            self.chunks_cap2 = L.b200moe_route_capacity_chunks(numel, self.E, 128)
            self.ce2, self.cr02, self.crows2 = z(self.chunks_cap2), z(self.chunks_cap2), z(self.chunks_cap2)
            self.counters2 = z(2)
            self.counts = z(4)
        self.out = torch.zeros(M, H, dtype=torch.bfloat16, device=device)
        if self.whole:
            # b200moe_layer's workspace: header zeroed (error word, counters
            # every call leaves at zero); the error word is self.err
            self.ws = torch.zeros(L.b200moe_layer_workspace_size(M, H, I, num_experts, self.E, topk),
                                  dtype=torch.uint8, device=device)
            self.err = self.ws[:4].view(torch.int32)
        self.router = None
        if router is not None:
            r = dict(router)
            bias = r.get("correction_bias")
            self.router = (({"softmax": 0, "sigmoid": 1}[r.get("scoring_func", "sigmoid")]),
                           None if bias is None else bias.to(device=device, dtype=torch.float32).contiguous(),
                           int(r.get("renormalize", True)), float(r.get("routed_scaling_factor", 1.0)))
            self.topk_weights = torch.zeros(M, topk, dtype=torch.float32, device=device)
            self.topk_ids = torch.zeros(M, topk, dtype=torch.int32, device=device)
            self.lscratch_ints = L.b200moe_route_logits_scratch_ints(numel, self.E)
            self.lscratch = z(self.lscratch_ints)  # zeroed: its first int is the router's CTA counter

    @property
    def launches(self) -> int:
        """Kernel launches per run() (run_from_logits: the same)."""
        if self.whole:
            return 1
        return (len(self.stages) + (1 if not self.split and self.tile > 64 else 0) +
                (1 if self.rscratch_ints > 0 and not self.heavy_rows else 0) + (2 if self.heavy_rows else 0))

    def run_from_logits(self, hidden, logits, w13, w13_scale, w2, w2_scale, events=None, grid_ctas: int = 0):
        """The layer from router logits: b200moe_route_logits (router + routing),
        then the same launches as run(). The selected ids and weights are left
        in self.topk_ids / self.topk_weights."""
        if self.router is None:
            raise ValueError("LayerPipeline was built without a router")
        L = _lib.lib()
        st = _stream(self.device)
        ev = events or [None] * (len(self.stages) + 1)
        rec = lambda i: ev[i].record() if ev[i] is not None else None  # noqa: E731
        scoring, bias, renorm, scale = self.router
        cnt = _ptr(self.counts)
        rec(0)
        if self.whole:
            _lib.check(L.b200moe_layer_logits(_ptr(hidden), self.M, self.H, self.I, self.num_experts, self.topk,
                                              _ptr(logits), int(logits.dtype == torch.bfloat16), scoring, _ptr(bias),
                                              renorm, scale, _ptr(w13), _ptr(w13_scale), _ptr(w2), _ptr(w2_scale),
                                              _ptr(self.expert_map), self.E, _ptr(self.topk_weights),
                                              _ptr(self.topk_ids), _ptr(self.out), _ptr(self.ws), self.ws.numel(),
                                              st), "layer_logits")
            rec(1)
            return self.out
        _lib.check(L.b200moe_route_logits(_ptr(logits), int(logits.dtype == torch.bfloat16), self.M, self.num_experts,
                                          self.topk, scoring, _ptr(bias), renorm, scale, _ptr(self.topk_weights),
                                          _ptr(self.topk_ids), _ptr(self.expert_map), self.E, self.tile,
                                          _ptr(self.sorted_ids), self.rows_cap, _ptr(self.ce), _ptr(self.cr0),
                                          _ptr(self.crows), self.chunks_cap, cnt, cnt + 4, _ptr(self.slot_pos),
                                          _ptr(self.ready), _ptr(self.lscratch), self.lscratch_ints, _ptr(self.err),
                                          st), "route_logits")
        rec(1)
        return self._after_route(hidden, self.topk_weights, w13, w13_scale, w2, w2_scale, rec, grid_ctas)

    def run(self, hidden, topk_ids, topk_weights, w13, w13_scale, w2, w2_scale, events=None, grid_ctas: int = 0):
        L = _lib.lib()
        st = _stream(self.device)
        ev = events or [None] * (len(self.stages) + 1)
        rec = lambda i: ev[i].record() if ev[i] is not None else None  # noqa: E731
        M, topk, E = self.M, self.topk, self.E
        cnt = _ptr(self.counts)
        rows = cnt + 4
        rec(0)
        if self.whole:
            _lib.check(L.b200moe_layer(_ptr(hidden), M, self.H, self.I, self.num_experts, topk, _ptr(w13),
                                       _ptr(w13_scale), _ptr(w2), _ptr(w2_scale), _ptr(topk_weights), _ptr(topk_ids),
                                       _ptr(self.expert_map), E, _ptr(self.out), _ptr(self.ws), self.ws.numel(), st),
                       "layer")
            rec(1)
            return self.out
        if self.heavy_rows:
            _lib.check(L.b200moe_route_mixed(_ptr(topk_ids), M, topk, self.num_experts, _ptr(self.expert_map), E,
                                             self.tile, self.heavy_rows, _ptr(self.sorted_ids), self.rows_cap,
                                             _ptr(self.ce), _ptr(self.cr0), _ptr(self.crows), self.chunks_cap,
                                             _ptr(self.ce2), _ptr(self.cr02), _ptr(self.crows2), self.chunks_cap2,
                                             cnt, _ptr(self.slot_pos), _ptr(self.ready), _ptr(self.counters2),
                                             _ptr(self.err), st), "route_mixed")
        else:
            _lib.check(L.b200moe_route(_ptr(topk_ids), M, topk, self.num_experts, _ptr(self.expert_map), E, self.tile,
                                       _ptr(self.sorted_ids), self.rows_cap, _ptr(self.ce), _ptr(self.cr0),
                                       _ptr(self.crows), self.chunks_cap, cnt, rows, _ptr(self.slot_pos),
                                       _ptr(self.ready), _ptr(self.rscratch), self.rscratch_ints, _ptr(self.err), st),
                       "route")
        rec(1)
        return self._after_route(hidden, topk_weights, w13, w13_scale, w2, w2_scale, rec, grid_ctas)

    def _after_route(self, hidden, topk_weights, w13, w13_scale, w2, w2_scale, rec, grid_ctas):
        L = _lib.lib()
        st = _stream(self.device)
        M, H, I, topk, E = self.M, self.H, self.I, self.topk, self.E
        cnt = _ptr(self.counts)
        if self.one_launch:
            _lib.check(L.b200moe_experts_fused(_ptr(hidden), M, topk, _ptr(self.slot_pos), _ptr(self.a1), _ptr(self.a1s),
                                               self.ld, self.rows_cap, _ptr(w13), _ptr(w13_scale), _ptr(w2),
                                               _ptr(w2_scale), E, H, I, _ptr(self.ce), _ptr(self.cr0), _ptr(self.crows),
                                               cnt, self.chunks_cap, _ptr(self.ready), self.tile, _ptr(self.a2),
                                               _ptr(self.a2s), _ptr(self.sorted_ids), _ptr(topk_weights),
                                               _ptr(self.pair), _ptr(self.out), _ptr(self.err), grid_ctas, st),
                       "experts_fused")
            rec(2)
            return self.out
        _lib.check(L.b200moe_gather_quant(_ptr(hidden), M, H, topk, _ptr(self.slot_pos), self.rows_cap,
                                          _ptr(self.a1), _ptr(self.a1s), self.ld, st), "gather_quant")
        rec(2)
        if not self.split:
            _lib.check(L.b200moe_experts(_ptr(self.a1), _ptr(self.a1s), self.ld, self.rows_cap, _ptr(w13),
                                         _ptr(w13_scale), _ptr(w2), _ptr(w2_scale), E, H, I, _ptr(self.ce),
                                         _ptr(self.cr0), _ptr(self.crows), cnt, self.chunks_cap, _ptr(self.ready),
                                         self.tile, _ptr(self.a2), _ptr(self.a2s), _ptr(self.sorted_ids),
                                         _ptr(topk_weights), M, topk, _ptr(self.pair), _ptr(self.err), grid_ctas,
                                         st), "experts")
            if self.heavy_rows:
                _lib.check(L.b200moe_experts_heavy(_ptr(self.a1), _ptr(self.a1s), self.ld, self.rows_cap, _ptr(w13),
                                                   _ptr(w13_scale), _ptr(w2), _ptr(w2_scale), E, H, I,
                                                   _ptr(self.ce2), _ptr(self.cr02), _ptr(self.crows2), cnt + 8,
                                                   self.chunks_cap2, _ptr(self.counters2), _ptr(self.a2),
                                                   _ptr(self.a2s), _ptr(self.sorted_ids), _ptr(topk_weights), M, topk,
                                                   _ptr(self.pair), _ptr(self.err), grid_ctas, st), "experts_heavy")
            rec(3)
            _lib.check(L.b200moe_combine_reduce(_ptr(self.pair), _ptr(self.slot_pos), self.sorted_rows, M, topk, H,
                                                _ptr(self.out), st),
                       "combine_reduce")
            rec(4)
            return self.out
        _lib.check(L.b200moe_gemm1_silu(_ptr(self.a1), _ptr(self.a1s), self.ld, self.rows_cap, _ptr(w13),
                                        _ptr(w13_scale), E, H, I, _ptr(self.ce), _ptr(self.cr0), _ptr(self.crows),
                                        cnt, self.chunks_cap, self.tile, _ptr(self.a2), _ptr(self.a2s),
                                        _ptr(self.err), grid_ctas, st), "gemm1_silu")
        rec(3)
        _lib.check(L.b200moe_gemm2_combine(_ptr(self.a2), _ptr(self.a2s), self.ld, self.rows_cap, _ptr(w2),
                                           _ptr(w2_scale), E, H, I, _ptr(self.ce), _ptr(self.cr0), _ptr(self.crows),
                                           cnt, self.chunks_cap, self.tile, _ptr(self.sorted_ids),
                                           _ptr(topk_weights), M, topk, _ptr(self.pair), _ptr(self.err), grid_ctas,
                                           st), "gemm2_combine")
        rec(4)
        _lib.check(L.b200moe_combine_reduce(_ptr(self.pair), _ptr(self.slot_pos), self.sorted_rows, M, topk, H,
                                                _ptr(self.out), st),
                   "combine_reduce")
        rec(5)
        return self.out
