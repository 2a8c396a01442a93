"""Expert-parallel MoE layer: one rank per GPU, experts sharded over ranks,
tokens exchanged either by the kernels themselves through NVLink peer memory
(exchange="peer", the default on GPUs) or with two equal-split all-to-alls
(exchange="nccl").

Rank r of G owns experts [r*E/G, (r+1)*E/G). Per forward call:
  1. quantise this rank's tokens 1x128 (fp8 + scales);
  2. pack one row per (token, owning rank) - fp8 row, scales, the token's top-k
     ids mapped to the destination's local experts (-1 elsewhere), weights -
     into G fixed-size blocks of `rows_per_rank` rows (b200moe_ep_dispatch);
  3. all-to-all the blocks;
  4. run the layer on every received row with this rank's experts
     (b200moe_layer_packed): one bf16 row per received row = the sum of that
     token's weighted outputs over this rank's experts;
  5. all-to-all those rows back;
  6. sum each token's returned rows in rank order (b200moe_ep_combine).
Blocks have a fixed size so the exchange needs no count all-to-all and no
host synchronisation; rows_per_rank is the largest token count any rank passes.

With exchange="peer" steps 2-3 are one kernel (the pack stores each block
straight into the destination's receive area, mapped through CUDA IPC, and
raises a flag there), the layer waits for the G flags, and steps 4-5 are one
kernel (the top-k reduce stores each result row straight into the source
rank's return area and raises a flag); step 6 waits for those flags. No NCCL
call on the data path (b200moe_ep_dispatch_peer, b200moe_layer_packed_peer,
b200moe_ep_combine_peer).

This is the dispatch/combine the reference consumes from DeepEP/Mori
(sglang_integration/aiter.py:554-756), with the reference's conventions:
per-group fp8 dispatch with fp32 scales (:614-617) and local ids, -1 for
experts elsewhere (:660-668).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .moe import FP8, _ptr, _stream


@dataclass
class Placement:
    """Where the experts' weights live: G ranks of `slots` physical experts;
    physical slot p = rank * slots + local index holds logical expert
    phys_to_logical[p]. A logical expert may have several replicas (EPLB,
    hot-expert replication); every logical expert has at least one."""
    num_experts: int
    G: int
    slots: int
    phys_to_logical: np.ndarray

    def __post_init__(self):
        p2l = np.asarray(self.phys_to_logical, dtype=np.int64)
        if p2l.shape != (self.G * self.slots,):
            raise ValueError("phys_to_logical must hold G * slots entries")
        if p2l.min() < 0 or p2l.max() >= self.num_experts:
            raise ValueError("phys_to_logical names an expert outside [0, num_experts)")
        if len(np.unique(p2l)) != self.num_experts:
            raise ValueError("every logical expert needs at least one physical slot")
        self.phys_to_logical = p2l

    @staticmethod
    def identity(num_experts: int, G: int) -> "Placement":
        if num_experts % G:
            raise ValueError("num_experts must be a multiple of the world size")
        return Placement(num_experts, G, num_experts // G, np.arange(num_experts))

    def replicas(self, e: int) -> np.ndarray:
        return np.nonzero(self.phys_to_logical == e)[0]

    @property
    def max_replicas(self) -> int:
        return int(np.bincount(self.phys_to_logical, minlength=self.num_experts).max())

    def table(self) -> np.ndarray:
        """(E, 1 + max_replicas) int32 rows [n, p_0, .., p_{n-1}, -1..] of the
        C ABI (b200moe_ep_dispatch's `replicas`)."""
        m = self.max_replicas
        t = np.full((self.num_experts, 1 + m), -1, dtype=np.int32)
        for e in range(self.num_experts):
            r = self.replicas(e)
            t[e, 0] = len(r)
            t[e, 1:1 + len(r)] = r
        return t

    def local_experts(self, rank: int) -> np.ndarray:
        """Logical expert of each of rank's slots, in slot order."""
        return self.phys_to_logical[rank * self.slots:(rank + 1) * self.slots]

    def is_identity(self) -> bool:
        return self.slots * self.G == self.num_experts and \
            bool((self.phys_to_logical == np.arange(self.num_experts)).all())


def eplb_placement(expert_load, G: int, slots_per_rank: int) -> Placement:
    """Hot-expert replication and balanced packing (the EPLB the reference
    plans to enable, moe_placement_glm52_mi355x.md:98-104; the algorithm is
    DeepSeek's published EPLB: replicate, then pack).

    expert_load (E,): tokens (or any load measure) per logical expert, e.g.
    counted from recent batches. The G * slots_per_rank - E spare slots go,
    one at a time, to the expert with the largest load per replica (at most G
    replicas each). The replicas, heaviest first (load / replicas), are then
    packed onto the rank with the least load that has a free slot and does not
    hold that expert yet. Within a rank, slots are in ascending expert order."""
    load = np.asarray(expert_load, dtype=np.float64)
    E = len(load)
    total = G * slots_per_rank
    if total < E:
        raise ValueError("G * slots_per_rank must be at least the number of experts")
    nrep = np.ones(E, dtype=np.int64)
    for _ in range(total - E):
        ratio = np.where(nrep < G, load / nrep, -np.inf)
        if not np.isfinite(ratio).any():
            ratio = load / nrep
        nrep[int(np.argmax(ratio))] += 1
    items = sorted(((load[e] / nrep[e], e) for e in range(E) for _ in range(nrep[e])), key=lambda x: (-x[0], x[1]))
    rank_load = np.zeros(G)
    held = [[] for _ in range(G)]
    for w, e in items:
        free = [r for r in range(G) if len(held[r]) < slots_per_rank]
        fresh = [r for r in free if e not in held[r]]
        cand = fresh or free
        r = min(cand, key=lambda r: (rank_load[r], r))
        held[r].append(e)
        rank_load[r] += w
    p2l = np.concatenate([np.sort(np.asarray(h, dtype=np.int64)) for h in held])
    return Placement(E, G, slots_per_rank, p2l)


def place_experts(w: torch.Tensor, placement: Placement, rank: int) -> torch.Tensor:
    """The (slots, ...) weights of rank `rank` from the (E, ...) weights of every expert."""
    idx = torch.as_tensor(placement.local_experts(rank), device=w.device)
    return w.index_select(0, idx).contiguous()


class CudaEPOps:
    """The rank-local steps on the GPU through the C ABI."""

    def row_bytes(self, H: int, topk: int) -> int:
        return _lib.lib().b200moe_ep_row_bytes(H, topk)

    def quant(self, hidden: torch.Tensor, q: torch.Tensor, s: torch.Tensor):
        M, H = hidden.shape
        _lib.check(_lib.lib().b200moe_quant_1x128(_ptr(hidden), M, H, H, _ptr(q), H, _ptr(s), H // 128, 1,
                                                  _stream(hidden.device)), "ep quant")

    def dispatch(self, q, s, topk_ids, topk_weights, num_experts, G, rows_per_rank, send, pos, tok_of, counts, err,
                 rank=0, placement=None):
        """placement: None (experts split evenly) or (table (E, 1+max_rep) int32
        device tensor, Placement)."""
        M, H = q.shape
        topk = topk_ids.shape[1]
        table, pl = placement if placement is not None else (None, None)
        _lib.check(_lib.lib().b200moe_ep_dispatch(
            _ptr(q), _ptr(s), _ptr(topk_ids), _ptr(topk_weights), M, H, topk, num_experts, G, rank, _ptr(table),
            pl.max_replicas if pl else 0, pl.slots if pl else 0, rows_per_rank,
            _ptr(send), _ptr(pos), _ptr(tok_of), _ptr(counts), _ptr(err), _stream(q.device)), "ep_dispatch")

    def workspace_bytes(self, R, H, I, E_local, topk) -> int:
        return _lib.lib().b200moe_layer_packed_workspace_size(R, H, I, E_local, topk)

    def layer_packed(self, rows, R, H, I, E_local, topk, w13, w13_scale, w2, w2_scale, out, ws, num_ranks=1):
        _lib.check(_lib.lib().b200moe_layer_packed(
            _ptr(rows), R, num_ranks, self.row_bytes(H, topk), H, I, E_local, topk, _ptr(w13), _ptr(w13_scale),
            _ptr(w2),
            _ptr(w2_scale), _ptr(out), _ptr(ws), ws.numel(), _stream(rows.device)), "layer_packed")

    def combine(self, returned, pos, M, H, G, rows_per_rank, out):
        _lib.check(_lib.lib().b200moe_ep_combine(_ptr(returned), _ptr(pos), M, H, G, rows_per_rank, _ptr(out),
                                                 _stream(out.device)), "ep_combine")


class PeerExchange:
    """This rank's exchange buffer and the device table of all G buffers as
    mapped in this process (b200moe_ep_peer_*). Collective: every rank of the
    group constructs it with the same arguments."""

    def __init__(self, rows_per_rank: int, H: int, topk: int, G: int, rank: int, group, device):
        lib = _lib.lib()
        nbytes = lib.b200moe_ep_peer_bytes(rows_per_rank, H, topk, G)
        if nbytes == 0:
            raise ValueError("unsupported exchange shape")
        base = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES)()
        _lib.check(lib.b200moe_ep_peer_alloc(nbytes, ctypes.byref(base), handle), "ep_peer_alloc")
        self.own = base.value
        self.opened = []
        handles = [bytes(handle)] * G
        if G > 1:
            dist.all_gather_object(handles, bytes(handle), group=group)
        ptrs = []
        for g in range(G):
            if g == rank:
                ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            h = (ctypes.c_uint8 * _lib.IPC_HANDLE_BYTES).from_buffer_copy(handles[g])
            _lib.check(lib.b200moe_ep_peer_open(h, ctypes.byref(p)), "ep_peer_open")
            self.opened.append(p.value)
            ptrs.append(p.value)
        self.bases = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.group = group
        self.G = G
        if G > 1:
            dist.barrier(group=group)  # every buffer mapped everywhere before any rank stores

    def close(self):
        """Collective: unmap the peers' buffers and free this rank's."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        if self.G > 1:
            dist.barrier(group=self.group)  # no rank still stores into a buffer being freed
        lib = _lib.lib()
        for p in self.opened:
            _lib.check(lib.b200moe_ep_peer_close(p), "ep_peer_close")
        _lib.check(lib.b200moe_ep_peer_free(self.own), "ep_peer_free")
        self.own, self.opened = None, []


class ExpertParallelMoE:
    """One rank's share of an expert-parallel MoE layer.

    w13 (E/G, 2I, H), w2 (E/G, H, I) fp8 with their 128x128 scales are the
    experts this rank owns. forward() takes this rank's tokens with GLOBAL
    top-k ids and returns their (M, H) bf16 outputs. Every rank must call
    forward() the same number of times (collectives).

    exchange: "peer" (kernels store into the other GPUs' memory; needs the
    CUDA ops) or "nccl" (all-to-alls; also runs with the oracle ops on gloo);
    None picks "peer" for the CUDA ops and "nccl" otherwise."""

    def __init__(self, w13, w13_scale, w2, w2_scale, num_experts: int, rows_per_rank: int,
                 group: Optional[dist.ProcessGroup] = None, ops=None, device=None, exchange: Optional[str] = None,
                 placement: Optional[Placement] = None):
        """placement: where the experts live (eplb_placement for hot-expert
        replication); None splits them evenly (num_experts / world_size per
        rank). w13 ... w2_scale are this rank's slots (place_experts)."""
        self.group = group
        self.G = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.E = num_experts
        self.E_local, self.I2, self.H = w13.shape
        if placement is not None and placement.is_identity():
            placement = None
        if placement is None:
            if num_experts % self.G:
                raise ValueError("num_experts must be a multiple of the world size")
            if self.E_local != num_experts // self.G:
                raise ValueError("w13 must hold num_experts / world_size experts")
        else:
            if placement.G != self.G or placement.num_experts != num_experts:
                raise ValueError("placement is for another world size or expert count")
            if self.E_local != placement.slots:
                raise ValueError("w13 must hold the placement's slots per rank")
        self.placement = placement
        self.I = self.I2 // 2
        self.w13, self.w13_scale, self.w2, self.w2_scale = w13, w13_scale.contiguous(), w2, w2_scale.contiguous()
        self.cap = int(rows_per_rank)
        self.ops = ops or CudaEPOps()
        self.device = torch.device(device) if device is not None else w13.device
        if exchange is None:
            exchange = "peer" if isinstance(self.ops, CudaEPOps) else "nccl"
        if exchange not in ("peer", "nccl"):
            raise ValueError(f"unknown exchange {exchange!r}")
        if exchange == "peer" and not isinstance(self.ops, CudaEPOps):
            raise ValueError("the peer exchange runs on the CUDA ops only")
        self.exchange = exchange
        self.peer = None
        self.epoch = 0
        self._topk = None
        self._place = None
        if placement is not None:
            self._place = (torch.as_tensor(placement.table(), device=self.device), placement)

    def _buffers(self, topk: int):
        if self._topk == topk:
            return
        G, cap, H, dev = self.G, self.cap, self.H, self.device
        rb = self.ops.row_bytes(H, topk)
        R = G * cap
        self.row_bytes = rb
        self.q = torch.empty(cap, H, dtype=FP8, device=dev)
        self.s = torch.empty(cap, H // 128, dtype=torch.float32, device=dev)
        if self.exchange == "peer":
            if self.peer is not None:
                self.peer.close()
            self.peer = PeerExchange(cap, H, topk, G, self.rank, self.group, dev)
            self.epoch = 0
        else:
            self.send = torch.empty(R * rb, dtype=torch.uint8, device=dev)
            self.recv = torch.empty(R * rb, dtype=torch.uint8, device=dev)
        self.pos = torch.empty(cap * G, dtype=torch.int32, device=dev)
        self.tok_of = torch.empty(R, dtype=torch.int32, device=dev)
        self.counts = torch.empty(G, dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        if self.exchange == "nccl":
            self.local_out = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
            self.returned = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
        self.ws = torch.empty(max(self.ops.workspace_bytes(R, H, self.I, self.E_local, topk), 256),
                              dtype=torch.uint8, device=dev)
        self.ws[:256].zero_()
        self._topk = topk

    def _all_to_all(self, out: torch.Tensor, inp: torch.Tensor):
        if self.G == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, group=self.group)

    STAGES = ("quant_dispatch", "all_to_all_dispatch", "layer_packed", "all_to_all_combine", "combine")

    def forward(self, hidden: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                out: Optional[torch.Tensor] = None, events=None) -> torch.Tensor:
        """events: optional list of 6 CUDA events recorded at the STAGES boundaries."""
        M, H = hidden.shape
        topk = topk_ids.shape[1]
        if M > self.cap:
            raise ValueError(f"{M} tokens exceed rows_per_rank={self.cap}")
        self._buffers(topk)
        ids = topk_ids.to(torch.int32).contiguous()
        tw = topk_weights.to(torch.float32).contiguous()
        if out is None:
            out = torch.empty(M, H, dtype=torch.bfloat16, device=self.device)
        rec = (lambda i: events[i].record()) if events is not None else (lambda i: None)
        q, s = self.q[:M], self.s[:M]
        if self.exchange == "peer":
            return self._forward_peer(hidden, ids, tw, q, s, out, rec)
        rec(0)
        self.ops.quant(hidden.contiguous(), q, s)
        self.ops.dispatch(q, s, ids, tw, self.E, self.G, self.cap, self.send, self.pos[: M * self.G],
                          self.tok_of, self.counts, self.err, rank=self.rank, placement=self._place)
        rec(1)
        self._all_to_all(self.recv, self.send)
        rec(2)
        R = self.G * self.cap
        self.ops.layer_packed(self.recv, R, H, self.I, self.E_local, topk, self.w13, self.w13_scale, self.w2,
                              self.w2_scale, self.local_out, self.ws, num_ranks=self.G)
        rec(3)
        self._all_to_all(self.returned.view(-1), self.local_out.view(-1))
        rec(4)
        self.ops.combine(self.returned, self.pos[: M * self.G], M, H, self.G, self.cap, out)
        rec(5)
        return out

    __call__ = forward

    def _forward_peer(self, hidden, ids, tw, q, s, out, rec):
        """forward() with the exchange inside the kernels: the two all-to-all
        stages record no time of their own."""
        lib, M, H, G, cap = _lib.lib(), hidden.shape[0], self.H, self.G, self.cap
        topk = ids.shape[1]
        self.epoch += 1
        st = _stream(self.device)
        bases, own = _ptr(self.peer.bases), self.peer.own
        rec(0)
        # the pack kernel quantises each token row on its way to the destinations
        table, pl = self._place if self._place is not None else (None, None)
        hidden = hidden.contiguous()  # held through the call
        _lib.check(lib.b200moe_ep_dispatch_peer(
            _ptr(hidden), None, None, _ptr(ids), _ptr(tw), M, H, topk, self.E, G, self.rank, _ptr(table),
            pl.max_replicas if pl else 0, pl.slots if pl else 0, cap, bases, own, self.epoch,
            _ptr(self.pos[: M * G]), _ptr(self.tok_of), _ptr(self.counts), _ptr(self.err), st), "ep_dispatch_peer")
        rec(1)
        rec(2)
        _lib.check(lib.b200moe_layer_packed_peer(
            own, bases, G, self.rank, cap, self.epoch, H, self.I, self.E_local, topk, _ptr(self.w13),
            _ptr(self.w13_scale), _ptr(self.w2), _ptr(self.w2_scale), _ptr(self.ws), self.ws.numel(), st),
            "layer_packed_peer")
        rec(3)
        rec(4)
        _lib.check(lib.b200moe_ep_combine_peer(own, _ptr(self.pos[: M * G]), M, H, topk, G, cap, self.epoch,
                                               _ptr(out), _ptr(self.err), st), "ep_combine_peer")
        rec(5)
        return out

    def close(self):
        """Collective with the peer exchange: release the exchange buffers."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def device_errors(self) -> int:
        """OR of the dispatch and layer device error words (synchronises)."""
        from .moe import read_device_error

        return read_device_error(self.err) | read_device_error(self.ws[:4].view(torch.int32))


def shard_experts(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The slice of an (E, ...) expert tensor that rank `rank` owns."""
    E = w.shape[0]
    per = E // world
    return w[rank * per:(rank + 1) * per].contiguous()
