"""Drop-in host API of the FP8 block-scaled MoE layer.

Mirrors the reference's operator surface for this path:
  * moe_decode_megakernel_full / _moe_decode_megakernel_full
      <- sglang_integration/aiter.py:74-177
  * fused_moe (per_128x128 / Silu / interleaved gate-up subset)
      <- the aiter fused_moe call at sglang_integration/aiter.py:459-478
  * moe_align_block_size        <- sglang op called at aiter.py:113-115
  * per_token_group_quant_fp8   <- sglang op called at aiter.py:132-133, 151-152
  * per_block_quant_fp8         <- phase5_orchestrator.py:35-41
Every op runs the CUDA kernels of libb200moe.so through its C ABI on the
current torch stream. Unsupported options raise NotImplementedError; there is
no fallback path.
"""
from __future__ import annotations

import ctypes
import threading
from enum import Enum
from typing import Optional

import torch

from . import _lib

FP8 = torch.float8_e4m3fn


# ----------------------------------------------------------------------------
# helpers
# ----------------------------------------------------------------------------
def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError("b200moe ops take CUDA tensors; there is no CPU implementation")
        if t.device != dev:
            raise ValueError("all tensors must be on the same device")
    return dev


class _Workspaces:
    """Grow-only per-(device, stream) workspace buffers. Their first 256 bytes
    are zeroed at allocation: the device error word (int 0), then the router's
    CTA counter and the whole-layer launch's sync words (ints 1..3, left at
    zero by every call)."""

    def __init__(self):
        self._bufs = {}
        self._lock = threading.Lock()

    def get(self, device: torch.device, nbytes: int) -> torch.Tensor:
        key = (device.index, _stream(device))
        with self._lock:
            buf = self._bufs.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
                buf[:256].zero_()
                self._bufs[key] = buf
            return buf


_workspaces = _Workspaces()


def read_device_error(err_word: torch.Tensor, clear: bool = True) -> int:
    """Returns the device error word (B200MOE_DEVERR_* bits) after the stream ran."""
    val = ctypes.c_int32()
    _lib.check(_lib.lib().b200moe_read_error(err_word.data_ptr(), ctypes.byref(val), int(clear),
                                             _stream(err_word.device)), "read_error")
    return int(val.value)


def layer_error_word(device: Optional[torch.device] = None) -> torch.Tensor:
    """The error word of the cached layer workspace for (device, current stream)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    return _workspaces.get(device, 256)[:4].view(torch.int32)


# ----------------------------------------------------------------------------
# routing and quantisation ops
# ----------------------------------------------------------------------------
def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int,
                         expert_map: Optional[torch.Tensor] = None, num_local_experts: Optional[int] = None,
                         err_word: Optional[torch.Tensor] = None):
    """Returns (sorted_token_ids, expert_ids, num_tokens_post_padded) with the
    reference's layout; see include/b200moe.h b200moe_align."""
    dev = _require_cuda(topk_ids)
    ids = topk_ids.to(torch.int32).contiguous()
    M, topk = ids.shape
    L = _lib.lib()
    E = num_local_experts if expert_map is not None else num_experts
    if expert_map is not None:
        expert_map = expert_map.to(device=dev, dtype=torch.int32).contiguous()
        if E is None:
            raise ValueError("num_local_experts is required with expert_map")
    cap = L.b200moe_align_capacity_rows(M * topk, E, block_size)
    cap_b = L.b200moe_align_capacity_blocks(M * topk, E, block_size)
    sorted_ids = torch.empty(cap, dtype=torch.int32, device=dev)
    expert_ids = torch.empty(cap_b, dtype=torch.int32, device=dev)
    ntp = torch.empty(1, dtype=torch.int32, device=dev)
    err = err_word if err_word is not None else layer_error_word(dev)
    _lib.check(L.b200moe_align(_ptr(ids), M, topk, num_experts, block_size, _ptr(expert_map), E or 0,
                               _ptr(sorted_ids), cap, _ptr(expert_ids), cap_b, _ptr(ntp), _ptr(err), _stream(dev)),
               "moe_align_block_size")
    return sorted_ids, expert_ids, ntp


def select_experts(router_logits: torch.Tensor, top_k: int, scoring_func: str = "softmax",
                   correction_bias: Optional[torch.Tensor] = None, renormalize: bool = True,
                   routed_scaling_factor: float = 1.0):
    """Router: (M, E) f32/bf16 logits -> (topk_weights (M, k) f32, topk_ids (M, k) int32).
    softmax: top-k softmax probabilities; sigmoid: top-k of sigmoid + correction_bias
    with the unbiased sigmoid as weights (GLM's routing). See b200moe_router_topk."""
    dev = _require_cuda(router_logits)
    if router_logits.dtype not in (torch.float32, torch.bfloat16):
        raise NotImplementedError("router logits must be float32 or bfloat16")
    scoring = {"softmax": 0, "sigmoid": 1}.get(scoring_func)
    if scoring is None:
        raise NotImplementedError(f"scoring_func {scoring_func!r}")
    logits = router_logits.contiguous()
    M, E = logits.shape
    w = torch.empty(M, top_k, dtype=torch.float32, device=dev)
    ids = torch.empty(M, top_k, dtype=torch.int32, device=dev)
    bias = None if correction_bias is None else correction_bias.to(device=dev, dtype=torch.float32).contiguous()
    _lib.check(_lib.lib().b200moe_router_topk(_ptr(logits), int(logits.dtype == torch.bfloat16), M, E, top_k,
                                              scoring, _ptr(bias), int(renormalize), float(routed_scaling_factor),
                                              _ptr(w), _ptr(ids), _stream(dev)), "select_experts")
    return w, ids


def per_token_group_quant_fp8(x: torch.Tensor, group_size: int = 128):
    """(M, K) bf16 -> (q e4m3 (M, K), s f32 (M, K/128))."""
    if group_size != 128:
        raise NotImplementedError("only 128-wide groups are supported")
    dev = _require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise NotImplementedError("per_token_group_quant_fp8 takes bf16 input")
    if x.dim() != 2 or x.stride(1) != 1:
        x = x.reshape(-1, x.shape[-1]).contiguous()
    M, K = x.shape
    q = torch.empty(M, K, dtype=FP8, device=dev)
    s = torch.empty(M, K // 128, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().b200moe_quant_1x128(_ptr(x), M, K, x.stride(0), _ptr(q), K, _ptr(s), K // 128, 1,
                                              _stream(dev)), "per_token_group_quant_fp8")
    return q, s


def per_block_quant_fp8(w: torch.Tensor, bn: int = 128, bk: int = 128):
    """(E, N, K) bf16 -> (q e4m3 (E, N, K), s f32 (E, N/128, K/128))."""
    if bn != 128 or bk != 128:
        raise NotImplementedError("only 128x128 blocks are supported")
    dev = _require_cuda(w)
    if w.dtype != torch.bfloat16:
        raise NotImplementedError("per_block_quant_fp8 takes bf16 input")
    w = w.contiguous()
    E, N, K = w.shape
    q = torch.empty(E, N, K, dtype=FP8, device=dev)
    s = torch.empty(E, N // 128, K // 128, dtype=torch.float32, device=dev)
    _lib.check(_lib.lib().b200moe_quant_block128(_ptr(w), E, N, K, _ptr(q), _ptr(s), _stream(dev)),
               "per_block_quant_fp8")
    return q, s


# ----------------------------------------------------------------------------
# the layer
# ----------------------------------------------------------------------------
def _check_layer_args(hidden, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids, a1_scale=None):
    dev = _require_cuda(hidden, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids)
    if hidden.dtype == FP8:
        if a1_scale is None or a1_scale.dim() != 2 or tuple(a1_scale.shape) != (hidden.shape[0], hidden.shape[1] // 128):
            raise NotImplementedError("fp8 hidden_states need a1_scale of shape (M, H/128) (1x128 per-token-group "
                                      "scales); per-token (M,) scales are not supported")
    elif hidden.dtype != torch.bfloat16:
        raise NotImplementedError("hidden_states must be bf16, or fp8 e4m3 with (M, H/128) a1_scale")
    if w13.dtype != FP8 or w2.dtype != FP8:
        raise NotImplementedError("weights must be float8_e4m3fn with 128x128 block scales")
    if w13_scale is None or w2_scale is None:
        raise ValueError("w13_scale and w2_scale are required")
    M, H = hidden.shape
    E, N2, H2 = w13.shape
    I = w2.shape[2]
    if H2 != H or N2 != 2 * I or w2.shape[:2] != (E, H):
        raise ValueError(f"shape mismatch: hidden {tuple(hidden.shape)}, w13 {tuple(w13.shape)}, "
                         f"w2 {tuple(w2.shape)}")
    if tuple(w13_scale.shape) != (E, N2 // 128, H // 128) or tuple(w2_scale.shape) != (E, H // 128, I // 128):
        raise ValueError("block scale shapes must be (E, N/128, K/128)")
    if topk_ids.shape != topk_weights.shape or topk_ids.shape[0] != M:
        raise ValueError("topk_ids and topk_weights must both be (M, topk)")
    return dev, M, H, I, E


def _run_layer(hidden, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids, expert_map, num_experts, out=None,
               a1_scale=None):
    dev, M, H, I, E_w = _check_layer_args(hidden, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids, a1_scale)
    topk = topk_ids.shape[1]
    if out is None:
        out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    if M == 0:
        return out
    hidden = hidden.contiguous()
    ids = topk_ids.to(torch.int32).contiguous()
    tw = topk_weights.to(torch.float32).contiguous()
    L = _lib.lib()
    n_local = E_w
    ws_bytes = L.b200moe_layer_workspace_size(M, H, I, num_experts, n_local, topk)
    ws = _workspaces.get(dev, ws_bytes)
    # Contiguous copies are bound to names so that they live until the call
    # returns: a copy whose pointer alone were passed could be freed, and its
    # memory reused by the next copy, before the kernels read it.
    w13_scale, w2_scale = w13_scale.contiguous(), w2_scale.contiguous()
    if hidden.dtype == FP8:
        a1 = a1_scale.to(torch.float32).contiguous()
        _lib.check(L.b200moe_layer_quantized(_ptr(hidden), _ptr(a1), M, H, I, num_experts, topk, _ptr(w13),
                                             _ptr(w13_scale), _ptr(w2), _ptr(w2_scale),
                                             _ptr(tw), _ptr(ids), _ptr(expert_map), n_local, _ptr(out), _ptr(ws),
                                             ws.numel(), _stream(dev)), "b200moe_layer_quantized")
        return out
    _lib.check(L.b200moe_layer(_ptr(hidden), M, H, I, num_experts, topk, _ptr(w13), _ptr(w13_scale),
                               _ptr(w2), _ptr(w2_scale), _ptr(tw), _ptr(ids), _ptr(expert_map),
                               n_local, _ptr(out), _ptr(ws), ws.numel(), _stream(dev)), "b200moe_layer")
    return out


def moe_decode_megakernel_full(hidden_states: torch.Tensor, w13_fp8: torch.Tensor, w13_scale: torch.Tensor,
                               w2_fp8: torch.Tensor, w2_scale: torch.Tensor, topk_weights: torch.Tensor,
                               topk_ids: torch.Tensor, a1_scale: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Full MoE layer, same arguments and result as the reference
    `_moe_decode_megakernel_full` (sglang_integration/aiter.py:74-177):
    (M, H) bf16 = sum_j topk_weights[:, j] * W2[e] . silu_mul(W13[e] . h).
    hidden_states may be bf16, or fp8 e4m3 already quantised 1x128 with
    a1_scale (M, H/128); the reference's per-token (M,) a1_scale form
    (aiter.py:126-130) cannot run there either and is rejected."""
    if hidden_states.dtype != FP8 and a1_scale is not None:
        raise ValueError("a1_scale is only meaningful with fp8 hidden_states")
    return _run_layer(hidden_states, w13_fp8, w13_scale, w2_fp8, w2_scale, topk_weights, topk_ids, None,
                      w13_fp8.shape[0], a1_scale=a1_scale)


_moe_decode_megakernel_full = moe_decode_megakernel_full


class QuantType(str, Enum):
    """aiter QuantType names (sglang_integration/aiter.py:180-184)."""
    No = "No"
    per_Token = "per_Token"
    per_128x128 = "per_128x128"
    per_1x32 = "per_1x32"


class ActivationType(str, Enum):
    Silu = "Silu"
    Gelu = "Gelu"
    Swiglu = "Swiglu"
    Situv2 = "Situv2"


def _enum_value(x) -> str:
    return x.value if isinstance(x, Enum) else (x.name if hasattr(x, "name") else str(x))


def expert_map_from_mask(expert_mask: torch.Tensor) -> torch.Tensor:
    """expert_mask (E_global,) of 0/1 -> map global id -> local weight index or -1."""
    m = expert_mask.to(torch.int32)
    local = torch.cumsum(m, 0, dtype=torch.int32) - 1
    return torch.where(m > 0, local, torch.full_like(local, -1)).contiguous()


def fused_moe(hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, topk_weight: torch.Tensor,
              topk_ids: torch.Tensor, quant_type=QuantType.per_128x128, activation=ActivationType.Silu,
              w1_scale: Optional[torch.Tensor] = None, w2_scale: Optional[torch.Tensor] = None,
              a1_scale: Optional[torch.Tensor] = None, a2_scale: Optional[torch.Tensor] = None,
              bias1: Optional[torch.Tensor] = None, bias2: Optional[torch.Tensor] = None,
              expert_mask: Optional[torch.Tensor] = None, doweight_stage1: bool = False, hidden_pad: int = 0,
              intermediate_pad: int = 0, gate_mode: str = "interleave", num_local_tokens=None, dtype=None,
              no_combine: bool = False, **extra) -> torch.Tensor:
    """The aiter fused_moe call of sglang_integration/aiter.py:459-478 for the
    block-scaled FP8 configuration (per_128x128, Silu, gate/up interleaved).

    expert_mask (E_global,) marks the experts whose weights w1/w2 hold (in
    ascending id order); slots routed elsewhere contribute nothing."""
    if _enum_value(quant_type) != QuantType.per_128x128.value:
        raise NotImplementedError(f"quant_type {quant_type!r}: only per_128x128 is supported")
    if _enum_value(activation) != ActivationType.Silu.value:
        raise NotImplementedError(f"activation {activation!r}: only Silu is supported")
    if str(_enum_value(gate_mode)).lower() not in ("interleave", "0"):
        raise NotImplementedError("only the interleaved gate/up weight layout is supported")
    if bias1 is not None or bias2 is not None:
        raise NotImplementedError("bias is not supported")
    if a2_scale is not None:
        raise NotImplementedError("static a2_scale is not supported (stage-2 activations are quantised per group)")
    if doweight_stage1 or hidden_pad or intermediate_pad:
        raise NotImplementedError("doweight_stage1 / hidden_pad / intermediate_pad are not supported")
    if no_combine:
        raise NotImplementedError("no_combine is not supported")
    if dtype not in (None, torch.bfloat16):
        raise NotImplementedError("output dtype must be bf16")
    if num_local_tokens is not None:
        raise NotImplementedError("num_local_tokens is not supported")
    if extra.pop("swiglu_limit", 0.0):
        raise NotImplementedError("swiglu_limit is not supported")
    if extra:
        raise NotImplementedError(f"unsupported arguments: {sorted(extra)}")
    if hidden_states.dtype != FP8 and a1_scale is not None:
        raise NotImplementedError("static a1_scale with bf16 hidden_states is not supported (activations are "
                                  "quantised per 1x128 group)")
    if hidden_states.shape[0] == 0:
        return hidden_states.new_empty((0, hidden_states.shape[1]), dtype=torch.bfloat16)
    if expert_mask is not None:
        emap = expert_map_from_mask(expert_mask.to(hidden_states.device))
        return _run_layer(hidden_states, w1, w1_scale, w2, w2_scale, topk_weight, topk_ids, emap,
                          int(expert_mask.numel()), a1_scale=a1_scale)
    return _run_layer(hidden_states, w1, w1_scale, w2, w2_scale, topk_weight, topk_ids, None, w1.shape[0],
                      a1_scale=a1_scale)


def moe_layer_from_logits(hidden_states: torch.Tensor, router_logits: torch.Tensor, w13_fp8: torch.Tensor,
                          w13_scale: torch.Tensor, w2_fp8: torch.Tensor, w2_scale: torch.Tensor, top_k: int,
                          scoring_func: str = "sigmoid", correction_bias: Optional[torch.Tensor] = None,
                          renormalize: bool = True, routed_scaling_factor: float = 1.0,
                          expert_map: Optional[torch.Tensor] = None):
    """Router + layer: select_experts(router_logits, ...) followed by
    moe_decode_megakernel_full, with the router inside routing's first launch
    (b200moe_layer_logits). Returns (out (M, H) bf16, topk_weights (M, k) f32,
    topk_ids (M, k) int32), bit-identical to the two calls. expert_map
    (num_experts,) maps a global id to a local weight index or -1 (the weights
    then hold only the mapped experts)."""
    dev = _require_cuda(hidden_states, router_logits, w13_fp8, w2_fp8)
    if hidden_states.dtype != torch.bfloat16:
        raise NotImplementedError("moe_layer_from_logits takes bf16 hidden_states")
    if router_logits.dtype not in (torch.float32, torch.bfloat16):
        raise NotImplementedError("router logits must be float32 or bfloat16")
    scoring = {"softmax": 0, "sigmoid": 1}.get(scoring_func)
    if scoring is None:
        raise NotImplementedError(f"scoring_func {scoring_func!r}")
    M, E_router = router_logits.shape
    tw = torch.empty(M, top_k, dtype=torch.float32, device=dev)
    ids = torch.empty(M, top_k, dtype=torch.int32, device=dev)
    _, _, H, I, E_w = _check_layer_args(hidden_states, w13_fp8, w13_scale, w2_fp8, w2_scale, tw, ids)
    out = torch.empty(M, H, dtype=torch.bfloat16, device=dev)
    if M == 0:
        return out, tw, ids
    if expert_map is not None:
        expert_map = expert_map.to(device=dev, dtype=torch.int32).contiguous()
    elif E_w != E_router:
        raise ValueError("without expert_map the weights must hold every routed expert")
    bias = None if correction_bias is None else correction_bias.to(device=dev, dtype=torch.float32).contiguous()
    logits = router_logits.contiguous()
    hidden = hidden_states.contiguous()
    w13_scale, w2_scale = w13_scale.contiguous(), w2_scale.contiguous()  # held through the call
    L = _lib.lib()
    ws = _workspaces.get(dev, L.b200moe_layer_workspace_size(M, H, I, E_router, E_w, top_k))
    _lib.check(L.b200moe_layer_logits(_ptr(hidden), M, H, I, E_router, top_k, _ptr(logits),
                                      int(logits.dtype == torch.bfloat16), scoring, _ptr(bias), int(renormalize),
                                      float(routed_scaling_factor), _ptr(w13_fp8), _ptr(w13_scale),
                                      _ptr(w2_fp8), _ptr(w2_scale), _ptr(expert_map), E_w, _ptr(tw),
                                      _ptr(ids), _ptr(out), _ptr(ws), ws.numel(), _stream(dev)),
               "b200moe_layer_logits")
    return out, tw, ids


def moe_layer_ep_local(hidden_states, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids, expert_map,
                       num_experts: int, out=None):
    """Layer over the experts this rank holds: ids are global, expert_map maps
    them to local weight rows (-1 = elsewhere). Used by the expert-parallel path."""
    return _run_layer(hidden_states, w13, w13_scale, w2, w2_scale, topk_weights, topk_ids, expert_map,
                      num_experts, out=out)
