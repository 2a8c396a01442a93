"""MoE runner adapter with the shape of the reference's aiter runner.

Mirrors, for this library's kernels, the runner pieces of
sglang_integration/aiter.py that sit around the hot path:
  * QuantType                       <- AiterQuantType (:180-184)
  * MoeQuantInfo / RunnerInput / RunnerOutput
                                    <- AiterMoeQuantInfo / AiterRunnerInput /
                                       AiterRunnerOutput (:187-233)
  * MoeRunnerConfig                 <- the MoeRunnerConfig fields run() reads
  * B200MoeRunnerCore.run           <- AiterRunnerCore.run (:358-483): empty
                                       batch, option checks, then the layer
  * pre_permute_standard / post_permute_standard
                                    <- pre_permute_standard_to_aiter (:491-515),
                                       post_permute_aiter_to_standard (:694-703)
  * pre_permute_deepep (DeepEP normal / low-latency and Mori dispatch
    outputs), post_permute_deepep_normal / _ll
                                    <- _pre_permute_deepep_to_aiter (:536-682),
                                       _post_permute_aiter_to_deepep (:706-756)
  * register_pre_permute / register_post_permute, MoeRunnerBackend.B200,
    MoeRunner                       <- sglang's permute registry as used at
                                       :491, :684-685, :694, :736, :748 and the
                                       backend property at :480-482
  * register_with_sglang            registers the permutes above with sglang's
                                    own registry when sglang is importable
  * fuse_shared_expert              the shared expert as one more routed slot
                                    (sglang's shared-experts fusion)
The runner needs no sglang import itself. Options the kernels do not
implement raise NotImplementedError (the reference runner raises for
unsupported no_combine the same way, :366-371); there is no fallback.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from enum import Enum
from typing import Any, Callable, Dict, Optional, Tuple

import torch

from . import moe


class QuantType:
    NONE = "No"
    PER_TOKEN = "per_Token"
    PER_128X128 = "per_128x128"
    PER_1X32 = "per_1x32"


@dataclass
class MoeRunnerConfig:
    activation: str = "silu"
    no_combine: bool = False
    apply_router_weight_on_input: bool = False
    gemm1_alpha: Optional[float] = None
    gemm1_clamp_limit: Optional[float] = None


@dataclass
class MoeQuantInfo:
    w13_weight: torch.Tensor
    w2_weight: torch.Tensor
    quant_type: str = QuantType.NONE
    w13_scale: Optional[torch.Tensor] = None
    w2_scale: Optional[torch.Tensor] = None
    a13_scale: Optional[torch.Tensor] = None
    a2_scale: Optional[torch.Tensor] = None
    b13: Optional[torch.Tensor] = None
    b2: Optional[torch.Tensor] = None
    expert_mask: Optional[torch.Tensor] = None
    doweight_stage1: bool = False
    hidden_pad: int = 0
    intermediate_pad: int = 0
    swiglu_limit: float = 0.0
    fused_moe_kwargs: Optional[dict] = None


@dataclass
class RunnerInput:
    hidden_states: torch.Tensor
    topk_ids: torch.Tensor       # int32
    topk_weights: torch.Tensor   # float32
    quant_type: str
    a1_scale: Optional[torch.Tensor] = None
    num_local_tokens: Optional[torch.Tensor] = None
    output_dtype: Optional[torch.dtype] = None


@dataclass
class RunnerOutput:
    hidden_states: torch.Tensor


@dataclass
class StandardDispatchOutput:
    """hidden_states and topk_output = (topk_weights, topk_ids, router_logits)."""
    hidden_states: torch.Tensor
    topk_output: tuple


@dataclass
class StandardCombineInput:
    hidden_states: torch.Tensor


class B200MoeRunnerCore:
    def __init__(self, config: Optional[MoeRunnerConfig] = None):
        self.config = config or MoeRunnerConfig()

    def run(self, runner_input: RunnerInput, quant_info: MoeQuantInfo, running_state: Optional[dict] = None,
            hooks: Any = None) -> RunnerOutput:
        cfg = self.config
        if cfg.no_combine:
            raise NotImplementedError("no_combine=True is not supported by the B200 MoE kernels")
        if runner_input.hidden_states.shape[0] == 0:
            return RunnerOutput(hidden_states=runner_input.hidden_states)
        if cfg.activation != "silu":
            raise NotImplementedError(f"activation {cfg.activation!r}: only silu is supported")
        if runner_input.quant_type != QuantType.PER_128X128:
            raise NotImplementedError(f"quant_type {runner_input.quant_type!r}: only per_128x128 is supported")
        if quant_info.b13 is not None or quant_info.b2 is not None or quant_info.swiglu_limit:
            raise NotImplementedError("bias and swiglu_limit are not supported")
        if quant_info.w13_scale is None or quant_info.w2_scale is None:
            raise ValueError("per_128x128 needs w13_scale and w2_scale")
        if runner_input.output_dtype not in (None, torch.bfloat16):
            raise NotImplementedError("output dtype must be bf16")
        a1_scale = runner_input.a1_scale if runner_input.a1_scale is not None else quant_info.a13_scale
        extra = dict(quant_info.fused_moe_kwargs or {})
        out = moe.fused_moe(
            hidden_states=runner_input.hidden_states, w1=quant_info.w13_weight, w2=quant_info.w2_weight,
            topk_weight=runner_input.topk_weights, topk_ids=runner_input.topk_ids,
            quant_type=moe.QuantType.per_128x128, activation=moe.ActivationType.Silu,
            w1_scale=quant_info.w13_scale, w2_scale=quant_info.w2_scale, a1_scale=a1_scale,
            a2_scale=quant_info.a2_scale, expert_mask=quant_info.expert_mask,
            doweight_stage1=quant_info.doweight_stage1, hidden_pad=quant_info.hidden_pad,
            intermediate_pad=quant_info.intermediate_pad, num_local_tokens=runner_input.num_local_tokens, **extra)
        return RunnerOutput(hidden_states=out)


def pre_permute_standard(dispatch_output: StandardDispatchOutput, quant_info: MoeQuantInfo,
                         runner_config: MoeRunnerConfig, running_state: Optional[dict] = None) -> RunnerInput:
    """Standard dispatch -> RunnerInput: f32 weights, int32 ids; with
    apply_router_weight_on_input (top-1 only) the weight is folded into the
    hidden states and replaced by ones."""
    hidden_states = dispatch_output.hidden_states
    topk_weights, topk_ids = dispatch_output.topk_output[0], dispatch_output.topk_output[1]
    topk_weights = topk_weights.to(torch.float32)
    if runner_config.apply_router_weight_on_input and not quant_info.doweight_stage1:
        if topk_weights.dim() != 2 or topk_weights.shape[-1] != 1:
            raise ValueError("apply_router_weight_on_input requires topk=1")
        hidden_states = hidden_states * topk_weights.to(hidden_states.dtype)
        topk_weights = torch.ones_like(topk_weights)
    return RunnerInput(hidden_states=hidden_states, topk_ids=topk_ids.to(torch.int32), topk_weights=topk_weights,
                       quant_type=quant_info.quant_type)


def post_permute_standard(runner_output: RunnerOutput, quant_info: MoeQuantInfo, runner_config: MoeRunnerConfig,
                          running_state: Optional[dict] = None) -> StandardCombineInput:
    return StandardCombineInput(hidden_states=runner_output.hidden_states)


# ----------------------------------------------------------------------------
# DeepEP / Mori dispatch formats
# ----------------------------------------------------------------------------
@dataclass
class DeepEPDispatchOutput:
    """What a DeepEP dispatcher (normal or low-latency) hands the runner: the
    rows received on this rank and their top-k ids among this rank's experts
    (-1 = expert on another rank)."""
    hidden_states: torch.Tensor
    topk_ids: torch.Tensor
    topk_weights: torch.Tensor


@dataclass
class MoriDispatchOutput:
    """Mori's dispatch output: received rows (bf16, or fp8 with group-128 fp32
    hidden_states_scale), local top-k ids and weights, the sender-side
    origin_topk_ids / origin_topk_weights its combine needs, the count of valid
    received rows (device tensor) and the output dtype."""
    hidden_states: torch.Tensor
    topk_ids: torch.Tensor
    topk_weights: torch.Tensor
    origin_topk_ids: torch.Tensor
    origin_topk_weights: torch.Tensor
    hidden_states_scale: Optional[torch.Tensor] = None
    num_recv_tokens_per_expert: Optional[torch.Tensor] = None
    out_dtype: Optional[torch.dtype] = None


@dataclass
class DeepEPCombineInput:
    """Combine input of the DeepEP / Mori formats (normal and low-latency have
    the same fields): the runner's rows and the ids / weights their combine
    routes them back with."""
    hidden_states: torch.Tensor
    topk_ids: torch.Tensor
    topk_weights: torch.Tensor
    is_mori: bool = False
    is_normal: bool = True


def _is_mori(dispatch_output: Any) -> bool:
    # Mori outputs carry the sender-side origin_topk_* that DeepEP's lack
    # (the same test as the reference, aiter.py:517-520).
    return hasattr(dispatch_output, "origin_topk_ids")


def mori_recv_bound(recv_rows: int, topk: int, per_rank_tokens=None, is_extend: bool = False) -> int:
    """Live rows of Mori's receive buffer at decode (0 = do not bound): every
    rank's tokens times topk, when the per-rank counts of the data-parallel
    sync are known and the batch is not a prefill; never more than the buffer
    (the rule of aiter.py:271-355, with the counts passed in instead of read
    from the serving runtime). Only with B200MOE_MORI_RECV_BOUND=1."""
    if os.environ.get("B200MOE_MORI_RECV_BOUND", "0").lower() not in ("1", "true"):
        return 0
    if is_extend or not per_rank_tokens:
        return 0
    bound = int(sum(per_rank_tokens)) * topk
    return bound if 0 < bound < recv_rows else 0


def pre_permute_deepep(dispatch_output: Any, quant_info: MoeQuantInfo, runner_config: "MoeRunnerConfig",
                       running_state: Optional[dict] = None, num_local_experts: Optional[int] = None,
                       max_input_rows: int = 0) -> RunnerInput:
    """DeepEP (normal / low-latency) or Mori dispatch output -> RunnerInput
    (aiter.py:536-682).

    DeepEP: -1 ids (experts on other ranks) are rerouted to the sink expert
    num_local_experts, which quant_info.expert_mask (num_local_experts + 1
    entries, 0 at the sink) masks off - the reference's convention; with no
    mask the layer drops -1 ids itself.
    Mori: fp8 rows with group-128 fp32 scales go in as they are (a1_scale);
    rows at or past the valid-row count (num_recv_tokens_per_expert) get ids
    -1; the first max_input_rows rows are kept when given (Mori's combine
    reads only those). FP4 dispatch and the other dtype pairs the reference
    upscales are refused (this path's weights are per_128x128 FP8)."""
    running_state = {} if running_state is None else running_state
    hidden_states = dispatch_output.hidden_states
    topk_ids = dispatch_output.topk_ids.to(torch.int32)
    topk_weights = dispatch_output.topk_weights.to(torch.float32)
    a1_scale = None
    output_dtype = None
    is_mori = _is_mori(dispatch_output)
    if is_mori:
        a1_scale = getattr(dispatch_output, "hidden_states_scale", None)
        output_dtype = getattr(dispatch_output, "out_dtype", None)
        fp4 = getattr(torch, "float4_e2m1fn_x2", None)
        if fp4 is not None and hidden_states.dtype == fp4:
            raise NotImplementedError("FP4 dispatch is not supported: this path runs per_128x128 FP8 weights")
        if a1_scale is not None and a1_scale.dtype != torch.float32:
            raise NotImplementedError("only group-128 fp32 dispatch scales are supported (no MX scales)")
        if max_input_rows > 0:
            hidden_states = hidden_states[:max_input_rows]
            a1_scale = None if a1_scale is None else a1_scale[:max_input_rows]
            topk_ids = topk_ids[:max_input_rows]
            topk_weights = topk_weights[:max_input_rows]
        n_valid = getattr(dispatch_output, "num_recv_tokens_per_expert", None)
        if n_valid is not None:
            # rows past the received count carry stale ids: drop them on the device
            rows = torch.arange(topk_ids.shape[0], device=topk_ids.device, dtype=torch.int32).unsqueeze(1)
            topk_ids = torch.where(rows < n_valid.reshape(-1)[:1].to(torch.int32), topk_ids,
                                   torch.full_like(topk_ids, -1))
        running_state["b200_combine_topk_ids"] = dispatch_output.origin_topk_ids
        running_state["b200_combine_topk_weights"] = dispatch_output.origin_topk_weights
    else:
        if num_local_experts is not None:
            topk_ids = torch.where(topk_ids == -1, torch.full_like(topk_ids, num_local_experts), topk_ids)
        running_state["b200_combine_topk_ids"] = dispatch_output.topk_ids
        running_state["b200_combine_topk_weights"] = dispatch_output.topk_weights
    running_state["b200_combine_is_mori"] = is_mori
    return RunnerInput(hidden_states=hidden_states, topk_ids=topk_ids, topk_weights=topk_weights,
                       quant_type=quant_info.quant_type, a1_scale=a1_scale, output_dtype=output_dtype)


def _post_permute_deepep(runner_output: RunnerOutput, running_state: dict, is_normal: bool) -> DeepEPCombineInput:
    return DeepEPCombineInput(hidden_states=runner_output.hidden_states,
                              topk_ids=running_state["b200_combine_topk_ids"],
                              topk_weights=running_state["b200_combine_topk_weights"],
                              is_mori=bool(running_state.get("b200_combine_is_mori")), is_normal=is_normal)


def post_permute_deepep_normal(runner_output: RunnerOutput, quant_info: MoeQuantInfo,
                               runner_config: "MoeRunnerConfig", running_state: dict) -> DeepEPCombineInput:
    return _post_permute_deepep(runner_output, running_state, True)


def post_permute_deepep_ll(runner_output: RunnerOutput, quant_info: MoeQuantInfo, runner_config: "MoeRunnerConfig",
                           running_state: dict) -> DeepEPCombineInput:
    return _post_permute_deepep(runner_output, running_state, False)


# ----------------------------------------------------------------------------
# Permute registry and the runner (the MoeRunnerBackend registration)
# ----------------------------------------------------------------------------
class MoeRunnerBackend(str, Enum):
    B200 = "b200"


_PRE: Dict[Tuple[str, str], Callable] = {}
_POST: Dict[Tuple[str, str], Callable] = {}


def register_pre_permute(dispatch_format: str, runner_backend: str):
    """Decorator: fn(dispatch_output, quant_info, runner_config, running_state)
    -> RunnerInput for (dispatch format, runner backend)."""
    def deco(fn):
        _PRE[(dispatch_format, str(getattr(runner_backend, "value", runner_backend)))] = fn
        return fn
    return deco


def register_post_permute(runner_backend: str, combine_format: str):
    """Decorator: fn(runner_output, quant_info, runner_config, running_state)
    -> combine input for (runner backend, combine format)."""
    def deco(fn):
        _POST[(str(getattr(runner_backend, "value", runner_backend)), combine_format)] = fn
        return fn
    return deco


def _pre_std(d, qi, cfg, state):
    return pre_permute_standard(d, qi, cfg, state)


def _pre_deepep(d, qi, cfg, state):
    n = qi.expert_mask.numel() - 1 if qi.expert_mask is not None else None
    return pre_permute_deepep(d, qi, cfg, state, num_local_experts=n,
                              max_input_rows=int(os.environ.get("B200MOE_MORI_MAX_INPUT_TOKENS", "0")))


register_pre_permute("standard", MoeRunnerBackend.B200)(_pre_std)
register_pre_permute("deepep_normal", MoeRunnerBackend.B200)(_pre_deepep)
register_pre_permute("deepep_ll", MoeRunnerBackend.B200)(_pre_deepep)
register_post_permute(MoeRunnerBackend.B200, "standard")(post_permute_standard)
register_post_permute(MoeRunnerBackend.B200, "deepep_normal")(post_permute_deepep_normal)
register_post_permute(MoeRunnerBackend.B200, "deepep_ll")(post_permute_deepep_ll)


class MoeRunner:
    """dispatch output -> pre-permute -> B200MoeRunnerCore.run -> post-permute,
    by (dispatch format, backend) and (backend, combine format), the way the
    serving framework drives a runner backend."""

    def __init__(self, config: Optional["MoeRunnerConfig"] = None, backend=MoeRunnerBackend.B200):
        self.config = config or MoeRunnerConfig()
        self.backend = str(getattr(backend, "value", backend))
        self.core = B200MoeRunnerCore(self.config)

    @property
    def runner_backend(self) -> MoeRunnerBackend:
        return MoeRunnerBackend(self.backend)

    def run(self, dispatch_output: Any, quant_info: MoeQuantInfo, dispatch_format: str = "standard",
            combine_format: Optional[str] = None):
        pre = _PRE.get((dispatch_format, self.backend))
        post = _POST.get((self.backend, combine_format or dispatch_format))
        if pre is None or post is None:
            raise NotImplementedError(f"no permute registered for {dispatch_format!r} -> {self.backend!r} -> "
                                      f"{combine_format or dispatch_format!r}")
        state: dict = {}
        ri = pre(dispatch_output, quant_info, self.config, state)
        return post(self.core.run(ri, quant_info, state), quant_info, self.config, state)


def register_with_sglang() -> bool:
    """Registers the pre/post-permutes above with sglang's runner registry
    (sglang.srt.layers.moe.moe_runner.base) under the backend name "b200".
    Returns False when sglang is not importable; nothing is patched then."""
    try:
        from sglang.srt.layers.moe.moe_runner import base as sg  # noqa: F401
    except Exception:  # sglang absent (or broken): nothing to register with
        return False
    for (fmt, backend), fn in _PRE.items():
        sg.register_pre_permute(fmt, backend)(fn)
    for (backend, fmt), fn in _POST.items():
        sg.register_post_permute(backend, fmt)(fn)
    return True


# ----------------------------------------------------------------------------
# Shared-expert fusion
# ----------------------------------------------------------------------------
def fuse_shared_expert(topk_weights: torch.Tensor, topk_ids: torch.Tensor, shared_expert_id: int,
                       shared_weight: float = 1.0):
    """Appends the shared expert as one more routed slot of every token
    (sglang's shared-experts fusion: the shared expert's weights are stored as
    expert `shared_expert_id`, after the routed ones, and every token routes
    to it with weight `shared_weight`). -> (topk_weights (M, k+1) f32,
    topk_ids (M, k+1) int32); the layer then computes routed + shared in one
    call."""
    M = topk_ids.shape[0]
    ids = torch.cat([topk_ids.to(torch.int32),
                     torch.full((M, 1), shared_expert_id, dtype=torch.int32, device=topk_ids.device)], dim=1)
    w = torch.cat([topk_weights.to(torch.float32),
                   torch.full((M, 1), float(shared_weight), dtype=torch.float32, device=topk_weights.device)], dim=1)
    return w.contiguous(), ids.contiguous()
