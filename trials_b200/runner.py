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
A serving framework registers these the way it registers the aiter ones; the
runner needs no sglang import itself. Options the kernels do not implement
raise NotImplementedError (the reference runner raises for unsupported
no_combine the same way, :366-371); there is no fallback.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional

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
