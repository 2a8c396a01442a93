"""Runner adapter: option checks on the CPU; the full path on the GPU."""
import pytest
import torch

from trials_b200 import runner


def _qi(**kw):
    w = torch.zeros(1)
    return runner.MoeQuantInfo(w13_weight=w, w2_weight=w, quant_type=runner.QuantType.PER_128X128, w13_scale=w,
                               w2_scale=w, **kw)


def _ri(M=2, qt=runner.QuantType.PER_128X128):
    return runner.RunnerInput(hidden_states=torch.zeros(M, 256, dtype=torch.bfloat16),
                              topk_ids=torch.zeros(M, 2, dtype=torch.int32), topk_weights=torch.ones(M, 2),
                              quant_type=qt)


def test_empty_batch_returns_input():
    core = runner.B200MoeRunnerCore()
    ri = _ri(M=0)
    assert core.run(ri, _qi()).hidden_states is ri.hidden_states


@pytest.mark.parametrize("cfg,qi,ri", [
    (runner.MoeRunnerConfig(no_combine=True), _qi(), _ri()),
    (runner.MoeRunnerConfig(activation="gelu"), _qi(), _ri()),
    (runner.MoeRunnerConfig(), _qi(), _ri(qt=runner.QuantType.PER_TOKEN)),
    (runner.MoeRunnerConfig(), _qi(b13=torch.zeros(1)), _ri()),
    (runner.MoeRunnerConfig(), _qi(swiglu_limit=7.0), _ri()),
])
def test_unsupported_options_raise(cfg, qi, ri):
    with pytest.raises(NotImplementedError):
        runner.B200MoeRunnerCore(cfg).run(ri, qi)


def test_pre_permute_standard():
    h = torch.ones(3, 256, dtype=torch.bfloat16)
    tw = torch.tensor([[0.5], [2.0], [1.0]], dtype=torch.bfloat16)
    ids = torch.tensor([[1], [0], [3]], dtype=torch.int64)
    d = runner.StandardDispatchOutput(hidden_states=h, topk_output=(tw, ids, None))
    ri = runner.pre_permute_standard(d, _qi(), runner.MoeRunnerConfig())
    assert ri.topk_ids.dtype == torch.int32 and ri.topk_weights.dtype == torch.float32
    ri2 = runner.pre_permute_standard(d, _qi(), runner.MoeRunnerConfig(apply_router_weight_on_input=True))
    assert torch.equal(ri2.topk_weights, torch.ones(3, 1))
    assert torch.allclose(ri2.hidden_states[:, 0].float(), tw[:, 0].float())


@pytest.mark.gpu
def test_runner_runs_the_layer(cuda_device):
    from oracle import moe_oracle as orc
    from trials_b200 import moe, synth

    L = synth.make_layer(synth.TINY, orc.per_block_quant_fp8, seed=0)
    qi = runner.MoeQuantInfo(w13_weight=L.w13.to(cuda_device), w2_weight=L.w2.to(cuda_device),
                             quant_type=runner.QuantType.PER_128X128, w13_scale=L.w13_scale.to(cuda_device),
                             w2_scale=L.w2_scale.to(cuda_device))
    d = runner.StandardDispatchOutput(hidden_states=L.hidden.to(cuda_device),
                                      topk_output=(L.topk_weights.to(cuda_device), L.topk_ids.to(cuda_device), None))
    cfg = runner.MoeRunnerConfig()
    ri = runner.pre_permute_standard(d, qi, cfg)
    out = runner.post_permute_standard(runner.B200MoeRunnerCore(cfg).run(ri, qi), qi, cfg).hidden_states
    ref = moe.moe_decode_megakernel_full(ri.hidden_states, qi.w13_weight, qi.w13_scale, qi.w2_weight, qi.w2_scale,
                                         ri.topk_weights, ri.topk_ids)
    assert torch.equal(out, ref)
