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


# ---- DeepEP / Mori formats, the permute registry, shared-expert fusion (CPU)
def test_pre_permute_deepep_reroutes_minus_one_to_the_sink():
    ids = torch.tensor([[0, -1], [-1, 2]], dtype=torch.int64)
    d = runner.DeepEPDispatchOutput(hidden_states=torch.zeros(2, 256, dtype=torch.bfloat16), topk_ids=ids,
                                    topk_weights=torch.ones(2, 2, dtype=torch.bfloat16))
    state = {}
    ri = runner.pre_permute_deepep(d, _qi(), runner.MoeRunnerConfig(), state, num_local_experts=3)
    assert ri.topk_ids.tolist() == [[0, 3], [3, 2]] and ri.topk_ids.dtype == torch.int32
    assert ri.topk_weights.dtype == torch.float32 and ri.a1_scale is None
    assert state["b200_combine_topk_ids"] is ids and state["b200_combine_is_mori"] is False
    # without a sink the layer drops -1 ids itself
    assert runner.pre_permute_deepep(d, _qi(), runner.MoeRunnerConfig(), {}).topk_ids.tolist() == [[0, -1], [-1, 2]]
    ci = runner.post_permute_deepep_ll(runner.RunnerOutput(hidden_states=torch.ones(2, 256)), _qi(),
                                       runner.MoeRunnerConfig(), state)
    assert ci.topk_ids is ids and not ci.is_normal and not ci.is_mori


def test_pre_permute_mori_keeps_fp8_rows_and_drops_rows_past_the_count():
    M, H = 5, 256
    q = torch.zeros(M, H, dtype=torch.float8_e4m3fn)
    sc = torch.ones(M, H // 128)
    ids = torch.arange(M * 2, dtype=torch.int32).view(M, 2) % 4
    d = runner.MoriDispatchOutput(hidden_states=q, topk_ids=ids, topk_weights=torch.ones(M, 2),
                                  origin_topk_ids=torch.zeros(3, 2, dtype=torch.int32),
                                  origin_topk_weights=torch.ones(3, 2), hidden_states_scale=sc,
                                  num_recv_tokens_per_expert=torch.tensor([3]), out_dtype=torch.bfloat16)
    state = {}
    ri = runner.pre_permute_deepep(d, _qi(), runner.MoeRunnerConfig(), state, max_input_rows=4)
    assert ri.hidden_states.shape[0] == 4 and ri.a1_scale.shape == (4, H // 128)
    assert ri.topk_ids[:3].tolist() == ids[:3].tolist() and (ri.topk_ids[3:] == -1).all()
    assert state["b200_combine_is_mori"] and state["b200_combine_topk_ids"] is d.origin_topk_ids
    ci = runner.post_permute_deepep_normal(runner.RunnerOutput(hidden_states=torch.ones(4, H)), _qi(),
                                           runner.MoeRunnerConfig(), state)
    assert ci.is_mori and ci.is_normal and ci.topk_weights is d.origin_topk_weights
    bad = runner.MoriDispatchOutput(hidden_states=q, topk_ids=ids, topk_weights=torch.ones(M, 2),
                                    origin_topk_ids=ids, origin_topk_weights=torch.ones(M, 2),
                                    hidden_states_scale=sc.to(torch.bfloat16))
    with pytest.raises(NotImplementedError):
        runner.pre_permute_deepep(bad, _qi(), runner.MoeRunnerConfig(), {})


def test_mori_recv_bound(monkeypatch):
    monkeypatch.delenv("B200MOE_MORI_RECV_BOUND", raising=False)
    assert runner.mori_recv_bound(4096, 9, [16, 16]) == 0  # off unless enabled
    monkeypatch.setenv("B200MOE_MORI_RECV_BOUND", "1")
    assert runner.mori_recv_bound(4096, 9, [16, 16, 8]) == 40 * 9
    assert runner.mori_recv_bound(4096, 9, [16, 16], is_extend=True) == 0
    assert runner.mori_recv_bound(100, 9, [16, 16]) == 0  # never grows the buffer
    assert runner.mori_recv_bound(4096, 9, None) == 0


def test_registry_and_runner_dispatch():
    assert runner.MoeRunner().runner_backend == runner.MoeRunnerBackend.B200
    with pytest.raises(NotImplementedError):
        runner.MoeRunner().run(None, _qi(), dispatch_format="unknown_format")
    seen = []

    @runner.register_pre_permute("test_fmt", "b200")
    def _pre(d, qi, cfg, state):
        seen.append("pre")
        state["x"] = 1
        return _ri(M=0)

    @runner.register_post_permute("b200", "test_fmt")
    def _post(out, qi, cfg, state):
        seen.append(("post", state["x"]))
        return out

    out = runner.MoeRunner().run(None, _qi(), dispatch_format="test_fmt")
    assert seen == ["pre", ("post", 1)] and out.hidden_states.shape[0] == 0


def test_register_with_sglang_uses_its_registry(monkeypatch):
    import sys
    import types

    assert runner.register_with_sglang() is False or "sglang" in sys.modules  # sglang is not installed here
    got = {"pre": [], "post": []}
    base = types.ModuleType("sglang.srt.layers.moe.moe_runner.base")
    base.register_pre_permute = lambda fmt, be: (lambda fn: got["pre"].append((fmt, be)) or fn)
    base.register_post_permute = lambda be, fmt: (lambda fn: got["post"].append((be, fmt)) or fn)
    names = ["sglang", "sglang.srt", "sglang.srt.layers", "sglang.srt.layers.moe", "sglang.srt.layers.moe.moe_runner"]
    for n in names:
        monkeypatch.setitem(sys.modules, n, types.ModuleType(n))
    monkeypatch.setitem(sys.modules, "sglang.srt.layers.moe.moe_runner.base", base)
    sys.modules["sglang.srt.layers.moe.moe_runner"].base = base
    assert runner.register_with_sglang() is True
    assert ("deepep_normal", "b200") in got["pre"] and ("b200", "deepep_ll") in got["post"]


def test_fuse_shared_expert():
    w, ids = runner.fuse_shared_expert(torch.full((3, 2), 0.5), torch.tensor([[1, 2], [0, 1], [2, 0]]), 8, 2.5)
    assert ids.tolist() == [[1, 2, 8], [0, 1, 8], [2, 0, 8]] and w[:, 2].tolist() == [2.5] * 3
    assert ids.dtype == torch.int32 and w.dtype == torch.float32


# ---- the same formats through the layer on the GPU
@pytest.mark.gpu
def test_deepep_and_mori_formats_run_the_layer(cuda_device):
    from oracle import moe_oracle as orc
    from trials_b200 import moe, synth

    dev = cuda_device
    L = synth.make_layer(synth.LayerShape(M=40, H=512, I=256, E=8, topk=4, scoring="sigmoid"), orc.per_block_quant_fp8,
                         seed=4)
    w = {k: getattr(L, k).to(dev) for k in ["w13", "w13_scale", "w2", "w2_scale", "hidden", "topk_weights"]}
    ids = L.topk_ids.to(dev).clone()
    ids[ids >= 6] = -1  # experts 6, 7 live on another rank: DeepEP marks them -1
    local = {k: w[k][:6].contiguous() for k in ["w13", "w13_scale", "w2", "w2_scale"]}
    mask = torch.ones(7, dtype=torch.int32, device=dev)
    mask[6] = 0  # the sink slot
    qi = runner.MoeQuantInfo(w13_weight=local["w13"], w2_weight=local["w2"], quant_type=runner.QuantType.PER_128X128,
                             w13_scale=local["w13_scale"], w2_scale=local["w2_scale"], expert_mask=mask)
    expect = moe.moe_decode_megakernel_full(w["hidden"], local["w13"], local["w13_scale"], local["w2"],
                                            local["w2_scale"], w["topk_weights"], ids)
    d = runner.DeepEPDispatchOutput(hidden_states=w["hidden"], topk_ids=ids, topk_weights=w["topk_weights"])
    ci = runner.MoeRunner().run(d, qi, dispatch_format="deepep_normal")
    assert torch.equal(ci.hidden_states, expect) and ci.topk_ids is ids
    # Mori: fp8 rows with group-128 scales, 30 valid rows of 40
    q, s = moe.per_token_group_quant_fp8(w["hidden"])
    m = runner.MoriDispatchOutput(hidden_states=q, topk_ids=ids, topk_weights=w["topk_weights"],
                                  origin_topk_ids=ids, origin_topk_weights=w["topk_weights"], hidden_states_scale=s,
                                  num_recv_tokens_per_expert=torch.tensor([30], device=dev), out_dtype=torch.bfloat16)
    qi_nomask = runner.MoeQuantInfo(w13_weight=local["w13"], w2_weight=local["w2"],
                                    quant_type=runner.QuantType.PER_128X128, w13_scale=local["w13_scale"],
                                    w2_scale=local["w2_scale"])
    out = runner.MoeRunner().run(m, qi_nomask, dispatch_format="deepep_ll").hidden_states
    assert torch.equal(out[:30], expect[:30]) and (out[30:] == 0).all()


@pytest.mark.gpu
def test_shared_expert_fusion_in_one_layer_call(cuda_device):
    """Routed experts plus a shared expert (stored as expert E) in one call
    equals the routed layer plus the shared expert's own layer, up to the bf16
    rounding of the two separate outputs."""
    from oracle import moe_oracle as orc
    from trials_b200 import moe, synth

    dev = cuda_device
    shape = synth.LayerShape(M=64, H=512, I=256, E=9, topk=4, scoring="sigmoid")
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=9, device=dev)
    g = torch.Generator(device=dev).manual_seed(1)
    tw, ids = synth.make_router(torch.randn(shape.M, 8, generator=g, device=dev), 4, "sigmoid")  # routed: 0..7
    fw, fids = runner.fuse_shared_expert(tw, ids, 8, 1.0)
    fused = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, fw, fids)
    routed = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, tw, ids)
    ones = torch.ones(shape.M, 1, device=dev)
    shared = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, ones,
                                            torch.full((shape.M, 1), 8, dtype=torch.int32, device=dev))
    assert orc.rel_l2(fused, routed.float() + shared.float()) < 5e-3
