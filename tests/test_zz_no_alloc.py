"""b200moe_layer_noalloc: the layer for callers that cannot allocate device
memory (a memory pool fixed at start-up, or a host framework that forbids
allocation inside an operator), so they cannot hand the layer a workspace.

It runs the same kernels on the same inputs as b200moe_layer, so it must give
the same bytes, call after call, although all calls share one static scratch
array that keeps the previous call's contents; and once its first call on the
device has looked up the array's address, its calls take no device memory.
This file is collected last so that a failure here stops a run only after
every other test has run.
"""
import pytest
import torch

from oracle import moe_oracle as orc
from trials_b200 import _lib, moe, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]


def _noalloc(L, out, err):
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    M, H = L.hidden.shape
    I = L.w2.shape[2]
    E = L.w13.shape[0]
    topk = L.topk_ids.shape[1]
    return _lib.lib().b200moe_layer_noalloc(
        ptr(L.hidden), M, H, I, E, topk, ptr(L.w13), ptr(L.w13_scale), ptr(L.w2), ptr(L.w2_scale),
        ptr(L.topk_weights), ptr(L.topk_ids), None, E, ptr(out), ptr(err),
        torch.cuda.current_stream().cuda_stream)


def _on(dev, L):
    for k in ["hidden", "topk_weights", "topk_ids", "w13", "w13_scale", "w2", "w2_scale"]:
        setattr(L, k, getattr(L, k).to(dev))
    return L


def test_noalloc_layer_matches_layer_on_two_calls_in_a_row(cuda_device):
    layers = [synth.make_layer(synth.glm(64), moe.per_block_quant_fp8, seed=3, device=cuda_device),
              _on(cuda_device, synth.make_layer(synth.TINY, orc.per_block_quant_fp8, seed=5))]
    for L in layers:
        expected = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale,
                                                  L.topk_weights, L.topk_ids)
        out = torch.full_like(expected, float("nan"))
        err = torch.full((1,), -1, dtype=torch.int32, device=cuda_device)
        assert _noalloc(L, out, err) == _lib.OK, _lib.lib().b200moe_last_error_message()
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(out, expected)


def test_noalloc_layer_takes_no_device_memory(cuda_device):
    L = synth.make_layer(synth.glm(64), moe.per_block_quant_fp8, seed=7, device=cuda_device)
    out = torch.empty(L.hidden.shape, dtype=torch.bfloat16, device=cuda_device)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    assert _noalloc(L, out, err) == _lib.OK  # first call on the device: looks up the scratch address
    torch.cuda.synchronize()
    first = out.clone()
    free_before, _ = torch.cuda.mem_get_info(cuda_device)
    for _ in range(3):
        assert _noalloc(L, out, err) == _lib.OK, _lib.lib().b200moe_last_error_message()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info(cuda_device)
    assert free_after == free_before
    assert torch.equal(out, first) and int(err.item()) == 0


def test_noalloc_rejects_layers_beyond_its_scratch(cuda_device):
    shape = synth.glm(1024)  # needs far more than the 64 MiB scratch
    dummy = torch.zeros(16, dtype=torch.uint8, device=cuda_device)
    p = dummy.data_ptr()
    st = _lib.lib().b200moe_layer_noalloc(p, shape.M, shape.H, shape.I, shape.E, shape.topk, p, p, p, p, p, p,
                                          None, shape.E, p, None, torch.cuda.current_stream().cuda_stream)
    assert st == _lib.ERR_WORKSPACE
    assert b"64 MiB" in _lib.lib().b200moe_last_error_message()
    # an invalid shape is reported as such, not as a size limit
    st = _lib.lib().b200moe_layer_noalloc(p, shape.M, 0, shape.I, shape.E, shape.topk, p, p, p, p, p, p,
                                          None, shape.E, p, None, torch.cuda.current_stream().cuda_stream)
    assert st == _lib.ERR_INVALID_ARG
