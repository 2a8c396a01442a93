"""The whole layer as one cooperative launch (routing, gather + quantise, both
GEMM stages, top-k reduce; b200moe_layer's choice for small batches) against
the same layer as separate launches, bit for bit, and against the oracle.
The launch count is read from a CUDA graph of the call."""
import contextlib
import ctypes
import types

import pytest
import torch

from oracle import moe_oracle as orc
from trials_b200 import _lib, moe, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]

WHOLE, SEPARATE = 1, 2


@contextlib.contextmanager
def launch_mode(mode):
    lib = _lib.lib()
    prev = lib.b200moe_set_layer_launch(mode)
    assert prev in (0, 1, 2)
    try:
        yield
    finally:
        lib.b200moe_set_layer_launch(prev)


def _layer(L, hidden, tw, ids, ws, out, expert_map=None, num_local=0, num_experts=None):
    s = L.shape
    lib = _lib.lib()
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    _lib.check(lib.b200moe_layer(ptr(hidden), hidden.shape[0], s.H, s.I, num_experts or s.E, s.topk, ptr(L.w13),
                                 ptr(L.w13_scale), ptr(L.w2), ptr(L.w2_scale), ptr(tw), ptr(ids), ptr(expert_map),
                                 num_local, ptr(out), ptr(ws), ws.numel(), torch.cuda.current_stream().cuda_stream),
               "layer")
    return out


def _workspace(shape, M, dev, num_local=0):
    lib = _lib.lib()
    n = lib.b200moe_layer_workspace_size(M, shape.H, shape.I, shape.E, num_local, shape.topk)
    return torch.zeros(max(n, 256), dtype=torch.uint8, device=dev)


SHAPES = {
    "tiny": synth.TINY,
    "small": synth.LayerShape(M=96, H=512, I=256, E=16, topk=4),
    "glm64": synth.glm(64),
    "glm1": synth.glm(1),
    "e512": synth.LayerShape(M=40, H=256, I=128, E=512, topk=8, scoring="sigmoid"),
    "e1024": synth.LayerShape(M=128, H=256, I=128, E=1024, topk=8),
    "tile64": synth.LayerShape(M=120, H=512, I=256, E=6, topk=2),  # 40 rows per expert: 64-token tiles
    "fanout": synth.LayerShape(M=128, H=512, I=256, E=64, topk=16),  # 2,048 slots: one gather warp per token
}


@pytest.mark.parametrize("name", list(SHAPES))
def test_whole_launch_equals_separate_launches(cuda_device, name):
    shape = SHAPES[name]
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=41, device=cuda_device)
    M = shape.M
    lib = _lib.lib()
    with launch_mode(WHOLE):
        assert lib.b200moe_layer_launches(M, shape.H, shape.I, shape.E, 0, shape.topk) == 1
    ws_a, ws_b = _workspace(shape, M, cuda_device), _workspace(shape, M, cuda_device)
    with launch_mode(SEPARATE):
        ref = _layer(L, L.hidden, L.topk_weights, L.topk_ids, ws_b, torch.empty_like(L.hidden))
    with launch_mode(WHOLE):
        for _ in range(3):  # the launch's sync words are left at zero for the next call
            out = _layer(L, L.hidden, L.topk_weights, L.topk_ids, ws_a, torch.empty_like(L.hidden))
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
            assert ws_a[:16].view(torch.int32).tolist() == [0, 0, 0, 0]


def test_whole_launch_matches_oracle(cuda_device):
    L = synth.make_layer(synth.TINY, orc.per_block_quant_fp8, seed=3)
    dev = cuda_device
    ref = orc.moe_layer(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights, L.topk_ids)
    Ld = synth.make_layer(synth.TINY, orc.per_block_quant_fp8, seed=3)
    for f in ("hidden", "w13", "w13_scale", "w2", "w2_scale", "topk_weights", "topk_ids"):
        setattr(Ld, f, getattr(L, f).to(dev))
    with launch_mode(WHOLE):
        out = _layer(Ld, Ld.hidden, Ld.topk_weights, Ld.topk_ids, _workspace(L.shape, L.shape.M, dev),
                     torch.empty_like(Ld.hidden))
    assert orc.rel_l2(out.cpu(), ref) < 5e-3


def test_whole_launch_with_expert_map_and_dropped_ids(cuda_device):
    """An expert-parallel rank's view: 16 of 64 experts local (expert_map),
    ids -1 for dropped slots and one id out of range (reported, dropped)."""
    shape = synth.LayerShape(M=50, H=512, I=256, E=64, topk=4)
    full = synth.make_layer(shape, moe.per_block_quant_fp8, seed=9, device=cuda_device)
    local = torch.arange(3, 64, 4)
    emap = torch.full((64,), -1, dtype=torch.int32)
    emap[local] = torch.arange(len(local), dtype=torch.int32)
    emap = emap.to(cuda_device)
    sel = local.to(cuda_device)
    L = types.SimpleNamespace(shape=shape, w13=full.w13[sel].contiguous(), w13_scale=full.w13_scale[sel].contiguous(),
                              w2=full.w2[sel].contiguous(), w2_scale=full.w2_scale[sel].contiguous())
    ids = full.topk_ids.clone()
    ids[::7, 0] = -1
    ids[5, 1] = 64  # out of range
    outs, errs = [], []
    for mode in (SEPARATE, WHOLE):
        ws = _workspace(shape, shape.M, cuda_device, num_local=len(local))
        with launch_mode(mode):
            outs.append(_layer(L, full.hidden, full.topk_weights, ids, ws, torch.empty_like(full.hidden), emap,
                               len(local), num_experts=64))
        errs.append(moe.read_device_error(ws[:4].view(torch.int32)))
    assert torch.equal(outs[0], outs[1])
    assert errs[0] == errs[1] != 0


def test_whole_launch_from_logits(cuda_device):
    """b200moe_layer_logits in one launch (the router runs first inside it)
    equals the router + separate launches: ids, weights and output."""
    shape = synth.glm(64)
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=5, device=cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(12)
    bias = torch.randn(shape.E, generator=g, device=cuda_device) * 0.05
    res = {}
    for mode in (SEPARATE, WHOLE):
        with launch_mode(mode):
            for M in (shape.M, 7, shape.M):
                logits = torch.randn(M, shape.E, generator=torch.Generator(device=cuda_device).manual_seed(M),
                                     device=cuda_device)
                h = L.hidden[:M]
                res[(mode, M)] = moe.moe_layer_from_logits(h, logits, L.w13, L.w13_scale, L.w2, L.w2_scale,
                                                           shape.topk, "sigmoid", bias, routed_scaling_factor=2.5)
    for M in (shape.M, 7):
        for a, b in zip(res[(SEPARATE, M)], res[(WHOLE, M)]):
            assert torch.equal(a, b)
    assert moe.read_device_error(moe.layer_error_word(cuda_device)) == 0


def test_whole_launch_with_fp8_input(cuda_device):
    shape = synth.LayerShape(M=64, H=512, I=256, E=32, topk=4)
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=17, device=cuda_device)
    xq, xs = moe.per_token_group_quant_fp8(L.hidden)
    outs = []
    for mode in (SEPARATE, WHOLE):
        with launch_mode(mode):
            outs.append(moe.moe_decode_megakernel_full(xq, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights,
                                                       L.topk_ids, a1_scale=xs))
    assert torch.equal(outs[0], outs[1])


def _kernel_nodes(graph) -> int:
    """Kernel nodes of a captured torch CUDA graph (driver API)."""
    cu = ctypes.CDLL("libcuda.so.1")
    h = ctypes.c_void_p(int(graph.raw_cuda_graph()))
    n = ctypes.c_size_t(0)
    assert cu.cuGraphGetNodes(h, None, ctypes.byref(n)) == 0
    nodes = (ctypes.c_void_p * n.value)()
    assert cu.cuGraphGetNodes(h, nodes, ctypes.byref(n)) == 0
    kinds = []
    for i in range(n.value):
        t = ctypes.c_int(-1)
        assert cu.cuGraphNodeGetType(ctypes.c_void_p(nodes[i]), ctypes.byref(t)) == 0
        kinds.append(t.value)
    return sum(1 for k in kinds if k == 0)  # CU_GRAPH_NODE_TYPE_KERNEL


@pytest.mark.parametrize("mode,launches", [(WHOLE, 1), (SEPARATE, 4)])
def test_whole_launch_is_one_kernel_in_a_cuda_graph(cuda_device, mode, launches):
    """Captured and replayed on new inputs: one kernel node for the whole
    layer (four for the separate launches), same results as eager calls."""
    shape = synth.glm(64)
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=0, device=cuda_device)
    g2 = torch.Generator(device=cuda_device).manual_seed(1)
    o_tw, o_ids = synth.make_router(torch.randn(shape.M, shape.E, generator=g2, device=cuda_device), shape.topk,
                                    shape.scoring)
    other = types.SimpleNamespace(hidden=torch.randn(shape.M, shape.H, generator=g2, device=cuda_device).to(
        torch.bfloat16), topk_weights=o_tw.float().contiguous(), topk_ids=o_ids.to(torch.int32).contiguous())
    lib = _lib.lib()
    with launch_mode(mode):
        assert lib.b200moe_layer_launches(shape.M, shape.H, shape.I, shape.E, 0, shape.topk) == launches
        h, tw, ids = L.hidden.clone(), L.topk_weights.clone(), L.topk_ids.clone()
        ws = _workspace(shape, shape.M, cuda_device)
        out = torch.empty_like(h)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            _layer(L, h, tw, ids, ws, out)  # warm-up on the capture stream
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph(keep_graph=True)  # the graph stays queryable until instantiate()
        with torch.cuda.graph(g):
            _layer(L, h, tw, ids, ws, out)
        assert _kernel_nodes(g) == launches
        g.instantiate()
        ws_e = _workspace(shape, shape.M, cuda_device)
        for src in (other, L, other):
            h.copy_(src.hidden)
            tw.copy_(src.topk_weights)
            ids.copy_(src.topk_ids)
            g.replay()
            eager = _layer(L, src.hidden, src.topk_weights, src.topk_ids, ws_e, torch.empty_like(h))
            torch.cuda.synchronize()
            assert torch.equal(out, eager)
        del g
