"""The layer on other models' geometries than GLM's: hidden sizes whose K
blocks, 1,024-column segments and 256-row units differ (DeepSeek-V3 7168,
Qwen3 4096 / 2048, and 2816 = 11 x 256 with I = 1408 for odd unit counts),
against the oracle (float64, evaluated on the GPU to keep the test short),
and the staged pipeline and the one-launch form against the layer bit for
bit. One token-major (prefill-sized) case at H = 7168."""
import contextlib

import pytest
import torch

from oracle import moe_oracle as orc
from trials_b200 import _lib, moe, stages, synth

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(900)]

SHAPES = {
    "deepseek_v3": synth.LayerShape(M=24, H=7168, I=2048, E=16, topk=4, scoring="sigmoid"),
    "qwen3_235b": synth.LayerShape(M=24, H=4096, I=1536, E=16, topk=4),
    "qwen3_30b": synth.LayerShape(M=24, H=2048, I=768, E=16, topk=4),
    "odd_units": synth.LayerShape(M=24, H=2816, I=1408, E=16, topk=4),
}
TOL = 5e-3


@contextlib.contextmanager
def launch_mode(mode):
    lib = _lib.lib()
    prev = lib.b200moe_set_layer_launch(mode)
    try:
        yield
    finally:
        lib.b200moe_set_layer_launch(prev)


def _check(shape, cuda_device, seed):
    L = synth.make_layer(shape, moe.per_block_quant_fp8, seed=seed, device=cuda_device)
    w = (L.w13, L.w13_scale, L.w2, L.w2_scale)
    out = moe.moe_decode_megakernel_full(L.hidden, *w, L.topk_weights, L.topk_ids)
    ref = orc.moe_layer(L.hidden, *w, L.topk_weights, L.topk_ids)
    err = orc.rel_l2(out.float(), ref.float())
    assert err < TOL, err
    pipe = stages.LayerPipeline(shape.M, shape.H, shape.I, shape.E, shape.topk, cuda_device, whole=False)
    staged = pipe.run(L.hidden, L.topk_ids, L.topk_weights, *w)
    torch.cuda.synchronize()
    assert torch.equal(staged, out)
    assert moe.read_device_error(pipe.err) == 0
    return L, out


@pytest.mark.parametrize("name", list(SHAPES))
def test_layer_on_model_geometries(cuda_device, name):
    shape = SHAPES[name]
    L, out = _check(shape, cuda_device, seed=len(name))
    with launch_mode(1):  # the whole layer in one launch: same bits
        one = moe.moe_decode_megakernel_full(L.hidden, L.w13, L.w13_scale, L.w2, L.w2_scale, L.topk_weights,
                                             L.topk_ids)
    assert torch.equal(one, out)
    assert moe.read_device_error(moe.layer_error_word(cuda_device)) == 0


def test_token_major_tiles_at_deepseek_width(cuda_device):
    """640 tokens, top-2 over 8 experts: 160 rows per expert, 128-row
    token-major tiles with 56 K blocks in stage 1 and 28 units per chunk in
    stage 2."""
    shape = synth.LayerShape(M=640, H=7168, I=2048, E=8, topk=2)
    assert stages.pick_tile_tokens(shape.M * shape.topk, shape.E) == 128
    _check(shape, cuda_device, seed=3)
