"""The C-ABI library: loads, exports every symbol include/b200moe.h declares,
and rejects bad arguments on the host (no GPU needed: these calls return
before anything is launched)."""
import re
from pathlib import Path

import pytest
import torch

from trials_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "b200moe.h"


def header_functions():
    text = HEADER.read_text()
    return re.findall(r"B200MOE_API\s+[\w\s\*]+?\b(b200moe_\w+)\s*\(", text)


def test_library_loads_and_exports_header_symbols():
    L = _lib.lib()
    names = header_functions()
    assert len(names) >= 19
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"


def test_version_and_status_strings():
    L = _lib.lib()
    assert L.b200moe_version() >= 100
    assert L.b200moe_status_string(0) == b"ok"
    assert L.b200moe_status_string(_lib.ERR_UNSUPPORTED) == b"unsupported shape or option"


def test_capacity_formulas():
    L = _lib.lib()
    # sglang sizing: numel + (E + 1) * (BM - 1); GLM decode M=64, k=8, E=256, BM=128 -> 259 blocks
    assert L.b200moe_align_capacity_rows(512, 256, 128) == 512 + 257 * 127
    assert L.b200moe_align_capacity_blocks(512, 256, 128) == 259
    assert L.b200moe_route_capacity_rows(512, 256) == 512 + 256 * 15
    rows = 512 + 256 * 15
    assert L.b200moe_route_capacity_chunks(512, 256, 32) == -(-rows // 32) + 256


def test_host_side_argument_checks():
    L = _lib.lib()
    # unsupported hidden size (not a multiple of 256)
    assert L.b200moe_layer(1, 4, 100, 128, 8, 2, 1, 1, 1, 1, 1, 1, None, 8, 1, 1, 1 << 30, None) == \
        _lib.ERR_UNSUPPORTED
    # K not a multiple of 128
    assert L.b200moe_quant_1x128(16, 4, 100, 100, 16, 100, 16, 1, 1, None) == _lib.ERR_INVALID_ARG
    # tile size outside {16, 32, 64, 128}
    assert L.b200moe_route(16, 4, 2, 8, None, 8, 48, 16, 1000, 16, 16, 16, 1000, 16, 16, None, None, None, 0, 16,
                           None) == \
        _lib.ERR_INVALID_ARG
    # too many experts
    assert L.b200moe_align(16, 4, 2, 2000, 128, None, 0, 16, 1 << 20, 16, 1 << 20, 16, 16, None) == \
        _lib.ERR_UNSUPPORTED
    # output capacity below the sglang sizing
    assert L.b200moe_align(16, 4, 2, 8, 128, None, 0, 16, 10, 16, 10, 16, 16, None) == _lib.ERR_WORKSPACE
    # workspace too small
    ws = L.b200moe_layer_workspace_size(4, 256, 128, 8, 8, 2)
    assert ws > 0
    assert L.b200moe_layer(256, 4, 256, 128, 8, 2, 256, 256, 256, 256, 256, 256, None, 8, 256, 256, ws - 1,
                           None) == _lib.ERR_WORKSPACE
    assert b"workspace" in L.b200moe_last_error_message()


def test_peer_exchange_host_checks():
    L = _lib.lib()
    H, topk, cap, G = 512, 4, 40, 4
    rb = L.b200moe_ep_row_bytes(H, topk)
    area_recv = -(-G * cap * rb // 256) * 256
    area_ret = -(-G * cap * H * 2 // 256) * 256
    assert L.b200moe_ep_peer_bytes(cap, H, topk, G) == 1024 + 2 * (area_recv + area_ret)
    assert L.b200moe_ep_peer_bytes(cap, H, topk, 65) == 0     # at most 64 ranks
    assert L.b200moe_ep_peer_bytes(cap, 100, topk, G) == 0    # H not a multiple of 128
    # epoch 0, a rank outside the group, an unaligned own buffer: refused before any launch
    args = [None, 16, 16, 16, 16, 8, H, topk, 16, G]
    ident = [None, 0, 0]
    assert L.b200moe_ep_dispatch_peer(*args, 0, *ident, cap, 256, 256, 0, 16, 16, 16, 16, None) == \
        _lib.ERR_INVALID_ARG
    assert L.b200moe_ep_dispatch_peer(*args, G, *ident, cap, 256, 256, 1, 16, 16, 16, 16, None) == \
        _lib.ERR_INVALID_ARG
    assert L.b200moe_ep_dispatch_peer(*args, 0, *ident, cap, 256, 260, 1, 16, 16, 16, 16, None) == \
        _lib.ERR_INVALID_ARG
    # replica tables: slots * G must cover the experts, 1 <= max_replicas <= G
    assert L.b200moe_ep_dispatch_peer(*args, 0, 16, 2, 3, cap, 256, 256, 1, 16, 16, 16, 16, None) == \
        _lib.ERR_INVALID_ARG
    assert L.b200moe_ep_dispatch_peer(*args, 0, 16, G + 1, 8, cap, 256, 256, 1, 16, 16, 16, 16, None) == \
        _lib.ERR_INVALID_ARG
    # without a table the experts must split evenly over the ranks
    assert L.b200moe_ep_dispatch(16, 16, 16, 16, 8, H, topk, 18, G, 0, None, 0, 0, cap, 16, 16, 16, 16, 16, None) \
        == _lib.ERR_INVALID_ARG
    assert L.b200moe_layer_packed_peer(256, 256, G, 0, cap, 0, H, 256, 4, topk, 16, 16, 16, 16, 256, 1 << 30,
                                       None) == _lib.ERR_INVALID_ARG
    assert L.b200moe_ep_combine_peer(256, 16, 8, H, topk, G, cap, 0, 16, 16, None) == _lib.ERR_INVALID_ARG
    assert L.b200moe_ep_peer_alloc(16, None, None) == _lib.ERR_INVALID_ARG


def test_python_errors_map_to_exceptions():
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED, "x")
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID_ARG, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA, "x")


def test_fused_moe_rejects_unsupported_options_before_launch():
    from trials_b200 import fused_moe, QuantType

    h = torch.zeros(2, 256, dtype=torch.bfloat16)
    w = torch.zeros(1)
    for kw in [dict(quant_type=QuantType.per_Token), dict(activation="Gelu"), dict(bias1=w),
               dict(no_combine=True), dict(gate_mode="separated"), dict(a2_scale=w), dict(swiglu_limit=7.0),
               dict(doweight_stage1=True)]:
        with pytest.raises(NotImplementedError):
            fused_moe(h, w, w, w, w, **kw)


def test_ops_refuse_cpu_tensors():
    from trials_b200 import moe_decode_megakernel_full

    h = torch.zeros(2, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        moe_decode_megakernel_full(h, h, h, h, h, h, h)


def test_packed_workspace_covers_every_tile():
    """The packed layers pick their tile from the slots expected per rank, so
    their workspace query covers the largest plan over the tile sizes: never
    less than the plain layer's workspace for the same rows, plus the unpacked
    ids and weights."""
    L = _lib.lib()
    H, I, topk = 6144, 2048, 8
    for R, E in ((64, 256), (512, 32), (4096, 128), (8192, 256)):
        packed = L.b200moe_layer_packed_workspace_size(R, H, I, E, topk)
        plain = L.b200moe_layer_workspace_size(R, H, I, E, E, topk)
        assert packed >= plain + R * topk * 8, (R, E)


def test_noalloc_layer_host_checks():
    """The no-allocation layer tells an invalid shape apart from a layer too
    large for its static scratch (both refused before any launch)."""
    L = _lib.lib()
    p = 256
    # H = 0: an invalid shape, not a size limit
    assert L.b200moe_layer_noalloc(p, 4, 0, 128, 8, 2, p, p, p, p, p, p, None, 8, p, None, None) == \
        _lib.ERR_INVALID_ARG
    assert b"bad argument" in L.b200moe_last_error_message()
    assert L.b200moe_layer_noalloc(p, -1, 256, 128, 8, 2, p, p, p, p, p, p, None, 8, p, None, None) == \
        _lib.ERR_INVALID_ARG
    # GLM-5-like layer at 1,024 tokens: far above the 64 MiB scratch
    assert L.b200moe_layer_noalloc(p, 1024, 6144, 2048, 256, 8, p, p, p, p, p, p, None, 256, p, None, None) == \
        _lib.ERR_WORKSPACE
    assert b"64 MiB" in L.b200moe_last_error_message()


def test_peer_wait_limit_setting():
    L = _lib.lib()
    default = L.b200moe_ep_peer_wait_limit_us(0)  # query only
    assert default == 10_000_000
    assert L.b200moe_ep_peer_wait_limit_us(20_000) == default
    assert L.b200moe_ep_peer_wait_limit_us(-5) == 20_000          # query: unchanged
    assert L.b200moe_ep_peer_wait_limit_us(10**12) == 20_000      # clamped to 60 s
    assert L.b200moe_ep_peer_wait_limit_us(default) == 60_000_000
    assert L.b200moe_ep_peer_wait_limit_us(0) == default


def test_layer_launch_policy():
    """The whole layer in one launch where it applies (tiles of 16..64, one-CTA
    routing, no mixed lists) under policy 1; separate launches under the
    default policy (measured faster) and policy 2."""
    L = _lib.lib()
    H, I, E, k = 6144, 2048, 256, 8
    prev = L.b200moe_set_layer_launch(0)
    try:
        assert L.b200moe_layer_launches(64, H, I, E, 0, k) == 4
        assert L.b200moe_layer_launches(1, H, I, E, 0, k) == 4
        assert L.b200moe_layer_launches(128, H, I, E, 0, k) == 4
        # above 128 tokens: mixed work lists (route, gather, experts, 2 heavy stages, reduce)
        assert L.b200moe_layer_launches(256, H, I, E, 0, k) == 6
        # prefill: two routing launches, gather, two token-major stages, reduce
        assert L.b200moe_layer_launches(8192, H, I, E, 0, k) == 6
        assert L.b200moe_layer_launches(0, H, I, E, 0, k) == 0
        assert L.b200moe_set_layer_launch(2) == 0
        assert L.b200moe_layer_launches(64, H, I, E, 0, k) == 4
        assert L.b200moe_set_layer_launch(1) == 2
        assert L.b200moe_layer_launches(64, H, I, E, 0, k) == 1
        assert L.b200moe_layer_launches(1, H, I, E, 0, k) == 1
        assert L.b200moe_layer_launches(128, H, I, E, 0, k) == 1
        assert L.b200moe_layer_launches(256, H, I, E, 0, k) == 6  # mixed lists: not applicable
        assert L.b200moe_layer_launches(8192, H, I, E, 0, k) == 6  # not applicable: token-major tiles
        assert L.b200moe_set_layer_launch(3) < 0
        assert L.b200moe_set_layer_launch(-1) < 0
    finally:
        L.b200moe_set_layer_launch(prev)
