"""ctypes binding of libb200moe.so (the C ABI declared in include/b200moe.h).

The library is required: there is no fallback implementation. Importing the
package works without it, but the first call into an op raises if the .so is
missing (build it with `python -m trials_b200.build`).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libb200moe.so"

OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED = -2
ERR_WORKSPACE = -3
ERR_CUDA = -4

DEVERR_BAD_EXPERT_ID = 1
DEVERR_TIMEOUT = 2
DEVERR_CAPACITY = 4

IPC_HANDLE_BYTES = 64

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_S = ctypes.c_size_t

# name -> (restype, argtypes); kept in the order of include/b200moe.h
SIGNATURES = {
    "b200moe_version": (_I, []),
    "b200moe_status_string": (ctypes.c_char_p, [_I]),
    "b200moe_last_error_message": (ctypes.c_char_p, []),
    "b200moe_align_capacity_rows": (_L, [_L, _I, _I]),
    "b200moe_align_capacity_blocks": (_L, [_L, _I, _I]),
    "b200moe_align": (_I, [_P, _L, _I, _I, _I, _P, _I, _P, _L, _P, _L, _P, _P, _P]),
    "b200moe_router_topk": (_I, [_P, _I, _L, _I, _I, _I, _P, _I, ctypes.c_float, _P, _P, _P]),
    "b200moe_quant_1x128": (_I, [_P, _L, _L, _L, _P, _L, _P, _L, _L, _P]),
    "b200moe_quant_block128": (_I, [_P, _L, _L, _L, _P, _P, _P]),
    "b200moe_layer_workspace_size": (_S, [_L, _L, _L, _I, _I, _I]),
    "b200moe_set_layer_launch": (_I, [_I]),
    "b200moe_layer_launches": (_I, [_L, _L, _L, _I, _I, _I]),
    "b200moe_layer": (_I, [_P, _L, _L, _L, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _S, _P]),
    "b200moe_layer_logits": (_I, [_P, _L, _L, _L, _I, _I, _P, _I, _I, _P, _I, ctypes.c_float, _P, _P, _P, _P, _P, _I,
                                  _P, _P, _P, _P, _S, _P]),
    "b200moe_layer_quantized": (_I, [_P, _P, _L, _L, _L, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _S, _P]),
    "b200moe_ep_row_bytes": (_L, [_L, _I]),
    "b200moe_ep_dispatch": (_I, [_P, _P, _P, _P, _L, _L, _I, _I, _I, _I, _P, _I, _I, _L, _P, _P, _P, _P, _P, _P]),
    "b200moe_layer_packed_workspace_size": (_S, [_L, _L, _L, _I, _I]),
    "b200moe_layer_packed": (_I, [_P, _L, _I, _L, _L, _L, _I, _I, _P, _P, _P, _P, _P, _P, _S, _P]),
    "b200moe_ep_combine": (_I, [_P, _P, _L, _L, _I, _L, _P, _P]),
    "b200moe_ep_peer_bytes": (_S, [_L, _L, _I, _I]),
    "b200moe_ep_peer_alloc": (_I, [_S, ctypes.POINTER(_P), _P]),
    "b200moe_ep_peer_open": (_I, [_P, ctypes.POINTER(_P)]),
    "b200moe_ep_peer_close": (_I, [_P]),
    "b200moe_ep_peer_free": (_I, [_P]),
    "b200moe_ep_dispatch_peer": (_I, [_P, _P, _P, _P, _P, _L, _L, _I, _I, _I, _I, _P, _I, _I, _L, _P, _P,
                                      ctypes.c_int32, _P, _P, _P, _P, _P]),
    "b200moe_layer_packed_peer": (_I, [_P, _P, _I, _I, _L, ctypes.c_int32, _L, _L, _I, _I, _P, _P, _P, _P, _P, _S,
                                       _P]),
    "b200moe_ep_combine_peer": (_I, [_P, _P, _L, _L, _I, _I, _L, ctypes.c_int32, _P, _P, _P]),
    "b200moe_ep_peer_wait_limit_us": (_L, [_L]),
    "b200moe_layer_noalloc": (_I, [_P, _L, _L, _L, _I, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P, _P, _P]),
    "b200moe_route_capacity_rows": (_L, [_L, _I]),
    "b200moe_route_capacity_chunks": (_L, [_L, _I, _I]),
    "b200moe_route_scratch_ints": (_L, [_L, _I]),
    "b200moe_route": (_I, [_P, _L, _I, _I, _P, _I, _I, _P, _L, _P, _P, _P, _L, _P, _P, _P, _P, _P, _L, _P, _P]),
    "b200moe_heavy_rows": (_I, [_L, _I, _I]),
    "b200moe_route_mixed": (_I, [_P, _L, _I, _I, _P, _I, _I, _I, _P, _L, _P, _P, _P, _L, _P, _P, _P, _L, _P, _P, _P,
                                 _P, _P, _P]),
    "b200moe_route_logits_scratch_ints": (_L, [_L, _I]),
    "b200moe_route_logits": (_I, [_P, _I, _L, _I, _I, _I, _P, _I, ctypes.c_float, _P, _P, _P, _I, _I, _P, _L, _P, _P,
                                  _P, _L, _P, _P, _P, _P, _P, _L, _P, _P]),
    "b200moe_gather_quant": (_I, [_P, _L, _L, _I, _P, _L, _P, _P, _L, _P]),
    "b200moe_gather_rows": (_I, [_P, _P, _L, _L, _L, _L, _I, _P, _L, _P, _P, _L, _P]),
    "b200moe_gemm1_silu": (_I, [_P, _P, _L, _L, _P, _P, _I, _L, _L, _P, _P, _P, _P, _L, _I, _P, _P, _P, _I, _P]),
    "b200moe_gemm2_combine": (_I, [_P, _P, _L, _L, _P, _P, _I, _L, _L, _P, _P, _P, _P, _L, _I, _P, _P, _L, _I,
                                   _P, _P, _I, _P]),
    "b200moe_experts": (_I, [_P, _P, _L, _L, _P, _P, _P, _P, _I, _L, _L, _P, _P, _P, _P, _L, _P, _I, _P, _P, _P, _P,
                             _L, _I, _P, _P, _I, _P]),
    "b200moe_experts_heavy": (_I, [_P, _P, _L, _L, _P, _P, _P, _P, _I, _L, _L, _P, _P, _P, _P, _L, _P, _P, _P, _P,
                                   _P, _L, _I, _P, _P, _I, _P]),
    "b200moe_experts_fused": (_I, [_P, _L, _I, _P, _P, _P, _L, _L, _P, _P, _P, _P, _I, _L, _L, _P, _P, _P, _P, _L,
                                   _P, _I, _P, _P, _P, _P, _P, _P, _P, _I, _P]),
    "b200moe_combine_reduce": (_I, [_P, _P, _I, _L, _I, _L, _P, _P]),
    "b200moe_read_error": (_I, [_P, _P, _I, _P]),
    "b200moe_selftest_wait_timeout": (_I, [_P, _I, _P]),
}

_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """Loads libb200moe.so once; raises RuntimeError if it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not LIB_PATH.exists():
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build the CUDA library with `python -m trials_b200.build`")
                L = ctypes.CDLL(str(LIB_PATH))
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


class B200MoeError(RuntimeError):
    def __init__(self, status: int, where: str):
        msg = lib().b200moe_last_error_message().decode(errors="replace")
        super().__init__(f"{where}: status {status} ({lib().b200moe_status_string(status).decode()}): {msg}")
        self.status = status


def check(status: int, where: str) -> None:
    """Raises the Python exception matching a C status code."""
    if status == OK:
        return
    err = B200MoeError(status, where)
    if status == ERR_INVALID_ARG:
        raise ValueError(str(err))
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(str(err))
    raise err
