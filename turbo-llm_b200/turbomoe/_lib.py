"""ctypes binding of libturbomoe.so (declarations mirror include/turbomoe.h).

The shared library is built in-tree by ``turbomoe/build.py``.  Loading it
never needs a GPU; calling a compute entry point does.  There is no fallback:
if the library is missing, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libturbomoe.so")

TM_OK = 0
TM_ERR_INVALID = -1
TM_ERR_CUDA = -2
TM_ERR_WORKSPACE = -3
TM_ERR_UNSUPPORTED = -4
TM_DTYPE_F32, TM_DTYPE_F16, TM_DTYPE_BF16 = 0, 1, 2
TM_STATUS_BAD_EXPERT_ID = 1

_p = C.c_void_p
_i = C.c_int
_i64 = C.c_int64

# name -> (restype, argtypes); the exact list of symbols include/turbomoe.h declares
SIGNATURES = {
    "tm_abi_version": (_i, []),
    "tm_last_error": (C.c_char_p, []),
    "tm_dequant_fp8_block": (_i, [_p, _p, _i64, _i64, _p, _i, _p]),
    "tm_packed_w13_bytes": (_i64, [_i, _i]),
    "tm_packed_s13_floats": (_i64, [_i, _i]),
    "tm_packed_w2_bytes": (_i64, [_i, _i]),
    "tm_packed_s2_floats": (_i64, [_i, _i]),
    "tm_pack_experts": (_i, [_p, _p, _p, _p, _p, _p, _i, _i, _i, _p, _p, _p, _p, _p]),
    "tm_unpack_expert": (_i, [_p, _p, _p, _p, _i, _i, _p, _p, _p, _i, _p]),
    "tm_workspace_bytes": (_i64, [_i64, _i, _i, _i, _i, _i]),
    "tm_workspace_init": (_i, [_p, _i64, _p]),
    "tm_workspace_status": (_i, [_p, _i64, C.POINTER(C.c_uint32), _p]),
    "tm_plan_offsets": (_i, [_i64, _i, _i, C.POINTER(C.c_int64)]),
    "tm_router_topk": (_i, [_p, _i64, _i, _i, _p, _i, _i, _p, _p, _p, _p, _i64, _p]),
    "tm_rmsnorm_router_topk": (_i, [_p, _i, _i, _p, C.c_float, _p, _p, _i, _i, _p, _p, _p, _p, _i64, _p]),
    "tm_rmsnorm_fp8_linear": (_i, [_p, _i, _i, _p, C.c_float, _i, _p, _p, _p, _p, _p, _p]),
    "tm_route_plan": (_i, [_p, _i64, _i, _i, _p, _i64, _p]),
    "tm_moe_decode_gateup": (_i, [_p, _i64, _i, _i, _i, _i, _i, _p, _p, _p, _p, _i, _p, _p, _i64, _p]),
    "tm_moe_decode_gateup_prefetch": (_i, [_p, _i64, _i, _i, _i, _i, _i, _p, _p, _p, _p, _i, _p, _p, _p, _p,
                                           _i64, _p]),
    "tm_moe_decode_down_combine": (_i, [_i64, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _i, _p, _p, _p,
                                        _i64, _p]),
    "tm_prefetch_experts_l2": (_i, [_p, _i64, _i, _p, _i, _p]),
    "tm_moe_prefill_grouped": (_i, [_p, _i64, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _p,
                                    _p, _p, _p, _i64, _p]),
    "tm_moe_grouped_f8": (_i, [_p, _i64, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _p,
                               _p, _p, _p, _i64, _p]),
    "tm_combine_slots": (_i, [_p, _p, _p, _i64, _i, _i, _i, _p, _p, _p]),
    "tm_moe_decode_layer_noalloc": (_i, [_p, _i64, _i, _i, _i, _i, _i, _p, _p, _p, _p, _p, _p, _p, _p, _p,
                                         _i, _p, _p, _p, _p, _p, _p, _p]),
    "tm_pack_linear": (_i, [_p, _i, _i, _p, _p]),
    "tm_fp8_linear": (_i, [_p, _i64, _i, _i, _i, _p, _p, _p, _p, _p, _p]),
    "tm_embed": (_i, [_p, _i64, _p, _i, _i64, _i, _p, _p, _p]),
    "tm_rmsnorm": (_i, [_p, _i64, _i, _i, _p, C.c_float, _p, _p]),
    "tm_qk_rope_kv": (_i, [_p, _i64, _i, _i, _i, _i, _p, _p, C.c_float, _p, _p, _i64, _p, _p, _p, _p, _p]),
    "tm_attn_decode_workspace_bytes": (_i64, [_i, _i, _i]),
    "tm_attn_decode": (_i, [_p, _p, _p, _p, _i64, _i, _i, _i, _i, C.c_float, _i, _p, _p, _i64, _p]),
    "tm_attn_decode_batched": (_i, [_p, _p, _p, _p, _i, _i64, _i64, _i, _i, _i, _i, C.c_float, _i, _p, _p]),
    "tm_qk_rope_attn_decode": (_i, [_p, _p, _p, C.c_float, _p, _p, _i64, _i, _i, _i, _i, C.c_float, _i, _p, _p, _p,
                                    _p]),
    "tm_lm_head_workspace_bytes": (_i64, []),
    "tm_lm_head_argmax": (_i, [_p, _i, _i, _p, _i64, _p, _p, _p, _i64, _p]),
    "tm_gdn_decode": (_i, [_p, _p, _p, _p, _i64, _i, _i, _i, _i, _i, _i, _p, _p, _p, _p, C.c_float, _p, _p,
                          _p, _p, _p]),
    "tm_ep_buffer_bytes": (_i64, [_i, _i64, _i, _i, _i, _i]),
    "tm_ep_create": (_i, [_i, _i, _i, _i, _i, _i, _i, _i64, _p, C.POINTER(_p)]),
    "tm_ep_connect": (_i, [_p, _p]),
    "tm_ep_connect_ptrs": (_i, [_p, C.POINTER(_p)]),
    "tm_ep_local_buffer": (_p, [_p]),
    "tm_ep_set_timeout": (_i, [_p, _i64]),
    "tm_ep_disconnect": (_i, [_p]),
    "tm_ep_destroy": (_i, [_p]),
    "tm_ep_owner_workspace_bytes": (_i64, [_p]),
    "tm_ep_status": (_i, [_p, C.POINTER(C.c_uint32), _p]),
    "tm_ep_dispatch": (_i, [_p, _p, _i64, _p, _p, _i64, _p]),
    "tm_ep_experts": (_i, [_p, _p, _p, _p, _p, _p, _i64, _p]),
    "tm_ep_combine": (_i, [_p, _p, _i64, _p, _i64, _p, _p, _p]),
}
TM_NOALLOC_SCRATCH_BYTES = 8 << 20
TM_EP_MAX_RANKS = 8
TM_EP_HANDLE_BYTES = 64
TM_STATUS_TIMEOUT = 2
TM_STATUS_PEER_FAILED = 4
TM_STATUS_BAD_TOKEN_ID = 8

_lock = threading.Lock()
_lib = None


class TurboMoEError(RuntimeError):
    pass


def lib():
    """The loaded library (raises if libturbomoe.so has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise TurboMoEError(
                    f"{LIB_PATH} is missing: build it with `python turbo-llm_b200/turbomoe/build.py` "
                    "(the MoE path has no CPU fallback)")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            if L.tm_abi_version() != 1:
                raise TurboMoEError("libturbomoe ABI version mismatch")
            _lib = L
    return _lib


def check(rc: int, what: str):
    if rc != TM_OK:
        msg = lib().tm_last_error()
        raise TurboMoEError(f"{what} failed ({rc}): {msg.decode() if msg else ''}")
