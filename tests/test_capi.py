"""The C-ABI library loads and exports every symbol include/turbomoe.h declares.

CPU only: nothing here launches a kernel.  Argument validation happens on
the host before any launch, so the error paths are testable without a GPU.
"""
import ctypes
import os
import re

import pytest

from turbomoe import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    txt = open(os.path.join(REPO, "include", "turbomoe.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(tm_[a-z0-9_]+)\s*\(", txt)))


def test_library_built_and_loads():
    assert os.path.exists(_lib.LIB_PATH), "run __graft_entry__.build() first"
    L = _lib.lib()
    assert L.tm_abi_version() == 1


def test_every_declared_symbol_exported_and_bound():
    L = ctypes.CDLL(_lib.LIB_PATH)
    syms = header_symbols()
    assert len(syms) >= 16
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/turbomoe.h but not exported"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature in turbomoe/_lib.py"
    assert set(_lib.SIGNATURES) == set(syms)


def test_packed_sizes():
    L = _lib.lib()
    H, I = 2048, 768
    assert L.tm_packed_w13_bytes(H, I) == 2 * H * I
    assert L.tm_packed_w2_bytes(H, I) == H * I
    assert L.tm_packed_s13_floats(H, I) == 2 * 6 * 16
    assert L.tm_packed_s2_floats(H, I) == 16 * 6


def test_workspace_bytes_monotone_and_header_fixed():
    L = _lib.lib()
    a = L.tm_workspace_bytes(1, 128, 8, 2048, 768, 0)
    b = L.tm_workspace_bytes(64, 128, 8, 2048, 768, 0)
    c = L.tm_workspace_bytes(64, 256, 8, 2048, 512, 512)
    assert 0 < a < b and c > 0
    assert L.tm_workspace_bytes(0, 128, 8, 2048, 768, 0) == -1
    # the plan regions sit at the same offsets whatever the expert sizes are
    o1 = (ctypes.c_int64 * 8)()
    assert L.tm_plan_offsets(64, 128, 8, o1) == 0
    assert list(o1)[1] > list(o1)[0]


def test_argument_errors_reported_without_launch():
    L = _lib.lib()
    # rows not a multiple of 128 -> TM_ERR_INVALID before any CUDA call
    rc = L.tm_dequant_fp8_block(16, 16, 100, 128, 16, 0, None)
    assert rc == _lib.TM_ERR_INVALID
    assert b"multiples of 128" in L.tm_last_error()
    rc = L.tm_dequant_fp8_block(None, 16, 128, 128, 16, 0, None)
    assert rc == _lib.TM_ERR_INVALID
    # workspace too small
    rc = L.tm_route_plan(256, 4, 8, 128, 256, 16, None)
    assert rc == _lib.TM_ERR_WORKSPACE
    assert b"workspace" in L.tm_last_error()
    # unaligned workspace
    rc = L.tm_route_plan(256, 4, 8, 128, 257, 1 << 30, None)
    assert rc == _lib.TM_ERR_INVALID
    # unknown act dtype
    rc = L.tm_unpack_expert(16, 16, 16, 16, 512, 256, None, None, None, 7, None)
    assert rc == _lib.TM_ERR_INVALID


def test_ops_refuse_cpu_tensors():
    import torch
    from turbomoe import ops
    with pytest.raises(_lib.TurboMoEError):
        ops.dequant_fp8_block(torch.zeros(128, 128, dtype=torch.uint8), torch.ones(1, 1))


def test_gateup_prefetch_argument_errors_without_launch():
    """tm_moe_decode_gateup_prefetch rejects missing down projections, bad
    shapes and unaligned pointers on the host, before any CUDA call."""
    L = _lib.lib()
    f = L.tm_moe_decode_gateup_prefetch
    # x, T, H, I, E, k, dtype, w13, s13, sh_w13, sh_s13, Is, sh_gate, w2, sh_w2, ws, ws_bytes, stream
    rc = f(16, 1, 2048, 768, 128, 8, 2, 16, 16, None, None, 0, None, None, None, 256, 1 << 30, None)
    assert rc == _lib.TM_ERR_INVALID and b"null" in L.tm_last_error()          # no w2
    rc = f(16, 1, 2000, 768, 128, 8, 2, 16, 16, None, None, 0, None, 16, None, 256, 1 << 30, None)
    assert rc == _lib.TM_ERR_INVALID and b"hidden" in L.tm_last_error()
    rc = f(16, 1, 2048, 768, 128, 8, 2, 16, 16, 16, 16, 512, 16, 16, None, 256, 1 << 30, None)
    assert rc == _lib.TM_ERR_INVALID and b"shared expert" in L.tm_last_error()  # shared w13 without sh_w2
    rc = f(16, 1, 2048, 768, 128, 8, 2, 24, 16, None, None, 0, None, 16, None, 256, 1 << 30, None)
    assert rc == _lib.TM_ERR_INVALID and b"aligned" in L.tm_last_error()


def test_prefetch_experts_argument_errors_without_launch():
    """tm_prefetch_experts_l2 rejects null pointers, bad counts, sizes that
    are not multiples of 16 and unaligned weights on the host."""
    L = _lib.lib()
    f = L.tm_prefetch_experts_l2
    # weights, expert_bytes, n_experts, expert_ids, n_ids, stream
    rc = f(None, 3145728, 128, 16, 8, None)
    assert rc == _lib.TM_ERR_INVALID and b"null" in L.tm_last_error()
    rc = f(16, 3145728, 128, 16, 0, None)
    assert rc == _lib.TM_ERR_INVALID and b"expert counts" in L.tm_last_error()
    rc = f(16, 3145720, 128, 16, 8, None)
    assert rc == _lib.TM_ERR_INVALID and b"multiple of 16" in L.tm_last_error()
    rc = f(24, 3145728, 128, 16, 8, None)
    assert rc == _lib.TM_ERR_INVALID and b"aligned" in L.tm_last_error()


def test_gdn_decode_argument_errors_without_launch():
    """tm_gdn_decode rejects null pointers, head dims other than 128, value
    heads that are not a multiple of the key heads, an unaligned recurrent
    state and overlapping conv-state buffers on the host."""
    L = _lib.lib()
    f = L.tm_gdn_decode
    BF16 = _lib.TM_DTYPE_BF16

    def call(qkv=256, batch=1, hk=16, hv=32, dk=128, dv=128, K=4, dt=BF16, cin=1 << 20, cout=1 << 24,
             state=1 << 26):
        # qkv, z, a, b, batch, Hk, Hv, dk, dv, K, dtype, conv_w, A_log, dt_bias, norm_w, eps, conv_in,
        # conv_out, state, out, stream
        return f(qkv, 512, 768, 1024, batch, hk, hv, dk, dv, K, dt, 2048, 4096, 8192, 16384, 1e-6, cin, cout,
                 state, 1 << 28, None)

    assert call(qkv=None) == _lib.TM_ERR_INVALID and b"null" in L.tm_last_error()
    assert call(dk=64) == _lib.TM_ERR_INVALID and b"head dims" in L.tm_last_error()
    assert call(hv=24) == _lib.TM_ERR_INVALID and b"value heads" in L.tm_last_error()
    assert call(K=9) == _lib.TM_ERR_INVALID and b"conv kernel" in L.tm_last_error()
    assert call(batch=0) == _lib.TM_ERR_INVALID and b"batch" in L.tm_last_error()
    assert call(dt=7) == _lib.TM_ERR_INVALID and b"dtype" in L.tm_last_error()
    assert call(state=(1 << 26) + 8) == _lib.TM_ERR_INVALID and b"16-byte" in L.tm_last_error()
    assert call(cout=(1 << 20) + 4096) == _lib.TM_ERR_INVALID and b"overlap" in L.tm_last_error()


# Destroying a NULL context is a no-op (like free(NULL)); the version query takes no arguments.
_NULL_OK = {"tm_abi_version", "tm_ep_destroy"}


@pytest.mark.skipif(__import__("torch").cuda.is_available(),
                    reason="all-NULL calls are only made where no device could be reached")
def test_every_entry_point_rejects_null_arguments_on_the_host():
    """Every int-returning entry point, called with NULL pointers and zero
    sizes, returns TM_ERR_INVALID with a message before any CUDA call (on a
    machine without a GPU a call that got as far as the runtime would return
    TM_ERR_CUDA instead)."""
    L = _lib.lib()
    checked = 0
    for name, (res, args) in sorted(_lib.SIGNATURES.items()):
        if res is not _lib._i or name in _NULL_OK:
            continue
        vals = [0.0 if a is ctypes.c_float else (0 if a in (_lib._i, _lib._i64) else None) for a in args]
        rc = getattr(L, name)(*vals)
        assert rc == _lib.TM_ERR_INVALID and L.tm_last_error(), (name, rc, L.tm_last_error())
        checked += 1
    assert checked >= 30
