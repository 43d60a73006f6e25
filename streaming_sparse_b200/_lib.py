"""ctypes binding of libssparse.so (the C ABI declared in include/ssparse.h).

Follows the reference's loading scheme for its sm_80 kernel library (ctypes.CDLL + argtypes,
raw data pointers, the current stream handle, nonzero status -> RuntimeError;
local_experiments/video_runtime_v1/fixed15_attention.py:13-33,120-124). There is no fallback:
if the library is missing or cannot be loaded, every op raises.
"""
from __future__ import annotations

import ctypes
import os
from functools import lru_cache

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libssparse.so")

SS_ERRORS = {
    1001: "inconsistent or unsupported sizes",
    1002: "null or misaligned pointer",
    1003: "workspace too small",
    1004: "extra exceeds the number of unforced blocks",
    1005: "block lists do not fit the attention kernel's shared memory",
    1006: "cuTensorMapEncodeTiled unavailable or failed",
    1007: "device ordinal beyond the library's 64-device table",
}
DEV_NONFINITE, DEV_TIMEOUT, DEV_BADID = 0x1, 0x2, 0x4

_P, _I, _I64, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t

SIGNATURES = {
    "ss_version": ([], _I),
    "ss_prepare_device": ([], _I),
    "ss_router_workspace_bytes": ([_I, _I, _I, _I, _I, ctypes.POINTER(_SZ)], _I),
    "ss_router_fast_workspace_bytes": ([_I, _I, _I, _I, _I, ctypes.POINTER(_SZ)], _I),
    "ss_router": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P, _P, _SZ, _P, _P], _I),
    "ss_router_noalloc": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P], _I),
    "ss_router_pool_keys": ([_P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P], _I),
    "ss_router_cached": ([_P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _I, _P, _I, _P, _P, _P, _SZ, _P,
                          _P], _I),
    "ss_router_fast": ([_P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _I, _P, _I, _P, _P, _P, _P, _SZ,
                        _P, _P], _I),
    "ss_router_pool_keys_ring": ([_P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _I, _I, _I, _P, _P, _P], _I),
    "ss_router_ring": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _I, _P, _I, _P, _P, _P, _I, _I, _I, _I,
                        _P, _P, _SZ, _P, _P], _I),
    "ss_attention_ring": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P, _I, _I, _I, _P, _P, _SZ, _P], _I),
    "ss_cache_append_ring": ([_P, _P, _I, _I, _P, _P, _I64, _I, _I, _I64, _I64, _I64, _I, _I, _I, _P,
                              ctypes.POINTER(_I64), ctypes.POINTER(_I), _P], _I),
    "ss_cache_ring_refresh": ([_P, _P, _I, _I, _I, _I, _P, _P], _I),
    "ss_qkv_norm_rope_ring": ([_P, _I64, _I, _I, _P, _P, _F, _P, _P, _P, _I64, _P, _P, _I64, _I, _I, _I64, _P, _I,
                               _P], _I),
    "ss_qkv_norm_rope_heads": ([_P, _I64, _I, _I, _P, _P, _F, _P, _P, _I, _I, _P, _I64, _P, _P, _I64, _I, _I, _I64,
                                _P, _I, _P], _I),
    "ss_cache_ring_commit": ([_P, _P, _I, _I, _I, _P, _I, _I, _P], _I),
    "ss_ipc_handle": ([_P, _P, ctypes.POINTER(_SZ)], _I),
    "ss_ipc_open": ([_P, _SZ, ctypes.POINTER(_P)], _I),
    "ss_ipc_close": ([_P, _SZ], _I),
    "ss_peer_barrier": ([_P, _I, _I, _P, _P, _P], _I),
    "ss_lse_merge_peers": ([_P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _P, _P], _I),
    "ss_attention_kv_parts": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _P, _I, _I, _I, _I, _P, _P, _SZ, _P], _I),
    "ss_lse_merge_gather": ([_P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _I, _P, _I, _P, _P, _P], _I),
    "ss_attention_heads": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _I, _I, _I, _P, _P, _I, _I, _I, _P, _P,
                            _SZ, _P], _I),
    "ss_attention": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P, _P], _I),
    "ss_attention_max_ids": ([_I, _I, ctypes.POINTER(_I)], _I),
    "ss_attention_workspace_bytes": ([_I, _I, ctypes.POINTER(_SZ)], _I),
    "ss_quant_k_pages": ([_P, _I, _I, _I, _I, _P, _P, _P], _I),
    "ss_attention_i8_workspace_bytes": ([_I, _I, ctypes.POINTER(_SZ)], _I),
    "ss_attention_i8": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P, _P, _SZ, _P], _I),
    "ss_quant_k_pages_ring": ([_P, _I, _I, _I, _I, _P, _P, _I, _I, _I, _P, _P], _I),
    "ss_attention_i8_ring": ([_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P, _I, _I, _I, _P, _P, _SZ,
                              _P], _I),
    "ss_attention_ws": ([_P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _P, _I, _P, _P, _P, _SZ, _P], _I),
    "ss_lse_merge": ([_P, _P, _I, _I, _I, _P, _I, _P, _P], _I),
    "ss_cache_append": ([_P, _P, _I, _I, _P, _P, _I64, _I, _I, _I64, _I64, _I64, _I, ctypes.POINTER(_I64), _P], _I),
    "ss_cache_rope_shift": ([_P, _I64, _P, _I64, _I, _I, _I, _P, _P], _I),
    "ss_qkv_norm_rope": ([_P, _I64, _I, _I, _P, _P, _F, _P, _P, _P, _I64, _P, _P, _I64, _P], _I),
    "ss_adaln": ([_P, _I, _I, _I, _P, _P, _I64, _P, _P, _F, _P, _P], _I),
    "ss_rms_norm": ([_P, _I64, _I, _I, _P, _F, _P, _P], _I),
    "ss_gate_residual": ([_P, _P, _I64, _I, _I, _I, _P, _I64, _P], _I),
}


@lru_cache(None)
def lib() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"libssparse.so not built ({LIB_PATH}); run `python -m streaming_sparse_b200.build`")
    handle = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.argtypes = args
        fn.restype = res
    return handle


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = SS_ERRORS.get(rc, f"CUDA error {rc}")
        raise RuntimeError(f"{what} failed: {msg} (status {rc})")


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
