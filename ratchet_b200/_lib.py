"""ctypes binding of the C ABI in include/fgg_api.h (library ratchet_b200/_fgg.so).

There is no fallback: if the native library is missing or fails to load,
every operator raises.  Build it with `python -m ratchet_b200.build`.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("_fgg.so")

FGG_OK = 0
FGG_EINVAL = 1
FGG_EBADSHAPE = 2
FGG_EALIGN = 3
FGG_EWORKSPACE = 4
FGG_ECUDA = 5
FGG_ETIMEOUT = 6
FGG_EARCH = 7
FGG_MAX_GROUPS = 512
FGG_NOALLOC_SCRATCH_BYTES = 32 << 20
FGG_DEBUG_NO_LOADS = 1

_VOIDP = ctypes.c_void_p
_PTRS = ctypes.POINTER(ctypes.c_void_p)


class FggNvfp4Weights(ctypes.Structure):
    _fields_ = [("num_groups", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("b", _VOIDP), ("b_sf", _VOIDP)]


class FggNvfp4Problem(ctypes.Structure):
    _fields_ = [("num_groups", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("m", _VOIDP), ("a", _VOIDP), ("a_sf", _VOIDP), ("alpha", _VOIDP),
                ("out", _VOIDP), ("b_index", _VOIDP), ("num_weight_groups", ctypes.c_int32)]


class FggNvfp4RowsProblem(ctypes.Structure):
    _fields_ = [("num_groups", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("max_rows", ctypes.c_int32), ("offsets", _VOIDP), ("a", _VOIDP), ("a_sf", _VOIDP),
                ("alpha", _VOIDP), ("out", _VOIDP), ("row_scale", _VOIDP), ("b_index", _VOIDP),
                ("num_weight_groups", ctypes.c_int32), ("max_group_rows", ctypes.c_int32)]


class FggMxProblem(ctypes.Structure):
    _fields_ = [("m_total", ctypes.c_int32), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("num_groups", ctypes.c_int32), ("a", _VOIDP), ("a_sf", _VOIDP), ("b", _VOIDP),
                ("b_sf", _VOIDP), ("m_indices", _VOIDP), ("c", _VOIDP),
                ("reuse_prepared", ctypes.c_int32)]


class FggMoeTokens(ctypes.Structure):
    _fields_ = [("num_tokens", ctypes.c_int32), ("topk", ctypes.c_int32), ("k", ctypes.c_int32),
                ("codes", _VOIDP), ("codes_stride", ctypes.c_int64),
                ("sf", _VOIDP), ("sf_stride", ctypes.c_int64),
                ("ids", _VOIDP), ("ids_stride", ctypes.c_int64),
                ("weights", _VOIDP), ("weights_stride", ctypes.c_int64),
                ("scale", _VOIDP), ("scale_stride", ctypes.c_int64),
                ("epoch", _VOIDP), ("parity_bytes", ctypes.c_int64)]


FGG_PEERS_MAX = 8


class FggMoePeers(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("capacity", ctypes.c_int32),
                ("n", ctypes.c_int32), ("epoch", _VOIDP), ("counters", _VOIDP), ("status", _VOIDP),
                ("gathered", _VOIDP * FGG_PEERS_MAX), ("recv", _VOIDP * FGG_PEERS_MAX),
                ("flags", _VOIDP * FGG_PEERS_MAX), ("owner", _VOIDP),
                ("num_experts", ctypes.c_int32), ("routes", _VOIDP),
                ("wait_ms", ctypes.c_int32)]


class FggError(RuntimeError):
    def __init__(self, code: int, where: str, detail: str):
        self.code = code
        super().__init__(f"{where}: {detail} (fgg error {code})")


# name -> (restype, argtypes)
_SIGS = {
    "fgg_error_string": (ctypes.c_char_p, [ctypes.c_int]),
    "fgg_last_error_detail": (ctypes.c_char_p, []),
    "fgg_version": (ctypes.c_char_p, []),
    "fgg_nvfp4_weight_pack_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "fgg_nvfp4_pack_weights": (ctypes.c_int, [ctypes.POINTER(FggNvfp4Weights), _VOIDP, ctypes.c_size_t, _VOIDP]),
    "fgg_nvfp4_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(FggNvfp4Problem)]),
    "fgg_nvfp4_grouped_gemm": (ctypes.c_int, [ctypes.POINTER(FggNvfp4Problem), _VOIDP, _VOIDP, ctypes.c_size_t, _VOIDP]),
    "fgg_nvfp4_prepare": (ctypes.c_int, [ctypes.POINTER(FggNvfp4Problem), _VOIDP, ctypes.c_size_t, _VOIDP]),
    "fgg_nvfp4_gemm": (ctypes.c_int, [ctypes.POINTER(FggNvfp4Problem), _VOIDP, _VOIDP, ctypes.c_size_t, _VOIDP]),
    "fgg_nvfp4_rows_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(FggNvfp4RowsProblem)]),
    "fgg_nvfp4_grouped_gemm_rows": (ctypes.c_int, [ctypes.POINTER(FggNvfp4RowsProblem), _VOIDP, _VOIDP, ctypes.c_size_t, _VOIDP]),
    "fgg_nvfp4_grouped_gemm_noalloc": (ctypes.c_int, [ctypes.POINTER(FggNvfp4Problem), _VOIDP, _VOIDP, _VOIDP]),
    "fgg_moe_plan": (ctypes.c_int, [_VOIDP, ctypes.c_int32, ctypes.c_int32, _VOIDP, _VOIDP, ctypes.c_int32,
                                    ctypes.c_int32, ctypes.c_int32, _VOIDP, _VOIDP, _VOIDP, _VOIDP, _VOIDP]),
    "fgg_moe_gather_rows": (ctypes.c_int, [_VOIDP, _VOIDP, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                                           _VOIDP, ctypes.c_int64, _VOIDP, _VOIDP, _VOIDP, _VOIDP]),
    "fgg_moe_combine": (ctypes.c_int, [_VOIDP, ctypes.c_int64, _VOIDP, _VOIDP, ctypes.c_int32, ctypes.c_int32,
                                       ctypes.c_int32, _VOIDP, _VOIDP, _VOIDP]),
    "fgg_moe_record_bytes": (ctypes.c_size_t, [ctypes.c_int32, ctypes.c_int32]),
    "fgg_moe_pack_tokens": (ctypes.c_int, [ctypes.POINTER(FggMoeTokens), _VOIDP, _VOIDP]),
    "fgg_moe_records_view": (ctypes.c_int, [_VOIDP, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.POINTER(FggMoeTokens)]),
    "fgg_moe_expand": (ctypes.c_int, [ctypes.POINTER(FggMoeTokens), _VOIDP, _VOIDP, ctypes.c_int32,
                                      ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _VOIDP, _VOIDP,
                                      _VOIDP, _VOIDP, _VOIDP, _VOIDP, _VOIDP, _VOIDP, _VOIDP]),
    "fgg_moe_reduce": (ctypes.c_int, [_VOIDP, ctypes.c_int32, _VOIDP, ctypes.POINTER(FggMoeTokens),
                                      ctypes.c_int32, _VOIDP, _VOIDP, _VOIDP]),
    "fgg_moe_sum_partials": (ctypes.c_int, [_VOIDP, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                            ctypes.c_int32, _VOIDP, _VOIDP]),
    "fgg_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(_VOIDP)]),
    "fgg_peer_free": (ctypes.c_int, [_VOIDP]),
    "fgg_peer_handle_bytes": (ctypes.c_size_t, []),
    "fgg_peer_export": (ctypes.c_int, [_VOIDP, _VOIDP]),
    "fgg_peer_import": (ctypes.c_int, [_VOIDP, ctypes.POINTER(_VOIDP)]),
    "fgg_peer_close": (ctypes.c_int, [_VOIDP]),
    "fgg_moe_dispatch_peers": (ctypes.c_int, [ctypes.POINTER(FggMoeTokens), ctypes.POINTER(FggMoePeers), _VOIDP]),
    "fgg_moe_wait_peers": (ctypes.c_int, [ctypes.POINTER(FggMoePeers), ctypes.c_int32, _VOIDP]),
    "fgg_moe_reduce_peers": (ctypes.c_int, [_VOIDP, ctypes.c_int32, _VOIDP, ctypes.POINTER(FggMoeTokens),
                                            ctypes.POINTER(FggMoePeers), _VOIDP, _VOIDP]),
    "fgg_moe_sum_peers": (ctypes.c_int, [ctypes.POINTER(FggMoePeers), ctypes.c_int32, _VOIDP, _VOIDP]),
    "fgg_nvfp4_grouped_gemm_silu_mul": (ctypes.c_int, [ctypes.POINTER(FggNvfp4Problem), _VOIDP, _VOIDP, ctypes.c_size_t, _VOIDP]),
    "fgg_mx_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(FggMxProblem)]),
    "fgg_mx_grouped_gemm": (ctypes.c_int, [ctypes.POINTER(FggMxProblem), _VOIDP, ctypes.c_size_t, _VOIDP]),
    "fgg_amax": (ctypes.c_int, [_VOIDP, ctypes.c_int32, ctypes.c_int64, _VOIDP, _VOIDP]),
    "fgg_nvfp4_quantize": (ctypes.c_int, [_VOIDP, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, _VOIDP, _VOIDP, _VOIDP, _VOIDP, _VOIDP]),
    "fgg_read_device_status": (ctypes.c_int, [_VOIDP, _VOIDP]),
    "fgg_debug_set_flags": (ctypes.c_int32, [ctypes.c_int32]),
}

_lock = threading.Lock()
_lib = None


def lib() -> ctypes.CDLL:
    """Load the native library once; raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"ratchet_b200: native library {LIB_PATH} is missing; build it with "
                    "`python -m ratchet_b200.build` (there is no CPU fallback)")
            L = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int, where: str) -> None:
    if rc == FGG_OK:
        return
    L = lib()
    detail = (L.fgg_last_error_detail() or b"").decode(errors="replace")
    if rc in (FGG_EINVAL, FGG_EBADSHAPE, FGG_EALIGN):
        raise ValueError(f"{where}: {detail} ({L.fgg_error_string(rc).decode()})")
    raise FggError(rc, where, detail or L.fgg_error_string(rc).decode())


def exported_symbols() -> list[str]:
    return list(_SIGS)
