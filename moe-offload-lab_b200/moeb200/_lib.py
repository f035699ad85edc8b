"""ctypes binding of libmoeb200.so (the C ABI declared in include/moeb200.h).

The library is built in-tree (moeb200/build.py) and loaded from next to this file. There is no
fallback: if the library is missing or a call fails, an exception is raised.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmoeb200.so"

F32, F16, BF16, I8, I4 = 0, 1, 2, 3, 4
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = 0, 1, 2, 3, 4
# MOEB200_NOALLOC_SCRATCH_BYTES of include/moeb200.h: the static scratch of the workspace-free entry point
NOALLOC_SCRATCH_BYTES = 1 << 20


class MoeB200Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"moeb200 error {code}: {msg}")
        self.code = code


class Layout(C.Structure):
    _fields_ = [("wtype", C.c_int32), ("hidden", C.c_int32), ("inter", C.c_int32), ("gs_up", C.c_int32),
                ("gs_dn", C.c_int32), ("_pad", C.c_int32), ("off_gu_q", C.c_int64), ("off_gu_s", C.c_int64),
                ("off_dn_q", C.c_int64), ("off_dn_s", C.c_int64), ("record_bytes", C.c_int64)]


class Policy(C.Structure):
    _fields_ = [("mode", C.c_int32), ("t1", C.c_float), ("t_mid", C.c_float), ("t2", C.c_float),
                ("thr", C.c_float)]


class ExpertTable(C.Structure):
    _fields_ = [("n_prec", C.c_int32), ("num_experts", C.c_int32), ("layout", Layout * 4),
                ("table", C.c_void_p), ("tma_base", C.c_int64)]


class PeerGroup(C.Structure):
    """moeb200_peer_group: device tables of every rank's mapped exchange buffers."""

    _fields_ = [("G", C.c_int32), ("rank", C.c_int32), ("T", C.c_int32), ("H", C.c_int32), ("k", C.c_int32),
                ("spin", C.c_uint32), ("rows", C.c_void_p), ("parts", C.c_void_p), ("flags", C.c_void_p),
                ("epoch", C.c_void_p), ("status", C.c_void_p)]


_P = C.c_void_p
_SIGS = {
    "moeb200_version": (C.c_char_p, []),
    "moeb200_last_error": (C.c_int, [C.c_char_p, C.c_size_t]),
    "moeb200_num_sms": (C.c_int, []),
    "moeb200_trace_begin": (C.c_int, []),
    "moeb200_path_used": (C.c_int, []),
    "moeb200_trace_end": (C.c_int, [C.POINTER(C.c_float), C.POINTER(C.c_float), C.POINTER(C.c_int32)]),
    "moeb200_router": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                 _P, _P, _P, _P, C.POINTER(Policy), _P, _P, _P, C.c_size_t, _P]),
    "moeb200_set_path": (C.c_int, [C.c_int32]),
    "moeb200_router_shared": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                        C.c_int32, _P, _P, _P, _P, C.POINTER(Policy), _P, _P, _P, C.c_size_t, _P]),
    "moeb200_levels_vote": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_double, _P]),
    "moeb200_set_item_tokens": (C.c_int, [C.c_int32]),
    "moeb200_router_workspace": (C.c_size_t, [C.c_int32, C.c_int32]),
    "moeb200_levels": (C.c_int, [_P, C.c_int32, C.c_int32, C.POINTER(Policy), _P, _P, _P]),
    "moeb200_dispatch": (C.c_int, [_P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, _P, _P, _P, _P,
                                   _P, C.c_size_t, _P]),
    "moeb200_dispatch_workspace": (C.c_size_t, [C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "moeb200_grouped_ffn": (C.c_int, [C.POINTER(Layout), _P, _P, C.c_int32, _P, C.c_int32, _P, _P, C.c_size_t,
                                      _P]),
    "moeb200_grouped_ffn_workspace": (C.c_size_t, [C.POINTER(Layout), C.c_int32]),
    "moeb200_grouped_ffn_noalloc": (C.c_int, [C.POINTER(Layout), _P, _P, C.c_int32, _P, C.c_int32, _P, _P]),
    "moeb200_noalloc_check_status": (C.c_int, [C.POINTER(C.c_int32), _P]),
    "moeb200_experts_forward": (C.c_int, [C.POINTER(ExpertTable), _P, C.c_int32, C.c_int32, _P, _P, C.c_int32,
                                          _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "moeb200_experts_workspace": (C.c_size_t, [C.POINTER(ExpertTable), C.c_int32, C.c_int32]),
    "moeb200_experts_forward_part": (C.c_int, [C.POINTER(ExpertTable), C.c_int32, C.c_int32, _P, C.c_int32,
                                               C.c_int32, _P, _P, C.c_int32, _P, _P, _P, _P, _P, C.c_size_t, _P]),
    "moeb200_combine_parts": (C.c_int, [_P, C.c_int32, C.c_int64, C.c_int32, _P, C.c_int32, _P]),
    "moeb200_ep_row_bytes": (C.c_size_t, [C.c_int32, C.c_int32, C.c_int32]),
    "moeb200_ep_pack": (C.c_int, [_P, _P, _P, _P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, _P]),
    "moeb200_ep_unpack": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, _P, _P, _P, _P, _P]),
    "moeb200_shared_expert": (C.c_int, [C.POINTER(Layout), _P, _P, _P, C.c_int32, C.c_int32, _P, C.c_int32, _P,
                                        C.c_size_t, _P]),
    "moeb200_shared_expert_workspace": (C.c_size_t, [C.POINTER(Layout), C.c_int32]),
    "moeb200_dense_int8_gemv": (C.c_int, [_P, _P, C.c_int32, C.c_int32, C.c_int32, _P, C.c_int32, C.c_int32, _P,
                                          _P, _P]),
    "moeb200_dense_int8_dequant": (C.c_int, [_P, _P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, _P]),
    "moeb200_quantize": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, _P, _P,
                                   _P]),
    "moeb200_peer_alloc": (C.c_int, [C.c_size_t, C.POINTER(C.c_void_p), _P]),
    "moeb200_peer_open": (C.c_int, [_P, C.POINTER(C.c_void_p)]),
    "moeb200_peer_close": (C.c_int, [_P]),
    "moeb200_peer_free": (C.c_int, [_P]),
    "moeb200_ep_signal": (C.c_int, [C.POINTER(PeerGroup), C.c_int32, _P]),
    "moeb200_ep_gather": (C.c_int, [C.POINTER(PeerGroup), C.c_int32, _P, _P, _P, _P, _P, _P]),
    "moeb200_ep_combine_peers": (C.c_int, [C.POINTER(PeerGroup), C.c_int32, _P, C.c_int32, _P]),
    "moeb200_check_workspace": (C.c_int, [_P, C.POINTER(C.c_int32), _P]),
}

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """The loaded library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise MoeB200Error(ERR_INVALID, f"{LIB_PATH} is missing: build it with moeb200/build.py "
                                            "(there is no fallback implementation)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> tuple[int, str]:
    buf = C.create_string_buffer(1024)
    code = lib().moeb200_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != OK:
        code, msg = last_error()
        raise MoeB200Error(rc, msg)


def exported_symbols() -> list[str]:
    return list(_SIGS)
