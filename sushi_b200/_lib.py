"""ctypes binding of libsushi_exl3_cuda.so (include/sushi_exl3.h).

The library is the product: every call below runs CUDA kernels on the device.  There is no CPU
fallback; a missing or unloadable library raises at import.
"""

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_NAME = "libsushi_exl3_cuda.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)


class SxDecode(ctypes.Structure):
    _fields_ = [("codebook", ctypes.c_int32), ("window_bits", ctypes.c_int32), ("table", ctypes.c_int32)]


class SxProj(ctypes.Structure):
    _fields_ = [
        ("trellis", ctypes.c_void_p),
        ("suh", ctypes.c_void_p),
        ("svh", ctypes.c_void_p),
        ("experts", ctypes.c_int32),
        ("in_features", ctypes.c_int32),
        ("out_features", ctypes.c_int32),
        ("n", ctypes.c_int32),
        ("tile_order", ctypes.c_int32),
    ]


class SxBank(ctypes.Structure):
    _fields_ = [("gate", SxProj), ("up", SxProj), ("down", SxProj)]


class SxRagged(ctypes.Structure):
    _fields_ = [
        ("trellis", ctypes.c_void_p * 3),
        ("suh", ctypes.c_void_p * 3),
        ("svh", ctypes.c_void_p * 3),
        ("meta", ctypes.c_void_p),
        ("experts", ctypes.c_int32),
        ("hidden", ctypes.c_int32),
        ("inter", ctypes.c_int32),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int32
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); every symbol include/sushi_exl3.h declares.
SIGNATURES = {
    "sx_status_name": (ctypes.c_char_p, [_I]),
    "sx_version": (ctypes.c_char_p, []),
    "sx_dequant_inner": (_I, [_P, ctypes.POINTER(SxProj), _I, ctypes.POINTER(SxDecode), _P]),
    "sx_decode_codewords": (_I, [_P, _I, ctypes.POINTER(SxDecode), _P]),
    "sx_tile_order_convert": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _I]),
    "sx_linear": (_I, [_P, ctypes.POINTER(SxProj), ctypes.POINTER(SxDecode), _P, _I, _I, _P]),
    "sx_linear_ex": (_I, [_P, ctypes.POINTER(SxProj), ctypes.POINTER(SxDecode), _P, _I, _I, _P, ctypes.c_uint32]),
    "sx_linear_gemm_workspace_bytes": (_SZ, [ctypes.POINTER(SxProj), _I]),
    "sx_linear_gemm": (_I, [_P, ctypes.POINTER(SxProj), ctypes.POINTER(SxDecode), _P, _I, _I, _P, _P, _SZ]),
    "sx_linear_shared": (_I, [_P, ctypes.POINTER(SxProj), _P, _I, ctypes.POINTER(SxDecode), _P, _I, _I, _P]),
    "sx_linear_shared_normed_workspace_bytes": (_SZ, [ctypes.POINTER(SxProj)]),
    "sx_linear_shared_normed": (_I, [_P, ctypes.POINTER(SxProj), _P, _I, ctypes.POINTER(SxDecode), _P, _I, _I, _P, _P,
                                     ctypes.c_float, _P, _SZ]),
    "sx_linear_grouped": (_I, [_P, ctypes.POINTER(SxProj), ctypes.POINTER(SxDecode), _P, _I, _I, _P]),
    "sx_router_topk": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, ctypes.c_float, _I, _I, _P, _P]),
    "sx_router_topk_gate": (_I, [_P, _P, _I, _P, _I, _I, _I, _I, _I, ctypes.c_float, _I, _I, _P, _P, _I, _I, _P, _P,
                                 _P]),
    "sx_moe_workspace_bytes": (_SZ, [ctypes.POINTER(SxBank), _I, _I]),
    "sx_moe": (_I, [_P, ctypes.POINTER(SxBank), ctypes.POINTER(SxDecode), _P, _I, _I, _P, _P, _I, _P, _P, _I, _P, _P, _SZ]),
    "sx_moe_ragged_workspace_bytes": (_SZ, [ctypes.POINTER(SxRagged), _I, _I]),
    "sx_moe_ragged": (_I, [_P, ctypes.POINTER(SxRagged), ctypes.POINTER(SxDecode), _P, _I, _I, _P, _P, _I, _P, _P, _I, _P,
                           _P, _SZ]),
    "sx_moe_static_scratch": (_I, [_P, ctypes.POINTER(SxBank), ctypes.POINTER(SxDecode), _P, _I, _I, _P, _P, _I, _P, _P, _I, _P]),
    "sx_moe_static_scratch_bytes": (_SZ, []),
    "sx_ep_unique_id": (_I, [_P]),
    "sx_ep_init": (_I, [_P, _I, _I, _P]),
    "sx_ep_destroy": (_I, [_P]),
    "sx_ep_abort": (_I, [_P]),
    "sx_ep_info": (_I, [_P, _P, _P]),
    "sx_ep_peer_bytes": (_SZ, [_P, _I, _I, _I, _I]),
    "sx_ep_reserve_peer": (_I, [_P, _SZ]),
    "sx_ep_peer_reserved": (_SZ, [_P]),
    "sx_ep_phase_timing": (_I, [_P, _I]),
    "sx_ep_phase_ms": (_I, [_P, _P]),
    "sx_ep_workspace_bytes": (_SZ, [_P, ctypes.POINTER(SxBank), _I, _I, _I]),
    "sx_ep_moe": (_I, [_P, _P, ctypes.POINTER(SxBank), _I, ctypes.POINTER(SxDecode), _P, _I, _I, _I, _P, _P, _I, _P,
                       _P, _I, _P, _P, _SZ]),
    "sx_moe_folded_workspace_bytes": (_SZ, [ctypes.POINTER(SxBank), ctypes.POINTER(SxBank), _P, _P, _I, _I]),
    "sx_moe_folded": (_I, [_P, ctypes.POINTER(SxBank), ctypes.POINTER(SxBank), _P, _P, _P, _I, _I, _P, _P, _I, _P, _I,
                           _P, _P, _SZ]),
    "sx_moe_ragged_folded_workspace_bytes": (_SZ, [ctypes.POINTER(SxRagged), ctypes.POINTER(SxBank), _P, _P, _I, _I]),
    "sx_moe_ragged_folded": (_I, [_P, ctypes.POINTER(SxRagged), ctypes.POINTER(SxBank), _P, _P, _P, _I, _I, _P, _P, _I,
                                  _P, _I, _P, _P, _SZ]),
    "sx_ep_ragged_workspace_bytes": (_SZ, [_P, ctypes.POINTER(SxRagged), _I, _I, _I]),
    "sx_ep_moe_ragged": (_I, [_P, _P, ctypes.POINTER(SxRagged), _I, ctypes.POINTER(SxDecode), _P, _I, _I, _I, _P, _P,
                              _I, _P, _P, _I, _P, _P, _SZ]),
    "sx_ep_folded_workspace_bytes": (_SZ, [_P, ctypes.POINTER(SxBank), ctypes.POINTER(SxBank), _I, _I, _I]),
    "sx_ep_moe_folded": (_I, [_P, _P, ctypes.POINTER(SxBank), ctypes.POINTER(SxBank), _I, _P, _P, _P, _I, _I, _I, _P,
                              _P, _I, _P, _I, _P, _P, _SZ]),
    "sx_ep_ragged_folded_workspace_bytes": (_SZ, [_P, ctypes.POINTER(SxRagged), ctypes.POINTER(SxBank), _I, _I, _I]),
    "sx_ep_moe_ragged_folded": (_I, [_P, _P, ctypes.POINTER(SxRagged), ctypes.POINTER(SxBank), _I, _P, _P, _P, _I, _I,
                                     _I, _P, _P, _I, _P, _I, _P, _P, _SZ]),
    "sx_device_error": (_I, [_P]),
    "sx_selftest_wait_timeout": (_I, [_P, _I]),
    "sx_last_error_detail": (ctypes.c_char_p, []),
}

# Library extras (not in the Zig-facing header): table introspection for the config parser.
EXTRAS = {
    "sx_table_row": (_I, [_I, _I, ctypes.POINTER(ctypes.c_uint32)]),
    "sx_table_info": (_I, [_I, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_I), ctypes.POINTER(_I),
                           ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)]),
}

_lib = None


def load():
    """The loaded library; raises if it is missing (build it with `make -C sushi_b200`)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C {HERE}` (no CPU fallback exists)")
    lib = ctypes.CDLL(LIB_PATH)
    for table in (SIGNATURES, EXTRAS):
        for name, (res, args) in table.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
    _lib = lib
    return lib
