"""sushi_b200: B200-native (sm_100a) EXL3 / STQ trellis-decode kernels behind a C ABI.

The product is libsushi_exl3_cuda.so (include/sushi_exl3.h); this package is its host-side mirror
of the reference's `sushi_exl3` module interface (see exl3.py).  Importing it loads the library
and fails loudly when it is missing: there is no CPU fallback.
"""

from . import _lib

_lib.load()

from .exl3 import (  # noqa: E402
    Bank,
    Codebook,
    Decode,
    Exl3Error,
    ExpertParallel,
    LINEAR_WEIGHTS_STATIC,
    Proj,
    Ragged,
    RouterMode,
    TileOrder,
    decode_codewords,
    dequant_inner,
    device_error,
    linear,
    linear_gemm,
    linear_grouped,
    linear_shared,
    linear_shared_normed,
    linear_shared_normed_workspace_bytes,
    moe,
    moe_clamped,
    moe_folded,
    moe_ragged,
    moe_with_gated_shared,
    moe_with_shared,
    router_topk,
    router_topk_gate,
    share_unique_id,
    table_info,
    table_row,
    tile_order_convert,
)

__all__ = [
    "Bank", "Codebook", "Decode", "Exl3Error", "ExpertParallel", "LINEAR_WEIGHTS_STATIC", "Proj", "Ragged", "RouterMode", "TileOrder", "decode_codewords",
    "dequant_inner", "device_error", "linear", "linear_gemm", "linear_grouped", "linear_shared", "linear_shared_normed",
    "linear_shared_normed_workspace_bytes", "moe", "moe_clamped", "moe_folded", "moe_ragged", "moe_with_gated_shared",
    "moe_with_shared", "router_topk", "router_topk_gate", "share_unique_id", "table_info", "table_row", "tile_order_convert",
]
