"""geode_b200 - a B200-native (sm_100a) backend for the Geode engine's speculative-decoding verify step.

The product is native: libgeode_cuda.so (CUDA kernels + the C ABI of include/geode_cuda.h) and libgeode_host.so
(the C++ host side: pack reader, Model-shaped verify / keep, the speculation step; include/geode_host.h). This
package only loads them (ctypes) for Python callers: tests, the benchmark. There is no CPU fallback: loading fails
loudly when a library is missing.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
CUDA_SO = os.path.join(PKG, "libgeode_cuda.so")
HOST_SO = os.path.join(PKG, "libgeode_host.so")

_cuda = None
_host = None


def cuda_lib() -> C.CDLL:
    """libgeode_cuda.so with its argument types declared. Raises when it was not built."""
    global _cuda
    if _cuda is not None:
        return _cuda
    if not os.path.exists(CUDA_SO):
        raise RuntimeError(f"{CUDA_SO} is missing: build it with `python -m geode_b200.build` (no CPU fallback)")
    L = C.CDLL(CUDA_SO, mode=C.RTLD_GLOBAL)
    vp, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t
    sig = {
        "gcuda_op_q4_tiled_bytes": (sz, [i64, i64]),
        "gcuda_op_q4_relayout": (i32, [vp, i64, i64, vp, vp]),
        "gcuda_op_quantize": (i32, [vp, i32, i32, vp, vp, vp, vp]),
        "gcuda_op_q4_gemv": (i32, [vp, i64, i64, f32, vp, vp, vp, i32, vp, vp]),
        "gcuda_op_q4_dequant": (i32, [vp, i64, f32, vp, i32, vp, vp]),
        "gcuda_op_bf16_gemv": (i32, [vp, i32, i32, vp, i32, vp, vp]),
        "gcuda_op_route_topk": (i32, [vp, i32, i32, i32, vp, vp, vp]),
        "gcuda_op_route_out_bytes": (sz, []),
        "gcuda_op_route_union": (i32, [vp, i32, i32, i32, vp, sz, vp]),
        "gcuda_op_greedy_verify": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, vp]),
        "gcuda_op_norm_quant": (i32, [vp, i32, i32, vp, f32, vp, vp, vp, vp, vp]),
        "gcuda_op_status": (i32, [i32]),
        "gcuda_op_q4_umma_bytes": (sz, [i64, i64]),
        "gcuda_op_q4_umma_relayout": (i32, [vp, i64, i64, vp, vp]),
        "gcuda_op_q4_gemm_umma": (i32, [vp, i64, i64, f32, vp, vp, vp, i32, vp, vp]),
        "gcuda_op_moe_lane_expert_bytes": (sz, [i32, i32]),
        "gcuda_op_moe_lane_work_bytes": (sz, [i32, i32, i32, i32]),
        "gcuda_op_moe_lane_relayout": (i32, [vp, sz, i32, i32, i32, vp, vp]),
        "gcuda_op_moe_lane": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp, i32, vp, vp, sz, vp]),
        "gcuda_op_moe_umma_expert_bytes": (sz, [i32, i32]),
        "gcuda_op_moe_umma_work_bytes": (sz, [i32, i32, i32, i32, i32]),
        "gcuda_op_moe_umma_relayout": (i32, [vp, sz, i32, i32, i32, vp, vp]),
        "gcuda_op_moe_umma": (i32, [vp, vp, i32, i32, i32, vp, vp, vp, i32, vp, i32, vp, vp, sz, vp]),
        "gcuda_debug_expf_table": (i32, [C.c_uint32, i64, vp, vp]),
    }
    for name, (res, args) in sig.items():
        if hasattr(L, name):
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
    _cuda = L
    return L
