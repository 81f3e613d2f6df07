"""ctypes binding of libq35k.so (the C ABI declared in include/q35k.h).

There is deliberately no fallback: if the shared library is missing or no
sm_100 GPU is present, every compute call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "libq35k.so")

OK, EINVAL, ENOTSUP, ENOMEM, ECUDA, ETIMEOUT, ENCCL, EDATA, EIO = 0, 1, 2, 3, 4, 5, 6, 7, 8
GATHER_NCCL, GATHER_PEER, GATHER_FUSED = 0, 1, 2
GEMM_EXACT, GEMM_FAST = 0, 1
MAX_SHARED = 4
NCCL_ID_BYTES = 128

# Symbols declared in include/q35k.h, with their ctypes signatures.
_vp, _i32, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
_pp = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = {
    "q35k_version": ([], ctypes.c_char_p),
    "q35k_create": ([_i32, _pp], _i32),
    "q35k_destroy": ([_vp], _i32),
    "q35k_last_error": ([_vp], ctypes.c_char_p),
    "q35k_sync": ([_vp], _i32),
    "q35k_weight_upload": ([_vp, _i32, _vp, _i32, _i32, _pp], _i32),
    "q35k_weight_free": ([_vp, _vp], _i32),
    "q35k_weight_info": ([_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                          ctypes.POINTER(_sz)], _i32),
    "q35k_matmul": ([_vp, _vp, _vp, _vp, _i32], _i32),
    "q35k_matmul_q8k": ([_vp, _vp, _vp, _vp, _i32], _i32),
    "q35k_matmul_dev": ([_vp, _vp, _vp, _vp, _i32, _vp], _i32),
    "q35k_host_register": ([_vp, _vp, _sz], _i32),
    "q35k_host_unregister": ([_vp, _vp], _i32),
    "q35k_matmul_argmax": ([_vp, _vp, _vp, _vp, _i32], _i32),
    "q35k_matmul_argmax_dev": ([_vp, _vp, _vp, _vp, _vp, _i32, _vp], _i32),
    "q35k_matmul_shared": ([_vp, _pp, _i32, _vp, _pp, _i32], _i32),
    "q35k_matmul_shared_dev": ([_vp, _pp, _i32, _vp, _pp, _i32, _vp], _i32),
    "q35k_matmul_silu": ([_vp, _vp, _vp, _vp, _vp, _i32], _i32),
    "q35k_matmul_silu_dev": ([_vp, _vp, _vp, _vp, _vp, _i32, _vp], _i32),
    "q35k_matmul_q8k_dev": ([_vp, _vp, _vp, _vp, _i32, _vp], _i32),
    "q35k_quantize_q8k": ([_vp, _vp, _vp, _i32, _i32], _i32),
    "q35k_quantize_q8k_dev": ([_vp, _vp, _vp, _i32, _i32, _vp], _i32),
    "q35k_quantize_q8k_silu": ([_vp, _vp, _vp, _vp, _i32, _i32], _i32),
    "q35k_quantize_q8k_silu_dev": ([_vp, _vp, _vp, _vp, _i32, _i32, _vp], _i32),
    "q35k_dequantize": ([_vp, _i32, _vp, _vp, _i32, _i32], _i32),
    "q35k_dequantize_dev": ([_vp, _i32, _vp, _vp, _i32, _i32, _vp], _i32),
    "q35k_shard_create": ([_i32, ctypes.POINTER(_i32), _pp], _i32),
    "q35k_nccl_unique_id": ([_vp], _i32),
    "q35k_shard_create_rank": ([_i32, _i32, _vp, _i32, _pp], _i32),
    "q35k_shard_destroy": ([_vp], _i32),
    "q35k_shard_last_error": ([_vp], ctypes.c_char_p),
    "q35k_shard_info": ([_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(_i32)], _i32),
    "q35k_shard_sync": ([_vp], _i32),
    "q35k_shard_weight_upload": ([_vp, _i32, _vp, _i32, _i32, _pp], _i32),
    "q35k_shard_weight_free": ([_vp, _vp], _i32),
    "q35k_shard_matmul_dev": ([_vp, _vp, _pp, _pp, _i32, _i32, _pp], _i32),
    "q35k_shard_matmul": ([_vp, _vp, _vp, _vp, _i32, _i32], _i32),
    "q35k_shard_set_wait_limit": ([_vp, _i32], _i32),
    "q35k_shard_reset": ([_vp], _i32),
    "q35k_shard_set_trace": ([_vp, _i32], _i32),
    "q35k_shard_trace": ([_vp, _i32, ctypes.POINTER(ctypes.c_uint64)], _i32),
    "q35k_set_gemm_mode": ([_vp, _i32], _i32),
    "q35k_matmul_static_dev": ([_vp, _vp, _vp, _i32, _vp], _i32),
    "q35k_gguf_open": ([ctypes.c_char_p, _pp], _i32),
    "q35k_gguf_close": ([_vp], _i32),
    "q35k_gguf_info": ([_vp, ctypes.POINTER(_i32), ctypes.POINTER(_i32), ctypes.POINTER(ctypes.c_uint32),
                        ctypes.POINTER(ctypes.c_uint64)], _i32),
    "q35k_gguf_find": ([_vp, ctypes.c_char_p], _i32),
    "q35k_gguf_tensor": ([_vp, _i32, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_i32), ctypes.POINTER(_i32),
                          ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_uint64)], _i32),
    "q35k_gguf_tensor_data": ([_vp, _i32, _sz, _pp], _i32),
    "q35k_gguf_get_int": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)], _i32),
    "q35k_gguf_get_float": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_double)], _i32),
    "q35k_gguf_get_string": ([_vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p)], _i32),
    "q35k_gguf_get_array": ([_vp, ctypes.c_char_p, ctypes.POINTER(_i32), ctypes.POINTER(ctypes.c_uint64)], _i32),
    "q35k_weight_upload_gguf": ([_vp, _vp, ctypes.c_char_p, _pp], _i32),
}

_lib = None
_lock = threading.Lock()


class LibraryNotBuilt(ImportError):
    pass


def load() -> ctypes.CDLL:
    """Load libq35k.so and declare every exported entry point."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise LibraryNotBuilt(
                f"{LIB_PATH} is not built; run `python qwen3.5sharp_b200/build.py` (there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
        return L


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
