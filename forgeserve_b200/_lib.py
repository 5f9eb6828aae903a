"""ctypes binding of the C ABI in include/forgeserve_b200.h (libforgeserve_b200.so, built in-tree).

There is no CPU implementation behind this module: if the library is missing or no CUDA device is
available, every call raises instead of falling back to anything else.
"""

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libforgeserve_b200.so")

FS_F32, FS_BF16 = 0, 1
FS_EPI_STORE, FS_EPI_RESIDUAL, FS_EPI_SWIGLU = 0, 1, 2
FS_EPI_SYSTEM_FENCE = 0x100
FS_IPC_HANDLE_BYTES = 64
FS_ERR_WAIT_TIMEOUT, FS_ERR_BAD_TOKEN, FS_ERR_BAD_SLOT, FS_ERR_BAD_POSITION = 1, 2, 4, 8
FS_ATTN_AUTO, FS_ATTN_CUDA_CORE, FS_ATTN_MMA_SYNC, FS_ATTN_TCGEN05 = 0, 1, 2, 3

c_i64, c_int, c_float, c_vp = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p


class KVCacheDesc(ctypes.Structure):
    """Mirror of fs_kv_cache."""

    _fields_ = [
        ("k", c_vp),
        ("v", c_vp),
        ("table", c_vp),
        ("table_stride", c_i64),
        ("table_cols", c_i64),
        ("block_size", c_i64),
        ("block_stride", c_i64),
        ("head_stride", c_i64),
        ("num_blocks", c_i64),
    ]


# name -> (restype, argtypes); every symbol declared in include/forgeserve_b200.h
SIGNATURES = {
    "fs_version": (c_int, []),
    "fs_last_error": (ctypes.c_char_p, []),
    "fs_device_error": (c_int, [c_int, ctypes.POINTER(ctypes.c_uint)]),
    "fs_launch_count": (c_i64, []),
    "fs_wait_selftest": (c_int, [c_i64, c_vp, c_vp]),
    "fs_set_persistent_sms": (c_int, [c_int]),
    "fs_set_gemm_pair_mode": (c_int, [c_int]),
    "fs_ipc_handle": (c_int, [c_vp, c_vp, ctypes.POINTER(c_i64)]),
    "fs_ipc_open": (c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "fs_ipc_close": (c_int, [c_vp]),
    "fs_copy_2d": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_vp]),
    "fs_rmsnorm": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_float, c_int, c_vp]),
    "fs_gemm": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_int, c_int,
                        c_vp]),
    "fs_gemm_simt": (c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_int,
                             c_int, c_vp]),
    "fs_rope_kv_write": (c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, c_vp, ctypes.POINTER(KVCacheDesc), c_i64, c_i64,
                                 c_i64, c_i64, c_i64, c_i64, c_int, c_int, c_int, c_vp]),
    "fs_kv_store": (c_int, [c_vp, c_vp, c_vp, ctypes.POINTER(KVCacheDesc), c_i64, c_i64, c_i64, c_i64, c_int, c_vp]),
    "fs_paged_gather": (c_int, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_vp, c_int, c_vp]),
    "fs_attention": (c_int, [c_vp, c_i64, ctypes.POINTER(KVCacheDesc), c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i64,
                             c_i64, c_i64, c_float, c_int, c_vp]),
    "fs_attention_impl": (c_int, [c_vp, c_i64, ctypes.POINTER(KVCacheDesc), c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                  c_i64, c_i64, c_i64, c_float, c_int, c_int, c_vp]),
    "fs_attention_decode_workspace": (c_i64, [c_i64, c_i64, c_i64, c_i64, c_i64]),
    "fs_attention_decode": (c_int, [c_vp, c_i64, ctypes.POINTER(KVCacheDesc), c_i64, c_vp, c_vp, c_i64, c_i64, c_i64,
                                    c_i64, c_i64, c_float, c_vp, c_i64, c_int, c_vp]),
    "fs_attention_decode_static": (c_int, [c_vp, c_i64, ctypes.POINTER(KVCacheDesc), c_i64, c_vp, c_vp, c_i64, c_i64,
                                           c_i64, c_i64, c_i64, c_float, c_int, c_vp]),
    "fs_embed": (c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_vp, c_int, c_vp]),
    "fs_argmax": (c_int, [c_vp, c_i64, c_i64, c_i64, c_vp, c_int, c_vp]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the kernel library once (raises RuntimeError if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m forgeserve_b200.build` (needs nvcc). "
                    "forgeserve_b200 has no CPU fallback.")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = load().fs_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed: {msg}")


def launch_count() -> int:
    return int(load().fs_launch_count())


def device_error(clear: bool = True) -> int:
    """Device error bits (FS_ERR_*) of the current device; synchronises it."""
    bits = ctypes.c_uint(0)
    check(load().fs_device_error(int(clear), ctypes.byref(bits)), "fs_device_error")
    return int(bits.value)
