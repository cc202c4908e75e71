"""ctypes binding of libmvb200.so — the only door to the CUDA kernels.

Loading fails loudly (``RuntimeError``) when the library has not been built:
there is no CPU or Triton fallback behind this module.  The argument types
below mirror ``include/mini_vllm_b200.h`` one to one.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libmvb200.so")

# element-type codes (MVB_DTYPE_*)
DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2

# host status codes (MVB_OK / MVB_ERR_*)
OK = 0
ERR_INVALID_ARG = -1
ERR_DTYPE = -2
ERR_HEAD_DIM = -3
ERR_BLOCK_SIZE = -4
ERR_ALIGNMENT = -5
ERR_CUDA = -6
ERR_WORKSPACE = -7
ERR_TENSOR_MAP = -8
ERR_VARIANT = -9
ERR_HEADS = -10

# device error bits (MVB_DEV_*)
DEV_KV_LEN = 1
DEV_BLOCK_ID = 2
DEV_TABLE_SHORT = 4
DEV_SLOT_RANGE = 8
DEV_DUP_SLOT = 16
DEV_TIMEOUT = 32
DEV_POSITION = 64
DEV_SCHEDULE = 128

# decode variants (MVB_DECODE_*)
DECODE_AUTO = 0
DECODE_FMA = 1
DECODE_MMA = 2
DECODE_STREAM = 3
DECODE_SCHED = 4
# flags ORed into the decode variant (MVB_DECODE_AFTER_WRITE, MVB_DECODE_SCHEDULE_READY)
DECODE_AFTER_WRITE = 0x100
DECODE_SCHEDULE_READY = 0x200

ABI_VERSION = 6

# Every symbol include/mini_vllm_b200.h declares, with (restype, argtypes).
_i32, _i64, _u32, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_float, ctypes.c_void_p
_p_i32, _p_i64 = ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int64)
SIGNATURES = {
    "mvb_abi_version": (_i32, []),
    "mvb_status_string": (ctypes.c_char_p, [_i32]),
    "mvb_kv_cache_write": (
        _i32,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
         _vp, _u32, _vp, _vp],
    ),
    "mvb_paged_decode_plan": (
        _i32,
        [_i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp,
         _p_i32, _p_i32, _p_i32, _p_i64, _p_i32],
    ),
    "mvb_paged_decode": (
        _i32,
        [_vp, _i64, _i64, _vp, _vp, _vp, _i64, _i32, _vp, _vp, _i64, _i64,
         _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _i32, _vp, _i64, _vp, _vp],
    ),
    "mvb_paged_decode_schedule": (
        _i32,
        [_vp, _vp, _i64, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _i64, _vp, _vp],
    ),
    "mvb_paged_gather": (
        _i32,
        [_vp, _vp, _vp, _i64, _i64, _i32, _vp, _vp, _vp, _vp, _i32, _i64, _i32, _i32, _i32, _i32, _i32,
         _vp, _vp, _vp],
    ),
    "mvb_paged_prefill": (
        _i32,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _i32, _vp, _vp, _vp, _i32,
         _i32, _vp, _i64, _i64, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _vp],
    ),
    "mvb_rope_kv_cache_write": (
        _i32,
        [_vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _vp, _i64,
         _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _u32, _vp, _vp],
    ),
    "mvb_build_step_metadata": (
        _i32,
        [_vp, _vp, _vp, _vp, _vp, _i32, _i64, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp],
    ),
    "mvb_test_decode_wait_timeout": (
        _i32,
        [_vp, _i64, _i64, _vp, _vp, _vp, _i64, _i32, _vp, _vp, _i64, _i64,
         _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _vp, _i64, _vp, _vp, _i32, _i32, _i32, _i32],
    ),
    "mvb_paged_decode_noalloc": (
        _i32,
        [_vp, _i64, _i64, _vp, _vp, _vp, _i64, _i32, _vp, _vp, _i64, _i64,
         _i32, _i32, _i32, _i32, _i32, _i32, _f32, _i32, _i32, _i32, _vp, _vp],
    ),
}

_lib = None
_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load (once) and return the library with typed entry points."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libmvb200.so not found at {LIB_PATH}: build it with "
                "__graft_entry__.build() (the paged-attention path has no CPU fallback)"
            )
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.mvb_abi_version() != ABI_VERSION:
            raise RuntimeError(
                f"libmvb200.so ABI {handle.mvb_abi_version()} != expected {ABI_VERSION}; rebuild it"
            )
        _lib = handle
        return _lib


TORCH_BINDING_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "_mvb_torch.so")
_DEFAULT_LIB_PATH = LIB_PATH
_fast = None


def fast():
    """The direct binding of the per-step calls (``lib/_mvb_torch.so``), or
    None when another ``libmvb200.so`` than the in-tree one is selected (the
    binding is linked against the in-tree library; calls then go through
    ctypes).  Raises when the binding has not been built."""
    global _fast
    if _fast is not None:
        return _fast
    if LIB_PATH != _DEFAULT_LIB_PATH:
        return None
    lib()  # the library the binding links, loaded and version-checked first
    with _lock:
        if _fast is None:
            if not os.path.exists(TORCH_BINDING_PATH):
                raise RuntimeError(
                    f"_mvb_torch.so not found at {TORCH_BINDING_PATH}: build it with __graft_entry__.build()"
                )
            import importlib.util

            spec = importlib.util.spec_from_file_location("_mvb_torch", TORCH_BINDING_PATH)
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            _fast = mod
    return _fast


def status_string(status: int) -> str:
    return lib().mvb_status_string(status).decode()
