"""ctypes binding of the C ABI in ``include/starkv_b200.h``.

This module is the only place Python touches the native library. There is no
fallback: if the library is missing or fails to load, every operator raises.
The struct layouts below mirror the header field for field; ``check_abi()``
compares their sizes with the library's own ``starkv_abi_sizeof``.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libstarkv_b200.so")

F16, BF16, F32, U8, I32, I64 = 0, 1, 2, 3, 4, 5
_DTYPES = {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32, torch.uint8: U8,
           torch.int32: I32, torch.int64: I64}

STATUS = {
    0: "ok", 22: "EINVAL", 100: "EALIGN", 101: "EDTYPE", 102: "EWORKSPACE", 103: "ECUDA",
    104: "ENODEV", 105: "EBOUNDS", 106: "ETIMEOUT",
}

p, i32, i64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float


class DecodeArgs(C.Structure):
    _fields_ = [
        ("query", p), ("q_stride", i64 * 3), ("q_dtype", i32),
        ("kv_cache", p), ("cache_stride", i64 * 3), ("cache_dtype", i32),
        ("num_blocks", i32), ("block_size", i32),
        ("block_table", p), ("bt_stride", i64 * 2), ("max_blocks", i32),
        ("seq_lens", p),
        ("n", i32), ("num_heads", i32), ("num_kv_heads", i32), ("head_dim", i32),
        ("max_seq_len", i32),
        ("k_up", p), ("k_up_stride", i64 * 2), ("k_up_dtype", i32),
        ("k_ranks", p), ("k_head_offsets", p),
        ("k_width", i32),
        ("v_up_by_q", p), ("v_up_stride", i64 * 3), ("v_up_dtype", i32),
        ("v_rank", i32),
        ("cos_sin_cache", p), ("cs_stride", i64 * 2), ("cs_dtype", i32), ("cs_rows", i32),
        ("scale", f32),
        ("out", p), ("out_stride", i64 * 3), ("out_dtype", i32),
        ("row_nbytes", i32), ("ks_off", i32), ("vs_off", i32), ("vq_off", i32),
        ("v_nout", i32), ("v_nbo", i32), ("v_bytes", i32),
        ("head_of_lane", p),
        ("tile_head", p), ("tile_nout", p), ("tile_last", p),
    ]


class PackArgs(C.Structure):
    _fields_ = [
        ("k_codes", p), ("k_stride0", i64), ("k_dtype", i32),
        ("v_codes", p), ("v_stride0", i64), ("v_dtype", i32),
        ("cache", p), ("cache_stride", i64 * 2),
        ("num_blocks", i32), ("block_size", i32),
        ("slot_mapping", p), ("slot_dtype", i32),
        ("n", i32), ("num_kv_heads", i32), ("k_width", i32), ("v_rank", i32),
        ("k_ranks", p), ("k_offsets", p), ("k_nouts", p),
        ("ks_off", i32), ("vs_off", i32), ("vq_off", i32), ("v_nout", i32), ("v_nbo", i32), ("v_bytes", i32),
        ("status", p),
    ]


class CacheWriteArgs(C.Structure):
    _fields_ = [
        ("key", p), ("key_stride0", i64), ("key_dtype", i32),
        ("value", p), ("value_stride0", i64), ("value_dtype", i32),
        ("cache", p), ("cache_stride", i64 * 3), ("cache_dtype", i32),
        ("num_blocks", i32), ("block_size", i32),
        ("slot_mapping", p), ("slot_dtype", i32),
        ("n", i32), ("k_width", i32), ("v_rank", i32),
        ("status", p),
    ]


EXPORTS = {
    "starkv_decode_workspace_bytes": (C.c_size_t, [i32, i32, i32, i32, i32, i32]),
    "starkv_paged_decode_bf16": (C.c_int, [C.POINTER(DecodeArgs), p, C.c_size_t, p]),
    "starkv_paged_decode_q32": (C.c_int, [C.POINTER(DecodeArgs), p, C.c_size_t, p]),
    "starkv_paged_decode_bf16_noalloc": (C.c_int, [C.POINTER(DecodeArgs), p]),
    "starkv_noalloc_read_status": (C.c_int, [C.POINTER(i32), i32, p]),
    "starkv_paged_decode_bf16_partial": (C.c_int, [C.POINTER(DecodeArgs), i32, i32, p, p, p, C.c_size_t, p]),
    "starkv_paged_decode_q32_partial": (C.c_int, [C.POINTER(DecodeArgs), i32, i32, p, p, p, C.c_size_t, p]),
    "starkv_cp_combine": (C.c_int, [p, i32, i32, i32, p, C.POINTER(i64), i32, p]),
    "starkv_selftest_wait_timeout": (C.c_int, [p, p]),
    "starkv_fold_q": (C.c_int, [p, C.POINTER(i64), i32, p, C.POINTER(i64), i32, p, i32, i32, i32, f32, p, p, p]),
    "starkv_pack_kv_q32": (C.c_int, [C.POINTER(PackArgs), p]),
    "starkv_kv_down_cache_write": (C.c_int, [p, i64, p, i64, i32, i32, i32, i32, p, C.POINTER(i64), i32, i32, p, i32,
                                             p, p]),
    "starkv_prefill_attention": (C.c_int, [p, C.POINTER(i64), p, C.POINTER(i64), p, C.POINTER(i64), i32, i32, i32, i32,
                                           i32, p, i32, i32, f32, p, C.POINTER(i64), p, p]),
    "starkv_cache_write_bf16": (C.c_int, [C.POINTER(CacheWriteArgs), p]),
    "starkv_read_status": (C.c_int, [p, C.POINTER(i32), i32, p]),
    "starkv_status_offset": (C.c_size_t, []),
    "starkv_abi_sizeof": (C.c_size_t, [i32]),
    "starkv_profile_begin": (C.c_int, [i32]),
    "starkv_profile_end": (C.c_int, [C.POINTER(f32), C.POINTER(i32)]),
    "starkv_version": (C.c_char_p, []),
    "starkv_strerror": (C.c_char_p, [C.c_int]),
}

_lib = None


def lib() -> C.CDLL:
    """Load the native library once; raise if it is not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"starkv_b200 native library not built: {LIB_PATH} "
                               "(run python star-kv-serve_b200/build.py)")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in EXPORTS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def check_abi() -> None:
    L = lib()
    for which, cls in enumerate((DecodeArgs, PackArgs, CacheWriteArgs)):
        got = L.starkv_abi_sizeof(which)
        if got != C.sizeof(cls):
            raise RuntimeError(f"ABI mismatch for {cls.__name__}: library {got} B, binding {C.sizeof(cls)} B")


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().starkv_strerror(status).decode()
        if status in (22, 101):
            raise ValueError(f"{what}: {msg} ({STATUS.get(status, status)})")
        raise RuntimeError(f"{what}: {msg} ({STATUS.get(status, status)})")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def i64s(values):
    arr = (i64 * len(values))(*[int(v) for v in values])
    return arr
