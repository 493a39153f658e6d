"""ctypes binding of the C ABI declared in include/q27_b200.h.

The shared library is built in-tree by ``python -m q27_b200.build``. There is no fallback:
if the library is missing, importing this module raises, and every call that needs a GPU
fails with the library's own status code.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libq27_b200.so"

MAX_LANES = 16
MAX_SLOTS = 8
MAX_SPLITS = 128
XCHG_HANDLE_BYTES = 64
MAX_RANKS = 8
NOALLOC_MAX_LANES = 4
PART_STRIDE = 258
KV_PAGE = 64
HEAD_DIM = 256
GQA = 6
T3_BLOCK_BYTES = 50
T5_BLOCK_BYTES = 82
I8_BLOCK_BYTES = 132

OK, ERR_INVALID_ARG, ERR_UNSUPPORTED_KIND, ERR_UNSUPPORTED_WIDTH, ERR_CUDA, ERR_TOO_LARGE = range(6)


class P3(C.Structure):
    _fields_ = [("p", C.c_void_p * MAX_LANES)]


class Slot(C.Structure):
    _fields_ = [
        ("ktab", C.c_void_p),
        ("vtab", C.c_void_p),
        ("q", P3),
        ("pos", P3),
        ("out", P3),
        ("scratch", C.c_void_p),
        ("ntok", C.c_int),
        ("row_base", C.c_int),
        ("row_count", C.c_int),
        ("reserved", C.c_int),
    ]


# name -> (restype, argtypes); mirrors include/q27_b200.h one to one
_vp, _i, _f, _i64, _sz = C.c_void_p, C.c_int, C.c_float, C.c_int64, C.c_size_t
SIGNATURES = {
    "q27_status_string": (C.c_char_p, [_i]),
    "q27_last_cuda_error": (_i, []),
    "q27_device_arch": (_i, []),
    "q27_launch_count": (C.c_longlong, []),
    "q27_wait_timeout_flag": (_i, [C.POINTER(_i)]),
    "q27_set_kernel_events": (_i, [_vp, _vp]),
    "q27_kv_row_bytes": (_i64, [_i, _i]),
    "q27_kv_row_bytes_side": (_i64, [_i, _i, _i]),
    "q27_decode_scratch_floats": (_i64, [_i, _i]),
    "q27_prefill_part_floats": (_i64, [_i, _i]),
    "q27_attn_decode": (_i, [_vp, _i, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _f, _vp, _i]),
    "q27_attn_decode3": (_i, [C.POINTER(P3), _i, _vp, _vp, C.POINTER(P3), _vp, C.POINTER(P3),
                              _i, _i, _i, _i, _f, _vp, _i, _i]),
    "q27_attn_verify_partials": (_i, [C.POINTER(P3), _i, _vp, _vp, _vp, C.POINTER(P3), _i, _i, _i,
                                      _f, _i, _i, _vp, _i]),
    "q27_attn_decode3_noalloc": (_i, [C.POINTER(P3), _i, _vp, _vp, C.POINTER(P3), C.POINTER(P3),
                                      _i, _i, _i, _f, _vp, _i, _i]),
    "q27_attn_decode_batched": (_i, [C.POINTER(Slot), _i, _i, _i, _i, _i, _f, _vp, _i]),
    "q27_attn_decode_batched_exact": (_i, [C.POINTER(Slot), _i, _i, _i, _i, _i, _f, _vp, _i]),
    "q27_attn_decode_partial": (_i, [C.POINTER(Slot), _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _i]),
    "q27_attn_merge_partials": (_i, [_vp, _i, _i64, _vp, _vp]),
    "q27_xchg_alloc": (_i, [_sz, C.POINTER(_vp), _vp]),
    "q27_xchg_open": (_i, [_vp, C.POINTER(_vp)]),
    "q27_xchg_close": (_i, [_vp]),
    "q27_xchg_free": (_i, [_vp]),
    "q27_xchg_mailbox_bytes": (_sz, [_i, _i64]),
    "q27_attn_decode_partial_push": (_i, [C.POINTER(Slot), _i, _i, _i, _i, _i, _i, _f,
                                          C.POINTER(_vp), _i, _i, C.c_uint, _vp, _i]),
    "q27_attn_merge_pushed": (_i, [_vp, _i, _i64, C.c_uint, _vp, _vp]),
    "q27_attn_decode_exchange": (_i, [C.POINTER(Slot), _i, _i, _i, _i, _i, _i, _f, C.POINTER(_vp), _i,
                                      _i, C.c_uint, _vp, _vp, _i, _i]),
    "q27_attn_prefill_T": (_i, [_vp, _i, _i, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _f,
                                _vp, _i]),
    "q27_attn_prefill_T_exact": (_i, [_vp, _i, _i, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i,
                                      _f, _vp, _i]),
    "q27_attn_decode3_wht": (_i, [C.POINTER(P3), _i, _vp, _vp, C.POINTER(P3), _vp, C.POINTER(P3),
                                  _i, _i, _i, _i, _f, _vp, _i, _i]),
    "q27_attn_decode_batched_wht": (_i, [C.POINTER(Slot), _i, _i, _i, _i, _i, _f, _vp, _i, _i]),
    "q27_attn_prefill_T_wht": (_i, [_vp, _i, _i, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _f,
                                    _vp, _i, _i]),
    "q27_attn_decode_partial_wht": (_i, [C.POINTER(Slot), _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _i]),
    "q27_attn_merge_partials_wht": (_i, [_vp, _i, _i64, _vp, _vp, _i]),
    "q27_attn_decode_partial_push_wht": (_i, [C.POINTER(Slot), _i, _i, _i, _i, _i, _i, _f,
                                              C.POINTER(_vp), _i, _i, C.c_uint, _vp, _i]),
    "q27_attn_merge_pushed_wht": (_i, [_vp, _i, _i64, C.c_uint, _vp, _vp, _i]),
    "q27_kv_dequant": (_i, [_vp, _i, _i, _i, _i, _vp, _vp]),
    "q27_kv_dequant_side": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp]),
    "q27_kv_store_T": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _i]),
    "q27_kv_store_T_t3": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _i]),
    "q27_wht_T": (_i, [_vp, _i, _i, _i, _i, _i, _i, _vp]),
    "q27_kv_store3": (_i, [C.POINTER(P3), C.POINTER(P3), _vp, _vp, C.POINTER(P3), _i, _vp, _i, _i]),
    "q27_kv_store_t3": (_i, [C.POINTER(P3), C.POINTER(P3), _vp, _vp, C.POINTER(P3), _i, _i, _vp, _i,
                             _i]),
    "q27_wht3": (_i, [C.POINTER(P3), _i, _i, _i, _i, _vp, _i]),
    "q27_kv_store_lanes_shard": (_i, [C.POINTER(P3), C.POINTER(P3), _vp, _vp, C.POINTER(P3), _i, _i,
                                      _vp, _i, _i, _i, _i]),
    "q27_kv_store_rows_shard": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _i, _i, _i]),
    "q27_mk_tab": (_i, [_vp, _sz, _i, _vp, _vp]),
    "q27_kvpool_create": (_vp, [_sz, _sz, _sz, _sz]),
    "q27_kvpool_destroy": (None, [_vp]),
    "q27_kvpool_npages": (_i, [_vp, _i]),
    "q27_kvpool_free_pages": (_i, [_vp, _i]),
    "q27_kvpool_page_bytes": (_sz, [_vp, _i]),
    "q27_kvpool_page_ptr": (_vp, [_vp, _i, _i]),
    "q27_kvpool_reserve": (_i, [_vp, _i, _i, C.POINTER(_i)]),
    "q27_kvpool_release": (None, [_vp, _i, C.POINTER(_i), _i]),
    "q27_kvlineage_create": (_vp, [_vp, _i, _i]),
    "q27_kvlineage_destroy": (None, [_vp]),
    "q27_kvlineage_entitle": (_i, [_vp, _i, C.POINTER(_i), _vp]),
    "q27_kvlineage_release": (None, [_vp]),
    "q27_kvlineage_rows": (_i, [_vp]),
    "q27_kvlineage_npages": (_i, [_vp]),
    "q27_kvlineage_pages_of": (_i, [_vp, _i, _i]),
    "q27_kvlineage_tab": (_vp, [_vp, _i, _i]),
    "q27_kvlineage_row": (_vp, [_vp, _i, _i, _i]),
    "q27_kv_snapshot_bytes": (_i64, [_i, _i, C.POINTER(_i), _sz, _sz]),
    "q27_kv_snapshot_export": (_i, [_vp, _i, _i, C.POINTER(_i), _vp, _vp]),
    "q27_kv_snapshot_import": (_i, [_vp, _i, _i, C.POINTER(_i), _vp, _vp]),
    "q27_pfx_fnv1a64": (C.c_uint64, [_vp, _sz, C.c_uint64]),
    "q27_pfx_compat_hash": (C.c_uint64, [C.c_char_p, C.c_uint64, _i, _i, _i, _i, _i, _i, _i, _i]),
}

_lib = None


class Q27Error(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        msg = lib().q27_status_string(status).decode()
        if status == ERR_CUDA:
            msg += f" [cudaError {lib().q27_last_cuda_error()}]"
        super().__init__(f"{where}: {msg} (status {status})")


def lib() -> C.CDLL:
    """Load (once) and return the shared library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m q27_b200.build` "
                "(there is no CPU or PyTorch fallback for this engine)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)  # AttributeError here = header/library drift
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(status: int, where: str) -> None:
    if status != OK:
        raise Q27Error(status, where)
