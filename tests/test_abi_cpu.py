"""CPU checks of the drop-in boundary: the C-ABI library loads and exports every symbol
include/q27_b200.h declares, argument validation answers without a GPU, and the ctypes
layer mirrors the header."""
import ctypes as C
import re
from pathlib import Path

import q27_b200
from q27_b200 import _lib as L

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    text = (ROOT / "include" / "q27_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q27_[A-Za-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported_and_bound():
    names = declared_functions()
    assert len(names) >= 20
    handle = C.CDLL(str(L.LIB_PATH))
    for n in names:
        assert hasattr(handle, n), f"{n} declared in the header but not exported"
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"
    assert sorted(L.SIGNATURES) == names


def test_struct_layout_matches_header():
    assert C.sizeof(L.P3) == 16 * 8
    assert C.sizeof(L.Slot) == 8 + 8 + 3 * 128 + 8 + 16
    assert L.Slot.scratch.offset == 16 + 3 * 128


def test_sizes_and_status_strings():
    lib = L.lib()
    assert lib.q27_kv_row_bytes(0, 4) == 2048 and lib.q27_kv_row_bytes(1, 4) == 1024
    assert lib.q27_kv_row_bytes(2, 4) == 400
    # kinds whose sides differ: K side by default (656 / 1056 B per row, src/server.cu:891-892),
    # V side turbo3 (Engine::kv_bytes, src/engine.cuh:868-876)
    assert [lib.q27_kv_row_bytes(k, 4) for k in (3, 4, 5)] == [2048, 656, 1056]
    assert [lib.q27_kv_row_bytes_side(k, 4, 1) for k in (2, 3, 4, 5)] == [400] * 4
    assert [lib.q27_kv_row_bytes_side(k, 4, 0) for k in (0, 1, 2)] == [2048, 1024, 400]
    for refused in (6, -1):         # outside the enum: refused, never mis-read
        assert lib.q27_kv_row_bytes(refused, 4) == -1 and lib.q27_kv_row_bytes_side(refused, 4, 1) == -1
    # ntok * n_q_heads * FD_MAXNS * FD_ST floats (src/spec3.cuh:109-127)
    assert q27_b200.decode_scratch_floats(12) == 12 * 24 * 128 * 258
    # n_q_heads * SB_rounded_to_16 * PF_SPLIT_MAX * 258 (src/prefill.cuh:86-88)
    assert q27_b200.prefill_part_floats(1000) == 24 * 1008 * 8 * 258
    assert lib.q27_status_string(2).decode().startswith("unsupported KV kind")


def test_validation_needs_no_gpu():
    lib = L.lib()
    one = 0x1000  # never dereferenced: validation fails first
    q = L.P3()
    q.p[0] = one
    # kinds outside the enum
    for kvk in (6, -1, 99):
        rc = lib.q27_attn_decode3(C.byref(q), 512, one, one, C.byref(q), one, C.byref(q), 0, 24, 4,
                                  256, 0.0625, None, 1, kvk)
        assert rc == L.ERR_UNSUPPORTED_KIND
    # widths outside 1..16 (the reference's `false`: caller must fall through)
    for ntok in (0, 17):
        rc = lib.q27_attn_decode3(C.byref(q), 512, one, one, C.byref(q), one, C.byref(q), 0, 24, 4,
                                  256, 0.0625, None, ntok, 0)
        assert rc == L.ERR_UNSUPPORTED_WIDTH
    # geometry other than 24/4/256
    assert lib.q27_attn_decode3(C.byref(q), 512, one, one, C.byref(q), one, C.byref(q), 0, 32, 4,
                                256, 0.0625, None, 1, 0) == L.ERR_UNSUPPORTED_WIDTH
    assert lib.q27_attn_decode3(C.byref(q), 512, one, one, C.byref(q), one, C.byref(q), 0, 24, 4,
                                128, 0.0625, None, 1, 0) == L.ERR_UNSUPPORTED_WIDTH
    # null pointers
    assert lib.q27_attn_decode(None, 512, one, one, one, one, one, 0, 24, 4, 256, 0.0625, None,
                               0) == L.ERR_INVALID_ARG
    assert lib.q27_attn_prefill_T(None, 512, 12288, one, one, one, 6144, None, 0, 0, 8, 24, 4, 256,
                                  0.0625, None, 0) == L.ERR_INVALID_ARG
    assert lib.q27_attn_prefill_T(one, 512, 12288, one, one, one, 6144, None, 0, 0, 8, 24, 4, 256,
                                  0.0625, None, 6) == L.ERR_UNSUPPORTED_KIND
    assert lib.q27_kv_dequant(one, 6, 0, 1, 4, one, None) == L.ERR_UNSUPPORTED_KIND
    assert lib.q27_kv_dequant_side(one, -1, 1, 0, 1, 4, one, None) == L.ERR_UNSUPPORTED_KIND
    # the block stores serve the kinds from turbo3 up; fp16 / fp8 have their own entry
    assert lib.q27_kv_store_T_t3(one, one, one, one, 0, 4, 256, 1, None, 1) == L.ERR_UNSUPPORTED_KIND
    assert lib.q27_kv_store_T_t3(one, one, one, one, 0, 4, 256, 1, None, 6) == L.ERR_UNSUPPORTED_KIND
    assert lib.q27_attn_merge_partials(None, 2, 10, one, None) == L.ERR_INVALID_ARG


def test_kvpool_disabled_without_pages():
    # either side with zero pages -> pool disabled (src/kv_pool.h:35-41); no GPU touched
    p = q27_b200.KvPool(100, 100, 2048, 2048)
    assert not p.enabled() and p.npages(0) == 0 and p.free_pages(1) == 0
