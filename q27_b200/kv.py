"""KV-cache formats, 64-row paging and the page pool: the host-side mirror of the
reference's ``KvKind`` (src/cuda_common.h:53), paged addressing (src/cuda_common.h:61-105),
``mk_tab`` (src/test_kernels.cu:27-36) and ``KvPool`` (src/kv_pool.h:24-72).

Device memory is held in torch tensors; every call into the engine goes through the C ABI.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib as L

KV_F16, KV_FP8, KV_T3 = 0, 1, 2
# From turbo3 up the V side is turbo3 blocks and only the K side varies: fp16 rows (turbo3v),
# 5-bit blocks (turbo5k), int8 blocks with a scale per 64 dims (int8-g64)
KV_T3V, KV_T5K, KV_I8G64 = 3, 4, 5
KV_PAGE = L.KV_PAGE
KIND_NAMES = {KV_F16: "fp16", KV_FP8: "fp8", KV_T3: "turbo3", KV_T3V: "turbo3v",
              KV_T5K: "turbo5k", KV_I8G64: "int8g64"}


def kv_k_rotated(kvk: int) -> bool:
    """Does K carry the WHT rotation, so that Q must be forward-rotated? (cuda_common.h:59)"""
    return kvk in (KV_T3, KV_T5K)


def row_bytes(kvk: int, n_kv_heads: int = 4, is_v: bool = False) -> int:
    """Bytes per cache row of one side of a kind (Engine::kv_bytes(is_v), src/engine.cuh:868)."""
    n = L.lib().q27_kv_row_bytes_side(kvk, n_kv_heads, int(is_v))
    if n < 0:
        raise L.Q27Error(L.ERR_UNSUPPORTED_KIND, "row_bytes")
    return int(n)


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def mk_tab(base: torch.Tensor, row_bytes_: int, rows: int) -> torch.Tensor:
    """Identity page table over a contiguous device buffer: entry j = base + j*64*row_bytes."""
    npages = (rows + KV_PAGE - 1) // KV_PAGE
    tab = torch.empty(max(npages, 1), dtype=torch.int64, device=base.device)
    L.check(L.lib().q27_mk_tab(base.data_ptr(), row_bytes_, rows, tab.data_ptr(),
                                stream_ptr()), "q27_mk_tab")
    return tab


@dataclass
class PagedSide:
    """One side (K or V) of a paged cache: backing bytes + its device page table."""
    data: torch.Tensor   # uint8 backing store (pages, possibly permuted)
    tab: torch.Tensor    # int64 device table of page pointers, logical page order
    rows: int


def paged_from_rows(rows_bytes: torch.Tensor, kvk: int, n_kv_heads: int = 4,
                    page_perm: torch.Tensor | None = None, is_v: bool = False) -> PagedSide:
    """Place logical cache rows (uint8 [rows, row_bytes], device) of one side into 64-row pages.

    With ``page_perm`` the pages are scattered: logical page j lives in physical page
    ``page_perm[j]`` (the reference's Q27_KV_SCATTER proof, src/engine.cuh:1294-1358).
    """
    rb = row_bytes(kvk, n_kv_heads, is_v)
    assert rows_bytes.dtype == torch.uint8 and rows_bytes.dim() == 2 and rows_bytes.shape[1] == rb
    rows = rows_bytes.shape[0]
    npages = max((rows + KV_PAGE - 1) // KV_PAGE, 1)
    page_bytes = KV_PAGE * rb
    store = torch.zeros(npages * page_bytes, dtype=torch.uint8, device=rows_bytes.device)
    if page_perm is None:
        store[: rows * rb] = rows_bytes.reshape(-1)
        tab = mk_tab(store, rb, rows)
        return PagedSide(store, tab, rows)
    perm = page_perm.to(device=rows_bytes.device, dtype=torch.int64)
    assert perm.numel() == npages
    padded = torch.zeros(npages * page_bytes, dtype=torch.uint8, device=rows_bytes.device)
    padded[: rows * rb] = rows_bytes.reshape(-1)
    store.view(npages, page_bytes)[perm] = padded.view(npages, page_bytes)
    tab = store.data_ptr() + perm * page_bytes
    return PagedSide(store, tab.contiguous(), rows)


class KvPool:
    """Process-wide page pool (src/kv_pool.h:24-72): two device allocations carved into
    64-row pages, LIFO free lists, ``page_ptr = base + idx * page_bytes``; no lock."""

    def __init__(self, k_bytes: int, v_bytes: int, k_row: int, v_row: int):
        self._h = L.lib().q27_kvpool_create(k_bytes, v_bytes, k_row, v_row)

    def enabled(self) -> bool:
        return bool(self._h)

    def npages(self, side: int) -> int:
        return L.lib().q27_kvpool_npages(self._h, side)

    def free_pages(self, side: int) -> int:
        return L.lib().q27_kvpool_free_pages(self._h, side)

    def page_bytes(self, side: int) -> int:
        return int(L.lib().q27_kvpool_page_bytes(self._h, side))

    def page_ptr(self, side: int, idx: int) -> int:
        return int(L.lib().q27_kvpool_page_ptr(self._h, side, idx) or 0)

    def reserve(self, side: int, n: int, out: list[int]) -> bool:
        buf = (C.c_int * max(n, 1))()
        if not L.lib().q27_kvpool_reserve(self._h, side, n, buf):
            return False
        out.extend(buf[i] for i in range(n))
        return True

    def release(self, side: int, pages: list[int]) -> None:
        buf = (C.c_int * max(len(pages), 1))(*pages)
        L.lib().q27_kvpool_release(self._h, side, buf, len(pages))
        pages.clear()

    def close(self) -> None:
        if self._h:
            L.lib().q27_kvpool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
