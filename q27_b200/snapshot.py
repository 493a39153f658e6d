"""Pooled pages of a conversation and the row-ordered snapshot of its caches, on one GPU or
over a cache split by rows across several: the host-side mirror of the reference's
``kv_entitle`` / ``kv_release_for_takeover`` / ``kv_row_host`` (src/engine.cuh:781-845), of the
KV section of ``pfx_export`` / ``pfx_import`` (src/engine.cuh:3786-3857) and of the entry format
of its prefix cache (``PfxHdr``, ``pfx_fnv1a64``, ``pfx_compat_hash``: src/prefix_cache.h:44-82).

A blob holds, pair by pair, the K rows then the V rows of the first ``L + extra[pair]`` logical
rows, whatever pages (and whichever GPUs) they live in, so an entry written by one geometry
restores into any other. On a sharded cache every rank gathers ITS rows with one kernel, and
only those bytes travel to the rank that assembles or deals out the blob; planning is plain
host arithmetic (``shard_plan``), the transport is torch.distributed point-to-point (NCCL on
GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

import ctypes as C
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

from . import _lib as L
from .kv import KvPool, stream_ptr

PFX_MAGIC, PFX_VERSION, PFX_HDR_BYTES = 0x50373251, 1, 64
_FNV_SEED = 1469598103934665603
_HDR = struct.Struct("<IIQQiiQQQQ")           # PfxHdr, packed, 64 bytes
assert _HDR.size == PFX_HDR_BYTES


def _ints(v, n):
    if v is None:
        return None
    assert len(v) == n
    return (C.c_int * n)(*[int(x) for x in v])


class KvLineage:
    """Pool pages of one conversation on this GPU and the page tables over them."""

    def __init__(self, pool: KvPool, pairs: int, max_rows: int):
        self.pool, self.pairs, self.max_rows = pool, pairs, max_rows
        self._h = L.lib().q27_kvlineage_create(pool._h, pairs, max_rows)
        if not self._h:
            raise RuntimeError("q27_kvlineage_create failed (disabled pool or out of memory)")

    def entitle(self, rows: int, extra=None, st=None) -> bool:
        """Make rows [0, rows + extra[pair]) addressable; False = the pool lacks the pages and
        nothing changed (the caller refuses the request, src/engine.cuh:781-811)."""
        rc = L.lib().q27_kvlineage_entitle(self._h, rows, _ints(extra, self.pairs), stream_ptr(st))
        if rc < 0:
            raise ValueError("q27_kvlineage_entitle: invalid argument")
        return rc == 1

    def release(self) -> None:
        L.lib().q27_kvlineage_release(self._h)

    def rows(self) -> int:
        return L.lib().q27_kvlineage_rows(self._h)

    def pages_of(self, side: int, pair: int) -> int:
        return L.lib().q27_kvlineage_pages_of(self._h, side, pair)

    def tab(self, side: int, pair: int) -> "TablePtr":
        return TablePtr(int(L.lib().q27_kvlineage_tab(self._h, side, pair)))

    def row_ptr(self, side: int, pair: int, r: int) -> int:
        return int(L.lib().q27_kvlineage_row(self._h, side, pair, r) or 0)

    def row_bytes(self, side: int) -> int:
        return self.pool.page_bytes(side) // L.KV_PAGE

    def snapshot_bytes(self, nrows: int, extra=None) -> int:
        return int(L.lib().q27_kv_snapshot_bytes(self.pairs, nrows, _ints(extra, self.pairs),
                                                 self.row_bytes(0), self.row_bytes(1)))

    def export_rows(self, nrows: int, extra=None, row0: int = 0, st=None) -> torch.Tensor:
        """Rows [row0, row0 + nrows + extra[pair]) of every pair, gathered into a device blob."""
        n = self.snapshot_bytes(nrows, extra)
        blob = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda")[:n]
        L.check(L.lib().q27_kv_snapshot_export(self._h, row0, nrows, _ints(extra, self.pairs),
                                               blob.data_ptr(), stream_ptr(st)), "q27_kv_snapshot_export")
        return blob

    def import_rows(self, blob: torch.Tensor, nrows: int, extra=None, row0: int = 0, st=None) -> None:
        assert blob.is_cuda and blob.dtype == torch.uint8 and blob.numel() == self.snapshot_bytes(nrows, extra)
        L.check(L.lib().q27_kv_snapshot_import(self._h, row0, nrows, _ints(extra, self.pairs),
                                               blob.data_ptr(), stream_ptr(st)), "q27_kv_snapshot_import")

    def close(self) -> None:
        if self._h:
            L.lib().q27_kvlineage_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class TablePtr:
    """A device page table owned by a lineage, usable wherever a table tensor is."""
    ptr: int

    def data_ptr(self) -> int:
        return self.ptr


# ---- snapshot identity and the entry file (src/prefix_cache.h) ---------------------------------

def fnv1a64(data: bytes | np.ndarray, seed: int = _FNV_SEED) -> int:
    buf = np.ascontiguousarray(np.frombuffer(data, dtype=np.uint8) if isinstance(data, (bytes, bytearray))
                               else data)
    return int(L.lib().q27_pfx_fnv1a64(buf.ctypes.data, buf.nbytes, seed))


def token_key(tokens, n: int) -> int:
    """Key of an entry: FNV-1a over the first n tokens as int32 (src/prefix_cache.h:186,229)."""
    return fnv1a64(np.ascontiguousarray(np.asarray(tokens[:n], dtype=np.int32)))


def compat_hash(model_path: str, model_bytes: int, n_layer: int, n_kv: int, head_dim: int,
                gdn_heads: int, gdn_dim: int, gdn_ch: int, kv_kind: int,
                format_version: int = PFX_VERSION) -> int:
    return int(L.lib().q27_pfx_compat_hash(model_path.encode(), model_bytes, n_layer, n_kv, head_dim,
                                           gdn_heads, gdn_dim, gdn_ch, kv_kind, format_version))


def entry_name(tokens, n: int) -> str:
    return f"{token_key(tokens, n):016x}-{n}.q27pc"


def write_entry(root, tokens, n: int, compat: int, gdn: bytes, kv: bytes) -> Path:
    """One entry file: header, the n tokens, the recurrent-state bytes (opaque here), the KV
    blob. Written whole to a .tmp beside it, then renamed (src/prefix_cache.h:224-263)."""
    toks = np.ascontiguousarray(np.asarray(tokens[:n], dtype=np.int32))
    hdr = _HDR.pack(PFX_MAGIC, PFX_VERSION, compat, token_key(tokens, n), n, 0, len(gdn), len(kv), 0, 0)
    final = Path(root) / entry_name(tokens, n)
    tmp = final.with_name(final.name + ".tmp")
    with open(tmp, "wb") as f:
        f.write(hdr)
        f.write(toks.tobytes())
        f.write(gdn)
        f.write(kv)
        f.flush()
        os.fsync(f.fileno())
    os.rename(tmp, final)
    return final


def read_entry(path, prompt, compat: int):
    """(L, gdn bytes, kv bytes) if the file is a well-formed entry of this compatibility class
    whose stored tokens equal the first L tokens of ``prompt`` ELEMENT BY ELEMENT and leave at
    least one token to decode from; otherwise None. The name's hash only picks candidates
    (src/prefix_cache.h:14-23,170-199)."""
    with open(path, "rb") as f:
        raw = f.read(PFX_HDR_BYTES)
        if len(raw) != PFX_HDR_BYTES:
            return None
        magic, version, comp, tok_hash, n, _pad, gdn_n, kv_n, _r0, _r1 = _HDR.unpack(raw)
        if magic != PFX_MAGIC or version != PFX_VERSION or comp != compat or n <= 0:
            return None
        if n + 1 > len(prompt):
            return None
        stored = np.frombuffer(f.read(4 * n), dtype=np.int32)
        if stored.size != n or not np.array_equal(stored, np.asarray(prompt[:n], dtype=np.int32)):
            return None
        gdn, kv = f.read(gdn_n), f.read(kv_n)
        if len(gdn) != gdn_n or len(kv) != kv_n:
            return None
        return n, gdn, kv


# ---- a cache split by rows over several GPUs ----------------------------------------------------

def local_rows(nrows: int, extra, pairs: int, lo: int, hi: int):
    """(rows, extra) of the part of rows [0, nrows + extra[pair]) that falls in [lo, hi), as
    local row counts of the rank that owns [lo, hi)."""
    extra = [0] * pairs if extra is None else list(extra)
    clip = lambda n: min(max(n, lo), hi) - lo
    base = clip(nrows)
    return base, [clip(nrows + e) - base for e in extra]


@dataclass
class Segment:
    rank: int
    blob_off: int      # where the piece sits in the whole blob
    local_off: int     # where it sits in the rank's own (gathered) blob
    nbytes: int


def shard_plan(nrows: int, extra, pairs: int, k_row: int, v_row: int, ranges) -> list[Segment]:
    """Where each rank's rows sit in the whole blob: one segment per (pair, side, rank) that
    holds any row. ``ranges``: the ranks' logical row ranges, ascending and disjoint."""
    extra = [0] * pairs if extra is None else list(extra)
    segs, blob_off = [], 0
    local_off = [0] * len(ranges)
    for c in range(pairs):
        n = nrows + extra[c]
        for rb in (k_row, v_row):
            for r, (lo, hi) in enumerate(ranges):
                a, b = min(max(0, lo), n), min(hi, n)
                if b > a:
                    segs.append(Segment(r, blob_off + a * rb, local_off[r], (b - a) * rb))
                    local_off[r] += (b - a) * rb
            blob_off += n * rb
    return segs


def assemble(plan: list[Segment], total: int, parts: dict[int, torch.Tensor]) -> torch.Tensor:
    """The whole blob from the ranks' gathered pieces (host tensors)."""
    out = torch.zeros(total, dtype=torch.uint8)
    for s in plan:
        out[s.blob_off:s.blob_off + s.nbytes] = parts[s.rank][s.local_off:s.local_off + s.nbytes]
    return out


def deal_out(plan: list[Segment], blob: torch.Tensor, rank: int) -> torch.Tensor:
    """The bytes of the whole blob that belong to ``rank``, in its local blob order."""
    mine = [s for s in plan if s.rank == rank]
    n = sum(s.nbytes for s in mine)
    out = torch.empty(n, dtype=torch.uint8)
    for s in mine:
        out[s.local_off:s.local_off + s.nbytes] = blob[s.blob_off:s.blob_off + s.nbytes]
    return out


def blob_bytes(nrows: int, extra, pairs: int, k_row: int, v_row: int) -> int:
    extra = [0] * pairs if extra is None else list(extra)
    return sum((nrows + e) * (k_row + v_row) for e in extra)


def export_sharded(local_blob: torch.Tensor, nrows: int, extra, pairs: int, k_row: int, v_row: int,
                   ranges, group=None, dst: int = 0):
    """Collective: every rank hands in the blob of ITS rows (``KvLineage.export_rows`` with the
    counts of ``local_rows``); rank ``dst`` returns the whole blob (host uint8), the others None."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    plan = shard_plan(nrows, extra, pairs, k_row, v_row, ranges)
    sizes = [sum(s.nbytes for s in plan if s.rank == r) for r in range(world)]
    assert local_blob.numel() == sizes[rank]
    if rank != dst:
        if sizes[rank]:
            dist.send(local_blob.contiguous(), dst, group=group)
        return None
    parts = {}
    for r in range(world):
        if r == rank:
            parts[r] = local_blob.cpu()
        elif sizes[r]:
            buf = torch.empty(sizes[r], dtype=torch.uint8, device=local_blob.device)
            dist.recv(buf, r, group=group)
            parts[r] = buf.cpu()
    return assemble(plan, blob_bytes(nrows, extra, pairs, k_row, v_row), parts)


def import_sharded(blob, nrows: int, extra, pairs: int, k_row: int, v_row: int, ranges, device,
                   group=None, src: int = 0) -> torch.Tensor:
    """Collective inverse of export_sharded: rank ``src`` holds the whole blob (host uint8); every
    rank returns the blob of ITS rows on ``device``, ready for ``KvLineage.import_rows``."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    plan = shard_plan(nrows, extra, pairs, k_row, v_row, ranges)
    sizes = [sum(s.nbytes for s in plan if s.rank == r) for r in range(world)]
    if rank == src:
        assert blob.numel() == blob_bytes(nrows, extra, pairs, k_row, v_row)
        for r in range(world):
            if r != rank and sizes[r]:
                dist.send(deal_out(plan, blob, r).to(device), r, group=group)
        return deal_out(plan, blob, rank).to(device)
    mine = torch.empty(sizes[rank], dtype=torch.uint8, device=device)
    if sizes[rank]:
        dist.recv(mine, src, group=group)
    return mine
