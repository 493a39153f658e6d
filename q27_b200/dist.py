"""KV-sequence sharding across GPUs: each rank holds a contiguous, page-aligned range of
every slot's cache rows behind its own page tables, computes un-normalised partials
{m, l, acc[256]} over its range, and the ranks' partials are merged with the log-sum-exp
combine (the reference's k_attn_fd_combine, src/spec3.cu:706-739, applied across GPUs
instead of across its 128 intra-GPU splits). Only the 258-float partials cross NVLink; no
KV row ever leaves its GPU.

One process per GPU; plumbing is torch.distributed (NCCL on GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib as L
from .attn import (FD_ST, attn_decode_exchange, attn_decode_partial, attn_decode_partial_push,
                   attn_merge_partials, attn_merge_pushed)

KV_PAGE = L.KV_PAGE


def shard_ranges(total_rows: int, world: int) -> list[tuple[int, int]]:
    """Contiguous page-aligned [lo, hi) row ranges, one per rank, covering [0, total_rows).
    Every boundary but the last is a multiple of 64 rows; trailing ranks may be empty."""
    pages = (total_rows + KV_PAGE - 1) // KV_PAGE
    per = (pages + world - 1) // world
    out = []
    for r in range(world):
        lo = min(r * per * KV_PAGE, total_rows)
        hi = min((r + 1) * per * KV_PAGE, total_rows)
        out.append((lo, hi))
    return out


def owner_of_row(row: int, ranges: list[tuple[int, int]]) -> int:
    """Rank whose shard holds `row` (where a newly stored draft row must be routed)."""
    for r, (lo, hi) in enumerate(ranges):
        if lo <= row < hi:
            return r
    raise ValueError(f"row {row} outside every shard")


@dataclass
class PartialExchange:
    """Buffers and geometry of one partial exchange: [world][nslots][lanes][n_q][258]."""
    nslots: int
    lanes: int
    n_q: int
    world: int
    local: torch.Tensor
    gathered: torch.Tensor

    @staticmethod
    def create(nslots: int, lanes: int, n_q: int, world: int, device) -> "PartialExchange":
        local = torch.empty((nslots, lanes, n_q, FD_ST), dtype=torch.float32, device=device)
        gathered = torch.empty((world, nslots, lanes, n_q, FD_ST), dtype=torch.float32,
                               device=device)
        return PartialExchange(nslots, lanes, n_q, world, local, gathered)

    @property
    def npairs(self) -> int:
        return self.nslots * self.lanes * self.n_q

    def bytes_per_rank(self) -> int:
        return self.local.numel() * 4


def all_gather_partials(ex: PartialExchange, group=None) -> torch.Tensor:
    """The single exchange step: every rank ends up with every rank's partials."""
    if ex.world == 1:
        ex.gathered[0].copy_(ex.local)
    else:
        # flat views: the concatenated form is accepted by NCCL and gloo alike
        dist.all_gather_into_tensor(ex.gathered.view(-1), ex.local.view(-1), group=group)
    return ex.gathered


def sharded_decode(slots, ex: PartialExchange, out: torch.Tensor, q_stride: int, n_kv_heads: int,
                   scale: float, kvk: int, group=None, st=None) -> torch.Tensor:
    """Decode / verify attention over KV-sequence shards.

    `slots` are this rank's SlotArgs (tables over local rows, row_base / row_count set to
    the rank's range). `out` receives the normalised [nslots*lanes*n_q][256] rows on every
    rank."""
    attn_decode_partial(slots, ex.lanes, q_stride, ex.n_q, n_kv_heads, L.HEAD_DIM, scale,
                        ex.local, st=st, kvk=kvk)
    all_gather_partials(ex, group)
    attn_merge_partials(ex.gathered, ex.world, ex.npairs, out, st=st)
    return out


class PeerMailboxes:
    """Peer-memory exchange of partials: one mailbox per rank in that rank's HBM, mapped into
    every other rank's process with CUDA IPC (the ranks are the processes of one node, one
    GPU each). A step is `attn_decode_partial_push` (partials + combine, then peer stores of
    the 258-float rows into every mailbox and a release flag) followed by `attn_merge_pushed`
    (device-side bounded wait for all flags, then the merge): no collective call, no host
    synchronisation. The handles are exchanged once, with `all_gather_object`."""

    def __init__(self, nslots: int, lanes: int, n_q: int, group=None, device_epoch: bool = False):
        import ctypes as C
        # device_epoch: the mailbox counts the exchanges itself, so every step's launches have
        # the same arguments and a step (or several) can be captured in a CUDA graph
        self.device_epoch = device_epoch
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > L.MAX_RANKS:
            raise ValueError(f"at most {L.MAX_RANKS} ranks share a split")
        self.nslots, self.lanes, self.n_q = nslots, lanes, n_q
        self.npairs = nslots * lanes * n_q
        self.epoch = 0
        nbytes = L.lib().q27_xchg_mailbox_bytes(self.world, self.npairs)
        # Set-up is collective: a rank whose allocation or mapping fails still takes part in
        # every exchange below, and all ranks then raise together (a caller can fall back to
        # the NCCL exchange on every rank instead of hanging the others).
        own, handle = C.c_void_p(), C.create_string_buffer(L.XCHG_HANDLE_BYTES)
        rc = L.lib().q27_xchg_alloc(nbytes, C.byref(own), handle)
        self.own = own.value if rc == 0 else None
        self.boxes, self._opened = [], []
        mine = handle.raw if rc == 0 else None
        handles = [mine] * self.world
        if self.world > 1:
            dist.all_gather_object(handles, mine, group=group)
        ok = all(h is not None for h in handles)
        if ok:
            for r in range(self.world):
                if r == self.rank:
                    self.boxes.append(self.own)
                    continue
                ptr = C.c_void_p()
                if L.lib().q27_xchg_open(C.create_string_buffer(handles[r], L.XCHG_HANDLE_BYTES),
                                         C.byref(ptr)) != 0:
                    ok = False
                    break
                self.boxes.append(ptr.value)
                self._opened.append(ptr.value)
        if self.world > 1:
            oks = [ok] * self.world
            dist.all_gather_object(oks, ok, group=group)   # also: every mailbox is mapped
            ok = all(oks)
        if not ok:
            self.close(group)
            raise RuntimeError("peer-memory mailboxes could not be set up on every rank "
                               "(CUDA IPC allocation or mapping failed)")

    def bytes_per_rank(self) -> int:
        return self.npairs * FD_ST * 4

    def decode(self, slots, out: torch.Tensor, q_stride: int, n_kv_heads: int, scale: float,
               kvk: int, st=None, wht: bool = False, two_kernels: bool = False) -> torch.Tensor:
        """One sharded decode / verify step; `out` [npairs][256] normalised on every rank.
        ``two_kernels``: the push and the merge as separate calls (what the single call falls
        back to when the rows of a step do not fit the GPU at once)."""
        self.epoch += 1
        epoch = 0 if self.device_epoch else self.epoch
        if two_kernels:
            attn_decode_partial_push(slots, self.lanes, q_stride, self.n_q, n_kv_heads, L.HEAD_DIM,
                                     scale, self.boxes, self.rank, epoch, st=st, kvk=kvk, wht=wht)
            attn_merge_pushed(self.own, self.world, self.npairs, epoch, out, st=st,
                              wht_kvk=kvk if wht else None)
        else:
            attn_decode_exchange(slots, self.lanes, q_stride, self.n_q, n_kv_heads, L.HEAD_DIM, scale,
                                 self.boxes, self.rank, epoch, out, st=st, kvk=kvk, wht=wht)
        return out

    def close(self, group=None):
        """Unmap the peers' mailboxes, then (after a barrier) free the own one."""
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        for ptr in self._opened:
            L.lib().q27_xchg_close(ptr)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=group)
        if self.own:
            L.check(L.lib().q27_xchg_free(self.own), "q27_xchg_free")
            self.own = None
