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
from .attn import FD_ST, attn_decode_partial, attn_merge_partials

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
