"""Host-side mirror of the reference's attention launch surface (same names, argument
meaning and error behaviour), over the C ABI:

* ``attn_decode``     <- q27k::attn_decode     (src/blocks.cuh:39-42)
* ``attn_decode3``    <- q27k::attn_decode3    (src/spec3.cuh:139-143)
* ``attn_prefill_T``  <- q27k::attn_prefill_T  (src/prefill.cuh:95-98)

plus the additive batched / sharded entries. Tensors are torch CUDA tensors owned by the
caller; nothing here allocates on the hot path except where a docstring says so.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib as L
from .kv import stream_ptr

INT_MAX = 2**31 - 1
FD_ST = L.PART_STRIDE


def decode_scratch_floats(ntok: int, n_q_heads: int = 24) -> int:
    return int(L.lib().q27_decode_scratch_floats(ntok, n_q_heads))


def prefill_part_floats(SB: int, n_q_heads: int = 24) -> int:
    return int(L.lib().q27_prefill_part_floats(SB, n_q_heads))


def _p3(tensors) -> L.P3:
    p = L.P3()
    for i, t in enumerate(tensors):
        p.p[i] = t.data_ptr() if isinstance(t, torch.Tensor) else int(t)
    return p


def attn_decode(q, q_stride, ktab, vtab, out, scratch, d_pos, max_ctx, n_q_heads, n_kv_heads,
                head_dim, scale, st=None, kvk=0):
    """Causal decode attention for one new token; seq_len = *d_pos + 1 read on device."""
    L.check(L.lib().q27_attn_decode(q.data_ptr(), q_stride, ktab.data_ptr(), vtab.data_ptr(),
                                    out.data_ptr(), scratch.data_ptr(), d_pos.data_ptr(), max_ctx,
                                    n_q_heads, n_kv_heads, head_dim, scale, stream_ptr(st), kvk),
            "q27_attn_decode")


def attn_decode3(q_lanes, q_stride, ktab, vtab, out_lanes, scratch, pos_lanes, max_ctx,
                 n_q_heads, n_kv_heads, head_dim, scale, st=None, ntok=3, kvk=0, wht=False):
    """ntok lanes against one pass over the cache; lane t attends cache[0 .. *pos_lanes[t]].

    q_lanes / out_lanes / pos_lanes: sequences of per-lane tensors (the reference's CP3 /
    P3 / IP3 bundles); entries beyond ntok are ignored. ``wht``: Q comes un-rotated and the
    output leaves un-rotated, the two rotations of the turbo kinds run inside the call."""
    q = _p3(q_lanes[:ntok])
    o = _p3(out_lanes[:ntok])
    p = _p3(pos_lanes[:ntok])
    fn = L.lib().q27_attn_decode3_wht if wht else L.lib().q27_attn_decode3
    L.check(fn(C.byref(q), q_stride, ktab.data_ptr(), vtab.data_ptr(), C.byref(o),
               scratch.data_ptr(), C.byref(p), max_ctx, n_q_heads, n_kv_heads, head_dim, scale,
               stream_ptr(st), ntok, kvk), "q27_attn_decode3")


def attn_verify_partials(q_lanes, q_stride, ktab, vtab, part, pos_lanes, n_kv_heads, gqa, head_dim,
                         scale, ns, st=None, kvk=0) -> bool:
    """The reference's fdmma::launch_fdmma / launch_fdmma_h16 (src/fdmma.cuh:460,808): ntok lanes
    against one pass over the cache, un-normalised partials at part[((t*n_q + h)*ns + sp)*258]
    for the caller's own combine. Returns False for a width that is not covered (the caller
    falls through), as the reference does."""
    ntok = len(q_lanes)
    q, p = _p3(q_lanes), _p3(pos_lanes)
    rc = L.lib().q27_attn_verify_partials(C.byref(q), q_stride, ktab.data_ptr(), vtab.data_ptr(),
                                          part.data_ptr(), C.byref(p), n_kv_heads, gqa, head_dim,
                                          scale, ns, ntok, stream_ptr(st), kvk)
    if rc == L.ERR_UNSUPPORTED_WIDTH:
        return False
    L.check(rc, "q27_attn_verify_partials")
    return True


def launch_count() -> int:
    """Kernels the library has launched from this thread so far."""
    return int(L.lib().q27_launch_count())


def attn_decode3_noalloc(q_lanes, q_stride, ktab, vtab, out_lanes, pos_lanes, n_q_heads,
                         n_kv_heads, head_dim, scale, st=None, ntok=1, kvk=0):
    """attn_decode3 for callers with no scratch buffer to give (no device allocator at
    hand, or allocation forbidden where they run): the split partials live in an array
    inside the library, sized for at most ``_lib.NOALLOC_MAX_LANES`` lanes. Calls share
    that array, so calls that overlap on the GPU race; the first call on a device should
    come before any stream capture."""
    q = _p3(q_lanes[:ntok])
    o = _p3(out_lanes[:ntok])
    p = _p3(pos_lanes[:ntok])
    L.check(L.lib().q27_attn_decode3_noalloc(C.byref(q), q_stride, ktab.data_ptr(),
                                             vtab.data_ptr(), C.byref(o), C.byref(p), n_q_heads,
                                             n_kv_heads, head_dim, scale, stream_ptr(st), ntok,
                                             kvk), "q27_attn_decode3_noalloc")


@dataclass
class SlotArgs:
    """One slot of a batched launch (q27_slot)."""
    ktab: torch.Tensor
    vtab: torch.Tensor
    q_lanes: list
    pos_lanes: list
    out_lanes: list = field(default_factory=list)
    scratch: torch.Tensor | None = None
    row_base: int = 0
    row_count: int = INT_MAX


def marshal_slots(slots) -> C.Array:
    """The q27_slot array of a list of SlotArgs, for callers that reuse it across steps (the
    caller keeps the SlotArgs alive)."""
    return _slots(slots)


def _slots(slots) -> C.Array:
    arr = (L.Slot * len(slots))()
    for i, s in enumerate(slots):
        arr[i].ktab = s.ktab.data_ptr()
        arr[i].vtab = s.vtab.data_ptr()
        arr[i].q = _p3(s.q_lanes)
        arr[i].pos = _p3(s.pos_lanes)
        arr[i].out = _p3(s.out_lanes)
        arr[i].scratch = s.scratch.data_ptr()
        arr[i].ntok = len(s.q_lanes)
        arr[i].row_base = s.row_base
        arr[i].row_count = s.row_count
    return arr


def attn_decode_batched(slots, q_stride, n_q_heads, n_kv_heads, head_dim, scale, st=None, kvk=0,
                        exact=False, wht=False):
    """All slots in one launch; per-slot semantics of attn_decode3."""
    arr = _slots(slots)
    if wht:
        L.check(L.lib().q27_attn_decode_batched_wht(arr, len(slots), q_stride, n_q_heads,
                                                    n_kv_heads, head_dim, scale, stream_ptr(st),
                                                    kvk, int(exact)), "q27_attn_decode_batched_wht")
        return
    fn = L.lib().q27_attn_decode_batched_exact if exact else L.lib().q27_attn_decode_batched
    L.check(fn(arr, len(slots), q_stride, n_q_heads, n_kv_heads, head_dim, scale, stream_ptr(st),
               kvk), "q27_attn_decode_batched")


class BatchedDecode:
    """attn_decode_batched with its argument block marshalled once. A decode loop calls the
    same slots every step (table, lane and scratch pointers are fixed for the life of the
    engine's captured graph; positions and Q change behind them), so the per-step cost on the
    host is one foreign call."""

    def __init__(self, slots, q_stride, n_q_heads, n_kv_heads, head_dim, scale, kvk=0,
                 exact=False, wht=False):
        self._keep = list(slots)                 # the tensors behind the raw pointers
        self._arr = _slots(self._keep)
        self._fn = (L.lib().q27_attn_decode_batched_wht if wht
                    else L.lib().q27_attn_decode_batched_exact if exact
                    else L.lib().q27_attn_decode_batched)
        self._args = (q_stride, n_q_heads, n_kv_heads, head_dim, scale)
        self._tail = (kvk, int(exact)) if wht else (kvk,)

    def __call__(self, st=None):
        L.check(self._fn(self._arr, len(self._keep), *self._args, stream_ptr(st), *self._tail),
                "q27_attn_decode_batched")


def attn_decode_partial(slots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim, scale,
                        partial_out, st=None, kvk=0, wht=False):
    """Un-normalised {m, l, acc} per (slot, lane, head) over each slot's row window."""
    arr = _slots(slots)
    fn = L.lib().q27_attn_decode_partial_wht if wht else L.lib().q27_attn_decode_partial
    L.check(fn(arr, len(slots), lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim, scale,
               partial_out.data_ptr(), stream_ptr(st), kvk), "q27_attn_decode_partial")


def attn_decode_partial_push(slots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim, scale,
                             mailboxes, rank, epoch, st=None, kvk=0, wht=False):
    """attn_decode_partial whose result lands in slot ``rank`` of every rank's mailbox
    (``mailboxes``: device addresses, one per rank, as mapped in this process)."""
    import ctypes as C
    arr = slots if isinstance(slots, C.Array) else _slots(slots)
    boxes = (C.c_void_p * len(mailboxes))(*mailboxes)
    fn = L.lib().q27_attn_decode_partial_push_wht if wht else L.lib().q27_attn_decode_partial_push
    L.check(fn(arr, len(arr), lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim, scale, boxes,
               len(mailboxes), rank, epoch, stream_ptr(st), kvk), "q27_attn_decode_partial_push")


def attn_decode_exchange(slots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim, scale,
                         mailboxes, rank, epoch, out, st=None, kvk=0, wht=False):
    """One sharded decode / verify step: partials, then combine + peer stores + wait + merge
    (one kernel when the rows fit the GPU at once); ``out`` [npairs][256] on every rank."""
    import ctypes as C
    arr = slots if isinstance(slots, C.Array) else _slots(slots)
    boxes = (C.c_void_p * len(mailboxes))(*mailboxes)
    L.check(L.lib().q27_attn_decode_exchange(arr, len(arr), lanes_stride, q_stride, n_q_heads,
                                             n_kv_heads, head_dim, scale, boxes, len(mailboxes), rank,
                                             epoch, out.data_ptr(), stream_ptr(st), kvk, int(wht)),
            "q27_attn_decode_exchange")


def attn_merge_pushed(mailbox, world, npairs, epoch, out, st=None, wht_kvk=None):
    """Device-side wait for every rank's push of ``epoch``, then the LSE merge into out.
    ``wht_kvk``: the cache kind, when the output rotation of that kind is to run here."""
    if wht_kvk is None:
        L.check(L.lib().q27_attn_merge_pushed(mailbox, world, npairs, epoch, out.data_ptr(),
                                              stream_ptr(st)), "q27_attn_merge_pushed")
    else:
        L.check(L.lib().q27_attn_merge_pushed_wht(mailbox, world, npairs, epoch, out.data_ptr(),
                                                  stream_ptr(st), wht_kvk), "q27_attn_merge_pushed_wht")


def attn_merge_partials(parts, nparts, npairs, out, st=None, wht_kvk=None):
    """LSE merge of ``nparts`` partial sets [nparts][npairs][258] -> out [npairs][256]."""
    if wht_kvk is None:
        L.check(L.lib().q27_attn_merge_partials(parts.data_ptr(), nparts, npairs, out.data_ptr(),
                                                stream_ptr(st)), "q27_attn_merge_partials")
    else:
        L.check(L.lib().q27_attn_merge_partials_wht(parts.data_ptr(), nparts, npairs,
                                                    out.data_ptr(), stream_ptr(st), wht_kvk),
                "q27_attn_merge_partials_wht")


def attn_prefill_T(qT, q_stride, q_row, ktab, vtab, outT, out_row, part, base_pos, t0, SB,
                   n_q_heads, n_kv_heads, head_dim, scale, st=None, kvk=0, exact=False, wht=False):
    """Causal GQA prefill attention for SB tokens starting at base_pos + t0."""
    if wht:
        L.check(L.lib().q27_attn_prefill_T_wht(
            qT.data_ptr(), q_stride, q_row, ktab.data_ptr(), vtab.data_ptr(), outT.data_ptr(),
            out_row, part.data_ptr() if part is not None else None, base_pos, t0, SB, n_q_heads,
            n_kv_heads, head_dim, scale, stream_ptr(st), kvk, int(exact)), "q27_attn_prefill_T_wht")
        return
    fn = L.lib().q27_attn_prefill_T_exact if exact else L.lib().q27_attn_prefill_T
    L.check(fn(qT.data_ptr(), q_stride, q_row, ktab.data_ptr(), vtab.data_ptr(), outT.data_ptr(),
               out_row, part.data_ptr() if part is not None else None, base_pos, t0, SB,
               n_q_heads, n_kv_heads, head_dim, scale, stream_ptr(st), kvk), "q27_attn_prefill_T")


def kv_dequant(tab, kvk, row0, nrows, n_kv_heads, out, st=None, is_v=False):
    """Bit-exact dequantisation of cache rows of one side to fp32 [nrows][n_kv_heads][256]."""
    L.check(L.lib().q27_kv_dequant_side(tab.data_ptr(), kvk, int(is_v), row0, nrows, n_kv_heads,
                                        out.data_ptr(), stream_ptr(st)), "q27_kv_dequant_side")


def kv_store_T(kT, vT, ktab, vtab, base_pos, rowlen, T, st=None, fp8=False):
    """Store T tokens' K/V rows (fp32 [T][rowlen]) at cache rows base_pos.. as fp16 / e4m3."""
    L.check(L.lib().q27_kv_store_T(kT.data_ptr(), vT.data_ptr(), ktab.data_ptr(), vtab.data_ptr(),
                                   base_pos, rowlen, T, stream_ptr(st), int(fp8)), "q27_kv_store_T")


def kv_store_T_t3(kT, vT, ktab, vtab, base_pos, n_kv_heads, head_dim, T, st=None, kvk=2):
    """Prefill store of the kinds from turbo3 up: per-128-group quantise of T tokens' V rows
    (turbo3) and K rows (the kind's K format)."""
    L.check(L.lib().q27_kv_store_T_t3(kT.data_ptr(), vT.data_ptr(), ktab.data_ptr(),
                                      vtab.data_ptr(), base_pos, n_kv_heads, head_dim, T,
                                      stream_ptr(st), kvk), "q27_kv_store_T_t3")


def wht_T(x, n_heads, head_dim, head_stride, row_stride, T, inv, st=None):
    """Per-128-group WHT rotate in place over a flat [T][row_stride] buffer."""
    L.check(L.lib().q27_wht_T(x.data_ptr(), n_heads, head_dim, head_stride, row_stride, T,
                              int(inv), stream_ptr(st)), "q27_wht_T")


def kv_store3(k_lanes, v_lanes, ktab, vtab, pos_lanes, rowlen, st=None, fp8=False):
    """Lane form of kv_store_T: lane t's fp32 K / V row to cache row *pos_lanes[t]."""
    import ctypes as C
    k, v, p = _p3(k_lanes), _p3(v_lanes), _p3(pos_lanes)
    L.check(L.lib().q27_kv_store3(C.byref(k), C.byref(v), ktab.data_ptr(), vtab.data_ptr(),
                                  C.byref(p), rowlen, stream_ptr(st), len(k_lanes), int(fp8)),
            "q27_kv_store3")


def kv_store_t3(k_lanes, v_lanes, ktab, vtab, pos_lanes, n_kv_heads, head_dim, st=None, kvk=2):
    """Lane form of kv_store_T_t3 (turbo3 encoder)."""
    import ctypes as C
    k, v, p = _p3(k_lanes), _p3(v_lanes), _p3(pos_lanes)
    L.check(L.lib().q27_kv_store_t3(C.byref(k), C.byref(v), ktab.data_ptr(), vtab.data_ptr(),
                                    C.byref(p), n_kv_heads, head_dim, stream_ptr(st),
                                    len(k_lanes), kvk), "q27_kv_store_t3")


def kv_store_lanes_shard(k_lanes, v_lanes, ktab, vtab, pos_lanes, n_kv_heads, head_dim, kvk,
                         row_base, row_count, st=None):
    """Lane-form store of any kind on a cache split by rows: only the lanes whose row falls in
    [row_base, row_base + row_count) are written, at row - row_base of these tables."""
    import ctypes as C
    k, v, p = _p3(k_lanes), _p3(v_lanes), _p3(pos_lanes)
    L.check(L.lib().q27_kv_store_lanes_shard(C.byref(k), C.byref(v), ktab.data_ptr(), vtab.data_ptr(),
                                             C.byref(p), n_kv_heads, head_dim, stream_ptr(st),
                                             len(k_lanes), kvk, row_base, row_count),
            "q27_kv_store_lanes_shard")


def kv_store_rows_shard(kT, vT, ktab, vtab, base_pos, n_kv_heads, head_dim, T, kvk, row_base,
                        row_count, st=None):
    """Chunk-form store (rows base_pos .. base_pos+T-1) of any kind on a cache split by rows."""
    L.check(L.lib().q27_kv_store_rows_shard(kT.data_ptr(), vT.data_ptr(), ktab.data_ptr(),
                                            vtab.data_ptr(), base_pos, n_kv_heads, head_dim, T,
                                            stream_ptr(st), kvk, row_base, row_count),
            "q27_kv_store_rows_shard")


def wht3(x_lanes, n_heads, head_dim, stride, inv, st=None):
    """Lane form of wht_T: rotate each lane's heads in place."""
    import ctypes as C
    x = _p3(x_lanes)
    L.check(L.lib().q27_wht3(C.byref(x), n_heads, head_dim, stride, int(inv), stream_ptr(st),
                             len(x_lanes)), "q27_wht3")
