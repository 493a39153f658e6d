"""GPU tests of pooled lineages, the row-ordered snapshot of their caches and the stores that
route rows to their owner on a cache split by rows (emulated here as several lineages on one
GPU; tests/test_multi_gpu.py runs the collective form on real ranks).

Gates: kv_entitle's all-or-nothing and aliasing rules (src/engine.cuh:781-811); the exported
blob equals the numpy restatement of pfx_export's walk (oracle/snapshot_oracle.py) byte for
byte whatever pages the rows live in; a blob imports into another pool geometry and another
number of owners and the cache then reads back bit-identically and attends identically."""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import q27_b200 as Q
from q27_b200 import snapshot as S
from q27_b200.dist import shard_ranges
from tests import synth
from tests.gpu_util import SCALE
from tests.oracle_lib import KV_F16, KV_T3, KV_T5K

sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "oracle"))
import snapshot_oracle as SO  # noqa: E402

pytestmark = pytest.mark.gpu
PAIRS, EXTRA = 3, [0, 0, 1]          # two attention layers and a draft-head pair one row longer


def make_pool(kvk, pages_k, pages_v):
    rk, rv = Q.row_bytes(kvk), Q.row_bytes(kvk, is_v=True)
    pool = Q.KvPool(pages_k * 64 * rk + 5, pages_v * 64 * rv + 5, rk, rv)   # rounded DOWN to pages
    assert pool.enabled() and pool.npages(0) == pages_k and pool.npages(1) == pages_v
    return pool


def test_entitle_is_all_or_nothing_and_tables_alias_the_first_page(cuda):
    pool = make_pool(KV_T3, 12, 12)
    lin = Q.KvLineage(pool, PAIRS, 64 * 6)
    assert lin.entitle(100, EXTRA)                     # 2 pages per pair and side
    assert [lin.pages_of(s, c) for s in (0, 1) for c in range(PAIRS)] == [2] * 6
    assert pool.free_pages(0) == 6 and lin.rows() == 100
    assert lin.entitle(128, EXTRA)                     # the draft pair needs row 128: one more page
    assert [lin.pages_of(0, c) for c in range(PAIRS)] == [2, 2, 3] and pool.free_pages(0) == 5
    assert not lin.entitle(300, EXTRA)                 # 5 pages per pair: not there -> nothing taken
    assert pool.free_pages(0) == 5 and lin.rows() == 128
    assert lin.entitle(64, EXTRA) and lin.rows() == 128          # never shrinks
    # the table: owned pages in order, every later entry aliases the pair's first page
    t = [lin.row_ptr(0, 2, 64 * j) for j in range(6)]
    assert len(set(t[:3])) == 3 and t[3:] == [t[0]] * 3
    assert lin.row_ptr(0, 2, 70) == t[1] + 6 * Q.row_bytes(KV_T3)           # kv_row_host
    lin.release()
    assert pool.free_pages(0) == 12 and pool.free_pages(1) == 12 and lin.rows() == 0
    lin.close()
    pool.close()


def fill(oracle, lin, kvk, rows, seed, row_base=0, row_count=2**31 - 1):
    """Store `rows` rows (+1 in the draft pair) of every pair through the lineage's tables with
    the chunk-form store; returns the CPU-encoded logical rows per pair."""
    ks, vs = [], []
    for c in range(PAIRS):
        n = rows + EXTRA[c]
        kf, vf = synth.make_kv(oracle, n, kvk, seed=seed + c)
        Q.kv_store_rows_shard(torch.from_numpy(kf.reshape(n, -1)).cuda(), torch.from_numpy(vf.reshape(n, -1)).cuda(),
                              lin.tab(0, c), lin.tab(1, c), 0, 4, 256, n, kvk, row_base, row_count)
        ks.append(synth.encode_rows(oracle, kf, kvk, is_v=False)[0])
        vs.append(synth.encode_rows(oracle, vf, kvk, is_v=True)[0])
    torch.cuda.synchronize()
    return ks, vs


@pytest.mark.parametrize("kvk", [KV_F16, KV_T3, KV_T5K])
def test_export_equals_the_reference_walk_and_imports_anywhere(oracle, cuda, kvk):
    rows = 300
    pool = make_pool(kvk, 40, 40)
    held = []
    pool.reserve(0, 3, held)                                # shift the K side against the V side
    lin = Q.KvLineage(pool, PAIRS, 64 * 8)
    assert lin.entitle(rows, EXTRA)
    ks, vs = fill(oracle, lin, kvk, rows, seed=40)
    for L in (300, 129, 64, 1, 0):
        blob = lin.export_rows(L, EXTRA)
        torch.cuda.synchronize()
        want = SO.kv_blob(ks, vs, L, EXTRA)
        assert blob.numel() == want.size == SO.kv_bytes(L, PAIRS - 1, Q.row_bytes(kvk), Q.row_bytes(kvk, is_v=True))
        assert (blob.cpu().numpy() == want).all()
    # into another pool, whose pages come out in another order, at another capacity
    blob = lin.export_rows(rows, EXTRA)
    pool2 = make_pool(kvk, 30, 30)
    scramble = []
    pool2.reserve(0, 7, scramble)
    pool2.release(0, scramble[::2])
    lin2 = Q.KvLineage(pool2, PAIRS, 64 * 5)
    assert lin2.entitle(rows, EXTRA)
    lin2.import_rows(blob, rows, EXTRA)
    for c in range(PAIRS):
        n = rows + EXTRA[c]
        for side, raw in ((0, ks[c]), (1, vs[c])):
            out = torch.empty((n, 4, 256), device=cuda)
            Q.kv_dequant(lin2.tab(side, c), kvk, 0, n, 4, out, is_v=bool(side))
            assert (out.cpu().numpy().view(np.uint32) ==
                    oracle.kv_dequant(raw, kvk, n, is_v=bool(side)).view(np.uint32)).all()
    for x in (lin, lin2):
        x.close()
    for p in (pool, pool2):
        p.close()


@pytest.mark.parametrize("kvk", [KV_T3, KV_F16])
def test_cache_split_by_rows_routes_stores_and_snapshots(oracle, cuda, kvk):
    """Three owners on one GPU. Chunk rows and draft-lane rows are handed to every owner alike
    and land only where they belong; the owners' exports assemble into the blob of the
    unsplit cache; that blob dealt out over two owners attends like the unsplit cache."""
    rows, cap = 700, 64 * 12
    ranges = shard_ranges(cap, 3)                          # (0,256) (256,512) (512,768)
    pools = [make_pool(kvk, 20, 20) for _ in range(3)]
    lins = [Q.KvLineage(p, PAIRS, hi - lo) for p, (lo, hi) in zip(pools, ranges)]
    for lin, (lo, hi) in zip(lins, ranges):
        n, ex = S.local_rows(rows, EXTRA, PAIRS, lo, hi)
        assert lin.entitle(n, ex)
    ks = vs = None
    for lin, (lo, hi) in zip(lins, ranges):
        ks, vs = fill(oracle, lin, kvk, rows - 4, seed=70, row_base=lo, row_count=hi - lo)
    # four draft rows at positions rows-4 .. rows-1 (+1 for the draft pair), lane form
    for c in range(PAIRS):
        n0 = rows - 4 + EXTRA[c]
        kf, vf = synth.make_kv(oracle, 4, kvk, seed=90 + c)
        kd = [torch.from_numpy(kf[t].reshape(-1).copy()).cuda() for t in range(4)]
        vd = [torch.from_numpy(vf[t].reshape(-1).copy()).cuda() for t in range(4)]
        pd = [torch.tensor([n0 + t], dtype=torch.int32, device=cuda) for t in range(4)]
        for lin, (lo, hi) in zip(lins, ranges):
            Q.kv_store_lanes_shard(kd, vd, lin.tab(0, c), lin.tab(1, c), pd, 4, 256, kvk, lo, hi - lo)
        ks[c] = np.concatenate([ks[c], synth.encode_rows(oracle, kf, kvk, is_v=False)[0]])
        vs[c] = np.concatenate([vs[c], synth.encode_rows(oracle, vf, kvk, is_v=True)[0]])
    torch.cuda.synchronize()
    want = SO.kv_blob(ks, vs, rows, EXTRA)
    rk, rv = Q.row_bytes(kvk), Q.row_bytes(kvk, is_v=True)
    plan = S.shard_plan(rows, EXTRA, PAIRS, rk, rv, ranges)
    parts = {}
    for r, (lin, (lo, hi)) in enumerate(zip(lins, ranges)):
        n, ex = S.local_rows(rows, EXTRA, PAIRS, lo, hi)
        parts[r] = lin.export_rows(n, ex).cpu()
    blob = S.assemble(plan, want.size, parts)
    assert (blob.numpy() == want).all()
    # deal the blob out over two owners and attend over pair 1 through partials + merge
    ranges2 = shard_ranges(cap, 2)
    pools2 = [make_pool(kvk, 30, 30) for _ in range(2)]
    lins2 = [Q.KvLineage(p, PAIRS, hi - lo) for p, (lo, hi) in zip(pools2, ranges2)]
    plan2 = S.shard_plan(rows, EXTRA, PAIRS, rk, rv, ranges2)
    for r, (lin, (lo, hi)) in enumerate(zip(lins2, ranges2)):
        n, ex = S.local_rows(rows, EXTRA, PAIRS, lo, hi)
        assert lin.entitle(n, ex)
        lin.import_rows(S.deal_out(plan2, blob, r).cuda(), n, ex)
    pos = [rows - 1, 400, 3]
    q = oracle.randn(3 * synth.Q_ROW, 5).reshape(3, 24, synth.Q_STRIDE)
    ql = [torch.from_numpy(q[t].reshape(-1).copy()).cuda() for t in range(3)]
    pl = [torch.tensor([p], dtype=torch.int32, device=cuda) for p in pos]
    parts_t = torch.empty((2, 3, 24, 258), device=cuda)
    for r, (lin, (lo, hi)) in enumerate(zip(lins2, ranges2)):
        scratch = torch.empty(Q.decode_scratch_floats(3), device=cuda)
        slot = Q.SlotArgs(lin.tab(0, 1), lin.tab(1, 1), ql, pl, [], scratch, row_base=lo, row_count=hi - lo)
        Q.attn_decode_partial([slot], 3, synth.Q_STRIDE, 24, 4, 256, SCALE, parts_t[r], kvk=kvk)
    out = torch.empty((3 * 24, 256), device=cuda)
    Q.attn_merge_partials(parts_t, 2, 3 * 24, out)
    torch.cuda.synchronize()
    ref = oracle.attn_decode(q, ks[1], vs[1], kvk, pos)
    assert synth.tolerance_ok(out.cpu().numpy().reshape(3, -1), ref)[0]
    for x in lins + lins2:
        x.close()
    for p in pools + pools2:
        p.close()
