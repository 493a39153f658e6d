"""KV-sequence sharding across real GPUs (skipped on a single-GPU box): two NCCL ranks, each
holding a page-aligned half of every slot's cache, exchange their 258-float partials -- once with an NCCL
all-gather, once through peer-memory mailboxes -- and merge; the result must equal attention
over the whole cache (oracle).
Run with `pytest -m gpu` on a box with >= 2 GPUs."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, kvk, q, k, v, pos, ranges, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist
    import q27_b200 as Q
    from q27_b200 import dist as qd
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    lo, hi = ranges[rank]
    lanes = len(pos)
    ks = Q.paged_from_rows(torch.from_numpy(k[lo:hi].copy()).to(dev), kvk)
    vs = Q.paged_from_rows(torch.from_numpy(v[lo:hi].copy()).to(dev), kvk)
    qd_ = [torch.from_numpy(q[t].copy()).to(dev) for t in range(lanes)]
    pd = [torch.tensor([p], dtype=torch.int32, device=dev) for p in pos]
    scratch = torch.full((Q.decode_scratch_floats(lanes),), float("nan"), device=dev)
    slot = Q.SlotArgs(ks.tab, vs.tab, qd_, pd, [], scratch, row_base=lo, row_count=hi - lo)
    ex = qd.PartialExchange.create(1, lanes, 24, world, dev)
    out = torch.zeros((lanes * 24, 256), device=dev)
    for _ in range(2):
        qd.sharded_decode([slot], ex, out, 512, 4, 1.0 / 16.0, kvk)
    torch.cuda.synchronize()
    # the same steps through peer memory: partials pushed into every rank's mailbox over
    # NVLink, flags, device-side wait, merge (no collective call per step)
    boxes = qd.PeerMailboxes(1, lanes, 24)
    out2 = torch.zeros((lanes * 24, 256), device=dev)
    for _ in range(3):
        boxes.decode([slot], out2, 512, 4, 1.0 / 16.0, kvk)      # one kernel: push, wait, merge
    torch.cuda.synchronize()
    out3 = torch.zeros((lanes * 24, 256), device=dev)
    for _ in range(2):
        boxes.decode([slot], out3, 512, 4, 1.0 / 16.0, kvk, two_kernels=True)
    boxes.decode([slot], out2, 512, 4, 1.0 / 16.0, kvk)          # and back: the two forms mix
    torch.cuda.synchronize()
    assert torch.equal(out2.view(torch.int32), out3.view(torch.int32))
    import ctypes as C
    flag = C.c_int(-1)
    Q._lib.check(Q._lib.lib().q27_wait_timeout_flag(C.byref(flag)), "q27_wait_timeout_flag")
    ret.put((rank, out.cpu().numpy(), out2.cpu().numpy(), flag.value))
    boxes.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("kvk", [0, 2])
def test_two_gpu_kv_split_matches_full_attention(oracle, kvk):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from tests import synth
    from q27_b200 import dist as qd
    import torch.multiprocessing as mp
    rows = 64 * 40
    pos = [rows - 1, rows - 2, rows - 3, 1000]
    c = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=5, outlier_frac=0.02 if kvk == 2 else 0.0)
    full = oracle.attn_decode(c.q, c.k, c.v, kvk, pos)
    ranges = qd.shard_ranges(rows, 2)
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, kvk, c.q, c.k, c.v, pos, ranges, ret))
             for r in range(2)]
    for p in procs:
        p.start()
    got = [ret.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, via_nccl, via_peers, flag in got:      # every rank ends up with the merged result
        assert synth.tolerance_ok(via_nccl.reshape(len(pos), -1), full)[0]
        assert flag == 0                             # no device-side wait ran out
        # same partials, same merge arithmetic: the two exchanges agree to the last bit
        assert np.array_equal(via_nccl, via_peers)


def _rank_snapshot(rank, world, port, kvk, rows, ret):
    """Each rank: a pool and a lineage over ITS rows; the same chunk and the same draft lanes
    are stored on every rank through the owner-routed stores; the ranks' exports are assembled
    on rank 0, dealt out again into fresh lineages, and the restored cache attends."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch.distributed as dist
    import q27_b200 as Q
    from q27_b200 import dist as qd
    from q27_b200 import snapshot as S
    from tests import synth
    from tests.oracle_lib import Oracle
    sys.path.insert(0, str(ROOT / "oracle"))
    import snapshot_oracle as SO
    oracle = Oracle()
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    pairs, extra, cap = 2, [0, 1], 64 * 16
    ranges = qd.shard_ranges(cap, world)
    lo, hi = ranges[rank]
    rk, rv = Q.row_bytes(kvk), Q.row_bytes(kvk, is_v=True)

    def fresh():
        pool = Q.KvPool(40 * 64 * rk, 40 * 64 * rv, rk, rv)
        lin = Q.KvLineage(pool, pairs, hi - lo)
        n, ex = S.local_rows(rows, extra, pairs, lo, hi)
        assert lin.entitle(n, ex)
        return pool, lin, n, ex

    pool, lin, n, ex = fresh()
    ks, vs = [], []
    for c in range(pairs):
        nr = rows + extra[c]
        kf, vf = synth.make_kv(oracle, nr, kvk, seed=11 + c)
        Q.kv_store_rows_shard(torch.from_numpy(kf[:nr - 3].reshape(nr - 3, -1)).to(dev),
                              torch.from_numpy(vf[:nr - 3].reshape(nr - 3, -1)).to(dev), lin.tab(0, c),
                              lin.tab(1, c), 0, 4, 256, nr - 3, kvk, lo, hi - lo)
        kd = [torch.from_numpy(kf[nr - 3 + t].reshape(-1).copy()).to(dev) for t in range(3)]
        vd = [torch.from_numpy(vf[nr - 3 + t].reshape(-1).copy()).to(dev) for t in range(3)]
        pd = [torch.tensor([nr - 3 + t], dtype=torch.int32, device=dev) for t in range(3)]
        Q.kv_store_lanes_shard(kd, vd, lin.tab(0, c), lin.tab(1, c), pd, 4, 256, kvk, lo, hi - lo)
        ks.append(synth.encode_rows(oracle, kf, kvk, is_v=False)[0])
        vs.append(synth.encode_rows(oracle, vf, kvk, is_v=True)[0])
    torch.cuda.synchronize()
    blob = S.export_sharded(lin.export_rows(n, ex), rows, extra, pairs, rk, rv, ranges)
    blob_ok = True
    if rank == 0:
        blob_ok = bool((blob.numpy() == SO.kv_blob(ks, vs, rows, extra)).all())
    lin.close()
    pool.close()
    pool, lin, n, ex = fresh()
    lin.import_rows(S.import_sharded(blob, rows, extra, pairs, rk, rv, ranges, dev), n, ex)
    pos = [rows - 1, rows // 2]
    q = oracle.randn(2 * synth.Q_ROW, 3).reshape(2, 24, synth.Q_STRIDE)
    ql = [torch.from_numpy(q[t].reshape(-1).copy()).to(dev) for t in range(2)]
    pl = [torch.tensor([p], dtype=torch.int32, device=dev) for p in pos]
    scratch = torch.empty(Q.decode_scratch_floats(2), device=dev)
    slot = Q.SlotArgs(lin.tab(0, 0), lin.tab(1, 0), ql, pl, [], scratch, row_base=lo, row_count=hi - lo)
    exg = qd.PartialExchange.create(1, 2, 24, world, dev)
    out = torch.zeros((2 * 24, 256), device=dev)
    qd.sharded_decode([slot], exg, out, 512, 4, 1.0 / 16.0, kvk)
    torch.cuda.synchronize()
    ref = oracle.attn_decode(q, ks[0], vs[0], kvk, pos)
    ret.put((rank, blob_ok, bool(synth.tolerance_ok(out.cpu().numpy().reshape(2, -1), ref)[0])))
    lin.close()
    pool.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("kvk", [2, 4])
def test_two_gpu_owner_routed_stores_and_snapshot(kvk):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_snapshot, args=(r, 2, port, kvk, 700, ret)) for r in range(2)]
    for p in procs:
        p.start()
    got = [ret.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(blob_ok and attn_ok for _, blob_ok, attn_ok in got), got
