"""CPU tests of the KV-sequence sharding host logic (q27_b200/dist.py): shard geometry, the
routing of new rows, and the exchange step run as world_size-2 gloo ranks. The per-shard
compute is stood in for by the oracle's windowed partials, so what is under test is the
plumbing: range arithmetic, buffer layout, all-gather order, merge input."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from q27_b200 import dist as qd  # noqa: E402


def test_shard_ranges_are_page_aligned_and_cover():
    for total, world in ((262144, 8), (262144, 1), (131072 * 3, 3), (1000, 4), (63, 2), (0, 2),
                         (64 * 5 + 1, 4)):
        r = qd.shard_ranges(total, world)
        assert len(r) == world and r[0][0] == 0 and r[-1][1] == total
        for (lo, hi), (lo2, _) in zip(r, r[1:]):
            assert hi == lo2 and lo <= hi
        for lo, hi in r[:-1]:
            assert lo % 64 == 0 and (hi % 64 == 0 or hi == total)
    # the sharded verify workload: 262144 rows over 8 GPUs -> 32768 rows (512 pages) each
    assert qd.shard_ranges(262144, 8)[3] == (3 * 32768, 4 * 32768)


def test_new_rows_route_to_the_owning_shard():
    r = qd.shard_ranges(1000, 4)          # 16 pages -> 4 pages (256 rows) per rank
    assert [qd.owner_of_row(x, r) for x in (0, 255, 256, 767, 999)] == [0, 0, 1, 2, 3]
    with pytest.raises(ValueError):
        qd.owner_of_row(1000, r)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q, kc, vc, pos, ranges, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from tests.oracle_lib import KV_T3, Oracle
    o = Oracle()
    lanes, n_q = len(pos), 24
    ex = qd.PartialExchange.create(1, lanes, n_q, world, "cpu")
    lo, hi = ranges[rank]
    part = o.attn_partial(q, kc, vc, KV_T3, pos, lo, hi)        # stand-in for the GPU kernel
    ex.local.copy_(torch.from_numpy(part).view(1, lanes, n_q, 258))
    g = qd.all_gather_partials(ex)
    merged = o.merge_partials(g.numpy().reshape(world, -1, 258))
    if rank == 1:
        ret.put(merged)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_exchange_reproduces_full_attention(oracle):
    from tests import synth
    from tests.oracle_lib import KV_T3
    rows = 64 * 6
    pos = [rows - 1, rows - 2, 200, 10]          # the last two lanes leave rank 1's shard (partly) empty
    c = synth.make_case(oracle, KV_T3, rows=rows, pos=pos, seed=71, outlier_frac=0.02)
    full = oracle.attn_decode(c.q, c.k, c.v, KV_T3, pos)
    ranges = qd.shard_ranges(rows, 2)
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, c.q, c.k, c.v, pos, ranges, ret))
             for r in range(2)]
    for p in procs:
        p.start()
    merged = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert np.abs(merged.reshape(len(pos), -1) - full).max() < 1e-5


def test_partial_exchange_geometry():
    ex = qd.PartialExchange.create(8, 6, 24, 8, "cpu")
    assert ex.npairs == 8 * 6 * 24
    assert ex.bytes_per_rank() == 8 * 6 * 24 * 258 * 4      # 1.19 MB for 8 slots x 6 lanes
    assert tuple(ex.gathered.shape) == (8, 8, 6, 24, 258)


def _mailbox_rank(rank, world, port, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        qd.PeerMailboxes(1, 2, 24)
        ret.put((rank, "constructed"))
    except RuntimeError as e:
        ret.put((rank, "raised: " + str(e)))
    dist.barrier()
    dist.destroy_process_group()


def test_mailbox_setup_fails_on_every_rank_together():
    """Without a GPU the mailbox allocation fails; the set-up is collective, so both ranks
    must come out of the constructor with the same error instead of one of them hanging in
    an exchange the other never joins (the caller then falls back to the NCCL form)."""
    if torch.cuda.is_available():
        pytest.skip("needs a box without a GPU")
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mailbox_rank, args=(r, 2, port, ret)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(ret.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(v.startswith("raised: peer-memory mailboxes could not be set up") for v in got.values())
