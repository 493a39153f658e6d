"""CPU tests of the snapshot format and of the planning for a cache split by rows: the numpy
oracle (oracle/snapshot_oracle.py) and the engine's host code against the fixture generated
from the reference's own header (tests/golden/pfx_identity.npz) and, when oracle/_ref was built,
against that header itself; entry files; the shard plan as an exact inverse pair; and the
collective export / import over two and three gloo ranks."""
import ctypes as C
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "oracle"))
import snapshot_oracle as SO  # noqa: E402

from q27_b200 import snapshot as S  # noqa: E402
from tests.oracle_lib import REF_CODEC_SO  # noqa: E402

G = np.load(ROOT / "tests" / "golden" / "pfx_identity.npz")


def test_hashes_and_header_match_the_reference_fixture():
    toks = G["tokens"]
    for n, key in zip(G["lens"], G["keys"]):
        assert SO.fnv1a64(toks[:n].tobytes()) == int(key)
        assert S.token_key(toks, int(n)) == int(key)
    path = G["path"].tobytes().decode()
    for g, want in zip(G["geoms"], G["compats"]):
        args = [int(v) for v in g]
        assert SO.compat_hash(path, *args) == int(want)
        assert S.compat_hash(path, *args) == int(want)
    assert int(G["magic"]) == SO.PFX_MAGIC == S.PFX_MAGIC and int(G["version"]) == SO.PFX_VERSION
    assert int(G["hdr_bytes"]) == 64 == S.PFX_HDR_BYTES
    want = G["hdr"].tobytes()
    assert SO.header(int(G["compats"][2]), toks, 4096, 123456, 7890123) == want
    assert S._HDR.pack(S.PFX_MAGIC, S.PFX_VERSION, int(G["compats"][2]), S.token_key(toks, 4096), 4096, 0,
                       123456, 7890123, 0, 0) == want


@pytest.mark.skipif(not REF_CODEC_SO.exists(), reason="oracle/_ref not built")
def test_hashes_match_the_reference_header_itself():
    ref = C.CDLL(str(REF_CODEC_SO))
    ref.q27ref_pfx_fnv1a64.restype = C.c_uint64
    ref.q27ref_pfx_fnv1a64.argtypes = [C.c_void_p, C.c_size_t]
    rng = np.random.default_rng(5)
    for n in (0, 1, 3, 1000, 70001):
        b = rng.integers(0, 256, n, dtype=np.uint8)
        want = ref.q27ref_pfx_fnv1a64(b.ctypes.data, n)
        assert SO.fnv1a64(b.tobytes()) == want == S.fnv1a64(b.tobytes())
    assert SO.kv_bytes(1000, 16, 656, 400) == 1000 * 16 * 1056 + 1001 * 1056   # pfx_kv_bytes


def test_entry_file_round_trip_and_the_strict_token_rule(tmp_path):
    toks = [int(t) for t in G["tokens"][:300]]
    compat = int(G["compats"][0])
    gdn, kv = os.urandom(1000), os.urandom(4096)
    p = S.write_entry(tmp_path, toks, 200, compat, gdn, kv)
    assert p.name == f"{SO.fnv1a64(np.asarray(toks[:200], '<i4').tobytes()):016x}-200.q27pc"
    assert not list(tmp_path.glob("*.tmp"))                       # published by rename only
    raw = p.read_bytes()
    assert raw[:64] == SO.header(compat, toks, 200, 1000, 4096)
    assert raw[64:64 + 800] == np.asarray(toks[:200], "<i4").tobytes() and raw[864:1864] == gdn
    assert S.read_entry(p, toks, compat) == (200, gdn, kv)
    other = list(toks)
    other[150] += 1                                              # same length, one token off
    assert S.read_entry(p, other, compat) is None
    assert S.read_entry(p, toks[:200], compat) is None            # nothing left to decode from
    assert S.read_entry(p, toks, compat ^ 1) is None              # another model / geometry
    p.write_bytes(raw[:500])
    assert S.read_entry(p, toks, compat) is None                  # truncated


def _caches(rng, pairs, rows, k_row, v_row):
    k = [rng.integers(0, 256, (rows, k_row), dtype=np.uint8) for _ in range(pairs)]
    v = [rng.integers(0, 256, (rows, v_row), dtype=np.uint8) for _ in range(pairs)]
    return k, v


def _ranges(total, world):
    from q27_b200.dist import shard_ranges
    return shard_ranges(total, world)


def _local_blob(k, v, L, extra, lo, hi):
    n, ex = S.local_rows(L, extra, len(k), lo, hi)
    return SO.kv_blob([a[lo:hi] for a in k], [a[lo:hi] for a in v], n, ex)


@pytest.mark.parametrize("world", [1, 2, 3, 5])
@pytest.mark.parametrize("L", [0, 1, 63, 64, 200, 447])
def test_shard_plan_assembles_the_reference_blob(world, L):
    rng = np.random.default_rng(100 + world)
    pairs, rows, k_row, v_row = 3, 448, 656, 400
    extra = [0, 0, 1]
    if L + 1 > rows:
        return
    k, v = _caches(rng, pairs, rows, k_row, v_row)
    whole = SO.kv_blob(k, v, L, extra)
    assert whole.size == S.blob_bytes(L, extra, pairs, k_row, v_row)
    ranges = _ranges(rows, world)
    plan = S.shard_plan(L, extra, pairs, k_row, v_row, ranges)
    parts = {r: torch.from_numpy(_local_blob(k, v, L, extra, *ranges[r])) for r in range(world)}
    for r in range(world):
        assert parts[r].numel() == sum(s.nbytes for s in plan if s.rank == r)
    got = S.assemble(plan, whole.size, parts)
    assert (got.numpy() == whole).all()
    for r in range(world):                                        # and back
        assert (S.deal_out(plan, got, r).numpy() == parts[r].numpy()).all()
    # segments tile the blob exactly once
    cover = np.zeros(whole.size, np.int32)
    for s in plan:
        cover[s.blob_off:s.blob_off + s.nbytes] += 1
    assert (cover == 1).all()


def _worker(rank, world, port, L, out_dir):
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(9)                 # the same caches on every rank
        pairs, rows, k_row, v_row, extra = 3, 320, 400, 400, [0, 0, 1]
        k, v = _caches(rng, pairs, rows, k_row, v_row)
        ranges = _ranges(rows, world)
        mine = torch.from_numpy(_local_blob(k, v, L, extra, *ranges[rank]))
        blob = S.export_sharded(mine, L, extra, pairs, k_row, v_row, ranges)
        if rank == 0:
            assert (blob.numpy() == SO.kv_blob(k, v, L, extra)).all()
        else:
            assert blob is None
        back = S.import_sharded(blob, L, extra, pairs, k_row, v_row, ranges, "cpu")
        assert (back.numpy() == mine.numpy()).all()
        # a blob is portable: the same bytes dealt out over a different number of owners
        if rank == 0:
            for w2 in (1, 4):
                r2 = _ranges(rows, w2)
                p2 = S.shard_plan(L, extra, pairs, k_row, v_row, r2)
                for q in range(w2):
                    assert (S.deal_out(p2, blob, q).numpy() == _local_blob(k, v, L, extra, *r2[q])).all()
        Path(out_dir, f"ok{rank}").write_text("ok")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,L", [(2, 200), (3, 130), (2, 10)])
def test_collective_export_import_over_gloo(tmp_path, world, L):
    port = 29600 + world * 7 + L % 50
    mp.spawn(_worker, args=(world, port, L, str(tmp_path)), nprocs=world, join=True)
    assert all((tmp_path / f"ok{r}").exists() for r in range(world))
