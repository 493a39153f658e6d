"""GPU tests of the loose ends of the drop-in boundary: attention over tables built from
KvPool pages the way the reference's engine builds them (src/engine.cuh:750-810: entries are
pool page pointers, entries past the slot's entitlement alias page 0), the verify launchers'
partial layout with a caller-chosen split count (src/fdmma.cuh:460-463, src/spec3.cu:1224-1235),
and the bounded wait of the peer-memory merge running out (a status, not a hang)."""
import ctypes as C
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import q27_b200 as Q
from q27_b200 import _lib as L
from tests import synth
from tests.gpu_util import SCALE
from tests.oracle_lib import KV_F16, KV_FP8, KV_T3

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def pool_tables(pool, rows, npages_tab, k_bytes, v_bytes, dev):
    """Reserve pages for `rows` rows, copy the cache bytes into them and build K / V tables of
    npages_tab entries whose tail (past the reserved pages) aliases page 0, as kv_entitle does."""
    need = (rows + 63) // 64
    tabs = []
    for side, data in ((0, k_bytes), (1, v_bytes)):
        idx = []
        assert pool.reserve(side, need, idx)
        pb = pool.page_bytes(side)
        ptrs = [pool.page_ptr(side, i) for i in idx]
        flat = data.reshape(-1)
        for j, ptr in enumerate(ptrs):
            chunk = flat[j * pb:(j + 1) * pb]
            if chunk.numel():
                _memcpy_d2d(ptr, chunk)      # pages are raw device memory owned by the pool
        tail = [pool.page_ptr(side, 0)] * (npages_tab - need)
        tabs.append((torch.tensor(ptrs + tail, dtype=torch.int64, device=dev), idx))
    return tabs


def _memcpy_d2d(dst_ptr: int, src: torch.Tensor):
    cudart = C.CDLL("libcudart.so")
    cudart.cudaMemcpy.argtypes = [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int]
    rc = cudart.cudaMemcpy(dst_ptr, src.data_ptr(), src.numel(), 3)   # cudaMemcpyDeviceToDevice
    assert rc == 0, rc


@pytest.mark.parametrize("kvk", [KV_F16, KV_T3])
def test_decode_and_prefill_over_pool_pages_with_aliased_tail(oracle, cuda, kvk):
    rows, lanes = 1000, 3
    c = synth.make_case(oracle, kvk, rows=rows, pos=[999, 998, 500], seed=41, outlier_frac=0.02 if kvk == KV_T3 else 0.0)
    rb = Q.row_bytes(kvk)
    pool = Q.KvPool(40 * 64 * rb, 40 * 64 * rb, rb, rb)
    assert pool.enabled() and pool.npages(0) == 40
    # scramble the free lists so that reserved pages are neither ordered nor contiguous
    for side in (0, 1):
        tmp = []
        assert pool.reserve(side, 11, tmp)
        pool.release(side, tmp[::2])
        pool.release(side, tmp[1::2])
    kb = torch.from_numpy(c.k.copy()).to(cuda)
    vb = torch.from_numpy(c.v.copy()).to(cuda)
    (ktab, kidx), (vtab, vidx) = pool_tables(pool, rows, 32, kb, vb, cuda)
    assert kidx != sorted(kidx)                    # scattered, as a long-running pool hands them out
    q = [torch.from_numpy(c.q[t].copy()).to(cuda) for t in range(lanes)]
    pos = [torch.tensor([p], dtype=torch.int32, device=cuda) for p in c.pos]
    out = [torch.full((synth.OUT_ROW,), float("nan"), device=cuda) for _ in range(lanes)]
    scratch = torch.full((Q.decode_scratch_floats(lanes),), float("nan"), device=cuda)
    ref = oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos)
    Q.attn_decode3(q, synth.Q_STRIDE, ktab, vtab, out, scratch, pos, 0, 24, 4, 256, SCALE, ntok=lanes, kvk=kvk)
    torch.cuda.synchronize()
    got = np.stack([o.cpu().numpy() for o in out])
    ok, excess, rel = synth.tolerance_ok(got, ref)
    assert ok, (excess, rel)
    # single-token entry over the same tables
    Q.attn_decode(q[0], synth.Q_STRIDE, ktab, vtab, out[0], scratch, pos[0], 0, 24, 4, 256, SCALE, kvk=kvk)
    torch.cuda.synchronize()
    assert synth.tolerance_ok(out[0].cpu().numpy()[None], ref[:1])[0]
    # prefill: the last 40 rows as a chunk over the first 960 as prefix
    base, T = rows - 40, 40
    qT = torch.from_numpy(oracle.randn(T * synth.Q_ROW, 99).reshape(T, synth.Q_ROW)).to(cuda)
    if kvk == KV_T3:
        qh = qT.cpu().numpy().reshape(T, 24, synth.Q_STRIDE).copy()
        qh[:, :, :256] = oracle.wht(np.ascontiguousarray(qh[:, :, :256]))
        qT = torch.from_numpy(qh.reshape(T, -1)).to(cuda)
    outT = torch.full((T, synth.OUT_ROW), float("nan"), device=cuda)
    part = torch.full((Q.prefill_part_floats(T),), float("nan"), device=cuda)
    Q.attn_prefill_T(qT, synth.Q_STRIDE, synth.Q_ROW, ktab, vtab, outT, synth.OUT_ROW, part, base, 0, T,
                     24, 4, 256, SCALE, kvk=kvk)
    torch.cuda.synchronize()
    refp = oracle.attn_prefill(qT.cpu().numpy().reshape(T, 24, synth.Q_STRIDE), c.k, c.v, kvk, base, 0, T)
    ok, excess, rel = synth.tolerance_ok(outT.cpu().numpy(), refp)
    assert ok, (excess, rel)
    pool.release(0, kidx)
    pool.release(1, vidx)
    assert pool.free_pages(0) == 40 and pool.free_pages(1) == 40
    pool.close()


@pytest.mark.parametrize("kvk", [KV_F16, KV_FP8, KV_T3])
@pytest.mark.parametrize("ns", [128, 85, 42, 15, 10, 7, 3, 2, 1])
def test_verify_partials_with_the_callers_split_count(oracle, cuda, kvk, ns):
    """The reference's tools/fdmma_test.cu pattern: NaN-poisoned scratch, partials for W lanes
    with ns splits, every cell the combine will read is written, merged result == oracle. The
    split counts leave a CTA 1, 2, 3, 5, 10, 15 or all 29 tiles (the last one 8 rows): the
    staging teams of the packed formats take alternate tiles, so even, odd and single-tile
    ranges are all walked."""
    rows, W = 1800, 6
    pos = [rows - W + t for t in range(W)]
    c = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=7 + ns, outlier_frac=0.02 if kvk == KV_T3 else 0.0)
    from tests.gpu_util import DeviceCase
    dc = DeviceCase(c, cuda)
    part = torch.full((W * 24 * ns * 258,), float("nan"), device=cuda)
    assert Q.attn_verify_partials(dc.q, synth.Q_STRIDE, dc.kside.tab, dc.vside.tab, part, dc.pos, 4, 6, 256,
                                  SCALE, ns, kvk=kvk)
    torch.cuda.synchronize()
    p = part.cpu().numpy().reshape(W * 24, ns, 258)
    assert np.isfinite(p[:, :, :2]).all()           # every {m, l} the combine reads was written
    live = p[:, :, 0] != np.float32(-3.4028234663852886e38)
    assert np.isfinite(p[live]).all()
    p = p.copy()
    p[~live, 1:] = 0.0                             # dead splits keep their sentinel m; the rest is never read
    merged = oracle.merge_partials(np.ascontiguousarray(p.transpose(1, 0, 2)))
    ref = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, pos))
    got = synth.scale_out(c, merged.reshape(W, -1))
    ok, excess, rel = synth.tolerance_ok(got, ref)
    assert ok, (kvk, ns, excess, rel)


def test_verify_partials_refuses_what_it_does_not_cover(cuda):
    one = torch.zeros(8, device=cuda)
    lanes = [one] * 17
    with pytest.raises(L.Q27Error):
        Q.attn_verify_partials([one], 512, one, one, one, [one], 4, 6, 256, SCALE, 16, kvk=6)   # outside KvKind
    # a kind without a tensor-core verify (turbo5k): `false`, the caller falls through to the
    # scalar entry as it does in the reference (src/spec3.cu:1118-1135)
    assert Q.attn_verify_partials([one] * 4, 512, one, one, one, [one] * 4, 4, 6, 256, SCALE, 16, kvk=4) is False
    assert Q.attn_verify_partials([one] * 4, 512, one, one, one, [one] * 4, 4, 8, 256, SCALE, 16) is False
    assert Q.attn_verify_partials([one] * 4, 512, one, one, one, [one] * 4, 4, 6, 256, SCALE, 129) is False
    del lanes


WAIT_RUNS_OUT = r'''
import ctypes as C, sys, time
sys.path.insert(0, %r)
import torch
import q27_b200 as Q
from q27_b200 import _lib as L
dev = torch.device("cuda:0")
lib = L.lib()
npairs, world = 24, 2                      # 24 blocks: all resident at once
nbytes = lib.q27_xchg_mailbox_bytes(world, npairs)
box = C.c_void_p()
L.check(lib.q27_xchg_alloc(nbytes, C.byref(box), None), "alloc")
out = torch.full((npairs, 256), float("nan"), device=dev)
flag = C.c_int(-1)
L.check(lib.q27_wait_timeout_flag(C.byref(flag)), "flag")
assert flag.value == 0
t0 = time.time()
# epoch 1 was pushed by nobody: the merge must give up on its own
Q.attn_merge_pushed(box.value, world, npairs, 1, out)
torch.cuda.synchronize()
dt = time.time() - t0
L.check(lib.q27_wait_timeout_flag(C.byref(flag)), "flag")
untouched = bool(torch.isnan(out).all().item())
print("RESULT", flag.value, untouched, round(dt, 2))
lib.q27_xchg_free(box)
''' % str(ROOT)


def test_merge_wait_runs_out_with_a_status_and_leaves_out_alone(cuda):
    """q27_attn_merge_pushed on an epoch nobody pushed: every block's bounded wait runs out
    (about half a second), the library's timeout flag is raised, `out` is not written, and
    the kernel returns by itself. Runs in a child process because the flag is sticky."""
    r = subprocess.run([sys.executable, "-c", WAIT_RUNS_OUT], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT")][-1].split()
    assert int(line[1]) != 0          # the flag says a wait timed out
    assert line[2] == "True"          # out untouched
    assert float(line[3]) < 30.0      # it came back on its own
