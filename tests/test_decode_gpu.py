"""GPU parity tests of decode / verify attention through the C ABI, against the CPU oracle
(and, when oracle/_ref was built, against the reference's own fd2 kernels on this GPU).

Matrix follows the reference's test_attn_fd2 (src/test_kernels.cu:843-1049): sequence
lengths {1, 47, 1024, 16384, 61440} x ntok {1, 5} x formats, NaN-poisoned scratch,
run-to-run bitwise repeat, and the scattered page table proof (Q27_KV_SCATTER)."""
import numpy as np
import pytest
import torch

import q27_b200 as Q
from tests import synth
from tests.gpu_util import SCALE, DeviceCase, RefGpu
from tests.oracle_lib import KV_F16, KV_FP8, KV_T3, REF_GPU_SO

pytestmark = pytest.mark.gpu
KINDS = [KV_F16, KV_FP8, KV_T3]

# tight bar for the fp32 "exact" family: max-abs/RMS, the reference's own gate for fd2
# (1e-4 fp16/fp8, 2e-4 turbo3: src/test_kernels.cu:981,1521)
EXACT_TOL = {KV_F16: 1e-4, KV_FP8: 1e-4, KV_T3: 2e-4}
# the named workloads draw plain N(0,1) for the fp16 / fp8 caches and add x8 outlier channels (2 %)
# only to the turbo3 configs, whose WHT rotation is there to spread them
OUTLIERS = {KV_F16: 0.0, KV_FP8: 0.0, KV_T3: 0.02}


def lanes_for(seq, ntok):
    # verify lanes sit at P+1+t (src/spec3.cu:1319-1326): the last lane sees the whole cache
    return [max(seq - ntok + t, 0) for t in range(ntok)]


@pytest.mark.parametrize("kvk", KINDS)
def test_dequant_is_bit_exact(oracle, cuda, kvk):
    c = synth.make_case(oracle, kvk, rows=200, pos=[199], seed=5, outlier_frac=0.02)
    dc = DeviceCase(c, cuda, scatter_seed=3)
    for side, raw in ((dc.kside, c.k), (dc.vside, c.v)):
        out = torch.empty((150, 4, 256), device=cuda)
        Q.kv_dequant(side.tab, kvk, 37, 150, 4, out)
        ref = oracle.kv_dequant(raw[37:187], kvk, 150)
        assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()


@pytest.mark.parametrize("kvk", KINDS)
@pytest.mark.parametrize("ntok", [1, 5])
@pytest.mark.parametrize("seq", [1, 47, 1024, 16384, 61440])
def test_decode_vs_oracle(oracle, cuda, kvk, ntok, seq):
    c = synth.make_case(oracle, kvk, rows=seq, pos=lanes_for(seq, ntok), seed=100 + seq % 97)
    ref = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos))
    dc = DeviceCase(c, cuda)
    exact = synth.scale_out(c, dc.run3(exact=True))
    rms = np.sqrt((ref.astype(np.float64) ** 2).mean()) + 1e-12
    assert np.abs(exact - ref).max() / rms < EXACT_TOL[kvk]
    got = synth.scale_out(c, dc.run3())
    ok, excess, rel = synth.tolerance_ok(got, ref)   # the parity bar: 2e-3 abs + 1e-3 rel
    assert ok, (excess, rel)
    assert rel < 1e-2                                 # the reference's fp16-MMA class bar
    again = synth.scale_out(c, dc.run3())
    assert (again.view(np.uint32) == got.view(np.uint32)).all()   # run-to-run bitwise


def test_turbo3_verify_margin_over_many_outlier_cases(oracle, cuda):
    """The tightest path against the parity bar is the six-lane verify over a turbo3 cache with
    2 % of the channels scaled by eight (fp16 operands: centroid x norm rounded once, P in fp16).
    Sixteen seeded cases of different lengths must all stay inside |a-b| <= 2e-3 + 1e-3*|b| (with
    the product rounded twice one case in a dozen went over)."""
    for seed in range(1, 17):
        rows = 1800 + 37 * seed
        pos = [rows - 6 + t for t in range(6)]
        c = synth.make_case(oracle, KV_T3, rows=rows, pos=pos, seed=seed, outlier_frac=0.02)
        ref = oracle.attn_decode(c.q, c.k, c.v, KV_T3, c.pos)
        got = DeviceCase(c, cuda).run3()
        ok, excess, rel = synth.tolerance_ok(got, ref)
        assert ok, (seed, excess, rel)


@pytest.mark.parametrize("kvk", KINDS)
def test_scattered_pages_and_untouched_gate(oracle, cuda, kvk):
    c = synth.make_case(oracle, kvk, rows=1500, pos=[1499, 700, 64], seed=77, outlier_frac=OUTLIERS[kvk])
    c.q[:, :, 256:] = np.nan                      # the gate half must never be read
    ref = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos))
    dc = DeviceCase(c, cuda, scatter_seed=11)
    qcopy = [t.clone() for t in dc.q]
    for exact in (True, False):
        got = synth.scale_out(c, dc.run3(exact=exact))
        ok, excess, rel = synth.tolerance_ok(got, ref)
        assert ok and np.isfinite(got).all(), (exact, excess, rel)
    for a, b in zip(dc.q, qcopy):
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))  # q||gate left as is


def test_attn_decode_single_token_entry(oracle, cuda):
    c = synth.make_case(oracle, KV_F16, rows=4096, pos=[4095], seed=1)   # the 4096-row fp16 single-token workload
    ref = oracle.attn_decode(c.q, c.k, c.v, KV_F16, c.pos)
    dc = DeviceCase(c, cuda)
    Q.attn_decode(dc.q[0], synth.Q_STRIDE, dc.kside.tab, dc.vside.tab, dc.out[0], dc.scratch,
                  dc.pos[0], 4096, 24, 4, 256, SCALE, kvk=KV_F16)
    torch.cuda.synchronize()
    ok, excess, rel = synth.tolerance_ok(dc.out[0].cpu().numpy(), ref[0])
    assert ok, (excess, rel)


def test_positions_are_read_on_device(oracle, cuda):
    # the same launch arguments, new *pos contents: graph-stable control (src/spec3.cu:628)
    c = synth.make_case(oracle, KV_FP8, rows=900, pos=[899, 500], seed=9)
    dc = DeviceCase(c, cuda)
    dc.run3()
    for newpos in ([10, 899], [0, 0]):
        for t, p in enumerate(newpos):
            dc.pos[t].fill_(p)
        got = synth.scale_out(c, dc.run3())
        ref = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, KV_FP8, newpos))
        assert synth.tolerance_ok(got, ref)[0]


@pytest.mark.parametrize("kvk", KINDS)
def test_batched_slots(oracle, cuda, kvk):
    cases = [synth.make_case(oracle, kvk, rows=r, pos=p, seed=s, outlier_frac=OUTLIERS[kvk])
             for r, p, s in ((700, [699], 1), (2300, [2299, 2298, 100], 2), (64, [63, 62], 3))]
    dcs = [DeviceCase(c, cuda, scatter_seed=i) for i, c in enumerate(cases)]
    for exact in (True, False):
        Q.attn_decode_batched([d.slot() for d in dcs], synth.Q_STRIDE, 24, 4, 256, SCALE, kvk=kvk,
                              exact=exact)
        torch.cuda.synchronize()
        for d, c in zip(dcs, cases):
            got = synth.scale_out(c, np.stack([o.cpu().numpy() for o in d.out]))
            ref = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos))
            assert synth.tolerance_ok(got, ref)[0]


@pytest.mark.parametrize("kvk", KINDS)
@pytest.mark.parametrize("nshards", [2, 4])
def test_kv_split_partials_merge(oracle, cuda, kvk, nshards):
    """KV-sequence sharding emulated on one GPU: every shard holds a page-aligned row range
    behind its own tables, emits un-normalised partials, and the LSE merge of the shards
    equals attention over the whole cache (and the oracle's partials, shard by shard)."""
    rows = 64 * 4 * nshards
    pos = [rows - 1, rows - 2, rows // 2 + 3, 70, 0]
    c = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=55, outlier_frac=OUTLIERS[kvk])
    full = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos))
    per = rows // nshards
    lanes_stride = 6
    parts = torch.empty((nshards, 1, lanes_stride, 24, 258), device=cuda)
    for g in range(nshards):
        dc = DeviceCase(c, cuda, row_lo=g * per, row_hi=(g + 1) * per)
        Q.attn_decode_partial([dc.slot()], lanes_stride, synth.Q_STRIDE, 24, 4, 256, SCALE,
                              parts[g], kvk=kvk)
        torch.cuda.synchronize()
        mine = parts[g, 0, : len(pos)].cpu().numpy()
        want = oracle.attn_partial(c.q, c.k, c.v, kvk, c.pos, g * per, (g + 1) * per)
        # partials agree after normalising each by its own l (m conventions may differ)
        live = want[:, :, 0] > -1e38
        assert ((mine[:, :, 0] > -1e38) == live).all()
        assert (mine[:, :, 1][~live] == 0).all()
        vs = np.ones(24, np.float32) if c.v_scale is None else np.repeat(c.v_scale, 6)
        vs = np.broadcast_to(vs[None, :], live.shape)[live][:, None]
        a = mine[live][:, 2:] / mine[live][:, 1:2] * vs
        b = want[live][:, 2:] / want[live][:, 1:2] * vs
        # a shard's own partial (as little as one key) is held to the reference's gate for
        # fp16-operand tensor-core paths (max-abs/RMS 1e-2, src/test_kernels.cu:1824-1962);
        # the parity bar applies to the merged output below
        assert np.abs(a - b).max() / (np.sqrt((b.astype(np.float64) ** 2).mean()) + 1e-12) < 1e-2
        # padded lane (index 5) is a well-formed empty partial
        assert (parts[g, 0, 5, :, 0].cpu().numpy() < -1e38).all()
    out = torch.empty((lanes_stride * 24, 256), device=cuda)
    Q.attn_merge_partials(parts, nshards, lanes_stride * 24, out)
    torch.cuda.synchronize()
    got = synth.scale_out(c, out.cpu().numpy().reshape(lanes_stride, -1)[: len(pos)])
    assert synth.tolerance_ok(got, full)[0]


@pytest.mark.parametrize("kvk", KINDS)
def test_kv_split_through_mailboxes(oracle, cuda, kvk):
    """The peer-memory exchange with both 'ranks' on this one GPU: two mailboxes, each rank's
    push lands in both (plain stores here, peer stores across GPUs), flags carry the epoch,
    and each rank's merge equals attention over the whole cache. Pushes and merges are
    separate launches in stream order, so no kernel ever waits on one that has not run.
    Three steps exercise both parities and the reuse of a parity."""
    import ctypes as C
    lib = Q._lib.lib()
    world, lanes_stride = 2, 4
    rows = 64 * 6
    npairs = lanes_stride * 24
    boxes = []
    for _ in range(world):
        ptr = C.c_void_p()
        Q._lib.check(lib.q27_xchg_alloc(lib.q27_xchg_mailbox_bytes(world, npairs), C.byref(ptr), None),
                     "q27_xchg_alloc")
        boxes.append(ptr.value)
    try:
        for epoch in (1, 2, 3):
            pos = [rows - 1, rows // 2 + epoch, 5 * epoch]
            c = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=90 + epoch,
                                outlier_frac=OUTLIERS[kvk])
            full = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos))
            keep = []
            for r in range(world):
                dc = DeviceCase(c, cuda, row_lo=r * rows // 2, row_hi=(r + 1) * rows // 2)
                keep.append(dc)
                Q.attn_decode_partial_push([dc.slot()], lanes_stride, synth.Q_STRIDE, 24, 4, 256,
                                           SCALE, boxes, r, epoch, kvk=kvk)
            for r in range(world):
                out = torch.empty((npairs, 256), device=cuda)
                Q.attn_merge_pushed(boxes[r], world, npairs, epoch, out)
                torch.cuda.synchronize()
                got = synth.scale_out(c, out.cpu().numpy().reshape(lanes_stride, -1)[: len(pos)])
                assert synth.tolerance_ok(got, full)[0]
        flag = C.c_int(-1)
        Q._lib.check(lib.q27_wait_timeout_flag(C.byref(flag)), "q27_wait_timeout_flag")
        assert flag.value == 0
    finally:
        torch.cuda.synchronize()
        for b in boxes:
            Q._lib.check(lib.q27_xchg_free(b), "q27_xchg_free")


@pytest.mark.parametrize("kvk,pos", [(KV_T3, [2999, 2000, 7]), (KV_F16, [2999])],
                         ids=["turbo3-three-lanes", "f16-one-lane"])
def test_one_call_exchange_with_a_single_owner(oracle, cuda, kvk, pos):
    """q27_attn_decode_exchange with one rank: the combine, the (empty) exchange and the merge in
    ONE kernel, device-counted epochs over several steps, equal to the plain decode bit for bit --
    also where the plain decode is the single launch that merges its own splits (one lane, short
    context): every merge of split records adds in one order. (With more owners the kernel waits
    for its peers' rows, which only real ranks on their own GPUs can provide:
    tests/test_multi_gpu.py.)"""
    import ctypes as C
    lib = Q._lib.lib()
    nl = len(pos)
    c = synth.make_case(oracle, kvk, rows=3000, pos=pos, seed=66, outlier_frac=OUTLIERS[kvk])
    ref = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos))
    dc = DeviceCase(c, cuda)
    npairs = nl * 24
    ptr = C.c_void_p()
    Q._lib.check(lib.q27_xchg_alloc(lib.q27_xchg_mailbox_bytes(1, npairs), C.byref(ptr), None), "q27_xchg_alloc")
    try:
        out = torch.full((npairs, 256), float("nan"), device=cuda)
        n0 = Q.launch_count()
        for _ in range(3):                          # epoch 0: the mailbox counts the steps itself
            Q.attn_decode_exchange([dc.slot()], nl, synth.Q_STRIDE, 24, 4, 256, SCALE, [ptr.value], 0, 0, out,
                                   kvk=kvk)
        torch.cuda.synchronize()
        assert Q.launch_count() - n0 == 3 * 2       # partial kernel + one exchange kernel per step
        assert synth.tolerance_ok(synth.scale_out(c, out.cpu().numpy().reshape(nl, -1)), ref)[0]
        n1 = Q.launch_count()
        plain = dc.run3()
        if nl == 1:
            assert Q.launch_count() - n1 == 1       # the decode kernel finished the step itself
        assert (out.cpu().numpy().reshape(nl, -1).view(np.uint32) == plain.view(np.uint32)).all()
    finally:
        torch.cuda.synchronize()
        Q._lib.check(lib.q27_xchg_free(ptr.value), "q27_xchg_free")


@pytest.mark.skipif(not REF_GPU_SO.exists(), reason="oracle/_ref not built")
@pytest.mark.parametrize("kvk", KINDS)
def test_against_reference_kernels_on_this_gpu(oracle, cuda, kvk):
    """The reference's own k_attn_fd2 + combine, recompiled for sm_100a from the reference
    tree, on the identical buffers: pins the oracle to the reference itself (<= 1e-4 / 2e-4
    max-abs/RMS, its own gate) and the engine to the reference within the parity bar."""
    ref_gpu = RefGpu()
    for seq, ntok in ((47, 1), (1024, 5), (16384, 5)):
        c = synth.make_case(oracle, kvk, rows=seq, pos=lanes_for(seq, ntok), seed=300 + seq % 89)
        oracle_out = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos))
        dc = DeviceCase(c, cuda)
        theirs = synth.scale_out(c, ref_gpu.decode3(dc).copy())
        rms = np.sqrt((oracle_out.astype(np.float64) ** 2).mean()) + 1e-12
        assert np.abs(theirs - oracle_out).max() / rms < EXACT_TOL[kvk]
        mine = synth.scale_out(c, dc.run3())
        assert synth.tolerance_ok(mine, theirs)[0]


def test_errors_are_status_codes(cuda, oracle):
    c = synth.make_case(oracle, KV_F16, rows=64, pos=[63], seed=2)
    dc = DeviceCase(c, cuda)
    with pytest.raises(Q._lib.Q27Error) as e:
        Q.attn_decode3(dc.q, synth.Q_STRIDE, dc.kside.tab, dc.vside.tab, dc.out, dc.scratch,
                       dc.pos, 0, 24, 4, 256, SCALE, ntok=1, kvk=6)     # outside the KvKind enum
    assert e.value.status == Q._lib.ERR_UNSUPPORTED_KIND
    assert torch.isnan(dc.out[0]).all()                                  # nothing was written


def test_kvpool_on_device(cuda):
    # src/kv_pool.h:24-72: sides rounded DOWN to whole pages, LIFO with low indices first
    rb = Q.row_bytes(KV_T3)
    pool = Q.KvPool(10 * 64 * rb + 17, 7 * 64 * rb, rb, rb)
    assert pool.enabled() and pool.npages(0) == 10 and pool.npages(1) == 7
    assert pool.page_bytes(0) == 64 * rb
    got = []
    assert pool.reserve(0, 3, got) and got == [0, 1, 2]
    assert pool.page_ptr(0, 2) - pool.page_ptr(0, 0) == 2 * 64 * rb
    assert not pool.reserve(1, 8, got) and pool.free_pages(1) == 7     # pops nothing
    pool.release(0, got)
    assert pool.free_pages(0) == 10 and got == []
    again = []
    assert pool.reserve(0, 1, again) and again == [2]                   # LIFO
    pool.close()


@pytest.mark.parametrize("kvk", KINDS)
def test_sixteen_lanes_ragged_positions(oracle, cuda, kvk):
    # the widest verify the lane bundles allow (p[16], src/kernels.cuh:67-68), lanes of very
    # different lengths, one of them a single key
    rows = 5000
    pos = [rows - 1 - 3 * t for t in range(12)] + [2500, 64, 63, 0]
    c = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=61, outlier_frac=OUTLIERS[kvk])
    ref = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos))
    dc = DeviceCase(c, cuda, scatter_seed=9)
    for exact in (True, False):
        got = synth.scale_out(c, dc.run3(exact=exact))
        ok, excess, rel = synth.tolerance_ok(got, ref)
        assert ok, (exact, excess, rel)


def test_other_head_counts_run_the_fp32_family(oracle, cuda):
    # geometry other than 24/4 but still 6 query heads per kv head: accepted, served by the
    # fp32 kernels (the tensor-core ring layouts are specialised for 4 kv heads)
    import ctypes as C
    from q27_b200 import _lib as L
    n_kv, n_q, rows = 2, 12, 300
    rng = np.random.default_rng(3)
    kf = oracle.randn(rows * n_kv * 256, 7).reshape(rows, n_kv, 256)
    vf = oracle.randn(rows * n_kv * 256, 8).reshape(rows, n_kv, 256)
    k = oracle.to_half_bits(kf).view(np.uint8).reshape(rows, -1)
    v = oracle.to_half_bits(vf).view(np.uint8).reshape(rows, -1)
    q = oracle.randn(n_q * 512, 9).reshape(1, n_q, 512)
    ref = oracle.attn_decode(q, k, v, KV_F16, [rows - 1], n_q=n_q, n_kv=n_kv)
    ks = Q.paged_from_rows(torch.from_numpy(k).to(cuda), KV_F16, n_kv_heads=n_kv)
    vs = Q.paged_from_rows(torch.from_numpy(v).to(cuda), KV_F16, n_kv_heads=n_kv)
    qd = torch.from_numpy(q[0].copy()).to(cuda)
    out = torch.zeros(n_q * 256, device=cuda)
    scratch = torch.empty(Q.decode_scratch_floats(1, n_q), device=cuda)
    pos = torch.tensor([rows - 1], dtype=torch.int32, device=cuda)
    Q.attn_decode(qd, 512, ks.tab, vs.tab, out, scratch, pos, 0, n_q, n_kv, 256, SCALE, kvk=KV_F16)
    torch.cuda.synchronize()
    assert synth.tolerance_ok(out.cpu().numpy()[None], ref)[0]
    # 5 query heads per kv head is not this model family: refused as a width
    rc = L.lib().q27_attn_decode(qd.data_ptr(), 512, ks.tab.data_ptr(), vs.tab.data_ptr(),
                                 out.data_ptr(), scratch.data_ptr(), pos.data_ptr(), 0, 10, 2, 256,
                                 SCALE, None, KV_F16)
    assert rc == L.ERR_UNSUPPORTED_WIDTH
