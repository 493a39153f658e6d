"""GPU parity tests of the KV kinds whose K side differs from the V side: turbo3v (fp16 K),
turbo5k (5-bit K blocks) and int8-g64 (int8 K with a scale per 64 dims), V always turbo3
(src/cuda_common.h:47-59). The reference serves them with its scalar kernel
(src/spec3.cu:1080-1088); here they run through the fp32 family, so every comparison with the
oracle is held to the reference's tight fd2 gate (2e-4 max-abs/RMS, src/test_kernels.cu:1521).
Codec gates follow tools/turbo5_test.cu and tools/i8g64_test.cu: the device encoders are
byte-equal to the CPU codecs (turbo5 in the device's tree order), dequant is bit-exact."""
import numpy as np
import pytest
import torch

import q27_b200 as Q
from tests import synth
from tests.gpu_util import SCALE, DeviceCase, RefGpu
from tests.oracle_lib import KV_I8G64, KV_T3V, KV_T5K, REF_GPU_SO

pytestmark = pytest.mark.gpu
KINDS = [KV_T3V, KV_T5K, KV_I8G64]
TIGHT = 2e-4


def rel_err(got, ref):
    rms = np.sqrt((ref.astype(np.float64) ** 2).mean()) + 1e-12
    return float(np.abs(got.astype(np.float64) - ref).max() / rms)


def k_blocks(oracle, kvk, x):
    """CPU encoding of K rows x [rows, 4, 256] -> uint8 [rows, row_bytes]"""
    return synth.encode_rows(oracle, x, kvk, is_v=False)[0]


@pytest.mark.parametrize("kvk", KINDS)
def test_dequant_is_bit_exact_on_both_sides(oracle, cuda, kvk):
    c = synth.make_case(oracle, kvk, rows=200, pos=[199], seed=5, outlier_frac=0.02)
    dc = DeviceCase(c, cuda, scatter_seed=3)
    for side, raw, is_v in ((dc.kside, c.k, False), (dc.vside, c.v, True)):
        out = torch.empty((150, 4, 256), device=cuda)
        Q.kv_dequant(side.tab, kvk, 37, 150, 4, out, is_v=is_v)
        ref = oracle.kv_dequant(raw[37:187], kvk, 150, is_v=is_v)
        assert (out.cpu().numpy().view(np.uint32) == ref.view(np.uint32)).all()


@pytest.mark.parametrize("kvk", KINDS)
@pytest.mark.parametrize("ntok", [1, 5])
@pytest.mark.parametrize("seq", [1, 47, 1024, 16384])
def test_decode_vs_oracle(oracle, cuda, kvk, ntok, seq):
    pos = [max(seq - ntok + t, 0) for t in range(ntok)]
    c = synth.make_case(oracle, kvk, rows=seq, pos=pos, seed=200 + seq % 97, outlier_frac=0.02)
    ref = oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos)
    dc = DeviceCase(c, cuda, scatter_seed=9)
    got = dc.run3()                       # the reference-shaped entry
    assert rel_err(got, ref) < TIGHT
    assert synth.tolerance_ok(got, ref)[0]
    again = dc.run3()
    assert (again.view(np.uint32) == got.view(np.uint32)).all()       # run-to-run bitwise
    assert (dc.run3(exact=True).view(np.uint32) == got.view(np.uint32)).all()   # same kernels


@pytest.mark.parametrize("kvk", KINDS)
def test_batched_slots_and_kv_split_merge(oracle, cuda, kvk):
    """Two slots in one launch, then the same cache cut into three row shards whose partials
    merge to the one-pass result (the multi-GPU KV split on one device)."""
    cases = [synth.make_case(oracle, kvk, rows=900 + 300 * i, pos=[899 + 300 * i, 400], seed=60 + i)
             for i in range(2)]
    dcs = [DeviceCase(c, cuda) for c in cases]
    Q.attn_decode_batched([d.slot() for d in dcs], synth.Q_STRIDE, 24, 4, 256, SCALE, kvk=kvk)
    torch.cuda.synchronize()
    for c, d in zip(cases, dcs):
        ref = oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos)
        assert rel_err(np.stack([o.cpu().numpy() for o in d.out]), ref) < TIGHT
    c = cases[1]
    bounds = [0, 448, 832, c.rows]
    parts = torch.empty((3, 2, 24, 258), device=cuda)
    for s in range(3):
        shard = DeviceCase(c, cuda, row_lo=bounds[s], row_hi=bounds[s + 1])
        Q.attn_decode_partial([shard.slot()], 2, synth.Q_STRIDE, 24, 4, 256, SCALE, parts[s], kvk=kvk)
    merged = torch.empty((2, 24 * 256), device=cuda)
    Q.attn_merge_partials(parts, 3, 2 * 24, merged)
    torch.cuda.synchronize()
    ref = oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos)
    assert rel_err(merged.cpu().numpy(), ref) < TIGHT


@pytest.mark.parametrize("kvk", KINDS)
@pytest.mark.parametrize("exact", [True, False])
def test_prefill_small(oracle, cuda, kvk, exact):
    base, T = 37, 23
    c = synth.make_case(oracle, kvk, rows=base + T, pos=[0] * T, seed=3)
    ref = oracle.attn_prefill(c.q, c.k, c.v, kvk, base, 0, T)
    perm = torch.from_numpy(np.random.default_rng(5).permutation((base + T + 63) // 64))
    ks = Q.paged_from_rows(torch.from_numpy(c.k).to(cuda), kvk, page_perm=perm)
    vs = Q.paged_from_rows(torch.from_numpy(c.v).to(cuda), kvk, page_perm=perm, is_v=True)
    qT = torch.from_numpy(c.q.reshape(T, -1).copy()).to(cuda)
    outT = torch.zeros((T, synth.OUT_ROW), device=cuda)
    part = torch.full((Q.prefill_part_floats(T),), float("nan"), device=cuda)
    Q.attn_prefill_T(qT, synth.Q_STRIDE, synth.Q_ROW, ks.tab, vs.tab, outT, synth.OUT_ROW, part,
                     base, 0, T, 24, 4, 256, SCALE, kvk=kvk, exact=exact)
    torch.cuda.synchronize()
    assert rel_err(outT.cpu().numpy(), ref) < TIGHT


def _empty_sides(cuda, kvk, rows, scatter):
    perm = torch.from_numpy(np.random.default_rng(scatter).permutation((rows + 63) // 64))
    zk = torch.zeros((rows, Q.row_bytes(kvk)), dtype=torch.uint8, device=cuda)
    zv = torch.zeros((rows, Q.row_bytes(kvk, is_v=True)), dtype=torch.uint8, device=cuda)
    return (Q.paged_from_rows(zk, kvk, page_perm=perm),
            Q.paged_from_rows(zv, kvk, page_perm=perm, is_v=True), perm)


def _read_rows(side, rb, rows, perm):
    pages = side.data.view((rows + 63) // 64, 64 * rb)[perm.to(side.data.device)]
    return pages.reshape(-1, rb)[:rows].cpu().numpy()


@pytest.mark.parametrize("kvk", KINDS)
def test_stores_match_cpu_codecs_bytewise(oracle, cuda, kvk):
    """kv_store_T_t3 over T rows and kv_store_t3 over draft lanes: K rows in the kind's K
    format, V rows as turbo3, every other row untouched."""
    base, T = 37, 150
    kf, vf = synth.make_kv(oracle, T, kvk, seed=17, outlier_frac=0.02)
    kf[3] = 0.0                                   # zero groups: zero scale / zero norm paths
    kf[4, :, 64:128] = 0.0
    kf[5] *= 1e-6
    ks, vs, perm = _empty_sides(cuda, kvk, base + T, scatter=4)
    Q.kv_store_T_t3(torch.from_numpy(kf.reshape(T, -1)).to(cuda),
                    torch.from_numpy(vf.reshape(T, -1)).to(cuda), ks.tab, vs.tab, base, 4, 256, T,
                    kvk=kvk)
    torch.cuda.synchronize()
    gk = _read_rows(ks, Q.row_bytes(kvk), base + T, perm)
    gv = _read_rows(vs, 400, base + T, perm)
    assert (gk[base:] == k_blocks(oracle, kvk, kf)).all() and (gk[:base] == 0).all()
    assert (gv[base:] == oracle.t3_quant(vf.reshape(-1, 128)).reshape(T, 400)).all()
    assert (gv[:base] == 0).all()
    # lane form
    rows, pos = 300, [299, 3, 64, 127, 128, 250]
    n = len(pos)
    ks, vs, perm = _empty_sides(cuda, kvk, rows, scatter=6)
    kd = [torch.from_numpy(kf[t].reshape(-1).copy()).to(cuda) for t in range(n)]
    vd = [torch.from_numpy(vf[t].reshape(-1).copy()).to(cuda) for t in range(n)]
    pd = [torch.tensor([p], dtype=torch.int32, device=cuda) for p in pos]
    Q.kv_store_t3(kd, vd, ks.tab, vs.tab, pd, 4, 256, kvk=kvk)
    torch.cuda.synchronize()
    gk = _read_rows(ks, Q.row_bytes(kvk), rows, perm)
    gv = _read_rows(vs, 400, rows, perm)
    wk = k_blocks(oracle, kvk, kf[:n])
    wv = oracle.t3_quant(vf[:n].reshape(-1, 128)).reshape(n, 400)
    for t, p in enumerate(pos):
        assert (gk[p] == wk[t]).all() and (gv[p] == wv[t]).all()
    untouched = np.ones(rows, bool)
    untouched[pos] = False
    assert (gk[untouched] == 0).all() and (gv[untouched] == 0).all()


@pytest.mark.parametrize("kvk", KINDS)
def test_store_then_attend_end_to_end(oracle, cuda, kvk):
    """Raw fp32 K/V and Q in, attention out, with the rotation steps of the engine
    (src/engine.cuh:1485-1506): Q rotated only where the K side is; the output un-rotated
    because V is turbo3. Against a plain softmax over the ORIGINAL values, the quantisation
    error is all that separates the two."""
    rows, ntok = 700, 3
    kf, vf = synth.make_kv(oracle, rows, kvk, seed=23)
    q = oracle.randn(ntok * synth.Q_ROW, 77).reshape(ntok, 24, synth.Q_STRIDE)
    ks, vs, perm = _empty_sides(cuda, kvk, rows, scatter=8)
    Q.kv_store_T_t3(torch.from_numpy(kf.reshape(rows, -1)).to(cuda),
                    torch.from_numpy(vf.reshape(rows, -1)).to(cuda), ks.tab, vs.tab, 0, 4, 256,
                    rows, kvk=kvk)
    ql = [torch.from_numpy(q[t].reshape(-1).copy()).to(cuda) for t in range(ntok)]
    if Q.kv_k_rotated(kvk):
        Q.wht3(ql, 24, 256, synth.Q_STRIDE, False)
    pos = [rows - 1, 300, 0]
    pl = [torch.tensor([p], dtype=torch.int32, device=cuda) for p in pos]
    out = [torch.empty(synth.OUT_ROW, device=cuda) for _ in range(ntok)]
    scratch = torch.empty(Q.decode_scratch_floats(ntok), device=cuda)
    Q.attn_decode3(ql, synth.Q_STRIDE, ks.tab, vs.tab, out, scratch, pl, 0, 24, 4, 256, SCALE,
                   ntok=ntok, kvk=kvk)
    Q.wht3(out, 24, 256, 256, True)
    torch.cuda.synchronize()
    got = np.stack([o.cpu().numpy() for o in out]).reshape(ntok, 24, 256)
    # the same pipeline on the CPU oracle: bit-identical caches, so the tight gate applies
    c = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=23)
    c.q[:, :, :256] = oracle.wht(np.ascontiguousarray(q[:, :, :256])) if Q.kv_k_rotated(kvk) else q[:, :, :256]
    ref_rot = oracle.attn_decode(c.q, c.k, c.v, kvk, pos).reshape(ntok, 24, 256)
    ref = oracle.wht(np.ascontiguousarray(ref_rot), inverse=True)
    assert rel_err(got, ref) < TIGHT
    # and against the unquantised truth: cosine of the outputs (V is 3-bit: >= 0.95)
    for t, p in enumerate(pos):
        for h in (0, 11, 23):
            s = kf[: p + 1, h // 6].astype(np.float64) @ q[t, h, :256].astype(np.float64) / 16.0
            w = np.exp(s - s.max())
            plain = (w[:, None] * vf[: p + 1, h // 6]).sum(0) / w.sum()
            cos = (got[t, h] * plain).sum() / np.sqrt((got[t, h] ** 2).sum() * (plain ** 2).sum())
            assert cos > 0.95, (kvk, t, h, cos)


@pytest.mark.skipif(not REF_GPU_SO.exists(), reason="oracle/_ref not built")
@pytest.mark.parametrize("kvk", KINDS)
def test_against_reference_kernels_on_this_gpu(oracle, cuda, kvk):
    """The reference's own device encoder and scalar decode kernel, recompiled for sm_100a
    from the reference tree, on identical inputs: K blocks byte-equal (turbo5k in the device's
    reduction order, int8-g64 and fp16 order-free), attention within the tight gate."""
    ref = RefGpu()
    T = 256
    kf, vf = synth.make_kv(oracle, T, kvk, seed=31, outlier_frac=0.02)
    kT = torch.from_numpy(kf.reshape(T, -1)).to(cuda)
    vT = torch.from_numpy(vf.reshape(T, -1)).to(cuda)
    mk, mv, perm = _empty_sides(cuda, kvk, T, scatter=1)
    rk, rv, _ = _empty_sides(cuda, kvk, T, scatter=1)
    Q.kv_store_T_t3(kT, vT, mk.tab, mv.tab, 0, 4, 256, T, kvk=kvk)
    ref.lib.q27ref_kv_store_T_t3(kT.data_ptr(), vT.data_ptr(), rk.tab.data_ptr(), rv.tab.data_ptr(),
                                 0, 4, 256, T, None, kvk)
    torch.cuda.synchronize()
    rb = Q.row_bytes(kvk)
    assert (_read_rows(mk, rb, T, perm) == _read_rows(rk, rb, T, perm)).all()
    for seq, ntok in ((47, 1), (1024, 5), (16384, 5)):
        pos = [max(seq - ntok + t, 0) for t in range(ntok)]
        c = synth.make_case(oracle, kvk, rows=seq, pos=pos, seed=300 + seq % 89)
        want = oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos)
        dc = DeviceCase(c, cuda)
        theirs = ref.decode3(dc).copy()
        assert rel_err(theirs, want) < TIGHT                 # pins the oracle to the reference
        assert rel_err(dc.run3(), theirs) < 2 * TIGHT
