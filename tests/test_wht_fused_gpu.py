"""GPU tests of attention with the rotation folded in: the `_wht` entries take the un-rotated
Q and write the un-rotated output. The gate is the reference's own three-launch sequence
(wht3 forward on Q where the K side is rotated -> attention -> wht3 inverse on the output,
src/engine.cuh:1482-1506) run through this engine's separate kernels: BITWISE equality, in
every kernel family (fp32 exact, mma.sync decode, tcgen05 verify, tcgen05 prefill with and
without split tail items, scalar prefill) and through the KV-sequence split. The separate
rotation kernels are themselves pinned bitwise to the CPU rotation (tests/test_kv_store_gpu.py)."""
import numpy as np
import pytest
import torch

import q27_b200 as Q
from tests import synth
from tests.gpu_util import SCALE, DeviceCase
from tests.oracle_lib import KV_F16, KV_I8G64, KV_T3, KV_T3V, KV_T5K

pytestmark = pytest.mark.gpu
TURBO = [KV_T3, KV_T3V, KV_T5K, KV_I8G64]


def raw_case(oracle, kvk, rows, pos, seed):
    """A case whose q is the UN-rotated query (the cache is encoded as usual)."""
    c = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=seed, outlier_frac=0.02)
    c.q = c.q_raw.copy()
    return c


def three_launches(dc, kvk, exact):
    """wht3 -> attention -> wht3 with the separate kernels, on copies of the lanes' Q."""
    q = [t.clone() for t in dc.q]
    if Q.kv_k_rotated(kvk):
        Q.wht3(q, 24, 256, synth.Q_STRIDE, False)
    slot = dc.slot()
    slot = Q.SlotArgs(slot.ktab, slot.vtab, q, slot.pos_lanes, slot.out_lanes, slot.scratch,
                      row_base=slot.row_base, row_count=slot.row_count)
    Q.attn_decode_batched([slot], synth.Q_STRIDE, 24, 4, 256, SCALE, kvk=kvk, exact=exact)
    if kvk >= KV_T3:
        Q.wht3(dc.out, 24, 256, 256, True)
    torch.cuda.synchronize()
    return np.stack([o.cpu().numpy() for o in dc.out])


@pytest.mark.parametrize("kvk", TURBO)
@pytest.mark.parametrize("exact", [True, False])
@pytest.mark.parametrize("ntok,seq", [(1, 47), (1, 5000), (5, 3000), (16, 700)])
def test_decode_bitwise_equals_three_launches(oracle, cuda, kvk, exact, ntok, seq):
    pos = [max(seq - ntok + t, 0) for t in range(ntok)]
    c = raw_case(oracle, kvk, seq, pos, seed=400 + seq % 91)
    c.q[:, :, 256:] = np.nan                           # the gate half is never read
    dc = DeviceCase(c, cuda, scatter_seed=5)
    want = three_launches(dc, kvk, exact)
    qcopy = [t.clone() for t in dc.q]
    for o in dc.out:
        o.fill_(float("nan"))
    Q.attn_decode_batched([dc.slot()], synth.Q_STRIDE, 24, 4, 256, SCALE, kvk=kvk, exact=exact,
                          wht=True)
    torch.cuda.synchronize()
    got = np.stack([o.cpu().numpy() for o in dc.out])
    assert np.isfinite(got).all()
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    for a, b in zip(dc.q, qcopy):                      # the caller's Q stays un-rotated
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    # and the result is attention: against the oracle's full pipeline (rotate, attend, un-rotate)
    cr = synth.make_case(oracle, kvk, rows=seq, pos=pos, seed=400 + seq % 91, outlier_frac=0.02)
    ref = oracle.wht(oracle.attn_decode(cr.q, cr.k, cr.v, kvk, pos).reshape(ntok, 24, 256), inverse=True)
    # (the element-wise parity bar is judged in the basis the kernels work in,
    # tests/test_decode_gpu.py; the rotation is orthonormal, so the RMS of the error is the
    # same in both bases and is what is checked here)
    err = got.reshape(ntok, 24, 256).astype(np.float64) - ref
    assert np.sqrt((err ** 2).mean() / (ref.astype(np.float64) ** 2).mean()) < (1e-4 if exact else 5e-3)


def test_reference_shaped_entry_and_plain_kinds(oracle, cuda):
    """q27_attn_decode3_wht, and the fp16 kind through it: no rotation, same bits as the plain
    entry."""
    c = raw_case(oracle, KV_T3, 900, [899, 500, 3], seed=7)
    dc = DeviceCase(c, cuda)
    want = three_launches(dc, KV_T3, False)
    Q.attn_decode3(dc.q, synth.Q_STRIDE, dc.kside.tab, dc.vside.tab, dc.out, dc.scratch, dc.pos, 0,
                   24, 4, 256, SCALE, ntok=3, kvk=KV_T3, wht=True)
    torch.cuda.synchronize()
    got = np.stack([o.cpu().numpy() for o in dc.out])
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    c = synth.make_case(oracle, KV_F16, rows=700, pos=[699], seed=8)
    dc = DeviceCase(c, cuda)
    plain = dc.run3()
    Q.attn_decode3(dc.q, synth.Q_STRIDE, dc.kside.tab, dc.vside.tab, dc.out, dc.scratch, dc.pos, 0,
                   24, 4, 256, SCALE, ntok=1, kvk=KV_F16, wht=True)
    torch.cuda.synchronize()
    assert (dc.out[0].cpu().numpy().view(np.uint32) == plain[0].view(np.uint32)).all()


@pytest.mark.parametrize("kvk", [KV_T3, KV_T5K])
def test_kv_split_bitwise(oracle, cuda, kvk):
    """Sharded cache: the partial side rotates Q, the merge side un-rotates the output."""
    rows, pos = 64 * 12, [64 * 12 - 1, 400, 70]
    c = raw_case(oracle, kvk, rows, pos, seed=13)
    cr = synth.make_case(oracle, kvk, rows=rows, pos=pos, seed=13, outlier_frac=0.02)   # rotated q
    bounds = [0, 256, 512, rows]

    def run(case, wht):
        parts = torch.empty((3, 3, 24, 258), device=cuda)
        for s in range(3):
            shard = DeviceCase(case, cuda, row_lo=bounds[s], row_hi=bounds[s + 1])
            Q.attn_decode_partial([shard.slot()], 3, synth.Q_STRIDE, 24, 4, 256, SCALE, parts[s],
                                  kvk=kvk, wht=wht)
        out = torch.empty((3 * 24, 256), device=cuda)
        Q.attn_merge_partials(parts, 3, 3 * 24, out, wht_kvk=kvk if wht else None)
        if not wht:
            Q.wht_T(out, 3 * 24, 256, 256, 3 * 24 * 256, 1, True)
        torch.cuda.synchronize()
        return out.cpu().numpy()

    assert (run(c, True).view(np.uint32) == run(cr, False).view(np.uint32)).all()


def _prefill(cuda, c, kvk, base, T, t0, SB, exact, wht, with_part=True):
    ks = Q.paged_from_rows(torch.from_numpy(c.k).to(cuda), kvk)
    vs = Q.paged_from_rows(torch.from_numpy(c.v).to(cuda), kvk, is_v=True)
    qT = torch.from_numpy(c.q.reshape(T, -1).copy()).to(cuda)
    outT = torch.zeros((T, synth.OUT_ROW), device=cuda)
    part = torch.full((Q.prefill_part_floats(SB),), float("nan"), device=cuda) if with_part else None
    if not wht:
        if Q.kv_k_rotated(kvk):
            Q.wht_T(qT, 24, 256, synth.Q_STRIDE, synth.Q_ROW, T, False)
    Q.attn_prefill_T(qT, synth.Q_STRIDE, synth.Q_ROW, ks.tab, vs.tab, outT, synth.OUT_ROW, part, base,
                     t0, SB, 24, 4, 256, SCALE, kvk=kvk, exact=exact, wht=wht)
    if not wht:
        # the engine rotates the rows the sub-batch wrote (src/prefill.cu:2598-2618)
        Q.wht_T(outT[t0:t0 + SB], 24, 256, 256, synth.OUT_ROW, SB, True)
    torch.cuda.synchronize()
    return outT.cpu().numpy()


@pytest.mark.parametrize("kvk", TURBO)
@pytest.mark.parametrize("exact", [True, False])
def test_prefill_bitwise_equals_three_launches(oracle, cuda, kvk, exact):
    base, T = 100, 48
    c = raw_case(oracle, kvk, base + T, [0] * T, seed=21)
    want = _prefill(cuda, c, kvk, base, T, 8, 30, exact, wht=False)
    got = _prefill(cuda, c, kvk, base, T, 8, 30, exact, wht=True)
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    assert (got[:8] == 0).all() and (got[38:] == 0).all()      # rows outside the sub-batch untouched


def test_prefill_split_tail_items_bitwise(oracle, cuda):
    """A chunk whose item count does not fill a wave: the tail items are cut into key ranges
    and the fix-up kernel holds the inverse rotation (with and without scratch for pieces)."""
    base, T = 2000, 64 * 21 + 9                   # 65 Q tiles x 4 kv heads = 260 items: 112 in the tail
    c = raw_case(oracle, KV_T3, base + T, [0] * T, seed=23)
    want = _prefill(cuda, c, KV_T3, base, T, 0, T, False, wht=False)
    got = _prefill(cuda, c, KV_T3, base, T, 0, T, False, wht=True)
    assert (got.view(np.uint32) == want.view(np.uint32)).all()
    nopart = _prefill(cuda, c, KV_T3, base, T, 0, T, False, wht=True, with_part=False)
    want_np = _prefill(cuda, c, KV_T3, base, T, 0, T, False, wht=False, with_part=False)
    assert (nopart.view(np.uint32) == want_np.view(np.uint32)).all()
