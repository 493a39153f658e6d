"""GPU parity tests of causal GQA prefill attention over a reused prefix, through the C ABI.
Cases follow the reference: T=23 at base 37 (test_attn_mma, src/test_kernels.cu:397-441), a
deep base (test_attn_split, :2207-2249), turbo3 at base 100 / T 48 (:2072-2201)."""
import numpy as np
import pytest
import torch

import q27_b200 as Q
from tests import synth
from tests.gpu_util import SCALE
from tests.oracle_lib import KV_F16, KV_FP8, KV_T3

pytestmark = pytest.mark.gpu


def run_prefill(oracle, cuda, kvk, base, T, t0=0, SB=None, seed=1, exact=False, scatter=None,
                bf16=False, with_part=True):
    SB = T - t0 if SB is None else SB
    c = synth.make_case(oracle, kvk, rows=base + T, pos=[0] * T, seed=seed, bf16=bf16)
    ref = synth.scale_out(c, oracle.attn_prefill(c.q, c.k, c.v, kvk, base, t0, SB))
    perm = None
    if scatter is not None:
        perm = torch.from_numpy(np.random.default_rng(scatter).permutation((base + T + 63) // 64))
    ks = Q.paged_from_rows(torch.from_numpy(c.k).to(cuda), kvk, page_perm=perm)
    vs = Q.paged_from_rows(torch.from_numpy(c.v).to(cuda), kvk, page_perm=perm)
    qT = torch.from_numpy(c.q.reshape(T, -1).copy()).to(cuda)
    outT = torch.zeros((T, synth.OUT_ROW), device=cuda)
    part = torch.full((Q.prefill_part_floats(SB),), float("nan"), device=cuda)
    Q.attn_prefill_T(qT, synth.Q_STRIDE, synth.Q_ROW, ks.tab, vs.tab, outT, synth.OUT_ROW,
                     part if with_part else None, base, t0, SB, 24, 4, 256, SCALE, kvk=kvk,
                     exact=exact)
    torch.cuda.synchronize()
    return synth.scale_out(c, outT.cpu().numpy()), ref


@pytest.mark.parametrize("kvk", [KV_F16, KV_FP8, KV_T3])
@pytest.mark.parametrize("exact", [True, False])
def test_prefill_small(oracle, cuda, kvk, exact):
    got, ref = run_prefill(oracle, cuda, kvk, base=37, T=23, seed=3, exact=exact, scatter=5)
    ok, excess, rel = synth.tolerance_ok(got, ref)
    assert ok, (excess, rel)
    if exact:
        assert rel < 2e-4


@pytest.mark.parametrize("exact", [True, False])
def test_prefill_sub_batch_leaves_other_rows(oracle, cuda, exact):
    got, ref = run_prefill(oracle, cuda, KV_F16, base=100, T=48, t0=16, SB=20, seed=4, exact=exact)
    assert synth.tolerance_ok(got[16:36], ref[16:36])[0]
    assert (got[:16] == 0).all() and (got[36:] == 0).all()


def test_prefill_turbo3_base100(oracle, cuda):
    got, ref = run_prefill(oracle, cuda, KV_T3, base=100, T=48, seed=6)
    assert synth.tolerance_ok(got, ref)[0]


def test_prefill_deep_prefix_bf16_values(oracle, cuda):
    # the prefill workload in miniature: bf16-rounded Q/K/V in an fp16 cache, a reused prefix
    # fully visible, the chunk causal
    got, ref = run_prefill(oracle, cuda, KV_F16, base=2048 + 64, T=256, seed=8, bf16=True)
    ok, excess, rel = synth.tolerance_ok(got, ref)
    assert ok, (excess, rel)


def test_prefill_no_prefix_first_row_is_v0(oracle, cuda):
    got, ref = run_prefill(oracle, cuda, KV_F16, base=0, T=70, seed=9)
    assert synth.tolerance_ok(got, ref)[0]


@pytest.mark.parametrize("kvk", [KV_F16, KV_T3])
def test_prefill_tail_items_split_into_key_ranges(oracle, cuda, kvk):
    """With scratch given, the items that do not fill a wave of SMs are cut into key-range
    pieces whose partials a fix-up kernel merges (here: 32 items, four pieces each; the
    scratch starts as NaN, so a piece that was skipped or read early would show). Without
    scratch the same call runs every item whole; both match the oracle and each other."""
    base, T = 4096 + 37, 160
    split, ref = run_prefill(oracle, cuda, kvk, base=base, T=T, seed=12, scatter=7)
    whole, _ = run_prefill(oracle, cuda, kvk, base=base, T=T, seed=12, scatter=7, with_part=False)
    assert np.isfinite(split).all()
    assert synth.tolerance_ok(split, ref)[0]
    assert synth.tolerance_ok(whole, ref)[0]
    # same tiles, same operands; the pieces round P against their own running maxima
    assert np.abs(split - whole).max() <= 1e-3 * np.abs(ref).max()


def test_prefill_tail_split_sub_batch(oracle, cuda):
    """A sub-batch (t0 > 0) through the split path: rows outside [t0, t0 + SB) stay untouched."""
    got, ref = run_prefill(oracle, cuda, KV_F16, base=6000, T=200, t0=30, SB=150, seed=13)
    assert synth.tolerance_ok(got[30:180], ref[30:180])[0]
    assert (got[:30] == 0).all() and (got[180:] == 0).all()
