"""The five named workloads at their FULL sizes, pinned to the CPU oracle.

Caches are drawn and encoded on the GPU with the workload generators of
``q27_b200.workloads`` (2 % of the channels scaled x8 for the turbo3 workloads, per-head absmax
scales for the fp8 one), copied to the host, and the oracle computes the same attention from
the same bytes: 4096 fp16 rows x 1 lane, 32768 fp8 rows x 6 lanes, 2 slots x 131072 turbo3
rows, one slot of 262144 turbo3 rows x 6 lanes (about three seconds of oracle), and a stated
sample of the query rows of the first and the last 2048-token prefill chunk. Bar: the
element-wise 2e-3 + 1e-3*|ref| of the headline metric.

On top come properties that hold at any size: identical V rows come back whatever the keys
are, and the log-sum-exp merge over KV shards equals attention over the whole cache."""
import numpy as np
import pytest
import torch

import q27_b200 as Q
from q27_b200 import workloads as W
from tests import synth
from tests.oracle_lib import KV_F16, KV_FP8, KV_T3

pytestmark = pytest.mark.gpu

N_Q, N_KV, HD, QS = W.N_Q, W.N_KV, W.HD, W.Q_STRIDE
SCALE = W.SCALE


def run_slots(caches, q, pos, kvk, exact=False):
    """q [nslots, lanes, 24*512] device, pos [nslots, lanes] int32 device -> [nslots, lanes, 6144]"""
    nslots, lanes = pos.shape
    dev = q.device
    out = torch.full((nslots, lanes, N_Q * HD), float("nan"), device=dev)
    scratch = [torch.full((Q.decode_scratch_floats(lanes),), float("nan"), device=dev)
               for _ in range(nslots)]
    slots = [Q.SlotArgs(c.ktab, c.vtab, [q[s, t] for t in range(lanes)],
                        [pos[s, t:t + 1] for t in range(lanes)], [out[s, t] for t in range(lanes)],
                        scratch[s]) for s, c in enumerate(caches)]
    Q.attn_decode_batched(slots, QS, N_Q, N_KV, HD, SCALE, kvk=kvk, exact=exact)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c5"])
def test_named_decode_workloads_against_the_oracle(oracle, cuda, name):
    wl = W.DECODE[name]
    nslots = 1 if name == "c5" else wl.slots          # one slot of the 8 x 262144 workload
    caches = [W.make_cache(wl.kvk, wl.rows, 300 + 10 * s, wl.outlier_frac, cuda)
              for s in range(nslots)]
    q_host = W.make_queries(nslots, wl.lanes, seed=17)
    pos_host = torch.tensor([[wl.rows - wl.lanes + t for t in range(wl.lanes)]] * nslots,
                            dtype=torch.int32)
    q_dev = q_host.to(cuda)
    if wl.kvk == KV_FP8:
        q_dev = torch.stack([W.fold_k_scale(q_dev[s], caches[s].k_scale) for s in range(nslots)])
    got = run_slots(caches, q_dev, pos_host.to(cuda), wl.kvk)
    for s, c in enumerate(caches):
        k, v = c.host_rows()
        ref = oracle.attn_decode(q_dev[s].cpu().numpy().reshape(wl.lanes, N_Q, QS), k, v, wl.kvk,
                                 pos_host[s].tolist())
        g = got[s]
        if wl.kvk == KV_FP8:       # parity is judged on the real-valued outputs
            g = W.apply_v_scale(g, c.v_scale)
            ref = W.apply_v_scale(torch.from_numpy(ref), c.v_scale.cpu()).numpy()
        ok, excess, rel = synth.tolerance_ok(g.cpu().numpy(), ref)
        assert ok, (name, s, excess, rel)


@pytest.mark.parametrize("base", [8192, 22528])
def test_prefill_chunks_against_the_oracle(oracle, cuda, base):
    """First and last chunk of the prefill workload (2048 new tokens over an 8192- / 22528-row
    prefix, bf16-rounded values in an fp16 cache). The kernel runs the whole chunk; the oracle
    checks query rows 0..63 and 1984..2047 of it (64 rows each: the chunk's first tile, which
    sees the prefix and almost nothing of the chunk, and its last, which sees all of it)."""
    SB = W.PREFILL_C4["chunk"]
    rows = base + SB
    g = torch.Generator(device=cuda)
    g.manual_seed(21 + base)
    rb = W.ROW_BYTES[KV_F16]
    stores = [torch.empty(((rows + 63) // 64) * 64 * rb, dtype=torch.uint8, device=cuda) for _ in range(2)]
    ktab, vtab = Q.mk_tab(stores[0], rb, rows), Q.mk_tab(stores[1], rb, rows)
    k = W.bf16_values((rows, N_KV * HD), g, cuda)
    v = W.bf16_values((rows, N_KV * HD), g, cuda)
    Q.kv_store_T(k, v, ktab, vtab, 0, N_KV * HD, rows)
    qT = W.bf16_values((SB, N_Q * QS), g, cuda)
    part = torch.full((Q.prefill_part_floats(SB),), float("nan"), device=cuda)
    outT = torch.full((SB, N_Q * HD), float("nan"), device=cuda)
    Q.attn_prefill_T(qT, QS, N_Q * QS, ktab, vtab, outT, N_Q * HD, part, base, 0, SB, N_Q, N_KV,
                     HD, SCALE, kvk=KV_F16)
    torch.cuda.synchronize()
    got = outT.cpu().numpy()
    assert np.isfinite(got).all()
    kh = stores[0][: rows * rb].cpu().numpy().reshape(rows, rb)
    vh = stores[1][: rows * rb].cpu().numpy().reshape(rows, rb)
    qh = qT.cpu().numpy().reshape(SB, N_Q, QS)
    for t0 in (0, SB - 64):
        ref = oracle.attn_prefill(qh, kh, vh, KV_F16, base, t0, 64)
        ok, excess, rel = synth.tolerance_ok(got[t0:t0 + 64], ref[t0:t0 + 64])
        assert ok, (base, t0, excess, rel)


def test_prefill_chunk_matches_the_scalar_kernel_everywhere(cuda):
    """Every query row of the last chunk: the tile kernel against the engine's fp32 scalar
    prefill (itself pinned to the oracle at small sizes), so no row between the two oracle
    samples above goes unchecked."""
    SB, base = W.PREFILL_C4["chunk"], 22528
    rows = base + SB
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    rb = W.ROW_BYTES[KV_F16]
    stores = [torch.empty(((rows + 63) // 64) * 64 * rb, dtype=torch.uint8, device=cuda) for _ in range(2)]
    ktab, vtab = Q.mk_tab(stores[0], rb, rows), Q.mk_tab(stores[1], rb, rows)
    Q.kv_store_T(W.bf16_values((rows, N_KV * HD), g, cuda), W.bf16_values((rows, N_KV * HD), g, cuda),
                 ktab, vtab, 0, N_KV * HD, rows)
    qT = W.bf16_values((SB, N_Q * QS), g, cuda)
    part = torch.full((Q.prefill_part_floats(SB),), float("nan"), device=cuda)
    outs = []
    for exact in (False, True):
        outT = torch.zeros((SB, N_Q * HD), device=cuda)
        Q.attn_prefill_T(qT, QS, N_Q * QS, ktab, vtab, outT, N_Q * HD, part, base, 0, SB, N_Q, N_KV,
                         HD, SCALE, kvk=KV_F16, exact=exact)
        torch.cuda.synchronize()
        outs.append(outT.cpu().numpy())
    ok, excess, rel = synth.tolerance_ok(outs[0], outs[1])
    assert ok, (excess, rel)


def test_identical_v_rows_come_back_at_131k(cuda):
    """Softmax weights sum to one: with every V row the same turbo3 row, the output is that
    row (dequantised), whatever 131072 keys say -- no row may be dropped, doubled or weighted
    by a stale norm anywhere along the ring."""
    rows = 131072
    c = W.make_cache(KV_T3, rows, 7, 0.02, cuda, same_v=True)
    v0 = torch.empty((1, N_KV, HD), device=cuda)
    Q.kv_dequant(c.vtab, KV_T3, 0, 1, N_KV, v0)
    q = W.make_queries(1, 1, seed=9).to(cuda)
    pos = torch.tensor([[rows - 1]], dtype=torch.int32, device=cuda)
    out = run_slots([c], q, pos, KV_T3)[0].cpu().numpy().reshape(N_Q, HD)
    want = np.repeat(v0.cpu().numpy().reshape(N_KV, HD), N_Q // N_KV, axis=0)
    assert synth.tolerance_ok(out, want)[0]


def test_shard_merge_equals_whole_at_131k(cuda):
    """KV-sequence split at full length: four page-aligned shards, partials merged with the
    log-sum-exp combine, against attention over the whole cache."""
    rows, nsh = 131072, 4
    c = W.make_cache(KV_T3, rows, 11, 0.02, cuda)
    q = W.make_queries(1, 1, seed=3).to(cuda)
    pos = torch.tensor([[rows - 1]], dtype=torch.int32, device=cuda)
    whole = run_slots([c], q, pos, KV_T3)[0].cpu().numpy()
    parts = torch.empty((nsh, 1, 1, N_Q, 258), device=cuda)
    per = rows // nsh
    scratch = torch.full((Q.decode_scratch_floats(1),), float("nan"), device=cuda)
    for s in range(nsh):
        # a shard sees the same tables from its first page on; its window is [s*per, (s+1)*per)
        slot = Q.SlotArgs(c.ktab[s * per // 64:], c.vtab[s * per // 64:], [q[0, 0]], [pos[0, 0:1]], [],
                          scratch, row_base=s * per, row_count=per)
        Q.attn_decode_partial([slot], 1, QS, N_Q, N_KV, HD, SCALE, parts[s], kvk=KV_T3)
    out = torch.empty((N_Q, HD), device=cuda)
    Q.attn_merge_partials(parts, nsh, N_Q, out)
    torch.cuda.synchronize()
    assert synth.tolerance_ok(out.cpu().numpy().reshape(1, -1), whole)[0]
