"""The BASELINE configurations at their FULL sizes, on data generated and encoded on the GPU.
The CPU oracle does not finish these in seconds, so the comparator is the library's own fp32
scalar family (`exact=True`: bit-exact element decode, fp32 FMA, expf), which the small-size
tests pin to the oracle and to the reference's recompiled kernels; on top of that come
properties that hold at any size: the log-sum-exp merge over KV shards equals attention over
the whole cache, identical V rows come back whatever the keys are, and the chunked prefill
equals the scalar prefill kernel."""
import numpy as np
import pytest
import torch

import q27_b200 as Q
from tests import synth
from tests.gpu_util import SCALE
from tests.oracle_lib import KV_F16, KV_FP8, KV_T3

pytestmark = pytest.mark.gpu

N_Q, N_KV, HD, QS = 24, 4, 256, 512
FP8_SCALE = 6.0 / 448.0


def device_cache(kvk, rows, seed, dev, same_v=False):
    """K / V caches of `rows` rows built on the device through the library's own stores (the
    turbo3 encoder is byte-identical to the CPU codec, tests/test_kv_store_gpu.py)."""
    rb = Q.row_bytes(kvk)
    sides = []
    for _ in range(2):
        store = torch.empty(((rows + 63) // 64) * 64 * rb, dtype=torch.uint8, device=dev)
        sides.append((store, Q.mk_tab(store, rb, rows)))
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    v_row = torch.randn((1, N_KV * HD), generator=g, device=dev).half().float()
    for r0 in range(0, rows, 8192):
        t = min(8192, rows - r0)
        k = torch.randn((t, N_KV * HD), generator=g, device=dev).half().float()
        v = v_row.expand(t, -1).contiguous() if same_v else \
            torch.randn((t, N_KV * HD), generator=g, device=dev).half().float()
        if kvk == KV_T3:
            Q.kv_store_T_t3(k, v, sides[0][1], sides[1][1], r0, N_KV, HD, t)
        else:
            s = FP8_SCALE if kvk == KV_FP8 else 1.0
            Q.kv_store_T(k / s, v / s, sides[0][1], sides[1][1], r0, N_KV * HD, t, fp8=kvk == KV_FP8)
    torch.cuda.synchronize()
    return sides


def decode(sides, kvk, q, pos, exact, row_base=0, row_count=2**31 - 1, partial=None):
    dev = q.device
    lanes = q.shape[0]
    out = torch.zeros((lanes, N_Q * HD), device=dev)
    scratch = torch.full((Q.decode_scratch_floats(lanes),), float("nan"), device=dev)
    slot = Q.SlotArgs(sides[0][1], sides[1][1], [q[t] for t in range(lanes)],
                      [pos[t:t + 1] for t in range(lanes)], [out[t] for t in range(lanes)], scratch,
                      row_base=row_base, row_count=row_count)
    if partial is not None:
        Q.attn_decode_partial([slot], lanes, QS, N_Q, N_KV, HD, SCALE, partial, kvk=kvk)
    else:
        Q.attn_decode_batched([slot], QS, N_Q, N_KV, HD, SCALE, kvk=kvk, exact=exact)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("kvk,rows,lanes", [(KV_F16, 4096, 1), (KV_FP8, 32768, 6), (KV_T3, 131072, 1),
                                             (KV_T3, 262144, 6)])
def test_decode_and_verify_at_baseline_sizes(cuda, kvk, rows, lanes):
    """Configs 1, 2, 3 (one slot) and 5 (one slot): tensor-core path against the fp32 scalar
    family on the same buffers, inside the BASELINE bar."""
    sides = device_cache(kvk, rows, seed=100 + kvk, dev=cuda)
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    q = torch.randn((lanes, N_Q * QS), generator=g, device=cuda) * (FP8_SCALE if kvk == KV_FP8 else 1.0)
    pos = torch.tensor([rows - lanes + t for t in range(lanes)], dtype=torch.int32, device=cuda)
    fast = decode(sides, kvk, q, pos, exact=False)
    slow = decode(sides, kvk, q, pos, exact=True)
    vs = FP8_SCALE if kvk == KV_FP8 else 1.0
    ok, excess, rel = synth.tolerance_ok(fast * vs, slow * vs)
    assert ok, (excess, rel)


def test_identical_v_rows_come_back_at_131k(cuda):
    """Softmax weights sum to one: with every V row the same turbo3 row, the output is that
    row (dequantised), whatever 131072 keys say -- no row may be dropped, doubled or weighted
    by a stale norm anywhere along the ring."""
    rows = 131072
    sides = device_cache(KV_T3, rows, seed=7, dev=cuda, same_v=True)
    v0 = torch.empty((1, N_KV, HD), device=cuda)
    Q.kv_dequant(sides[1][1], KV_T3, 0, 1, N_KV, v0)
    g = torch.Generator(device=cuda)
    g.manual_seed(9)
    q = torch.randn((1, N_Q * QS), generator=g, device=cuda)
    pos = torch.tensor([rows - 1], dtype=torch.int32, device=cuda)
    out = decode(sides, KV_T3, q, pos, exact=False).reshape(N_Q, HD)
    want = np.repeat(v0.cpu().numpy().reshape(N_KV, HD), N_Q // N_KV, axis=0)
    assert synth.tolerance_ok(out, want)[0]


def test_shard_merge_equals_whole_at_131k(cuda):
    """KV-sequence split at full length: four page-aligned shards, partials merged with the
    log-sum-exp combine, against attention over the whole cache."""
    rows, nsh = 131072, 4
    sides = device_cache(KV_T3, rows, seed=11, dev=cuda)
    g = torch.Generator(device=cuda)
    g.manual_seed(3)
    q = torch.randn((1, N_Q * QS), generator=g, device=cuda)
    pos = torch.tensor([rows - 1], dtype=torch.int32, device=cuda)
    whole = decode(sides, KV_T3, q, pos, exact=False)
    parts = torch.empty((nsh, 1, 1, N_Q, 258), device=cuda)
    per = rows // nsh
    for s in range(nsh):
        # a shard sees the same tables; its window is [s*per, (s+1)*per)
        shard = [(sides[0][0], sides[0][1][s * per // 64:]), (sides[1][0], sides[1][1][s * per // 64:])]
        decode(shard, KV_T3, q, pos, exact=False, row_base=s * per, row_count=per, partial=parts[s])
    out = torch.empty((N_Q, HD), device=cuda)
    Q.attn_merge_partials(parts, nsh, N_Q, out)
    torch.cuda.synchronize()
    assert synth.tolerance_ok(out.cpu().numpy().reshape(1, -1), whole)[0]


@pytest.mark.parametrize("base", [8192, 22528])
def test_prefill_chunk_at_baseline_size(cuda, base):
    """Config 4, its first and its last chunk: 2048 new tokens over an 8192- / 22528-token
    prefix, bf16-rounded values in an fp16 cache; tile kernel (whole items at the short
    prefix, the tail wave cut into key ranges at the long one) against the fp32 scalar
    prefill kernel."""
    SB = 2048
    rows = base + SB
    sides = []
    for _ in range(2):
        store = torch.empty(((rows + 63) // 64) * 64 * 2048, dtype=torch.uint8, device=cuda)
        sides.append((store, Q.mk_tab(store, 2048, rows)))
    g = torch.Generator(device=cuda)
    g.manual_seed(21)
    k = torch.randn((rows, N_KV * HD), generator=g, device=cuda).bfloat16().float()
    v = torch.randn((rows, N_KV * HD), generator=g, device=cuda).bfloat16().float()
    Q.kv_store_T(k, v, sides[0][1], sides[1][1], 0, N_KV * HD, rows)
    qT = torch.randn((SB, N_Q * QS), generator=g, device=cuda).bfloat16().float()
    part = torch.full((Q.prefill_part_floats(SB),), float("nan"), device=cuda)
    outs = []
    for exact in (False, True):
        outT = torch.zeros((SB, N_Q * HD), device=cuda)
        Q.attn_prefill_T(qT, QS, N_Q * QS, sides[0][1], sides[1][1], outT, N_Q * HD, part, base, 0, SB,
                         N_Q, N_KV, HD, SCALE, kvk=KV_F16, exact=exact)
        torch.cuda.synchronize()
        outs.append(outT.cpu().numpy())
    ok, excess, rel = synth.tolerance_ok(outs[0], outs[1])
    assert ok, (excess, rel)
