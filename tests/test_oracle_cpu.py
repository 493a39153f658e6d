"""CPU tests of the oracle: pinned against the reference's own CPU codec (when the
reference tree was available to build oracle/_ref), against the committed golden
fixtures, and against the known-answer properties the reference's tests hold."""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest

from tests.oracle_lib import (ALL_KINDS, KV_F16, KV_FP8, KV_I8G64, KV_T3, KV_T3V, KV_T5K, HD,
                              REF_CODEC_SO, Oracle, RefCodec)
from tests import synth

GOLDEN = Path(__file__).resolve().parent / "golden"
_fp = C.POINTER(C.c_float)


@pytest.fixture(scope="module")
def ref():
    if not REF_CODEC_SO.exists():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    return RefCodec()


def test_block_is_50_bytes_and_zero_vector_packs_index_4(oracle):
    # sizeof(block_turbo3) == 50 (src/turbo3.cuh:33-34); a zero vector maps to centroid
    # index 4: low bits all 0, high bits all 1 (src/metal/test_metal_ops.cpp:304-311)
    blk = oracle.t3_quant(np.zeros(128, np.float32))
    assert blk.shape == (1, 50)
    assert (blk[0, 2:34] == 0).all() and (blk[0, 34:50] == 255).all()
    assert oracle.row_bytes(KV_T3) == 400 and oracle.row_bytes(KV_FP8) == 1024
    assert oracle.row_bytes(KV_F16) == 2048 and oracle.row_bytes(6) == -1
    # K rows of the kinds whose sides differ (656 / 1056 B: src/server.cu:891-892); V is turbo3
    assert [oracle.row_bytes(k) for k in (KV_T3V, KV_T5K, KV_I8G64)] == [2048, 656, 1056]
    assert all(oracle.row_bytes(k, is_v=True) == 400 for k in (KV_T3, KV_T3V, KV_T5K, KV_I8G64))


def test_tables_match_reference_header(oracle, ref):
    for mine, theirs, n in ((oracle.lib.q27o_t3_centroids(), ref.lib.q27ref_hdr_centroids(), 8),
                            (oracle.lib.q27o_t3_s1(), ref.lib.q27ref_hdr_s1(), 128),
                            (oracle.lib.q27o_t3_s2(), ref.lib.q27ref_hdr_s2(), 128)):
        assert [mine[i] for i in range(n)] == [theirs[i] for i in range(n)]
    assert ref.lib.q27ref_block_bytes() == 50
    for v in np.linspace(-0.25, 0.25, 4001, dtype=np.float32):
        assert oracle.lib.q27o_t3_nearest(float(v)) == ref.lib.q27ref_hdr_nearest(float(v)) \
            == ref.lib.q27ref_cpu_nearest(float(v))


def test_codec_bitwise_vs_reference_cpu_codec(oracle, ref):
    rng = np.random.default_rng(7)
    n = 4000
    x = (rng.standard_normal((n, 128)) * rng.choice([1e-3, 1, 8, 50], size=(n, 1))).astype(np.float32)
    x[0] = 0
    mine = oracle.t3_quant(x)
    theirs = np.zeros_like(mine)
    for i in range(n):
        ref.lib.q27ref_cpu_quant(x[i].ctypes.data_as(_fp), theirs[i].ctypes.data_as(C.c_void_p))
    assert (mine == theirs).all()
    deq = oracle.kv_dequant(mine.reshape(n // 8, 400), KV_T3, n // 8).reshape(n, 128)
    y = np.zeros(128, np.float32)
    for i in range(0, n, 17):
        ref.lib.q27ref_cpu_dequant(theirs[i].ctypes.data_as(C.c_void_p), y.ctypes.data_as(_fp))
        assert (deq[i].view(np.uint32) == y.view(np.uint32)).all()
    a, b = x[:256].copy(), x[:256].copy()
    for i in range(256):
        ref.lib.q27ref_cpu_fwht(b[i].ctypes.data_as(_fp))
    assert (oracle.wht(a).view(np.uint32) == b.view(np.uint32)).all()
    for i in range(256):
        ref.lib.q27ref_cpu_fwht_inv(b[i].ctypes.data_as(_fp))
    assert (oracle.wht(oracle.wht(a), inverse=True).view(np.uint32) == b.view(np.uint32)).all()


def test_turbo5_tables_and_codec_vs_reference_cpu_codec(oracle, ref):
    c, t = oracle.lib.q27o_t5_centroids(), oracle.lib.q27o_t5_thresholds()
    rc, rt = ref.lib.q27ref_hdr5_centroids(), ref.lib.q27ref_hdr5_thresholds()
    assert [c[i] for i in range(32)] == [rc[i] for i in range(32)]
    assert [t[i] for i in range(31)] == [rt[i] for i in range(31)]
    assert ref.lib.q27ref_block5_bytes() == 82
    probe = np.concatenate([np.linspace(-0.3, 0.3, 6001, dtype=np.float32),
                            np.array([t[i] for i in range(31)], np.float32)])
    for v in probe:
        assert oracle.lib.q27o_t5_nearest(float(v)) == ref.lib.q27ref_hdr5_nearest(float(v)) \
            == ref.lib.q27ref_cpu5_nearest(float(v))
    rng = np.random.default_rng(17)
    n = 3000
    x = (rng.standard_normal((n, 128)) * rng.choice([1e-3, 1, 8, 50], size=(n, 1))).astype(np.float32)
    x[0] = 0
    vp = C.c_void_p
    for tree in (True, False):
        mine = oracle.t5_quant(x, tree=tree)
        theirs = np.zeros_like(mine)
        for i in range(n):
            ref.lib.q27ref_cpu_quant5(x[i].ctypes.data_as(_fp), theirs[i].ctypes.data_as(vp), int(tree))
        assert (mine == theirs).all()
    mine = oracle.t5_quant(x)
    deq = oracle.kv_dequant(mine.reshape(n // 8, 656), KV_T5K, n // 8).reshape(n, 128)
    y = np.zeros(128, np.float32)
    for i in range(0, n, 13):
        ref.lib.q27ref_cpu_dequant5(mine[i].ctypes.data_as(vp), y.ctypes.data_as(_fp))
        assert (deq[i].view(np.uint32) == y.view(np.uint32)).all()


def test_int8_g64_codec_vs_reference_cpu_codec(oracle, ref):
    assert ref.lib.q27ref_block_i8_bytes() == 132
    rng = np.random.default_rng(19)
    n = 3000
    x = (rng.standard_normal((n, 128)) * rng.choice([1e-7, 1e-3, 1, 8, 300], size=(n, 1))).astype(np.float32)
    x[0] = 0
    x[1, :64] = 0
    x[2] = np.float32(65504.0 * 127)      # scale at the top of fp16
    vp = C.c_void_p
    mine = oracle.i8_quant(x)
    theirs = np.zeros_like(mine)
    for i in range(n):
        ref.lib.q27ref_i8_quant(x[i].ctypes.data_as(_fp), theirs[i].ctypes.data_as(vp))
    assert (mine == theirs).all()          # order-independent codec: exact, no tie class
    assert (mine[0] == 0).all() and (mine[1, :64] == 0).all() and (mine[1, 128:130] == 0).all()
    deq = oracle.kv_dequant(mine.reshape(n // 8, 1056), KV_I8G64, n // 8).reshape(n // 2, 256)
    y = np.zeros(256, np.float32)
    for r in range(0, n // 2, 11):
        ref.lib.q27ref_i8_dequant_row(mine[2 * r:].ctypes.data_as(vp), y.ctypes.data_as(_fp))
        assert (deq[r].view(np.uint32) == y.view(np.uint32)).all()


def test_converters_vs_cuda_host_converters(oracle, ref):
    for h in range(0, 65536, 3):
        a, b = oracle.lib.q27o_half_to_float(h), ref.lib.q27ref_half_to_float(h)
        assert a == b or (a != a and b != b)
    for b8 in range(256):
        a, b = oracle.lib.q27o_e4m3_to_float(b8), ref.lib.q27ref_e4m3_to_float(b8)
        assert a == b or (a != a and b != b)
    rng = np.random.default_rng(3)
    xs = np.concatenate([rng.standard_normal(3000).astype(np.float32) * s
                         for s in (1e-8, 1e-5, 1e-3, 1, 30, 500, 70000)])
    for x in xs:
        assert oracle.lib.q27o_float_to_half(float(x)) == ref.lib.q27ref_float_to_half(float(x))
        assert oracle.lib.q27o_float_to_e4m3(float(x)) == ref.lib.q27ref_float_to_e4m3(float(x))


def test_golden_fixtures(oracle):
    g = np.load(GOLDEN / "turbo3_codec.npz")
    assert (oracle.t3_quant(g["x"]) == g["blocks"]).all()
    deq = oracle.kv_dequant(g["blocks"].reshape(-1, 400), KV_T3, g["blocks"].shape[0] // 8)
    assert (deq.reshape(-1, 128).view(np.uint32) == g["dequant"].view(np.uint32)).all()
    assert (oracle.wht(g["x"]).view(np.uint32) == g["fwht"].view(np.uint32)).all()
    assert (oracle.to_half_bits(g["conv_in"]) == g["half_bits"]).all()
    assert (oracle.to_e4m3(g["conv_in"]) == g["e4m3_bits"]).all()
    e = np.array([oracle.lib.q27o_e4m3_to_float(int(b)) for b in range(256)], np.float32)
    nan = np.isnan(g["e4m3_table"])
    assert nan.sum() == 2 and (np.isnan(e) == nan).all()          # 0x7f and 0xff only
    assert (e.view(np.uint32)[~nan] == g["e4m3_table"].view(np.uint32)[~nan]).all()


def test_golden_fixtures_of_the_k_side_codecs(oracle):
    g = np.load(GOLDEN / "k_codecs.npz")
    assert (oracle.t5_quant(g["x"], tree=True) == g["t5_tree"]).all()
    assert (oracle.t5_quant(g["x"], tree=False) == g["t5_serial"]).all()
    n = g["x"].shape[0]
    d5 = oracle.kv_dequant(g["t5_tree"].reshape(n // 8, 656), KV_T5K, n // 8)
    assert (d5.reshape(n, 128).view(np.uint32) == g["t5_dequant"].view(np.uint32)).all()
    assert (oracle.i8_quant(g["x"]) == g["i8_blocks"]).all()
    d8 = oracle.kv_dequant(g["i8_blocks"].reshape(n // 8, 1056), KV_I8G64, n // 8)
    assert (d8.reshape(n // 2, 256).view(np.uint32) == g["i8_dequant"].view(np.uint32)).all()
    # the V side of both kinds is turbo3: same bytes, same dequant as the turbo3 kind
    t3 = np.load(GOLDEN / "turbo3_codec.npz")
    for kvk in (KV_T3V, KV_T5K, KV_I8G64):
        dv = oracle.kv_dequant(t3["blocks"].reshape(-1, 400), kvk, t3["blocks"].shape[0] // 8, is_v=True)
        assert (dv.reshape(-1, 128).view(np.uint32) == t3["dequant"].view(np.uint32)).all()


def test_k_side_codecs_round_trip_quality(oracle):
    # turbo5 round-trip cosine >= 0.998 predicted from its distortion (src/turbo5.cuh:57-60);
    # int8-g64 error <= half a step of each group's scale (src/i8g64.cuh:14-21)
    x = oracle.randn(256 * 128, 15).reshape(256, 128)
    d5 = oracle.kv_dequant(oracle.t5_quant(x).reshape(32, 656), KV_T5K, 32).reshape(256, 128)
    rec = oracle.wht(d5, inverse=True)
    assert (rec * x).sum() / np.sqrt((rec ** 2).sum() * (x ** 2).sum()) > 0.998
    blk = oracle.i8_quant(x)
    d8 = oracle.kv_dequant(blk.reshape(32, 1056), KV_I8G64, 32).reshape(512, 64)
    scale = blk[:, 128:132].copy().view(np.float16).astype(np.float32).reshape(512, 1)
    assert (np.abs(d8 - x.reshape(512, 64)) <= 0.5 * scale * (1 + 1e-6) + 1e-12).all()


def test_wht_round_trip_and_dot_invariance(oracle):
    # WHT round trip (src/test_kernels.cu:1320-1357) and the read contract
    # WHT(q).deq(K) ~ q.K (tools/turbo3_test.cu:126-147: score cosine >= 0.97)
    x = oracle.randn(512 * 128, 5).reshape(512, 128)
    back = oracle.wht(oracle.wht(x), inverse=True)
    assert np.abs(back - x).max() < 1e-5
    blocks = oracle.t3_quant(x)
    deq = oracle.kv_dequant(blocks.reshape(-1, 400), KV_T3, 64).reshape(512, 128)
    q = oracle.randn(512 * 128, 6).reshape(512, 128)
    lhs = (oracle.wht(q).astype(np.float64) * deq).sum(1)
    rhs = (q.astype(np.float64) * x).sum(1)
    cos = (lhs * rhs).sum() / np.sqrt((lhs ** 2).sum() * (rhs ** 2).sum())
    assert cos > 0.97
    rec = oracle.wht(deq, inverse=True)
    c2 = (rec * x).sum() / np.sqrt((rec ** 2).sum() * (x ** 2).sum())
    assert c2 > 0.97


@pytest.mark.parametrize("kvk", ALL_KINDS)
def test_attention_vs_plain_numpy_softmax(oracle, kvk):
    # independent double-precision restatement in numpy over the oracle's own dequant
    c = synth.make_case(oracle, kvk, rows=97, pos=[96, 40, 0], seed=11)
    out = oracle.attn_decode(c.q, c.k, c.v, kvk, c.pos)
    kd = oracle.kv_dequant(c.k, kvk, c.rows).astype(np.float64)
    vd = oracle.kv_dequant(c.v, kvk, c.rows, is_v=True).astype(np.float64)
    for t, p in enumerate(c.pos):
        for h in range(24):
            s = kd[: p + 1, h // 6] @ c.q[t, h, :HD].astype(np.float64) / 16.0
            w = np.exp(s - s.max())
            ref = (w[:, None] * vd[: p + 1, h // 6]).sum(0) / w.sum()
            assert np.abs(out[t, h * HD:(h + 1) * HD] - ref).max() < 1e-6 * max(1.0, np.abs(ref).max())


def test_partials_merge_to_full_attention(oracle):
    # the (m, l, acc) monoid: windows merged by the combine rule equal the one-pass result
    c = synth.make_case(oracle, KV_T3, rows=300, pos=[299, 150, 10], seed=21)
    full = oracle.attn_decode(c.q, c.k, c.v, KV_T3, c.pos)
    bounds = [0, 64, 128, 192, 300]
    parts = np.stack([oracle.attn_partial(c.q, c.k, c.v, KV_T3, c.pos, lo, hi).reshape(-1, 258)
                      for lo, hi in zip(bounds[:-1], bounds[1:])])
    assert parts[3, 2 * 24, 0] == np.float32(-3.4028234663852886e38)  # lane 2 empty in last window
    merged = oracle.merge_partials(parts)
    assert np.abs(merged.reshape(3, -1) - full).max() < 1e-6
    two_step = oracle.merge_partials(np.stack([oracle.merge_partials(parts[:2], normalise=False),
                                               oracle.merge_partials(parts[2:], normalise=False)]))
    assert np.abs(two_step.reshape(3, -1) - full).max() < 1e-6


def test_prefill_matches_decode_row_by_row(oracle):
    # token t of a chunk at base_pos attends rows [0, base_pos + t + 1): same as a decode
    # lane at pos = base_pos + t (src/test_kernels.cu:2116)
    base, T = 37, 5
    c = synth.make_case(oracle, KV_F16, rows=base + T, pos=[base + t for t in range(T)], seed=31)
    dec = oracle.attn_decode(c.q, c.k, c.v, KV_F16, c.pos)
    pf = oracle.attn_prefill(c.q, c.k, c.v, KV_F16, base, 0, T)
    assert np.abs(pf - dec).max() == 0.0
    pf2 = oracle.attn_prefill(c.q, c.k, c.v, KV_F16, base, 2, 2)
    assert np.abs(pf2[2:4] - dec[2:4]).max() == 0.0 and (pf2[:2] == 0).all()


def test_fp8_scale_folding_identity(oracle):
    # C2's per-head absmax scale folds outside the scale-free entry points: scaling Q by
    # s_K and the output by s_V reproduces attention over the scaled dequantised cache
    c = synth.make_case(oracle, KV_FP8, rows=128, pos=[127], seed=41)   # c.q = q_raw * s_K
    out = synth.scale_out(c, oracle.attn_decode(c.q, c.k, c.v, KV_FP8, c.pos)).reshape(1, 24, HD)
    kd = oracle.kv_dequant(c.k, KV_FP8, 128).astype(np.float64) * c.k_scale[None, :, None]
    vd = oracle.kv_dequant(c.v, KV_FP8, 128).astype(np.float64) * c.v_scale[None, :, None]
    for h in (0, 7, 23):
        s = kd[:, h // 6] @ c.q_raw[0, h, :HD].astype(np.float64) / 16.0
        w = np.exp(s - s.max())
        ref = (w[:, None] * vd[:, h // 6]).sum(0) / w.sum()
        assert np.abs(out[0, h] - ref).max() < 1e-5
    # and the scaled cache tracks the fp16 source to e4m3 precision
    assert np.abs(kd - c.kf).max() / np.abs(c.kf).max() < 0.07


def test_generator_is_seeded_and_normal(oracle):
    a, b = oracle.randn(100000, 9), oracle.randn(100000, 9)
    assert (a == b).all() and not (a == oracle.randn(100000, 10)).all()
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1) < 0.02
    assert (oracle.randn(100001, 9, nthreads=1)[:100000] == a).all()
