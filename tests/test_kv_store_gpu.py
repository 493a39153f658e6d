"""GPU tests of the KV row stores and the WHT rotation (the steps either side of attention):
device turbo3 encoder vs the serial CPU codec (test_kv_turbo3_store,
src/test_kernels.cu:1150-1316), fp8/fp16 stores vs the host converters bitwise
(test_kv_fp8_store, :446-489), device WHT == CPU fwht bitwise and inverse round trip
(test_wht3, :1320-1357), and the rotated end-to-end pipeline (test_attn_fd2_turbo3,
:1366-1589)."""
import ctypes as C

import numpy as np
import pytest
import torch

import q27_b200 as Q
from tests import synth
from tests.gpu_util import SCALE, RefGpu
from tests.oracle_lib import KV_F16, KV_FP8, KV_T3, REF_GPU_SO

pytestmark = pytest.mark.gpu


def empty_cache(cuda, kvk, rows, scatter=None):
    rb = Q.row_bytes(kvk)
    perm = None
    if scatter is not None:
        perm = torch.from_numpy(np.random.default_rng(scatter).permutation((rows + 63) // 64))
    z = torch.zeros((rows, rb), dtype=torch.uint8, device=cuda)
    return Q.paged_from_rows(z, kvk, page_perm=perm), Q.paged_from_rows(z, kvk, page_perm=perm), perm


def read_rows(side, kvk, rows, perm):
    rb = Q.row_bytes(kvk)
    npages = (rows + 63) // 64
    pages = side.data.view(npages, 64 * rb)
    if perm is not None:
        pages = pages[perm.to(pages.device)]
    return pages.reshape(-1, rb)[:rows].cpu().numpy()


def test_turbo3_store_matches_cpu_codec_bytewise(oracle, cuda):
    base, T = 37, 150
    kf, vf = synth.make_kv(oracle, T, KV_T3, seed=17, outlier_frac=0.02)
    kf[3] = 0.0                                   # a zero group: index-4 packing, norm 0
    ks, vs, perm = empty_cache(cuda, KV_T3, base + T, scatter=4)
    kT = torch.from_numpy(kf.reshape(T, -1)).to(cuda)
    vT = torch.from_numpy(vf.reshape(T, -1)).to(cuda)
    Q.kv_store_T_t3(kT, vT, ks.tab, vs.tab, base, 4, 256, T)
    torch.cuda.synchronize()
    for side, src in ((ks, kf), (vs, vf)):
        got = read_rows(side, KV_T3, base + T, perm)
        want = oracle.t3_quant(src.reshape(-1, 128)).reshape(T, 400)
        assert (got[base:] == want).all()
        assert (got[:base] == 0).all()            # rows before base_pos untouched


@pytest.mark.parametrize("fp8", [False, True])
def test_scalar_store_matches_host_converters_bitwise(oracle, cuda, fp8):
    kvk = KV_FP8 if fp8 else KV_F16
    base, T = 70, 90
    kf, vf = synth.make_kv(oracle, T, kvk, seed=19)
    kf *= 40.0                                     # exercises e4m3 saturation at +-448
    ks, vs, perm = empty_cache(cuda, kvk, base + T, scatter=2)
    Q.kv_store_T(torch.from_numpy(kf.reshape(T, -1)).to(cuda),
                 torch.from_numpy(vf.reshape(T, -1)).to(cuda), ks.tab, vs.tab, base, 1024, T,
                 fp8=fp8)
    torch.cuda.synchronize()
    for side, src in ((ks, kf), (vs, vf)):
        got = read_rows(side, kvk, base + T, perm)[base:]
        want = (oracle.to_e4m3(src) if fp8 else oracle.to_half_bits(src).view(np.uint8)).reshape(T, -1)
        assert (got == want).all()


def test_wht_bitwise_and_round_trip(oracle, cuda):
    T = 7
    x = oracle.randn(T * synth.Q_ROW, 23).reshape(T, 24, synth.Q_STRIDE)
    d = torch.from_numpy(x.reshape(T, -1).copy()).to(cuda)
    Q.wht_T(d, 24, 256, synth.Q_STRIDE, synth.Q_ROW, T, False)
    torch.cuda.synchronize()
    got = d.cpu().numpy().reshape(T, 24, synth.Q_STRIDE)
    want = oracle.wht(np.ascontiguousarray(x[:, :, :256]))
    assert (got[:, :, :256].view(np.uint32) == want.view(np.uint32)).all()   # bitwise
    assert (got[:, :, 256:].view(np.uint32) == x[:, :, 256:].view(np.uint32)).all()  # gate half
    Q.wht_T(d, 24, 256, synth.Q_STRIDE, synth.Q_ROW, T, True)
    torch.cuda.synchronize()
    back = d.cpu().numpy().reshape(T, 24, synth.Q_STRIDE)
    assert np.abs(back - x).max() < 1e-5
    inv = oracle.wht(want, inverse=True)
    assert (back[:, :, :256].view(np.uint32) == inv.view(np.uint32)).all()


def test_turbo3_pipeline_end_to_end(oracle, cuda):
    """rope'd q -> forward WHT -> store -> attention in the rotated basis -> inverse WHT:
    equals the oracle's rotated pipeline and tracks un-quantised fp16 attention (cosine)."""
    rows, pos = 900, [899, 898, 500]
    c = synth.make_case(oracle, KV_T3, rows=rows, pos=pos, seed=29, outlier_frac=0.02)
    ks, vs, _ = empty_cache(cuda, KV_T3, rows)
    Q.kv_store_T_t3(torch.from_numpy(c.kf.reshape(rows, -1)).to(cuda),
                    torch.from_numpy(c.vf.reshape(rows, -1)).to(cuda), ks.tab, vs.tab, 0, 4, 256,
                    rows)
    q = torch.from_numpy(c.q_raw.reshape(len(pos), -1).copy()).to(cuda)     # lanes contiguous
    Q.wht_T(q, 24, 256, synth.Q_STRIDE, synth.Q_ROW, len(pos), False)
    out = torch.zeros((len(pos), synth.OUT_ROW), device=cuda)
    scratch = torch.empty(Q.decode_scratch_floats(len(pos)), device=cuda)
    posd = [torch.tensor([p], dtype=torch.int32, device=cuda) for p in pos]
    Q.attn_decode3(list(q), synth.Q_STRIDE, ks.tab, vs.tab, list(out), scratch, posd, 0, 24, 4, 256,
                   SCALE, ntok=len(pos), kvk=KV_T3)
    torch.cuda.synchronize()
    rot_got = out.cpu().numpy()                   # the engine's own output: rotated basis
    Q.wht_T(out, 24, 256, 256, synth.OUT_ROW, len(pos), True)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    rot = oracle.attn_decode(c.q, c.k, c.v, KV_T3, pos)
    want = oracle.wht(rot.reshape(-1, 128), inverse=True).reshape(rot.shape)
    # after the inverse rotation every output mixes 128 rotated ones: judged with the
    # reference's own gate for its tensor-core paths (max-abs/RMS, src/test_kernels.cu:1521)
    assert synth.tolerance_ok(rot_got, rot)[0]    # the parity bar on the attention output
    rms = np.sqrt((want.astype(np.float64) ** 2).mean())
    assert np.abs(got - want).max() / rms < 3e-2  # x8 outlier channels, 900 keys, 3 lanes
    c16 = synth.make_case(oracle, KV_F16, rows=rows, pos=pos, seed=29, outlier_frac=0.02)
    plain = oracle.attn_decode(c16.q, c16.k, c16.v, KV_F16, pos)
    cos = (got * plain).sum() / np.sqrt((got ** 2).sum() * (plain ** 2).sum())
    assert cos > 0.9


@pytest.mark.skipif(not REF_GPU_SO.exists(), reason="oracle/_ref not built")
def test_store_vs_reference_device_encoder(oracle, cuda):
    """Against the reference's own device encoder on this GPU, with its own bars
    (src/test_kernels.cu:1150-1316): >= 95 % of blocks bit-equal, <= 0.2 % index ties,
    norms within 1 fp16 ULP."""
    ref = RefGpu()
    T = 256
    kf, vf = synth.make_kv(oracle, T, KV_T3, seed=31, outlier_frac=0.02)
    kT = torch.from_numpy(kf.reshape(T, -1)).to(cuda)
    vT = torch.from_numpy(vf.reshape(T, -1)).to(cuda)
    ks, vs, _ = empty_cache(cuda, KV_T3, T)
    rk, rv, _ = empty_cache(cuda, KV_T3, T)
    Q.kv_store_T_t3(kT, vT, ks.tab, vs.tab, 0, 4, 256, T)
    ref.lib.q27ref_kv_store_T_t3(kT.data_ptr(), vT.data_ptr(), rk.tab.data_ptr(), rv.tab.data_ptr(),
                                 0, 4, 256, T, None, KV_T3)
    torch.cuda.synchronize()
    for mine, theirs in ((ks, rk), (vs, rv)):
        a = read_rows(mine, KV_T3, T, None).reshape(-1, 50)
        b = read_rows(theirs, KV_T3, T, None).reshape(-1, 50)
        equal = (a == b).all(1).mean()
        assert equal >= 0.95
        na, nb = a[:, :2].copy().view(np.uint16)[:, 0], b[:, :2].copy().view(np.uint16)[:, 0]
        assert np.abs(na.astype(np.int32) - nb.astype(np.int32)).max() <= 1
        # index ties: unpack and count differing 3-bit indices
        def idx(x):
            qs, sg = x[:, 2:34], x[:, 34:50]
            low = np.stack([(qs >> (2 * i)) & 3 for i in range(4)], -1).reshape(len(x), 128)
            hi = np.stack([(sg >> i) & 1 for i in range(8)], -1).reshape(len(x), 128)
            return low | (hi << 2)
        assert (idx(a) != idx(b)).mean() <= 0.002


@pytest.mark.parametrize("kvk", [KV_F16, KV_FP8, KV_T3])
def test_lane_form_stores_match_cpu_codec_bytewise(oracle, cuda, kvk):
    """kv_store3 / kv_store_t3 (src/spec3.cu:512-588): one row per draft lane, row index
    read on the device from the lane's position pointer; rows land at scattered positions
    and every other row of the cache stays untouched."""
    rows = 300
    pos = [299, 3, 64, 127, 128, 250]
    n = len(pos)
    kf, vf = synth.make_kv(oracle, n, kvk, seed=29, outlier_frac=0.02 if kvk == KV_T3 else 0.0)
    if kvk == KV_FP8:
        kf *= 40.0
    ks, vs, perm = empty_cache(cuda, kvk, rows, scatter=6)
    kd = [torch.from_numpy(kf[t].reshape(-1).copy()).to(cuda) for t in range(n)]
    vd = [torch.from_numpy(vf[t].reshape(-1).copy()).to(cuda) for t in range(n)]
    pd = [torch.tensor([p], dtype=torch.int32, device=cuda) for p in pos]
    if kvk == KV_T3:
        Q.kv_store_t3(kd, vd, ks.tab, vs.tab, pd, 4, 256)
    else:
        Q.kv_store3(kd, vd, ks.tab, vs.tab, pd, 1024, fp8=kvk == KV_FP8)
    torch.cuda.synchronize()
    for side, src in ((ks, kf), (vs, vf)):
        got = read_rows(side, kvk, rows, perm)
        if kvk == KV_T3:
            want = oracle.t3_quant(src.reshape(-1, 128)).reshape(n, 400)
        elif kvk == KV_FP8:
            want = oracle.to_e4m3(src).reshape(n, -1)
        else:
            want = oracle.to_half_bits(src).view(np.uint8).reshape(n, -1)
        for t, p in enumerate(pos):
            assert (got[p] == want[t]).all()
        untouched = np.ones(rows, bool)
        untouched[pos] = False
        assert (got[untouched] == 0).all()


def test_lane_form_wht_bitwise(oracle, cuda):
    """wht3 (src/spec3.cu:595-614) on q||gate rows: bitwise the CPU rotation, gate half kept."""
    n = 5
    x = oracle.randn(n * synth.Q_ROW, 31).reshape(n, 24, synth.Q_STRIDE)
    lanes = [torch.from_numpy(x[t].reshape(-1).copy()).to(cuda) for t in range(n)]
    Q.wht3(lanes, 24, 256, synth.Q_STRIDE, False)
    torch.cuda.synchronize()
    got = np.stack([l.cpu().numpy().reshape(24, synth.Q_STRIDE) for l in lanes])
    want = oracle.wht(np.ascontiguousarray(x[:, :, :256]))
    assert (got[:, :, :256].view(np.uint32) == want.view(np.uint32)).all()
    assert (got[:, :, 256:] == x[:, :, 256:]).all()
    Q.wht3(lanes, 24, 256, synth.Q_STRIDE, True)
    torch.cuda.synchronize()
    back = np.stack([l.cpu().numpy().reshape(24, synth.Q_STRIDE) for l in lanes])
    assert np.abs(back[:, :, :256] - x[:, :, :256]).max() < 1e-5
