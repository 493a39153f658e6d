"""Seeded synthetic inputs for the parity tests, built on the CPU with the oracle's own
generator and codecs (so the oracle and the CUDA path see byte-identical caches)."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from tests.oracle_lib import KV_F16, KV_FP8, KV_T3, KV_T3V, KV_T5K, KV_I8G64, HD, Oracle

N_Q, N_KV, GQA = 24, 4, 6
Q_STRIDE = 2 * HD          # interleaved [q | gate] per head (src/engine.cuh: q||gate layout)
Q_ROW = N_Q * Q_STRIDE     # 12288
OUT_ROW = N_Q * HD         # 6144


@dataclass
class Case:
    kvk: int
    rows: int
    q: np.ndarray        # [ntok, N_Q, Q_STRIDE] fp32 (already WHT-rotated for turbo3)
    q_raw: np.ndarray    # un-rotated q
    k: np.ndarray        # uint8 [rows, row_bytes]
    v: np.ndarray
    pos: list
    k_scale: np.ndarray | None = None   # per-kv-head dequant scales (fp8 absmax), else None
    v_scale: np.ndarray | None = None
    kf: np.ndarray | None = None        # the fp32 K/V values before encoding [rows, N_KV, HD]
    vf: np.ndarray | None = None


def k_rotated(kvk: int) -> bool:
    """Does the K side carry the rotation, so that Q must be rotated to match?
    (kv_k_rotated, src/cuda_common.h:59)"""
    return kvk in (KV_T3, KV_T5K)


def encode_rows(o: Oracle, x: np.ndarray, kvk: int, is_v: bool = False):
    """x [rows, N_KV, HD] fp32 -> (uint8 [rows, row_bytes], per-head scale or None). From
    turbo3 up the V side is turbo3 blocks whatever the K side holds (src/cuda_common.h:47-53)."""
    rows = x.shape[0]
    if kvk >= KV_T3:
        if is_v or kvk == KV_T3:
            return o.t3_quant(x.reshape(-1, 128)).reshape(rows, -1), None
        if kvk == KV_T3V:
            return o.to_half_bits(x).view(np.uint8).reshape(rows, -1), None
        if kvk == KV_T5K:
            return o.t5_quant(x.reshape(-1, 128)).reshape(rows, -1), None
        if kvk == KV_I8G64:
            return o.i8_quant(x.reshape(-1, 128)).reshape(rows, -1), None
        raise ValueError(kvk)
    if kvk == KV_F16:
        return o.to_half_bits(x).view(np.uint8).reshape(rows, -1), None
    if kvk == KV_FP8:
        # values pass through fp16 first, then per-(side, kv head) absmax scaling to +-448
        xh = o.to_half_bits(x).view(np.float16).astype(np.float32)
        a = np.abs(xh).max(axis=(0, 2))
        a = np.where(a > 0, a, 1.0).astype(np.float32)
        scaled = xh * (np.float32(448.0) / a)[None, :, None]
        return o.to_e4m3(scaled).reshape(rows, -1), (a / np.float32(448.0)).astype(np.float32)
    raise ValueError(kvk)


def make_kv(o: Oracle, rows: int, kvk: int, seed: int, outlier_frac: float = 0.0):
    kf = o.randn(rows * N_KV * HD, seed * 2 + 1).reshape(rows, N_KV, HD)
    vf = o.randn(rows * N_KV * HD, seed * 2 + 2).reshape(rows, N_KV, HD)
    if outlier_frac > 0:
        rng = np.random.default_rng(seed)
        nch = max(1, int(round(outlier_frac * N_KV * HD)))
        for side in (kf, vf):
            ch = rng.choice(N_KV * HD, size=nch, replace=False)
            side.reshape(rows, -1)[:, ch] *= np.float32(8.0)
    return kf, vf


def make_case(o: Oracle, kvk: int, rows: int, pos: list, seed: int,
              outlier_frac: float = 0.0, bf16: bool = False) -> Case:
    ntok = len(pos)
    kf, vf = make_kv(o, rows, kvk, seed, outlier_frac)
    q_raw = o.randn(ntok * N_Q * Q_STRIDE, seed * 2 + 1000003).reshape(ntok, N_Q, Q_STRIDE)
    if bf16:
        kf, vf, q_raw = o.round_bf16(kf), o.round_bf16(vf), o.round_bf16(q_raw)
    k, ks = encode_rows(o, kf, kvk, is_v=False)
    v, vs = encode_rows(o, vf, kvk, is_v=True)
    q = q_raw.copy()
    if k_rotated(kvk):  # the engine receives Q already rotated (src/engine.cuh:1485-1488)
        q[:, :, :HD] = o.wht(np.ascontiguousarray(q_raw[:, :, :HD]))
    if kvk == KV_FP8:
        # the reference's fp8 cache is scale-free (src/cuda_common.h:110-121): the per-head
        # absmax scale of the K side is folded into Q by the caller, the V side's into the
        # output (Case.scale_out)
        q[:, :, :HD] *= np.repeat(ks, GQA)[None, :, None]
    return Case(kvk, rows, q, q_raw, k, v, list(pos), ks, vs, kf, vf)


def scale_out(case: Case, out: np.ndarray) -> np.ndarray:
    """Apply the V-side dequant scale (fp8 absmax) to [lanes, N_Q*HD] outputs; identity for
    the other kinds. Parity is judged on these real-valued outputs."""
    if case.v_scale is None:
        return out
    o3 = np.asarray(out).reshape(out.shape[0], N_Q, HD)
    return (o3 * np.repeat(case.v_scale, GQA)[None, :, None]).reshape(out.shape)


def tolerance_ok(got: np.ndarray, ref: np.ndarray, atol=2e-3, rtol=1e-3):
    """The parity bar of the headline metric: |a-b| <= 2e-3 + 1e-3*|b| element-wise; returns (ok, max excess,
    max-abs/RMS as the reference's own tests report it, src/test_kernels.cu:885-893)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    err = np.abs(got - ref)
    excess = float((err - (atol + rtol * np.abs(ref))).max())
    rms = float(np.sqrt((ref ** 2).mean()) + 1e-12)
    return excess <= 0.0, excess, float(err.max() / rms)
