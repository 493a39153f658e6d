"""ctypes access to the CPU oracle (oracle/build/libq27_oracle.so) and, when they were
built, to the libraries compiled from the reference's own sources (oracle/_ref/).

Test infrastructure: imported by tests/, __graft_entry__.smoke() and bench.py's CPU
baseline leg only."""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
ORACLE_SO = ROOT / "oracle" / "build" / "libq27_oracle.so"
REF_CODEC_SO = ROOT / "oracle" / "_ref" / "libq27ref_codec.so"
REF_GPU_SO = ROOT / "oracle" / "_ref" / "libq27ref_gpu.so"

KV_F16, KV_FP8, KV_T3, KV_T3V, KV_T5K, KV_I8G64 = range(6)
ALL_KINDS = (KV_F16, KV_FP8, KV_T3, KV_T3V, KV_T5K, KV_I8G64)
HD, FD_ST, T3_BLOCK, T5_BLOCK, I8_BLOCK = 256, 258, 50, 82, 132

_fp = C.POINTER(C.c_float)
_vp = C.c_void_p


def build_oracle() -> Path:
    """gcc-compile the oracle if the library is missing (seconds)."""
    if not ORACLE_SO.exists():
        subprocess.run(["make", "-C", str(ROOT / "oracle"), "oracle"], check=True,
                       capture_output=True)
    return ORACLE_SO


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_fp)


class Oracle:
    def __init__(self):
        self.lib = C.CDLL(str(build_oracle()))
        L = self.lib
        L.q27o_half_to_float.restype = C.c_float
        L.q27o_half_to_float.argtypes = [C.c_uint16]
        L.q27o_float_to_half.restype = C.c_uint16
        L.q27o_float_to_half.argtypes = [C.c_float]
        L.q27o_e4m3_to_float.restype = C.c_float
        L.q27o_e4m3_to_float.argtypes = [C.c_uint8]
        L.q27o_float_to_e4m3.restype = C.c_uint8
        L.q27o_float_to_e4m3.argtypes = [C.c_float]
        L.q27o_round_bf16.restype = C.c_float
        L.q27o_round_bf16.argtypes = [C.c_float]
        for f in ("q27o_t3_centroids", "q27o_t3_s1", "q27o_t3_s2"):
            getattr(L, f).restype = _fp
        L.q27o_t3_nearest.argtypes = [C.c_float]
        L.q27o_row_bytes.restype = C.c_int64
        L.q27o_row_bytes_side.restype = C.c_int64
        for f in ("q27o_t5_centroids", "q27o_t5_thresholds"):
            getattr(L, f).restype = _fp
        L.q27o_t5_nearest.argtypes = [C.c_float]
        L.q27o_t5_quant_groups.argtypes = [_fp, C.c_int64, _vp, C.c_int, C.c_int]
        L.q27o_i8_quant_groups.argtypes = [_fp, C.c_int64, _vp, C.c_int]
        L.q27o_kv_dequant_side.argtypes = [_vp, C.c_int, C.c_int, C.c_int64, C.c_int, _fp, C.c_int]
        L.q27o_splitmix64.restype = C.c_uint64
        L.q27o_splitmix64.argtypes = [C.c_uint64]
        L.q27o_randn.argtypes = [_fp, C.c_int64, C.c_uint64, C.c_int]
        L.q27o_t3_quant_groups.argtypes = [_fp, C.c_int64, _vp, C.c_int]
        L.q27o_wht_groups.argtypes = [_fp, C.c_int64, C.c_int, C.c_int]
        L.q27o_kv_dequant.argtypes = [_vp, C.c_int, C.c_int64, C.c_int, _fp, C.c_int]
        L.q27o_float_to_half_n.argtypes = [_fp, C.c_int64, _vp]
        L.q27o_float_to_e4m3_n.argtypes = [_fp, C.c_int64, _vp]
        L.q27o_round_bf16_n.argtypes = [_fp, C.c_int64]
        L.q27o_attn_decode.argtypes = [_fp, C.c_int64, C.c_int, _vp, _vp, C.c_int,
                                       C.POINTER(C.c_int), C.c_int, C.c_int, C.c_int, C.c_float,
                                       _fp, C.c_int]
        L.q27o_attn_partial.argtypes = [_fp, C.c_int64, C.c_int, _vp, _vp, C.c_int,
                                        C.POINTER(C.c_int), C.c_int, C.c_int, C.c_int, C.c_float,
                                        C.c_int64, C.c_int64, _fp, C.c_int]
        L.q27o_merge_partials.argtypes = [_fp, C.c_int, C.c_int64, _fp, C.c_int]
        L.q27o_attn_prefill.argtypes = [_fp, C.c_int, C.c_int, _vp, _vp, C.c_int, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_int, C.c_float, _fp, C.c_int, C.c_int]

    # ---- generators / codecs -------------------------------------------------------
    def randn(self, n: int, seed: int, nthreads: int = 0) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        self.lib.q27o_randn(out.ctypes.data_as(_fp), n, seed, nthreads)
        return out

    def to_half_bits(self, x) -> np.ndarray:
        x, px = _f32(x)
        out = np.empty(x.shape, dtype=np.uint16)
        self.lib.q27o_float_to_half_n(px, x.size, out.ctypes.data_as(_vp))
        return out

    def to_e4m3(self, x) -> np.ndarray:
        x, px = _f32(x)
        out = np.empty(x.shape, dtype=np.uint8)
        self.lib.q27o_float_to_e4m3_n(px, x.size, out.ctypes.data_as(_vp))
        return out

    def round_bf16(self, x) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        self.lib.q27o_round_bf16_n(x.ctypes.data_as(_fp), x.size)
        return x

    def t3_quant(self, x) -> np.ndarray:
        """x [..., 128k] fp32 -> uint8 blocks [ngroups, 50]"""
        x, px = _f32(x)
        ng = x.size // 128
        out = np.zeros((ng, T3_BLOCK), dtype=np.uint8)
        self.lib.q27o_t3_quant_groups(px, ng, out.ctypes.data_as(_vp), 0)
        return out

    def t5_quant(self, x, tree: bool = True) -> np.ndarray:
        """x [..., 128k] fp32 -> uint8 turbo5 blocks [ngroups, 82]; tree = the reduction order
        of the reference's device encoder"""
        x, px = _f32(x)
        ng = x.size // 128
        out = np.zeros((ng, T5_BLOCK), dtype=np.uint8)
        self.lib.q27o_t5_quant_groups(px, ng, out.ctypes.data_as(_vp), int(tree), 0)
        return out

    def i8_quant(self, x) -> np.ndarray:
        """x [..., 128k] fp32 -> uint8 int8-g64 blocks [ngroups, 132]"""
        x, px = _f32(x)
        ng = x.size // 128
        out = np.zeros((ng, I8_BLOCK), dtype=np.uint8)
        self.lib.q27o_i8_quant_groups(px, ng, out.ctypes.data_as(_vp), 0)
        return out

    def wht(self, x, inverse: bool = False) -> np.ndarray:
        x = np.array(x, dtype=np.float32, copy=True, order="C")
        self.lib.q27o_wht_groups(x.ctypes.data_as(_fp), x.size // 128, int(inverse), 0)
        return x

    def row_bytes(self, kvk: int, n_kv: int = 4, is_v: bool = False) -> int:
        return int(self.lib.q27o_row_bytes_side(kvk, n_kv, int(is_v)))

    def kv_dequant(self, cache: np.ndarray, kvk: int, rows: int, n_kv: int = 4,
                   is_v: bool = False) -> np.ndarray:
        cache = np.ascontiguousarray(cache)
        out = np.empty((rows, n_kv, HD), dtype=np.float32)
        rc = self.lib.q27o_kv_dequant_side(cache.ctypes.data_as(_vp), kvk, int(is_v), rows, n_kv,
                                           out.ctypes.data_as(_fp), 0)
        assert rc == 0
        return out

    # ---- attention -----------------------------------------------------------------
    def attn_decode(self, q, kcache, vcache, kvk, pos, n_q=24, n_kv=4, scale=0.0625,
                    nthreads=0) -> np.ndarray:
        """q: [ntok, n_q, q_stride] fp32; returns [ntok, n_q*256]"""
        q, pq = _f32(q)
        ntok, _, q_stride = q.shape
        kcache, vcache = np.ascontiguousarray(kcache), np.ascontiguousarray(vcache)
        posa = (C.c_int * ntok)(*[int(p) for p in pos])
        out = np.empty((ntok, n_q * HD), dtype=np.float32)
        rc = self.lib.q27o_attn_decode(pq, n_q * q_stride, q_stride, kcache.ctypes.data_as(_vp),
                                       vcache.ctypes.data_as(_vp), kvk, posa, ntok, n_q, n_kv,
                                       scale, out.ctypes.data_as(_fp), nthreads)
        assert rc == 0
        return out

    def attn_partial(self, q, kcache, vcache, kvk, pos, lo, hi, n_q=24, n_kv=4, scale=0.0625,
                     nthreads=0) -> np.ndarray:
        q, pq = _f32(q)
        ntok, _, q_stride = q.shape
        kcache, vcache = np.ascontiguousarray(kcache), np.ascontiguousarray(vcache)
        posa = (C.c_int * ntok)(*[int(p) for p in pos])
        out = np.empty((ntok, n_q, FD_ST), dtype=np.float32)
        rc = self.lib.q27o_attn_partial(pq, n_q * q_stride, q_stride, kcache.ctypes.data_as(_vp),
                                        vcache.ctypes.data_as(_vp), kvk, posa, ntok, n_q, n_kv,
                                        scale, lo, hi, out.ctypes.data_as(_fp), nthreads)
        assert rc == 0
        return out

    def merge_partials(self, parts, normalise: bool = True) -> np.ndarray:
        """parts [nparts, npairs, 258] -> [npairs, 256] (or [npairs, 258] un-normalised)"""
        parts, pp = _f32(parts)
        nparts, npairs, _ = parts.shape
        out = np.empty((npairs, HD if normalise else FD_ST), dtype=np.float32)
        self.lib.q27o_merge_partials(pp, nparts, npairs, out.ctypes.data_as(_fp), int(normalise))
        return out

    def attn_prefill(self, qT, kcache, vcache, kvk, base_pos, t0, SB, n_q=24, n_kv=4,
                     scale=0.0625, nthreads=0) -> np.ndarray:
        """qT [T, n_q, q_stride]; returns outT [T, n_q*256] with rows t0..t0+SB-1 written"""
        qT, pq = _f32(qT)
        T, _, q_stride = qT.shape
        kcache, vcache = np.ascontiguousarray(kcache), np.ascontiguousarray(vcache)
        out = np.zeros((T, n_q * HD), dtype=np.float32)
        rc = self.lib.q27o_attn_prefill(pq, q_stride, n_q * q_stride, kcache.ctypes.data_as(_vp),
                                        vcache.ctypes.data_as(_vp), kvk, base_pos, t0, SB, n_q,
                                        n_kv, scale, out.ctypes.data_as(_fp), n_q * HD, nthreads)
        assert rc == 0
        return out


class RefCodec:
    """The reference's own CPU turbo3 codec and table header, plus the CUDA toolkit's host
    converters, compiled from the reference tree (absent on the GPU box)."""

    def __init__(self):
        if not REF_CODEC_SO.exists():
            raise FileNotFoundError(REF_CODEC_SO)
        self.lib = C.CDLL(str(REF_CODEC_SO))
        L = self.lib
        for f in ("q27ref_hdr_centroids", "q27ref_hdr_s1", "q27ref_hdr_s2"):
            getattr(L, f).restype = _fp
        L.q27ref_cpu_nearest.argtypes = [C.c_float]
        L.q27ref_hdr_nearest.argtypes = [C.c_float]
        L.q27ref_float_to_half.restype = C.c_uint16
        L.q27ref_float_to_half.argtypes = [C.c_float]
        L.q27ref_half_to_float.restype = C.c_float
        L.q27ref_half_to_float.argtypes = [C.c_uint16]
        L.q27ref_float_to_e4m3.restype = C.c_uint8
        L.q27ref_float_to_e4m3.argtypes = [C.c_float]
        L.q27ref_e4m3_to_float.restype = C.c_float
        L.q27ref_e4m3_to_float.argtypes = [C.c_uint8]
        L.q27ref_cpu_quant.argtypes = [_fp, _vp]
        L.q27ref_cpu_dequant.argtypes = [_vp, _fp]
        L.q27ref_cpu_fwht.argtypes = [_fp]
        L.q27ref_cpu_fwht_inv.argtypes = [_fp]
        # the 5-bit and int8-g64 K codecs (tools/turbo5_test.cu, tools/i8g64_test.cu)
        for f in ("q27ref_hdr5_centroids", "q27ref_hdr5_thresholds"):
            getattr(L, f).restype = _fp
        L.q27ref_cpu5_nearest.argtypes = [C.c_float]
        L.q27ref_hdr5_nearest.argtypes = [C.c_float]
        L.q27ref_cpu_quant5.argtypes = [_fp, _vp, C.c_int]
        L.q27ref_cpu_dequant5.argtypes = [_vp, _fp]
        L.q27ref_i8_quant.argtypes = [_fp, _vp]
        L.q27ref_i8_dequant_row.argtypes = [_vp, _fp]
