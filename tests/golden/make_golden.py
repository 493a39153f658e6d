"""Generates tests/golden/turbo3_codec.npz and tests/golden/k_codecs.npz from the REFERENCE's
own code: the CPU turbo3 / turbo5 / int8-g64 codecs in tools/turbo3_test.cu,
tools/turbo5_test.cu and tools/i8g64_test.cu and the CUDA toolkit's host fp16/e4m3 converters,
all built from the reference tree into oracle/_ref/libq27ref_codec.so by oracle/Makefile.

Run in a container that has the reference tree:  make -C oracle ref && python tests/golden/make_golden.py
The inputs come from an LCG of the kind the reference's tools use
(tools/turbo3_test.cu:95-96); no oracle code is involved in producing the fixture."""
import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent.parent
sys.path.insert(0, str(ROOT))
from tests.oracle_lib import RefCodec  # noqa: E402

_fp = C.POINTER(C.c_float)


def lcg_floats(n, seed, scale):
    s = np.uint32(seed)
    out = np.empty(n, np.float32)
    with np.errstate(over="ignore"):
        for i in range(n):
            s = np.uint32(s * np.uint32(1664525) + np.uint32(1013904223))
            out[i] = (float((int(s) >> 8) & 0xFFFF) / 65536.0 - 0.5) * scale
    return out


def main():
    ref = RefCodec()
    ngroups = 128  # 16 rows x 4 kv heads x 2 blocks
    x = lcg_floats(ngroups * 128, 1234567, 2.0).reshape(ngroups, 128)
    x[::7] *= 8.0
    x[5] = 0.0
    blocks = np.zeros((ngroups, 50), np.uint8)
    deq = np.zeros((ngroups, 128), np.float32)
    fw = x.copy()
    for i in range(ngroups):
        ref.lib.q27ref_cpu_quant(x[i].ctypes.data_as(_fp), blocks[i].ctypes.data_as(C.c_void_p))
        ref.lib.q27ref_cpu_dequant(blocks[i].ctypes.data_as(C.c_void_p), deq[i].ctypes.data_as(_fp))
        ref.lib.q27ref_cpu_fwht(fw[i].ctypes.data_as(_fp))
    conv_in = np.concatenate([lcg_floats(2048, 99, s) for s in (1e-6, 1e-3, 1.0, 40.0, 1000.0, 2e5)])
    half_bits = np.array([ref.lib.q27ref_float_to_half(float(v)) for v in conv_in], np.uint16)
    e4m3_bits = np.array([ref.lib.q27ref_float_to_e4m3(float(v)) for v in conv_in], np.uint8)
    e4m3_table = np.array([ref.lib.q27ref_e4m3_to_float(b) for b in range(256)], np.float32)
    np.savez_compressed(Path(__file__).parent / "turbo3_codec.npz", x=x, blocks=blocks, dequant=deq,
                        fwht=fw, conv_in=conv_in, half_bits=half_bits, e4m3_bits=e4m3_bits,
                        e4m3_table=e4m3_table)
    print("wrote turbo3_codec.npz", blocks.shape, conv_in.shape)

    # K-side codecs of the turbo5k and int8-g64 kinds: same inputs plus scale extremes
    xk = x.copy()
    xk[9] *= 1e-6                        # tiny group: fp16 scale underflow territory for int8
    xk[11, 64:] = 0.0                    # one all-zero 64-group inside a live block
    b5_tree = np.zeros((ngroups, 82), np.uint8)
    b5_serial = np.zeros((ngroups, 82), np.uint8)
    d5 = np.zeros((ngroups, 128), np.float32)
    b8 = np.zeros((ngroups, 132), np.uint8)
    d8 = np.zeros((ngroups // 2, 256), np.float32)
    vp = C.c_void_p
    for i in range(ngroups):
        ref.lib.q27ref_cpu_quant5(xk[i].ctypes.data_as(_fp), b5_tree[i].ctypes.data_as(vp), 1)
        ref.lib.q27ref_cpu_quant5(xk[i].ctypes.data_as(_fp), b5_serial[i].ctypes.data_as(vp), 0)
        ref.lib.q27ref_cpu_dequant5(b5_tree[i].ctypes.data_as(vp), d5[i].ctypes.data_as(_fp))
        ref.lib.q27ref_i8_quant(xk[i].ctypes.data_as(_fp), b8[i].ctypes.data_as(vp))
    b8 = np.ascontiguousarray(b8)
    for r in range(ngroups // 2):
        ref.lib.q27ref_i8_dequant_row(b8[2 * r:].ctypes.data_as(vp), d8[r].ctypes.data_as(_fp))
    np.savez_compressed(Path(__file__).parent / "k_codecs.npz", x=xk, t5_tree=b5_tree,
                        t5_serial=b5_serial, t5_dequant=d5, i8_blocks=b8, i8_dequant=d8)
    print("wrote k_codecs.npz", b5_tree.shape, b8.shape, int((b5_tree != b5_serial).sum()))

    # identity of a prefix-snapshot entry (src/prefix_cache.h): hashes, compat hash, header bytes
    L_ = ref.lib
    L_.q27ref_pfx_fnv1a64.restype = C.c_uint64
    L_.q27ref_pfx_fnv1a64.argtypes = [C.c_void_p, C.c_size_t]
    L_.q27ref_pfx_compat_hash.restype = C.c_uint64
    L_.q27ref_pfx_compat_hash.argtypes = [C.c_char_p, C.c_uint64] + [C.c_int] * 8
    L_.q27ref_pfx_fill_hdr.argtypes = [C.c_void_p, C.c_uint64, C.c_void_p, C.c_int, C.c_uint64, C.c_uint64]
    toks = (lcg_floats(5000, 77, 60000.0).astype(np.int32) % 151936).astype(np.int32)
    lens = np.array([1, 2, 7, 64, 4096, 5000], np.int32)
    keys = np.array([L_.q27ref_pfx_fnv1a64(toks.ctypes.data, int(n) * 4) for n in lens], np.uint64)
    geoms = np.array([[15_000_000_000, 64, 4, 256, 32, 128, 8192, k, 1] for k in range(6)]
                     + [[1, 2, 3, 4, 5, 6, 7, 2, 2]], np.int64)
    path = b"/models/q27-q4.gguf"
    compats = np.array([L_.q27ref_pfx_compat_hash(path, *[int(v) for v in g]) for g in geoms], np.uint64)
    hdr = np.zeros(64, np.uint8)
    L_.q27ref_pfx_fill_hdr(hdr.ctypes.data, int(compats[2]), toks.ctypes.data, 4096, 123456, 7890123)
    np.savez_compressed(Path(__file__).parent / "pfx_identity.npz", tokens=toks, lens=lens, keys=keys,
                        geoms=geoms, path=np.frombuffer(path, np.uint8), compats=compats, hdr=hdr,
                        magic=np.uint32(L_.q27ref_pfx_magic()), version=np.uint32(L_.q27ref_pfx_version()),
                        hdr_bytes=np.int32(L_.q27ref_pfx_hdr_bytes()))
    print("wrote pfx_identity.npz", [hex(int(k)) for k in keys[:2]])


if __name__ == "__main__":
    main()
