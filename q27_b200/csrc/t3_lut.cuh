// turbo3 centroid lookup in registers: 3-bit selectors assembled 8 per 32-bit word, centroids
// (fp16 bit patterns of src/turbo3.cuh:38-40) looked up four at a time with PRMT from
// low-byte / high-byte tables. Shared by the decode and the tile kernels.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "t3_tables.cuh"

namespace q27b {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// fp16 bit patterns of the centroids (src/turbo3.cuh:38-40), split into low and high bytes
// and packed as PRMT pools: pool byte i (0..7) = byte of centroid i.
struct T3Tab {
    uint32_t lo_a, lo_b, hi_a, hi_b;
};
__device__ __forceinline__ T3Tab t3_tables() {
    uint32_t lo[2] = {0, 0}, hi[2] = {0, 0};
    const float c[8] = {Q27_T3_CENTROID_LIST};
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint32_t bits = __half_as_ushort(__float2half_rn(c[i]));
        lo[i >> 2] |= (bits & 0xffu) << (8 * (i & 3));
        hi[i >> 2] |= (bits >> 8) << (8 * (i & 3));
    }
    return T3Tab{lo[0], lo[1], hi[0], hi[1]};
}
// The same pools for the centroids times one block norm: the fp32 centroid times the norm,
// rounded ONCE to fp16 -- the nearest fp16 to the dequantised value (turbo3_deq_elem,
// src/turbo3.cuh:134, is that fp32 product); an fp16 centroid times the fp16 norm would round
// twice. 8 FMUL + 4 packs + 4 PRMT per block instead of one HMUL2 per two elements.
__device__ __forceinline__ T3Tab t3_tables_scaled(float norm) {
    const float c[8] = {Q27_T3_CENTROID_LIST};
    uint32_t p[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const __half2 v = __floats2half2_rn(c[2 * i] * norm, c[2 * i + 1] * norm);
        p[i] = *reinterpret_cast<const uint32_t*>(&v);
    }
    return T3Tab{prmt(p[0], p[1], 0x6420u), prmt(p[2], p[3], 0x6420u), prmt(p[0], p[1], 0x7531u),
                 prmt(p[2], p[3], 0x7531u)};
}
// 16 elements: qs word Q (2 bits each) + 16 sign bits -> selectors with one nibble
// (hi<<2 | low2) per element; ze holds elements 0,2,..,14 and zo elements 1,3,..,15.
__device__ __forceinline__ void t3_selectors(uint32_t Q, uint32_t S16, uint32_t& ze, uint32_t& zo) {
    // byte LUT spreading sign bits (b0, b2 of a nibble) to bit 2 of two output nibbles
    const uint32_t he = prmt(0x04000400u, 0x44404440u, S16 & 0x7777u);
    const uint32_t ho = prmt(0x04000400u, 0x44404440u, (S16 >> 1) & 0x7777u);
    ze = (Q & 0x33333333u) | he;
    zo = ((Q >> 2) & 0x33333333u) | ho;
}
// 8 selector nibbles -> 4 half2 registers (nibbles 2i, 2i+1 -> h[i])
__device__ __forceinline__ void t3_lookup(const T3Tab& t, uint32_t z, uint32_t* h) {
    const uint32_t zh = z >> 16;
    const uint32_t l0 = prmt(t.lo_a, t.lo_b, z), h0 = prmt(t.hi_a, t.hi_b, z);
    const uint32_t l1 = prmt(t.lo_a, t.lo_b, zh), h1 = prmt(t.hi_a, t.hi_b, zh);
    h[0] = prmt(l0, h0, 0x5140u);
    h[1] = prmt(l0, h0, 0x7362u);
    h[2] = prmt(l1, h1, 0x5140u);
    h[3] = prmt(l1, h1, 0x7362u);
}


} // namespace q27b
