// The per-128-group signed Walsh-Hadamard rotation of the turbo formats, as a warp-level
// routine over a 128-float buffer in shared memory: forward = s1 -> butterfly -> inv_sqrt * s2
// (t3_fwht), inverse = s2 -> butterfly -> inv_sqrt * s1 (t3_fwht_inv; src/test_kernels.cu:1065-1087,
// src/spec3.cu:595-614). Every output of every stage is ONE rounded add, subtract or multiply
// of fixed inputs, so the result does not depend on how the work is spread over threads: it is
// bitwise the serial CPU loop, whether it runs as a kernel of its own or inside the staging
// loop or the epilogue of an attention kernel.
#pragma once
#include "common.cuh"

namespace q27b {

constexpr float INV_SQRT_128 = 0.08838834764831845f;
__device__ __forceinline__ float wht_sign(const uint32_t* m, int j) {
    return (m[j >> 5] >> (j & 31)) & 1u ? -1.f : 1.f;
}

// SKEW: element j of the group lives at x[j + SKEW * (j >> 5)] (a buffer whose 32-element
// blocks are SKEW floats apart, for bank-conflict-free readers; 0 = contiguous).
template <int SKEW>
__device__ __forceinline__ int wht_at(int j) { return j + SKEW * (j >> 5); }

// 128-point butterfly over a warp's shared buffer: element pairs (j, j^h), lo+hi / lo-hi.
template <int SKEW = 0>
__device__ __forceinline__ void butterfly128(float* x, int lane) {
#pragma unroll
    for (int h = 1; h < 128; h <<= 1) {
        __syncwarp();
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int j = lane + 32 * i;
            const float a = x[wht_at<SKEW>(j)], b = x[wht_at<SKEW>(j ^ h)];
            v[i] = (j & h) ? __fsub_rn(b, a) : __fadd_rn(a, b);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 4; i++) x[wht_at<SKEW>(lane + 32 * i)] = v[i];
    }
    __syncwarp();
}

// rotation of one group in place by one warp (all 32 lanes; x visible to the warp on entry,
// result visible to the warp on return)
template <bool INV, int SKEW = 0>
__device__ __forceinline__ void wht_group(float* x, int lane) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int j = lane + 32 * i;
        x[wht_at<SKEW>(j)] = __fmul_rn(x[wht_at<SKEW>(j)], wht_sign(INV ? kS2Neg : kS1Neg, j));
    }
    butterfly128<SKEW>(x, lane);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int j = lane + 32 * i;
        x[wht_at<SKEW>(j)] = __fmul_rn(x[wht_at<SKEW>(j)], __fmul_rn(INV_SQRT_128, wht_sign(INV ? kS1Neg : kS2Neg, j)));
    }
    __syncwarp();
}

// What a fused attention call does about the rotation (bit set): rotate every Q head forward
// while it is staged / un-rotate every output head before it is written.
enum : int { WHT_Q = 1, WHT_OUT = 2 };
// The engine's rule (src/engine.cuh:1482-1506): Q is rotated where the K side is
// (kv_k_rotated, src/cuda_common.h:59); the output is un-rotated wherever V is turbo3.
inline int wht_flags_for(int kvk) {
    return ((kvk == Q27_KV_T3 || kvk == Q27_KV_T5K) ? WHT_Q : 0) | (kvk >= Q27_KV_T3 ? WHT_OUT : 0);
}

} // namespace q27b
