// The turbo3 / turbo5 codec constants, stated ONCE for every kernel of the engine (decoders,
// fragment lookups, encoders, rotation). Values follow src/turbo3.cuh:38-43,57-66 and
// src/turbo5.cuh:63-80 of the reference; the CPU oracle keeps its own independent statement
// and the tests compare the two bit for bit.
#pragma once
#include <stdint.h>

namespace q27b {

// centroid of index idx = low2 | hi << 2 (src/turbo3.cuh:38-40); c[7 - i] == -c[i]
#define Q27_T3_CENTROID_LIST \
    -0.190207f, -0.118786f, -0.066822f, -0.021663f, 0.021663f, 0.066822f, 0.118786f, 0.190207f
// decision thresholds between neighbouring centroids (src/turbo3.cuh:57-66)
#define Q27_T3_MIDPOINT_LIST \
    -0.154496f, -0.092804f, -0.044243f, 0.000000f, 0.044243f, 0.092804f, 0.154496f
// the two sign diagonals of the rotation as bit masks: bit j set <=> element j is -1
// (src/turbo3.cuh:42-43)
#define Q27_T3_S1_NEG_LIST 0xE46A0359u, 0x42F85949u, 0xA4C63BBBu, 0x49F250A9u
#define Q27_T3_S2_NEG_LIST 0x16ACEE90u, 0x3F628FDCu, 0xB7A5357Au, 0xBEA56562u

// turbo5, the 5-bit K side: centroid of index idx = low4 | hi << 4 (src/turbo5.cuh:63-71) and the
// 31 decision thresholds between neighbours (src/turbo5.cuh:72-80); both odd-symmetric
#define Q27_T5_CENTROID_LIST \
    -0.28821075f, -0.23786362f, -0.20486116f, -0.17931595f, -0.15797059f, -0.13932019f, \
    -0.12253633f, -0.10710939f, -0.09270022f, -0.07906913f, -0.06603809f, -0.05346908f, \
    -0.04125080f, -0.02928998f, -0.01750547f, -0.00582388f, 0.00582388f, 0.01750547f, \
    0.02928998f, 0.04125080f, 0.05346908f, 0.06603809f, 0.07906913f, 0.09270022f, \
    0.10710939f, 0.12253633f, 0.13932019f, 0.15797059f, 0.17931595f, 0.20486116f, \
    0.23786362f, 0.28821075f
#define Q27_T5_THRESHOLD_LIST \
    -0.26303717f, -0.22136238f, -0.19208856f, -0.16864327f, -0.14864540f, -0.13092826f, \
    -0.11482286f, -0.09990481f, -0.08588468f, -0.07255360f, -0.05975358f, -0.04735994f, \
    -0.03527039f, -0.02339773f, -0.01166468f, 0.00000000f, 0.01166468f, 0.02339773f, \
    0.03527039f, 0.04735994f, 0.05975358f, 0.07255360f, 0.08588468f, 0.09990481f, \
    0.11482286f, 0.13092826f, 0.14864540f, 0.16864327f, 0.19208856f, 0.22136238f, \
    0.26303717f

static __device__ __constant__ float kT5Centroid[32] = {Q27_T5_CENTROID_LIST};
static __device__ __constant__ float kT5Threshold[31] = {Q27_T5_THRESHOLD_LIST};
static __device__ __constant__ float kT3Centroid[8] = {Q27_T3_CENTROID_LIST};
static __device__ __constant__ float kT3Midpoint[7] = {Q27_T3_MIDPOINT_LIST};
static __device__ __constant__ uint32_t kS1Neg[4] = {Q27_T3_S1_NEG_LIST};
static __device__ __constant__ uint32_t kS2Neg[4] = {Q27_T3_S2_NEG_LIST};

} // namespace q27b
