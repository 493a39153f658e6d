// The turbo3 codec constants, stated ONCE for every kernel of the engine (decoders, fragment
// lookups, encoder, rotation). Values follow src/turbo3.cuh:38-43,57-66 of the reference; the
// CPU oracle keeps its own independent statement and the tests compare the two bit for bit.
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

static __device__ __constant__ float kT3Centroid[8] = {Q27_T3_CENTROID_LIST};
static __device__ __constant__ float kT3Midpoint[7] = {Q27_T3_MIDPOINT_LIST};
static __device__ __constant__ uint32_t kS1Neg[4] = {Q27_T3_S1_NEG_LIST};
static __device__ __constant__ uint32_t kS2Neg[4] = {Q27_T3_S2_NEG_LIST};

} // namespace q27b
