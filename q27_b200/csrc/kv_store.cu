// KV row stores and the per-128-group Walsh-Hadamard rotation: the steps either side of
// attention in every call stack of the reference (kv_store_T / kv_store_T_t3 / wht_T,
// src/prefill.cu:1221-1243,2556-2618; kv_store3 / kv_store_t3 / wht3, src/spec3.cu:512-614).
//
// The turbo3 encoder follows the reference's serial CPU codec (t3_quant,
// src/test_kernels.cu:1089-1103) operation for operation -- serial fp32 sums in element
// order, separate multiply and add -- so its blocks are byte-identical to that codec. (The
// reference's own device encoder reduces in a tree and is allowed <= 0.2 % index ties
// against the same CPU codec, src/test_kernels.cu:1150-1316.)
//
// K legs of the kinds above turbo3 (src/spec3.cu:564-578, src/prefill.cu:2570-2584): turbo3v
// stores plain fp16 rows; turbo5k runs the same normalise / rotate / nearest / norm-correction
// pipeline over 32 centroids, with the two norms summed in the halving-tree order of the
// reference's device encoder (turbo5_quant_group, src/turbo5.cuh:129-162), whose bit-for-bit
// gate is its CPU oracle in tree mode (tools/turbo5_test.cu:58-84); int8-g64 takes the absmax
// of each 64 dims, rounds absmax/127 to fp16 and quantises with the reciprocal of the ROUNDED
// scale (i8g64_quant_group, src/i8g64.cuh:48-64) -- order-independent, hence exact.
#include "common.cuh"
#include "wht.cuh"

namespace q27b {
namespace {

__device__ __forceinline__ int t3_nearest(float v) { // src/turbo3.cuh:57-66
    int idx = 0;
#pragma unroll
    for (int i = 0; i < 7; i++) idx += v < kT3Midpoint[i] ? 0 : 1;   // thresholds ascend
    return idx;
}

constexpr int ST_WARPS = 8;

// One warp encodes one 128-element group into a 50-byte block.
__device__ __forceinline__ void t3_encode_group(const float* __restrict__ src, uint8_t* blk,
                                                float* xs, int lane) {
#pragma unroll
    for (int i = 0; i < 4; i++) xs[lane + 32 * i] = src[lane + 32 * i];
    __syncwarp();
    float gn = 0.f;
    if (lane == 0) { // serial sum in element order, as the CPU codec does
        float nsq = 0.f;
        for (int j = 0; j < 128; j++) nsq = __fadd_rn(nsq, __fmul_rn(xs[j], xs[j]));
        gn = sqrtf(nsq);
    }
    gn = __shfl_sync(0xffffffffu, gn, 0);
    const float inv = gn > 1e-10f ? __fdiv_rn(1.f, gn) : 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) xs[lane + 32 * i] = __fmul_rn(xs[lane + 32 * i], inv);
    __syncwarp();
    wht_group<false>(xs, lane);
    // lane owns elements 4*lane .. 4*lane+3: one qs byte, half a signs byte
    int idx[4];
    uint32_t qs = 0, hb = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        idx[i] = t3_nearest(xs[4 * lane + i]);
        qs |= (uint32_t)(idx[i] & 3) << (2 * i);
        hb |= (uint32_t)((idx[i] >> 2) & 1) << i;
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float cv = kT3Centroid[idx[i]];
        xs[4 * lane + i] = __fmul_rn(cv, cv);
    }
    __syncwarp();
    const uint32_t hb_hi = __shfl_down_sync(0xffffffffu, hb, 1);
    blk[2 + lane] = (uint8_t)qs;
    if ((lane & 1) == 0) blk[34 + (lane >> 1)] = (uint8_t)(hb | (hb_hi << 4));
    if (lane == 0) {
        float rsq = 0.f;
        for (int j = 0; j < 128; j++) rsq = __fadd_rn(rsq, xs[j]);
        const float rn = sqrtf(rsq);
        const float corr = rn > 1e-10f ? __fdiv_rn(gn, rn) : gn;
        *reinterpret_cast<__half*>(blk) = __float2half_rn(corr);
    }
    __syncwarp();
}

__device__ __forceinline__ int t5_nearest(float v) { // src/turbo5.cuh:95-107
    int idx = 0;
#pragma unroll
    for (int i = 0; i < 31; i++) idx += v >= kT5Threshold[i] ? 1 : 0;
    return idx;
}

// Sum of a group's 128 values, lane holding elements lane + 32 i, in the order of the loop
// `for (s = 64; s > 0; s >>= 1) r[j] += r[j + s]  (j < s)`: result valid in lane 0.
__device__ __forceinline__ float tree_sum128(const float (&v)[4], int lane) {
    float a = __fadd_rn(__fadd_rn(v[0], v[2]), __fadd_rn(v[1], v[3]));   // s = 64, then s = 32
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, s));
    return a;
}

// One warp encodes one 128-element group into an 82-byte turbo5 block.
__device__ __forceinline__ void t5_encode_group(const float* __restrict__ src, uint8_t* blk,
                                                float* xs, int lane) {
    float v[4], sq[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        v[i] = src[lane + 32 * i];
        sq[i] = __fmul_rn(v[i], v[i]);
    }
    const float gn = __shfl_sync(0xffffffffu, sqrtf(tree_sum128(sq, lane)), 0);
    const float inv = gn > 1e-10f ? __fdiv_rn(1.f, gn) : 0.f;
#pragma unroll
    for (int i = 0; i < 4; i++) xs[lane + 32 * i] = __fmul_rn(v[i], inv);
    __syncwarp();
    wht_group<false>(xs, lane);
    // lane owns elements 4*lane .. 4*lane+3: two qs bytes, half a hi byte
    int idx[4];
    uint32_t qs = 0, hb = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        idx[i] = t5_nearest(xs[4 * lane + i]);
        qs |= (uint32_t)(idx[i] & 15) << (4 * i);
        hb |= (uint32_t)((idx[i] >> 4) & 1) << i;
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float cv = kT5Centroid[idx[i]];
        xs[4 * lane + i] = __fmul_rn(cv, cv);
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; i++) sq[i] = xs[lane + 32 * i];
    const float rn = sqrtf(tree_sum128(sq, lane));
    const uint32_t hb_hi = __shfl_down_sync(0xffffffffu, hb, 1);
    *reinterpret_cast<uint16_t*>(blk + 2 + 2 * lane) = (uint16_t)qs;          // block is 2-aligned
    if ((lane & 1) == 0) blk[66 + (lane >> 1)] = (uint8_t)(hb | (hb_hi << 4));
    if (lane == 0) {
        const float corr = rn > 1e-10f ? __fdiv_rn(gn, rn) : gn;
        *reinterpret_cast<__half*>(blk) = __float2half_rn(corr);
    }
    __syncwarp();
}

// One warp encodes one 128-element group into a 132-byte int8-g64 block: lane holds elements
// lane + 32 i, so i = 0, 1 belong to the first 64-group and i = 2, 3 to the second.
__device__ __forceinline__ void i8_encode_group(const float* __restrict__ src, uint8_t* blk,
                                                int lane) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = src[lane + 32 * i];
    float am[2] = {fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))};
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        am[0] = fmaxf(am[0], __shfl_xor_sync(0xffffffffu, am[0], off));
        am[1] = fmaxf(am[1], __shfl_xor_sync(0xffffffffu, am[1], off));
    }
#pragma unroll
    for (int g = 0; g < 2; g++) {
        const __half sh = __float2half_rn(__fdiv_rn(am[g], 127.0f));
        const float sw = __half2float(sh);                 // the ROUNDED scale
        const float inv = sw > 0.f ? __fdiv_rn(1.0f, sw) : 0.f;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int q = min(127, max(-127, __float2int_rn(__fmul_rn(v[2 * g + i], inv))));
            reinterpret_cast<int8_t*>(blk)[64 * g + 32 * i + lane] = (int8_t)(sw > 0.f ? q : 0);
        }
        if (lane == 0) *reinterpret_cast<__half*>(blk + 128 + 2 * g) = sh;
    }
}

// One (row, group) of a side in the side's storage format; `cell` = (row in page) * groups per
// row + group. V sides and turbo3 K go through the turbo3 encoder.
__device__ __forceinline__ void encode_group(int fmt, const float* __restrict__ src, uint8_t* page,
                                             size_t cell, float* xs, int lane) {
    if (fmt == RF_T3) {
        t3_encode_group(src, page + cell * T3_BLK, xs, lane);
    } else if (fmt == RF_T5) {
        t5_encode_group(src, page + cell * T5_BLK, xs, lane);
    } else if (fmt == RF_I8) {
        i8_encode_group(src, page + cell * I8_BLK, lane);
    } else {                                                // RF_F16: 128 plain halves
        __half* d = reinterpret_cast<__half*>(page) + cell * 128;
#pragma unroll
        for (int i = 0; i < 4; i++) d[lane + 32 * i] = __float2half_rn(src[lane + 32 * i]);
    }
}

// rows base_pos .. base_pos+T-1; kT/vT: [T][n_kv*256] fp32
__global__ void __launch_bounds__(ST_WARPS * 32)
k_kv_store_T_t3(const float* __restrict__ kT, const float* __restrict__ vT, void* const* ktab,
                void* const* vtab, int base_pos, int n_kv, int T, int kfmt, int row_base, int row_count) {
    __shared__ float xs[ST_WARPS][128];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gpr = n_kv * 2; // groups per row per side
    const int64_t total = (int64_t)T * gpr * 2;
    for (int64_t w = (int64_t)blockIdx.x * ST_WARPS + warp; w < total;
         w += (int64_t)gridDim.x * ST_WARPS) {
        const int side = (int)(w & 1);
        const int64_t gidx = w >> 1;
        const int t = (int)(gidx / gpr), gi = (int)(gidx % gpr);
        const int p = base_pos + t - row_base;     // row of this GPU's tables, if it owns the row
        if (p < 0 || p >= row_count) continue;
        uint8_t* page = static_cast<uint8_t*>((side ? vtab : ktab)[p >> PAGE_SHIFT]);
        encode_group(side ? RF_T3 : kfmt, (side ? vT : kT) + (size_t)t * gpr * 128 + (size_t)gi * 128,
                     page, (size_t)(p & (PAGE - 1)) * gpr + gi, xs[warp], lane);
    }
}

template <bool FP8>
__global__ void __launch_bounds__(256)
k_kv_store_T(const float* __restrict__ kT, const float* __restrict__ vT, void* const* ktab,
             void* const* vtab, int base_pos, int rowlen, int T, int row_base, int row_count) {
    const int64_t total = (int64_t)T * rowlen;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / rowlen), e = (int)(i % rowlen);
        const int p = base_pos + t - row_base;
        if (p < 0 || p >= row_count) continue;
        const size_t off = (size_t)(p & (PAGE - 1)) * rowlen + e;
        if (FP8) {
            static_cast<__nv_fp8_e4m3*>(ktab[p >> PAGE_SHIFT])[off] = __nv_fp8_e4m3(kT[i]);
            static_cast<__nv_fp8_e4m3*>(vtab[p >> PAGE_SHIFT])[off] = __nv_fp8_e4m3(vT[i]);
        } else {
            static_cast<__half*>(ktab[p >> PAGE_SHIFT])[off] = __float2half_rn(kT[i]);
            static_cast<__half*>(vtab[p >> PAGE_SHIFT])[off] = __float2half_rn(vT[i]);
        }
    }
}

// In-place rotation of the first head_dim floats of every head of T rows.
template <bool INV>
__global__ void __launch_bounds__(ST_WARPS * 32)
k_wht_T(float* __restrict__ x, int n_heads, int head_stride, int row_stride, int T) {
    __shared__ float xs[ST_WARPS][128];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t total = (int64_t)T * n_heads * 2;
    for (int64_t w = (int64_t)blockIdx.x * ST_WARPS + warp; w < total;
         w += (int64_t)gridDim.x * ST_WARPS) {
        const int half = (int)(w & 1), h = (int)((w >> 1) % n_heads), t = (int)((w >> 1) / n_heads);
        float* g = x + (size_t)t * row_stride + (size_t)h * head_stride + half * 128;
#pragma unroll
        for (int i = 0; i < 4; i++) xs[warp][lane + 32 * i] = g[lane + 32 * i];
        __syncwarp();
        wht_group<INV>(xs[warp], lane);
#pragma unroll
        for (int i = 0; i < 4; i++) g[lane + 32 * i] = xs[warp][lane + 32 * i];
        __syncwarp();
    }
}

// ---- lane forms: one row per draft lane, source rows and positions behind lane bundles ----
// [row_base, row_base + row_count): the logical rows this GPU's tables hold (everything, or
// its shard of a cache split by rows: a lane whose row lives elsewhere is skipped here and
// stored by the GPU that owns it, every GPU running the same call on the same lanes).
struct LaneRows {
    const float* k[Q27_MAX_LANES];
    const float* v[Q27_MAX_LANES];
    const int* pos[Q27_MAX_LANES];
    int row_base, row_count;
};
struct LaneVecs {
    float* x[Q27_MAX_LANES];
};

// grid (groups per row x 2 sides / ST_WARPS, ntok): lane t's K and V rows into cache row *pos[t]
__global__ void __launch_bounds__(ST_WARPS * 32)
k_kv_store3_t3(const __grid_constant__ LaneRows L, void* const* ktab, void* const* vtab, int n_kv,
               int kfmt) {
    __shared__ float xs[ST_WARPS][128];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.y, gpr = n_kv * 2;
    const int w = blockIdx.x * ST_WARPS + warp;          // (group, side)
    if (w >= gpr * 2) return;
    const int side = w & 1, gi = w >> 1;
    const int p = __ldg(L.pos[t]) - L.row_base;
    if (p < 0 || p >= L.row_count) return;
    uint8_t* page = static_cast<uint8_t*>((side ? vtab : ktab)[p >> PAGE_SHIFT]);
    encode_group(side ? RF_T3 : kfmt, (side ? L.v[t] : L.k[t]) + (size_t)gi * 128, page,
                 (size_t)(p & (PAGE - 1)) * gpr + gi, xs[warp], lane);
}

template <bool FP8>
__global__ void __launch_bounds__(256)
k_kv_store3(const __grid_constant__ LaneRows L, void* const* ktab, void* const* vtab, int rowlen) {
    const int e = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (e >= rowlen) return;
    const int p = __ldg(L.pos[t]) - L.row_base;
    if (p < 0 || p >= L.row_count) return;
    const size_t off = (size_t)(p & (PAGE - 1)) * rowlen + e;
    if (FP8) {
        static_cast<__nv_fp8_e4m3*>(ktab[p >> PAGE_SHIFT])[off] = __nv_fp8_e4m3(L.k[t][e]);
        static_cast<__nv_fp8_e4m3*>(vtab[p >> PAGE_SHIFT])[off] = __nv_fp8_e4m3(L.v[t][e]);
    } else {
        static_cast<__half*>(ktab[p >> PAGE_SHIFT])[off] = __float2half_rn(L.k[t][e]);
        static_cast<__half*>(vtab[p >> PAGE_SHIFT])[off] = __float2half_rn(L.v[t][e]);
    }
}

// grid (heads x 2 groups / ST_WARPS, ntok): rotate the first 256 floats of every head in place
template <bool INV>
__global__ void __launch_bounds__(ST_WARPS * 32)
k_wht3(const __grid_constant__ LaneVecs V, int n_heads, int stride) {
    __shared__ float xs[ST_WARPS][128];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int w = blockIdx.x * ST_WARPS + warp;
    if (w >= n_heads * 2) return;
    float* g = V.x[blockIdx.y] + (size_t)(w >> 1) * stride + (w & 1) * 128;
#pragma unroll
    for (int i = 0; i < 4; i++) xs[warp][lane + 32 * i] = g[lane + 32 * i];
    __syncwarp();
    wht_group<INV>(xs[warp], lane);
#pragma unroll
    for (int i = 0; i < 4; i++) g[lane + 32 * i] = xs[warp][lane + 32 * i];
}

unsigned blocks_for(int64_t units, int per_block) {
    int64_t b = (units + per_block - 1) / per_block;
    return (unsigned)(b < 1 ? 1 : b > 148 * 16 ? 148 * 16 : b);
}

} // namespace

int launch_kv_store_T(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                      int base_pos, int n_kv, int T, cudaStream_t st, int kvk, int row_base,
                      int row_count) {
    if (T == 0) return Q27_OK;
    if (kvk >= Q27_KV_T3 && kind_known(kvk)) {
        k_kv_store_T_t3<<<blocks_for((int64_t)T * n_kv * 4, ST_WARPS), ST_WARPS * 32, 0, st>>>(
            kT, vT, ktab, vtab, base_pos, n_kv, T, k_fmt(kvk), row_base, row_count);
    } else if (kvk == Q27_KV_FP8) {
        k_kv_store_T<true><<<blocks_for((int64_t)T * n_kv * HD, 256), 256, 0, st>>>(
            kT, vT, ktab, vtab, base_pos, n_kv * HD, T, row_base, row_count);
    } else if (kvk == Q27_KV_F16) {
        k_kv_store_T<false><<<blocks_for((int64_t)T * n_kv * HD, 256), 256, 0, st>>>(
            kT, vT, ktab, vtab, base_pos, n_kv * HD, T, row_base, row_count);
    } else {
        return Q27_ERR_UNSUPPORTED_KIND;
    }
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

int launch_kv_store3(const float* const* k, const float* const* v, const int* const* pos,
                     void* const* ktab, void* const* vtab, int n_kv, int ntok, cudaStream_t st,
                     int kvk, int row_base, int row_count) {
    if (ntok == 0) return Q27_OK;
    LaneRows L{};
    L.row_base = row_base;
    L.row_count = row_count;
    for (int t = 0; t < ntok; t++) {
        L.k[t] = k[t];
        L.v[t] = v[t];
        L.pos[t] = pos[t];
    }
    if (kvk >= Q27_KV_T3 && kind_known(kvk)) {
        dim3 grid((n_kv * 4 + ST_WARPS - 1) / ST_WARPS, ntok);
        k_kv_store3_t3<<<grid, ST_WARPS * 32, 0, st>>>(L, ktab, vtab, n_kv, k_fmt(kvk));
    } else if (kvk == Q27_KV_FP8 || kvk == Q27_KV_F16) {
        const int rowlen = n_kv * HD;
        dim3 grid((rowlen + 255) / 256, ntok);
        if (kvk == Q27_KV_FP8) k_kv_store3<true><<<grid, 256, 0, st>>>(L, ktab, vtab, rowlen);
        else k_kv_store3<false><<<grid, 256, 0, st>>>(L, ktab, vtab, rowlen);
    } else {
        return Q27_ERR_UNSUPPORTED_KIND;
    }
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

int launch_wht3(float* const* x, int n_heads, int stride, int ntok, bool inv, cudaStream_t st) {
    if (ntok == 0 || n_heads == 0) return Q27_OK;
    LaneVecs V{};
    for (int t = 0; t < ntok; t++) V.x[t] = x[t];
    dim3 grid((n_heads * 2 + ST_WARPS - 1) / ST_WARPS, ntok);
    if (inv) k_wht3<true><<<grid, ST_WARPS * 32, 0, st>>>(V, n_heads, stride);
    else k_wht3<false><<<grid, ST_WARPS * 32, 0, st>>>(V, n_heads, stride);
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

int launch_wht_T(float* x, int n_heads, int head_stride, int row_stride, int T, bool inv,
                 cudaStream_t st) {
    if (T == 0 || n_heads == 0) return Q27_OK;
    const unsigned blocks = blocks_for((int64_t)T * n_heads * 2, ST_WARPS);
    if (inv) k_wht_T<true><<<blocks, ST_WARPS * 32, 0, st>>>(x, n_heads, head_stride, row_stride, T);
    else k_wht_T<false><<<blocks, ST_WARPS * 32, 0, st>>>(x, n_heads, head_stride, row_stride, T);
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

} // namespace q27b
