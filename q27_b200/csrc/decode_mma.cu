// Tensor-core split-KV decode for sm_100a.
//
// One CTA = (slot, lane, position split [, kv head]). A producer warp streams the split's
// K and V rows into a shared-memory ring with asynchronous copies (cp.async.bulk for whole
// turbo3 rows, 16-byte cp.async for fp16 / fp8 slices; completion on an mbarrier); consumer
// warps turn ring rows straight into mma.sync fragments in registers -- no dequantised tile
// is ever written back to shared memory -- and run
//     S^T = K . Q^T        (16 keys x 8 query columns per MMA, fp16 operands, fp32 accum)
//     O^T += V^T . P^T     (16 dims x 8 query columns, contraction over 16 keys)
// with an online softmax per query column. The six GQA heads of a KV head are the columns
// (8 with padding), so one read of a row serves all of them.
//
// turbo3 rows are never multiplied out to centroid*norm per element: the per-block fp16
// norm is factored out of the dot product (two accumulators per tile, one per 128-dim
// block, recombined as nK0*D0 + nK1*D1) and folded into P for the V side, so the MMA
// operands are the eight centroid constants, looked up 4 elements per PRMT. The bit-exact
// centroid*norm product lives in the exact family and q27_kv_dequant.
//
// turbo3 is bound by the integer pipe (selector assembly and lookups: about 2.4 PRMT / LOP3 /
// SHF lane-operations per cache element against 64 per clock and SM). A consumer warp takes
// BOTH 16-key tiles of a ring stage at once: two independent score streams keep the pipe fed
// while one waits on a lookup or an MMA, and one online-softmax step covers the 32 keys.
//
// Dimension and key indices inside a tile are permuted per format so that every thread's
// fragment registers come from contiguous packed bytes; Q^T fragments and the output rows
// use the same maps (kdim_* / vdim_* below), so the permutation cancels.
//
// Small launches finish in the same kernel: when a (slot, lane, kv group) has few splits, its
// CTAs wait for one another once their partials are written (cooperative launch, bounded wait)
// and each merges its share of the group's outputs and writes the normalised values, so a short
// decode is ONE launch.
#include <limits.h>

#include "decode_mma.cuh"
#include "t3_lut.cuh"
#include "wht.cuh"
#include "finish.cuh"

namespace q27b {

__device__ int g_wait_timeout_flag = 0; // set when a bounded mbarrier wait ran out

namespace {

constexpr int STAGE_ROWS = 32;    // rows per ring stage (= 2 key tiles; never crosses a page)
constexpr int TILE = 16;          // keys per MMA tile
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;
constexpr int FUSE_MAX_SPLITS = FINISH_MAX_SPLITS;
// A launch finishes itself while its partials are few (measured: c1, 6 heads x 37 splits, 21.9 ->
// 14.3 us per step); long launches are better off with the combine kernel, whose launch hides
// behind the partial kernel's tail (c3, 24 heads x 74 splits: 94 us that way, 101 us fused).
constexpr int FUSE_MAX_BYTES = 288 * 1024;

template <int KVK> struct Fmt;
template <> struct Fmt<Q27_KV_F16> {
    static constexpr int KVH = 1;               // kv heads per CTA
    static constexpr int PITCH = 512 + 16;      // one (row, head) slice + pad: conflict-free ldmatrix
    static constexpr int SLICE = 512;
    static constexpr int STAGES = 5;
    static constexpr int NCW = 8;               // consumer warps
};
template <> struct Fmt<Q27_KV_FP8> {
    static constexpr int KVH = 1;
    static constexpr int PITCH = 256 + 16;
    static constexpr int SLICE = 256;
    static constexpr int STAGES = 8;
    static constexpr int NCW = 8;
};
template <> struct Fmt<Q27_KV_T3> {
    static constexpr int KVH = 4;               // whole 400-byte rows: all four kv heads
    static constexpr int PITCH = 400;
    static constexpr int SLICE = 400;
    static constexpr int STAGES = 5;
    static constexpr int NCW = 8;
};
template <int KVK> constexpr int n_threads() { return (Fmt<KVK>::NCW + 1) * 32; }   // + the producer warp
constexpr int HEADER_BYTES = 256;                 // ring barriers
template <int KVK> constexpr int stage_bytes() { return 2 * STAGE_ROWS * Fmt<KVK>::PITCH; }
template <int KVK> constexpr int ring_bytes() { return stage_bytes<KVK>() * Fmt<KVK>::STAGES; }
// per-warp partials for the final merge
template <int KVK> constexpr int merge_bytes() { return Fmt<KVK>::NCW * GQA * PART * 4; }
template <int KVK> constexpr int work_bytes() {
    return ring_bytes<KVK>() > merge_bytes<KVK>() ? ring_bytes<KVK>() : merge_bytes<KVK>();
}
// The staged Q heads are read back as Q^T fragments by lanes that differ in head (g) and in
// thread column (c). At a pitch of 256 floats every head starts on the same bank: 6 (fp16 /
// fp8) or 24 (turbo3, where the columns are 32 floats apart as well) lanes of a load collide,
// and the eight warps build their fragments through one shared-memory port (1.6 us of a short
// decode). So the pitch is padded -- fp16 reads 8-byte pairs at banks 8 g + 2 c, fp8 at 4 g +
// 16 c (two ways at best: its columns are 16 floats apart) -- and turbo3 also skews the row:
// every 32-float block sits one float further on and the second 128-group four more, which puts
// lane (g, c) on bank 12 g + c: no two alike.
template <int KVK> constexpr int q_pitch() { return KVK == Q27_KV_F16 ? HD + 8 : KVK == Q27_KV_T3 ? HD + 12 : HD + 4; }
constexpr int Q_SKEW_T3 = 1;                 // floats between the 32-float blocks of a turbo3 Q row
template <int KVK>
__host__ __device__ __forceinline__ int q_at(int d) {     // where dim d of a staged head lives in its row
    return KVK == Q27_KV_T3 ? d + Q_SKEW_T3 * ((d >> 5) & 3) + 4 * (d >> 7) : d;
}
template <int KVK> constexpr int qstage_bytes() { return Fmt<KVK>::KVH * GQA * q_pitch<KVK>() * 4; }
template <int KVK> constexpr int smem_bytes() {
    return HEADER_BYTES + work_bytes<KVK>() + qstage_bytes<KVK>();
}

// ---- PTX helpers ----------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
                 "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait: gives up after ~1M polls, records it, and lets the caller bail out.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity) {
    for (int i = 0; i < (1 << 20); i++) {
        if (mbar_try_wait(b, parity)) return true;
        if (i > 4096) __nanosleep(128);
    }
    atomicExch(&g_wait_timeout_flag, 1);
    return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(x));
    return d;
}
// a pointer held by lane `src` of the warp
__device__ __forceinline__ const void* shfl_ptr(const void* p, int src) {
    const unsigned long long v = (unsigned long long)(uintptr_t)p;
    const uint32_t lo = __shfl_sync(0xffffffffu, (uint32_t)v, src);
    const uint32_t hi = __shfl_sync(0xffffffffu, (uint32_t)(v >> 32), src);
    return reinterpret_cast<const void*>((uintptr_t)(((unsigned long long)hi << 32) | lo));
}
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}
// shared-space loads on 32-bit shared addresses (no generic-pointer arithmetic)
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// 32 bits starting at a 2-byte-aligned shared address. The unaligned form glues two 16-bit
// loads with a multiply-add: that instruction runs on the FMA pipe, which this kernel leaves
// idle, where a funnel shift would compete with the lookups for the integer pipe.
__device__ __forceinline__ uint32_t lds32_a2(uint32_t a, bool aligned4) {
    if (aligned4) return lds32(a);
    const uint32_t lo = lds16(a), hi = lds16(a + 2);
    uint32_t r;
    asm("mad.lo.u32 %0, %1, 65536, %2;" : "=r"(r) : "r"(hi), "r"(lo));
    return r;
}
__device__ __forceinline__ float lds_half(uint32_t a) {
    return __half2float(__ushort_as_half((unsigned short)lds16(a)));
}

// ---- index maps: (MMA-logical index) -> (actual dimension / key) -------------------------
// K side: contraction step s (0..15), thread column c (0..3), register r (0: logical k
// 2c,2c+1; 1: logical k 2c+8,2c+9), element e (0/1) -> dimension of the head.
template <int KVK>
__host__ __device__ __forceinline__ int kdim(int s, int c, int r, int e) {
    if (KVK == Q27_KV_F16) return 16 * s + 2 * c + 8 * r + e;
    if (KVK == Q27_KV_FP8) return 16 * (c + 4 * (s >> 2)) + 4 * (s & 3) + 2 * r + e;
    // turbo3: s = 8*block + 4*group + i; the thread owns dims [32c, 32c+32) of the block
    const int b = s >> 3, w = (s >> 2) & 1, i = s & 3;
    const int e16 = (i & 1) * 8 + (i >> 1) + 4 * r + 2 * e;
    return 128 * b + 32 * c + 16 * w + e16;
}
// V side: output tile mt (0..15), row rr (0..15) of O^T -> dimension of the head.
__host__ __device__ __forceinline__ int t3_vorder(int i) {
    // order in which the interleaved selectors yield a thread's 16 dims of a block
    return ((i >> 2) == 0 ? 0 : (i >> 2) == 1 ? 2 : (i >> 2) == 2 ? 1 : 3) + 4 * (i & 3);
}
template <int KVK>
__host__ __device__ __forceinline__ int vdim(int mt, int rr) {
    if (KVK == Q27_KV_F16) return 16 * mt + rr;
    if (KVK == Q27_KV_FP8) {
        const int g = rr & 7;
        return 16 * (4 * (g & 1) + (g >> 1) + 8 * (mt >> 3)) + 2 * (mt & 7) + (rr >> 3);
    }
    const int b = mt >> 3, j = mt & 7;
    return 128 * b + 16 * (rr & 7) + t3_vorder(2 * j + (rr >> 3));
}
// logical key index (row of S^T / contraction index of PV) -> key within the 16-key tile
template <int KVK>
__host__ __device__ __forceinline__ int keyperm(int k) {
    if (KVK == Q27_KV_FP8) return ((k >> 1) & 3) + 4 * (k & 1) + 8 * (k >> 3);
    return k;
}

// ---- per-warp state -----------------------------------------------------------------------
struct WarpAcc {
    float o[16][4];   // O^T: tile mt, regs {(row g, col 2c), (g, 2c+1), (g+8, 2c), (g+8, 2c+1)}
    float m[2];       // running max (log2 domain) of columns 2c, 2c+1
    float l[2];       // this thread's share of the running sum
};

// Online-softmax update for one 16-key tile. s[4] = scores (already scaled to log2 domain)
// for rows g, g+8 and columns 2c, 2c+1; valid rows carry real scores, masked rows -inf.
// Returns P as two half2 registers (rows g / g+8), columns (2c, 2c+1).
__device__ __forceinline__ void softmax_tile(WarpAcc& A, const float (&s)[4], float (&p)[4]) {
    float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(A.m[0], mx0), mn1 = fmaxf(A.m[1], mx1);
    if (mn0 > A.m[0] || mn1 > A.m[1]) { // rescale (every thread of a column group agrees)
        const float a0 = ex2(A.m[0] - mn0), a1 = ex2(A.m[1] - mn1);
        A.l[0] *= a0;
        A.l[1] *= a1;
#pragma unroll
        for (int mt = 0; mt < 16; mt++) {
            A.o[mt][0] *= a0; A.o[mt][1] *= a1; A.o[mt][2] *= a0; A.o[mt][3] *= a1;
        }
        A.m[0] = mn0;
        A.m[1] = mn1;
    }
    p[0] = ex2(s[0] - A.m[0]);
    p[1] = ex2(s[1] - A.m[1]);
    p[2] = ex2(s[2] - A.m[0]);
    p[3] = ex2(s[3] - A.m[1]);
    A.l[0] += p[0] + p[2];
    A.l[1] += p[1] + p[3];
}

// The same for two tiles (32 keys) in one step: one max, one rescale.
__device__ __forceinline__ void softmax_pair(WarpAcc& A, const float (&s)[4], const float (&t)[4],
                                             float (&p)[4], float (&q)[4]) {
    float mx0 = fmaxf(fmaxf(s[0], s[2]), fmaxf(t[0], t[2]));
    float mx1 = fmaxf(fmaxf(s[1], s[3]), fmaxf(t[1], t[3]));
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(A.m[0], mx0), mn1 = fmaxf(A.m[1], mx1);
    if (mn0 > A.m[0] || mn1 > A.m[1]) { // rescale (every thread of a column group agrees)
        const float a0 = ex2(A.m[0] - mn0), a1 = ex2(A.m[1] - mn1);
        A.l[0] *= a0;
        A.l[1] *= a1;
#pragma unroll
        for (int mt = 0; mt < 16; mt++) {
            A.o[mt][0] *= a0; A.o[mt][1] *= a1; A.o[mt][2] *= a0; A.o[mt][3] *= a1;
        }
        A.m[0] = mn0;
        A.m[1] = mn1;
    }
    p[0] = ex2(s[0] - A.m[0]);
    p[1] = ex2(s[1] - A.m[1]);
    p[2] = ex2(s[2] - A.m[0]);
    p[3] = ex2(s[3] - A.m[1]);
    q[0] = ex2(t[0] - A.m[0]);
    q[1] = ex2(t[1] - A.m[1]);
    q[2] = ex2(t[2] - A.m[0]);
    q[3] = ex2(t[3] - A.m[1]);
    A.l[0] += (p[0] + p[2]) + (q[0] + q[2]);
    A.l[1] += (p[1] + p[3]) + (q[1] + q[3]);
}

// ---- tile processors ------------------------------------------------------------------
// Each consumes one 16-key tile of one kv head from the ring stage. `valid` = number of
// real keys in the tile (rows >= valid are masked). qf = Q^T fragments, 2 regs per step.

template <int KVK>
__device__ __forceinline__ void tile_f16(WarpAcc& A, uint32_t ks, uint32_t vs,
                                         const uint32_t (&qf)[16][2], int valid, float sc2,
                                         int lane) {
    constexpr int P = Fmt<Q27_KV_F16>::PITCH;
    const int g = lane >> 2;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8, col = (lane >> 4) * 8;
        const uint32_t base = ks + row * P + col * 2;
#pragma unroll
        for (int s = 0; s < 16; s++) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4(base + s * 32, a0, a1, a2, a3);
            mma16816(d, a0, a1, a2, a3, qf[s][0], qf[s][1]);
        }
    }
    float sv[4], p[4];
    sv[0] = g < valid ? d[0] * sc2 : -INFINITY;
    sv[1] = g < valid ? d[1] * sc2 : -INFINITY;
    sv[2] = g + 8 < valid ? d[2] * sc2 : -INFINITY;
    sv[3] = g + 8 < valid ? d[3] * sc2 : -INFINITY;
    softmax_tile(A, sv, p);
    const uint32_t b0 = movmatrix_t(pack_h2(p[0], p[1]));
    const uint32_t b1 = movmatrix_t(pack_h2(p[2], p[3]));
    {
        const int row = (lane & 7) + (lane >> 4) * 8, col = ((lane >> 3) & 1) * 8;
        const uint32_t base = vs + row * P + col * 2;
#pragma unroll
        for (int mt = 0; mt < 16; mt++) {
            uint32_t a0, a1, a2, a3;
            ldsm_x4_t(base + mt * 32, a0, a1, a2, a3);
            mma16816(A.o[mt], a0, a1, a2, a3, b0, b1);
        }
    }
}

__device__ __forceinline__ uint32_t e4m3x2_to_h2(uint32_t two_bytes) {
    __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two_bytes, __NV_E4M3);
    return (uint32_t)h.x | ((uint32_t)h.y << 16);
}

__device__ __forceinline__ void tile_fp8(WarpAcc& A, uint32_t ks, uint32_t vs,
                                         const uint32_t (&qf)[16][2], int valid, float sc2,
                                         int lane) {
    constexpr int P = Fmt<Q27_KV_FP8>::PITCH;
    const int g = lane >> 2, c = lane & 3;
    const int r0 = keyperm<Q27_KV_FP8>(g), r1 = keyperm<Q27_KV_FP8>(g + 8);
    float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint4 x = lds128(ks + r0 * P + 16 * (c + 4 * j));
        const uint4 y = lds128(ks + r1 * P + 16 * (c + 4 * j));
        const uint32_t xw[4] = {x.x, x.y, x.z, x.w}, yw[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int s = 4 * j + i;
            mma16816(d, e4m3x2_to_h2(xw[i] & 0xffffu), e4m3x2_to_h2(yw[i] & 0xffffu),
                     e4m3x2_to_h2(xw[i] >> 16), e4m3x2_to_h2(yw[i] >> 16), qf[s][0], qf[s][1]);
        }
    }
    float sv[4], p[4];
    sv[0] = r0 < valid ? d[0] * sc2 : -INFINITY;
    sv[1] = r0 < valid ? d[1] * sc2 : -INFINITY;
    sv[2] = r1 < valid ? d[2] * sc2 : -INFINITY;
    sv[3] = r1 < valid ? d[3] * sc2 : -INFINITY;
    softmax_tile(A, sv, p);
    const uint32_t b0 = movmatrix_t(pack_h2(p[0], p[1]));
    const uint32_t b1 = movmatrix_t(pack_h2(p[2], p[3]));
    // V: this thread's four keys are c, c+4, c+8, c+12; dims: two 16-byte chunks by g
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
        const int ch = 4 * (g & 1) + (g >> 1) + 8 * hh;
        const uint4 k0 = lds128(vs + (c) * P + 16 * ch);
        const uint4 k1 = lds128(vs + (c + 4) * P + 16 * ch);
        const uint4 k2 = lds128(vs + (c + 8) * P + 16 * ch);
        const uint4 k3 = lds128(vs + (c + 12) * P + 16 * ch);
        const uint32_t w0[4] = {k0.x, k0.y, k0.z, k0.w}, w1[4] = {k1.x, k1.y, k1.z, k1.w};
        const uint32_t w2[4] = {k2.x, k2.y, k2.z, k2.w}, w3[4] = {k3.x, k3.y, k3.z, k3.w};
#pragma unroll
        for (int m8 = 0; m8 < 8; m8++) {
            // dims u = 2*m8, 2*m8+1 of this chunk: bytes (2*m8 & 3), +1 of word m8 >> 1
            const uint32_t sel = (m8 & 1) ? 0x7362u : 0x5140u;
            const uint32_t x01 = prmt(w0[m8 >> 1], w1[m8 >> 1], sel); // (k0[u],k1[u],k0[u+1],k1[u+1])
            const uint32_t x23 = prmt(w2[m8 >> 1], w3[m8 >> 1], sel);
            mma16816(A.o[8 * hh + m8], e4m3x2_to_h2(x01 & 0xffffu), e4m3x2_to_h2(x01 >> 16),
                     e4m3x2_to_h2(x23 & 0xffffu), e4m3x2_to_h2(x23 >> 16), b0, b1);
        }
    }
}

// turbo3, one 16-key tile, K side: centroid dot products per 128-dim block recombined with the
// block norms; s[4] = scores in the log2 domain for rows g, g+8 and columns 2c, 2c+1
// (masked rows -inf).
__device__ __forceinline__ void t3_scores(uint32_t ks, int kvh, const uint32_t (&qf)[16][2],
                                          int valid, float sc2, int lane, const T3Tab& tab,
                                          float (&sv)[4]) {
    constexpr int P = Fmt<Q27_KV_T3>::PITCH;
    const int g = lane >> 2, c = lane & 3;
    float dk[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const uint32_t kr0 = ks + g * P + kvh * 100;
    const uint32_t kr1 = kr0 + 8 * P;
#pragma unroll
    for (int b = 0; b < 2; b++) {
        // block b starts at +50b: 4-byte aligned for b == 1, 2 mod 4 for b == 0; qs at +2,
        // signs at +34
        const bool al = (b == 1);
        const uint32_t q0 = kr0 + 50 * b + 2 + 8 * c;
        const uint32_t q1 = kr1 + 50 * b + 2 + 8 * c;
        const uint32_t s0 = lds32_a2(kr0 + 50 * b + 34 + 4 * c, al);
        const uint32_t s1 = lds32_a2(kr1 + 50 * b + 34 + 4 * c, al);
#pragma unroll
        for (int w = 0; w < 2; w++) {
            uint32_t ze0, zo0, ze1, zo1, h0[8], h1[8];
            t3_selectors(lds32_a2(q0 + 4 * w, al), w ? s0 >> 16 : s0 & 0xffffu, ze0, zo0);
            t3_selectors(lds32_a2(q1 + 4 * w, al), w ? s1 >> 16 : s1 & 0xffffu, ze1, zo1);
            t3_lookup(tab, ze0, h0);
            t3_lookup(tab, zo0, h0 + 4);
            t3_lookup(tab, ze1, h1);
            t3_lookup(tab, zo1, h1 + 4);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int s = 8 * b + 4 * w + i;
                mma16816(dk[b], h0[2 * i], h1[2 * i], h0[2 * i + 1], h1[2 * i + 1], qf[s][0],
                         qf[s][1]);
            }
        }
    }
    const float nk00 = lds_half(kr0), nk01 = lds_half(kr0 + 50);
    const float nk10 = lds_half(kr1), nk11 = lds_half(kr1 + 50);
    sv[0] = g < valid ? (dk[0][0] * nk00 + dk[1][0] * nk01) * sc2 : -INFINITY;
    sv[1] = g < valid ? (dk[0][1] * nk00 + dk[1][1] * nk01) * sc2 : -INFINITY;
    sv[2] = g + 8 < valid ? (dk[0][2] * nk10 + dk[1][2] * nk11) * sc2 : -INFINITY;
    sv[3] = g + 8 < valid ? (dk[0][3] * nk10 + dk[1][3] * nk11) * sc2 : -INFINITY;
}

// turbo3, one 16-key tile, V side: O^T += V^T . P^T with the V norms folded into P.
__device__ __forceinline__ void t3_values(float (&o)[16][4], uint32_t vs, int kvh,
                                          const float (&p)[4], int valid, int lane,
                                          const T3Tab& tab) {
    constexpr int P = Fmt<Q27_KV_T3>::PITCH;
    const int g = lane >> 2, c = lane & 3;
    const uint32_t vr0 = vs + g * P + kvh * 100;
    const uint32_t vr1 = vr0 + 8 * P;
    uint32_t pb[2][2]; // [block][key half] P^T fragments with the V norm folded in
#pragma unroll
    for (int b = 0; b < 2; b++) {
        // masked rows may hold stale bytes: keep their weight an exact zero
        const float n0 = g < valid ? lds_half(vr0 + 50 * b) : 0.f;
        const float n1 = g + 8 < valid ? lds_half(vr1 + 50 * b) : 0.f;
        pb[b][0] = movmatrix_t(pack_h2(p[0] * n0, p[1] * n0));
        pb[b][1] = movmatrix_t(pack_h2(p[2] * n1, p[3] * n1));
    }
    // this thread's keys are 2c, 2c+1 (pair 0) and 2c+8, 2c+9 (pair 1); its dims are
    // [16g, 16g+16) of each block: one qs word + 16 sign bits per (key, block)
#pragma unroll
    for (int b = 0; b < 2; b++) {
        const bool al = (b == 1);
        uint32_t ze[4], zo[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int key = 2 * c + (k & 1) + 8 * (k >> 1);
            const uint32_t blk = vs + key * P + kvh * 100 + 50 * b;
            t3_selectors(lds32_a2(blk + 2 + 4 * g, al), lds16(blk + 34 + 2 * g), ze[k], zo[k]);
        }
        uint32_t hp[2][16]; // [pair][dim order] half2 = (key A, key B) of one dim
#pragma unroll
        for (int pr = 0; pr < 2; pr++) {
            const uint32_t ea = ze[2 * pr], eb = ze[2 * pr + 1], oa = zo[2 * pr], ob = zo[2 * pr + 1];
            const uint32_t ze_lo = (ea & 0x0F0F0F0Fu) | ((eb << 4) & 0xF0F0F0F0u);
            const uint32_t ze_hi = ((ea >> 4) & 0x0F0F0F0Fu) | (eb & 0xF0F0F0F0u);
            const uint32_t zo_lo = (oa & 0x0F0F0F0Fu) | ((ob << 4) & 0xF0F0F0F0u);
            const uint32_t zo_hi = ((oa >> 4) & 0x0F0F0F0Fu) | (ob & 0xF0F0F0F0u);
            t3_lookup(tab, ze_lo, hp[pr]);       // dims e16 = 0, 4, 8, 12
            t3_lookup(tab, ze_hi, hp[pr] + 4);   // 2, 6, 10, 14
            t3_lookup(tab, zo_lo, hp[pr] + 8);   // 1, 5, 9, 13
            t3_lookup(tab, zo_hi, hp[pr] + 12);  // 3, 7, 11, 15
        }
#pragma unroll
        for (int j = 0; j < 8; j++)
            mma16816(o[8 * b + j], hp[0][2 * j], hp[0][2 * j + 1], hp[1][2 * j],
                     hp[1][2 * j + 1], pb[b][0], pb[b][1]);
    }
}

// turbo3: both 16-key tiles of a ring stage at once. rows = real keys among the 32 (1..32);
// a missing second tile costs nothing.
__device__ __forceinline__ void stage_t3(WarpAcc& A, uint32_t ks, uint32_t vs, int kvh,
                                         const uint32_t (&qf)[16][2], int rows, float sc2,
                                         int lane, const T3Tab& tab) {
    constexpr int P = Fmt<Q27_KV_T3>::PITCH;
    float s0[4], s1[4], p0[4], p1[4];
    if (rows > TILE) {
        t3_scores(ks, kvh, qf, TILE, sc2, lane, tab, s0);
        t3_scores(ks + TILE * P, kvh, qf, rows - TILE, sc2, lane, tab, s1);
        softmax_pair(A, s0, s1, p0, p1);
        t3_values(A.o, vs, kvh, p0, TILE, lane, tab);
        t3_values(A.o, vs + TILE * P, kvh, p1, rows - TILE, lane, tab);
    } else {
        t3_scores(ks, kvh, qf, rows, sc2, lane, tab, s0);
        softmax_tile(A, s0, p0);
        t3_values(A.o, vs, kvh, p0, rows, lane, tab);
    }
}

// ---- the kernel -------------------------------------------------------------------------
// FUSE: the variant that also finishes the launch (b.fuse is set for it and only for it); the
// plain variant does not carry that code.
template <int KVK, bool FUSE>
__global__ void __launch_bounds__(n_threads<KVK>(), 1)
k_decode_mma(const __grid_constant__ DevBatch b) {
    using F = Fmt<KVK>;
    constexpr int NCW = F::NCW;
    constexpr int WAYS = NCW / F::KVH;             // consumer warps per kv head
    constexpr int NHEADS = F::KVH * GQA;           // query heads this CTA serves
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + 16;
    uint8_t* ring = smem + HEADER_BYTES;
    float* q_stage = reinterpret_cast<float*>(ring + work_bytes<KVK>());
    constexpr int QP = q_pitch<KVK>();
    __shared__ int s_fail, s_grp_ok;
    __shared__ float s_fin[FUSE ? FINISH_SMEM_FLOATS : 1];
    __shared__ float s_wt[NHEADS][WAYS], s_mb[NHEADS], s_lb[NHEADS];

    pdl_trigger();               // a combine kernel may be scheduled; it waits for this grid
    const int t = blockIdx.x, sp = blockIdx.y;
    const int groups = b.n_kv / F::KVH;
    const int slot = blockIdx.z / groups, kvg = blockIdx.z % groups;
    const DevSlot& S = b.s[slot];
    if (t >= S.ntok) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    unsigned long long* ticket = nullptr;
    if (FUSE) {
        // the two counters of this (lane, kv group) -- arrivals, departures -- behind the last
        // split's partials in the slot's scratch (nsplit <= 127 of the 128 splits the scratch
        // has room for); words that do not carry the tag yet (first use of this scratch, or
        // partials of a call with more splits written over them) are armed here, long before
        // anybody arrives on them
        ticket = group_counters(S.scratch, S.ntok, b.n_q, b.nsplit, t * groups + kvg);
        if (threadIdx.x == 0) group_arm(ticket);
    }
    int max_len = 0;
    for (int u = 0; u < S.ntok; u++)
        max_len = max(max_len, local_len(__ldg(S.pos[u]), S.row_base, S.row_count));
    const int my_len = local_len(__ldg(S.pos[t]), S.row_base, S.row_count);
    const int chunk = split_chunk(max_len, b.nsplit, b.unit);
    const int lo = sp * chunk, hi = min(my_len, lo + chunk);
    const int kvh0 = kvg * F::KVH;
    float* dst0 = S.scratch + (((size_t)t * b.n_q + kvh0 * GQA) * b.nsplit + sp) * PART;

    if (lo >= hi) {
        // empty window: stamp the sentinel so that whoever merges can skip it
        if (threadIdx.x < NHEADS) {
            float* d = dst0 + (size_t)threadIdx.x * b.nsplit * PART;
            d[0] = NEG_SENTINEL;
            d[1] = 0.f;
        }
    } else {
        const int nstages = (hi - lo + STAGE_ROWS - 1) / STAGE_ROWS;
        if (threadIdx.x == 0) {
            s_fail = 0;
            for (int s = 0; s < F::STAGES; s++) {
                mbar_init(&full[s], KVK == Q27_KV_T3 ? 1 : 32);   // tx bytes, or 32 lane arrivals
                mbar_init(&empty[s], NCW);        // every consumer warp releases every stage
            }
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();         // barriers are live: the producer starts while Q is staged

        const float sc2 = b.scale * LOG2E;
        const uint32_t ring_s = smem_u32(ring);
        const int g = lane >> 2, c = lane & 3;
        float* ring_f = reinterpret_cast<float*>(ring);

        if (warp == NCW) {
            // ---------------- producer ----------------
            // page pointers are fetched 32 pages at a time, one per lane, so that no stage
            // waits on a dependent table load
            const int last_page = (hi - 1) >> PAGE_SHIFT;
            const void* kpl = nullptr;
            const void* vpl = nullptr;
            int pbase = INT_MIN / 2;
            int issued = 0;
            for (int i = 0; i < nstages; i++) {
                const int s = i % F::STAGES;
                const uint32_t ph = (uint32_t)((i / F::STAGES) & 1);
                const int row0 = lo + i * STAGE_ROWS;
                const int pg = row0 >> PAGE_SHIFT;
                if (pg - pbase >= 32) {
                    pbase = pg;
                    if (pg + lane <= last_page) {
                        kpl = S.ktab[pg + lane];
                        vpl = S.vtab[pg + lane];
                    }
                }
                const uint8_t* kpage = static_cast<const uint8_t*>(shfl_ptr(kpl, pg - pbase));
                const uint8_t* vpage = static_cast<const uint8_t*>(shfl_ptr(vpl, pg - pbase));
                if (i >= F::STAGES && !mbar_wait(&empty[s], ph ^ 1)) { s_fail = 1; break; }
                const int nrows = min(STAGE_ROWS, hi - row0);
                uint8_t* kdst = ring + (size_t)s * stage_bytes<KVK>();
                uint8_t* vdst = kdst + STAGE_ROWS * F::PITCH;
                if (KVK == Q27_KV_T3) {
                    if (lane == 0) {
                        const uint32_t bytes = (uint32_t)nrows * F::SLICE;
                        const size_t off = (size_t)(row0 & (PAGE - 1)) * F::SLICE;
                        mbar_expect_tx(&full[s], 2 * bytes);
                        bulk_g2s(kdst, kpage + off, bytes, &full[s]);
                        bulk_g2s(vdst, vpage + off, bytes, &full[s]);
                    }
                } else {
                    // fp16 / fp8: the rows of one kv head are 512 / 256-byte slices 2048 / 1024 B
                    // apart, and each goes to a padded pitch, so there is no single large copy.
                    // One bulk copy per slice is bound by the copy rate (about one per 70 cycles:
                    // a third of the HBM rate at 131K rows); 16-byte asynchronous copies by the
                    // whole warp are not. Each lane's arrival is counted when its copies land.
                    constexpr int CPR = F::SLICE / 16;        // 16-byte chunks per row slice
                    constexpr int RPI = 32 / CPR;             // row slices per warp instruction
                    const size_t off = ((size_t)(row0 & (PAGE - 1)) * b.n_kv + kvh0) * F::SLICE;
                    const uint8_t* kp = kpage + off;
                    const uint8_t* vp = vpage + off;
                    const int c16 = (lane % CPR) * 16;
                    for (int r = lane / CPR; r < nrows; r += RPI) {
                        const size_t src = (size_t)r * b.n_kv * F::SLICE + c16;
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                                     ::"r"(smem_u32(kdst + r * F::PITCH + c16)), "l"(kp + src) : "memory");
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                                     ::"r"(smem_u32(vdst + r * F::PITCH + c16)), "l"(vp + src) : "memory");
                    }
                    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];"
                                 ::"r"(smem_u32(&full[s])) : "memory");
                }
                issued = i + 1;
            }
            // No copy may still be in flight when the CTA hands its shared memory back (or reuses
            // it below), also when a consumer gave up early: wait, bounded, for what was issued.
            if (KVK != Q27_KV_T3) {
                asm volatile("cp.async.wait_all;" ::: "memory");
            } else {
                for (int i = max(0, issued - F::STAGES); i < issued; i++)
                    if (!mbar_wait(&full[i % F::STAGES], (uint32_t)((i / F::STAGES) & 1))) s_fail = 1;
            }
        } else {
            // ---------------- consumers ----------------
            const int ctid = threadIdx.x;         // 0 .. NCW*32-1
            // the CTA's query heads, fp32, staged once with coalesced loads, all of a thread's
            // loads in flight together (one after the other they cost a trip to L2 each: 4 us for
            // the 24 heads of a turbo3 CTA)
            {
                constexpr int NQ4 = NHEADS * (HD / 4);
                constexpr int QL = (NQ4 + NCW * 32 - 1) / (NCW * 32);
                float4 qv[QL];
#pragma unroll
                for (int u = 0; u < QL; u++) {
                    const int i = ctid + u * NCW * 32;
                    const int h = min(i, NQ4 - 1) / (HD / 4), d4 = i % (HD / 4);
                    qv[u] = __ldg(reinterpret_cast<const float4*>(S.q[t] + (size_t)(kvh0 * GQA + h) * b.q_stride) + d4);
                }
#pragma unroll
                for (int u = 0; u < QL; u++) {
                    const int i = ctid + u * NCW * 32;
                    if (i < NQ4) {
                        float* dst = q_stage + (i / (HD / 4)) * QP + q_at<KVK>((i % (HD / 4)) * 4);
                        if constexpr (KVK == Q27_KV_T3) {     // the skew leaves the row 4-byte aligned
                            dst[0] = qv[u].x; dst[1] = qv[u].y; dst[2] = qv[u].z; dst[3] = qv[u].w;
                        } else {
                            *reinterpret_cast<float4*>(dst) = qv[u];
                        }
                    }
                }
            }
            if (b.wht & WHT_Q) {
                // the forward rotation of wht3 (src/spec3.cu:595-614) on the staged heads, a
                // 128-group per warp at a time, while the producer is already filling the ring
                asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32));
                for (int gi = warp; gi < NHEADS * 2; gi += NCW)
                    wht_group<false, KVK == Q27_KV_T3 ? Q_SKEW_T3 : 0>(q_stage + (gi >> 1) * QP + q_at<KVK>((gi & 1) * 128), lane);
            }
            // Rows past the end of a ragged last stage are never copied; their weights are exact
            // zeros, so what the ring holds there only has to decode to finite numbers. Any
            // turbo3 byte pattern decodes to a centroid (its norms are masked). fp16 / fp8
            // patterns may be NaN or Inf: if the last stage's slot was never filled before, the
            // rows the copies will not touch are cleared (bytes the copies do not write).
            if (KVK != Q27_KV_T3 && nstages <= F::STAGES) {
                const int il = nstages - 1, nlast = hi - lo - il * STAGE_ROWS;
                uint8_t* kdst = ring + (size_t)(il % F::STAGES) * stage_bytes<KVK>();
                const int per_row = F::PITCH / 16;
                for (int i = ctid; i < (STAGE_ROWS - nlast) * per_row * 2; i += NCW * 32) {
                    const int side = i / ((STAGE_ROWS - nlast) * per_row);
                    const int j = i % ((STAGE_ROWS - nlast) * per_row);
                    reinterpret_cast<uint4*>(kdst + side * STAGE_ROWS * F::PITCH +
                                             (size_t)(nlast + j / per_row) * F::PITCH)[j % per_row] =
                        make_uint4(0, 0, 0, 0);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32));

            const int hq = warp % F::KVH, way = warp / F::KVH;
            // Q^T fragments: column n = g is head (kvh0 + hq)*6 + g (columns 6, 7 are zero padding)
            uint32_t qf[16][2];
            {
                // padding columns read what a live lane of their half-warp reads (a broadcast)
                const float* qh = q_stage + (size_t)(hq * GQA + (g < GQA ? g : g - 2)) * QP;
#pragma unroll
                for (int s = 0; s < 16; s++)
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        float x0, x1;
                        if constexpr (KVK == Q27_KV_T3) {
                            x0 = qh[q_at<KVK>(kdim<KVK>(s, c, r, 0))];
                            x1 = qh[q_at<KVK>(kdim<KVK>(s, c, r, 1))];
                        } else {            // the two elements of a register are neighbours
                            const float2 x = *reinterpret_cast<const float2*>(qh + kdim<KVK>(s, c, r, 0));
                            x0 = x.x;
                            x1 = x.y;
                        }
                        qf[s][r] = g < GQA ? pack_h2(x0, x1) : 0u;
                    }
            }
            WarpAcc A;
#pragma unroll
            for (int mt = 0; mt < 16; mt++) A.o[mt][0] = A.o[mt][1] = A.o[mt][2] = A.o[mt][3] = 0.f;
            A.m[0] = A.m[1] = -INFINITY;
            A.l[0] = A.l[1] = 0.f;
            const T3Tab tab = t3_tables();
            (void)tab;
            const int ntiles = (hi - lo + TILE - 1) / TILE;
            // Every consumer warp observes every phase of every ring slot, in order (waits on
            // `full`, arrives on `empty`), whether or not it owns a tile of that stage: a warp
            // that skipped phases could not tell them apart by parity.
            for (int i = 0; i < nstages; i++) {
                const int s = i % F::STAGES;
                const uint32_t ph = (uint32_t)((i / F::STAGES) & 1);
                if (!mbar_wait(&full[s], ph)) { s_fail = 1; break; }
                if (KVK == Q27_KV_T3) {
                    if (i % WAYS == way) {
                        const uint32_t ks = ring_s + s * stage_bytes<KVK>();
                        stage_t3(A, ks, ks + STAGE_ROWS * F::PITCH, hq, qf,
                                 min(STAGE_ROWS, hi - lo - i * STAGE_ROWS), sc2, lane, tab);
                    }
                } else {
#pragma unroll
                    for (int half = 0; half < 2; half++) {
                        const int tile = 2 * i + half;
                        if (i % WAYS == way && tile < ntiles) {
                            const int valid = min(TILE, hi - lo - tile * TILE);
                            const uint32_t ks = ring_s + s * stage_bytes<KVK>() + half * TILE * F::PITCH;
                            const uint32_t vs = ks + STAGE_ROWS * F::PITCH;
                            if (KVK == Q27_KV_F16) tile_f16<KVK>(A, ks, vs, qf, valid, sc2, lane);
                            else tile_fp8(A, ks, vs, qf, valid, sc2, lane);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
            }
            // every consumer is past its last ring read once all of them reach this barrier
            asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32));
            // column sums: add the shares of the 8 threads of a column group
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                A.l[0] += __shfl_xor_sync(0xffffffffu, A.l[0], off);
                A.l[1] += __shfl_xor_sync(0xffffffffu, A.l[1], off);
            }
            // per-warp partial [head j][258] into the (now idle) ring; natural-log domain for m
            float* wp = ring_f + (size_t)warp * GQA * PART;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int j = 2 * c + e;
                if (j < GQA) {
                    if (g == 0) {
                        wp[j * PART] = A.m[e] == -INFINITY ? NEG_SENTINEL : A.m[e] * LN2;
                        wp[j * PART + 1] = A.l[e];
                    }
#pragma unroll
                    for (int mt = 0; mt < 16; mt++) {
                        wp[j * PART + 2 + vdim<KVK>(mt, g)] = A.o[mt][e];
                        wp[j * PART + 2 + vdim<KVK>(mt, g + 8)] = A.o[mt][2 + e];
                    }
                }
            }
            asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32));
            // Merge the WAYS partial sets of each head in a fixed order. One thread per head
            // forms the weights e^{m_w - M} once; then every thread owns one dim of all heads.
            // A CTA that gave up on a wait publishes empty partials instead.
            const bool failed = s_fail != 0;
            if (ctid < NHEADS) {
                const int h = ctid / GQA, j = ctid % GQA;
                const float* src = ring_f + (size_t)h * GQA * PART + j * PART;
                float mb = NEG_SENTINEL;
#pragma unroll
                for (int w = 0; w < WAYS; w++) mb = fmaxf(mb, src[(size_t)w * NHEADS * PART]);
                float lb = 0.f;
#pragma unroll
                for (int w = 0; w < WAYS; w++) {
                    const float* pw = src + (size_t)w * NHEADS * PART;
                    const float e = pw[0] == NEG_SENTINEL ? 0.f : expf(pw[0] - mb);
                    s_wt[ctid][w] = e;
                    lb += pw[1] * e;
                }
                s_mb[ctid] = failed ? NEG_SENTINEL : mb;
                s_lb[ctid] = failed ? 0.f : lb;
            }
            asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32));
            if (ctid < HD) {
#pragma unroll 6
                for (int hj = 0; hj < NHEADS; hj++) {
                    const float* src = ring_f + (size_t)(hj / GQA) * GQA * PART + (hj % GQA) * PART;
                    float acc = 0.f, v[WAYS];
#pragma unroll
                    for (int w = 0; w < WAYS; w++) v[w] = src[(size_t)w * NHEADS * PART + 2 + ctid];
#pragma unroll
                    for (int w = 0; w < WAYS; w++) {
                        // a set that saw no key has weight 0: selected, never added
                        const float e = s_wt[hj][w], x = v[w] * e;
                        acc += e != 0.f ? x : 0.f;
                    }
                    float* d = dst0 + (size_t)hj * b.nsplit * PART;
                    if (ctid == 0) { d[0] = s_mb[hj]; d[1] = s_lb[hj]; }
                    d[2 + ctid] = acc;
                }
            }
        }
        __syncthreads();         // the producer has drained: shared memory is quiet from here on
    }

    if (FUSE) {
        // Every CTA of this (slot, lane, kv group) waits for the group's partials (the launch is
        // cooperative: all CTAs are resident), merges its share of the group's outputs and
        // leaves; the last one to leave clears the counters for the next launch.
        const unsigned n = (unsigned)b.nsplit;
        __syncthreads();                          // this CTA's partial rows are written
        if (threadIdx.x == 0) {
            const bool ok = group_wait(ticket, n);
            if (!ok) atomicExch(&g_wait_timeout_flag, 1);
            s_grp_ok = ok ? 1 : 0;
        }
        __syncthreads();
        if (s_grp_ok) {
            // CTA `sp` of `n` takes the half heads sp, sp + n, ... of the group's 2 NHEADS
            const int used = min(b.nsplit, (max_len + chunk - 1) / chunk);
            const float* base = S.scratch + ((size_t)t * b.n_q + kvh0 * GQA) * b.nsplit * PART;
            for (int g = sp; g < 2 * NHEADS; g += (int)n)
                merge_half_head(base + (size_t)(g >> 1) * b.nsplit * PART, used, g & 1,
                                S.out[t] + (size_t)(kvh0 * GQA + (g >> 1)) * HD + (g & 1) * 128, b.wht, s_fin);
        }
        __syncthreads();
        if (threadIdx.x == 0) group_leave(ticket, n);
    }
}

template <int KVK>
int launch_one(DevBatch& b, int sm_count, bool may_fuse, cudaStream_t st) {
    using F = Fmt<KVK>;
    static DeviceOnce once;      // the attribute belongs to a device, not to the process
    int rc = device_once(once, []() -> int {
        Q27_CUDA_TRY(cudaFuncSetAttribute(k_decode_mma<KVK, false>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          smem_bytes<KVK>()));
        Q27_CUDA_TRY(cudaFuncSetAttribute(k_decode_mma<KVK, true>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          smem_bytes<KVK>()));
        return Q27_OK;
    });
    if (rc) return rc;
    const int groups = b.n_kv / F::KVH;
    const int per_split = b.nslots * b.max_ntok * groups;
    int ns = sm_count / per_split;
    ns = ns < 1 ? 1 : ns > Q27_MAX_SPLITS ? Q27_MAX_SPLITS : ns;
    // The launch finishes in this kernel when nobody else wants the partials: the CTAs of a
    // (slot, lane, kv group) wait for one another and share the merge of the group's outputs
    // (and the un-rotation of the output, if asked). The counters sit behind the last split's
    // partials in the scratch.
    b.fuse = 0;
    if (may_fuse && ns <= FUSE_MAX_SPLITS && F::KVH * GQA * ns * PART * 4 <= FUSE_MAX_BYTES) {
        b.fuse = 1;
        for (int i = 0; i < b.nslots; i++)
            if ((uintptr_t)b.s[i].scratch & 7) b.fuse = 0;    // 64-bit counters in the scratch
    }
    b.nsplit = ns;
    b.unit = STAGE_ROWS;
    dim3 grid(b.max_ntok, b.nsplit, b.nslots * groups);
    if (b.fuse) {
        // the CTAs of a group wait for one another: a cooperative launch, which the runtime
        // refuses unless every CTA can be resident at once
        void* args[] = {const_cast<DevBatch*>(&b)};
        const cudaError_t e = cudaLaunchCooperativeKernel(
            reinterpret_cast<const void*>(&k_decode_mma<KVK, true>), grid, dim3(n_threads<KVK>()), args,
            smem_bytes<KVK>(), st);
        if (e == cudaSuccess) {
            Q27_COUNT_LAUNCH();
            return Q27_OK;
        }
        (void)cudaGetLastError();                 // not launchable that way here: two launches
        b.fuse = 0;
    }
    k_decode_mma<KVK, false><<<grid, n_threads<KVK>(), smem_bytes<KVK>(), st>>>(b);
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

} // namespace

int launch_decode_mma(DevBatch& b, int kvk, int sm_count, bool may_fuse, cudaStream_t st,
                      bool* done) {
    *done = false;
    if (kind_known(kvk) && !kind_has_tensor_path(kvk)) return Q27_OK;   // served by the fp32 family
    b.fuse = 0;
    if (b.n_kv != 4) return Q27_OK; // the ring layouts assume 4 kv heads per row
    if (b.q_stride & 3) return Q27_OK; // Q heads are staged with 16-byte loads
    for (int i = 0; i < b.nslots; i++)
        for (int t = 0; t < b.s[i].ntok; t++)
            if ((uintptr_t)b.s[i].q[t] & 15) return Q27_OK;
    int rc;
    if (kvk == Q27_KV_F16) rc = launch_one<Q27_KV_F16>(b, sm_count, may_fuse, st);
    else if (kvk == Q27_KV_FP8) rc = launch_one<Q27_KV_FP8>(b, sm_count, may_fuse, st);
    else if (kvk == Q27_KV_T3) rc = launch_one<Q27_KV_T3>(b, sm_count, may_fuse, st);
    else return Q27_ERR_UNSUPPORTED_KIND;
    if (rc == Q27_OK) *done = true;
    return rc;
}

int read_wait_timeout_flag(int* out) {
    Q27_CUDA_TRY(cudaMemcpyFromSymbol(out, g_wait_timeout_flag, sizeof(int)));
    return Q27_OK;
}

} // namespace q27b
