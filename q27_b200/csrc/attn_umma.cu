// Attention on the 5th-generation tensor cores (tcgen05.mma, accumulators in tensor memory).
//
// One CTA = one Q tile of up to 128 rows against a range of cache rows of ONE kv head. The
// rows of the tile are (token, GQA head) pairs -- 21 tokens x 6 heads for prefill, ntok lanes
// x 6 heads for verify -- so every K/V tile that is staged serves all six heads (and, for
// verify, all draft lanes: one pass over the cache). Each row carries its own causal bound.
//
//   S  = Q . K^T   M=128 rows, N=64 keys, K=256 dims     -> TMEM (two S buffers)
//   O += P . V     M=128 rows, N=256 dims, K=64 keys      -> TMEM (256 columns)
//
// Operands are fp16 in shared memory in the 128-byte-swizzled canonical layouts (Q and K
// K-major, V MN-major = its natural [key][dim] rows, P K-major), accumulation is fp32.
// Warp roles: warps 0-3 softmax (thread = row = TMEM lane); warp 4 issues the S MMAs and warp 5
// the PV MMAs (two independent issue streams, ordered only by mbarriers); warps 6-13 stage
// K/V tiles (cp.async for fp16 rows, registers + convert for fp8 / turbo3). The running
// max is only advanced when it grows by more than 2^8, so O in TMEM is rarely rescaled.
// Every mbarrier wait is bounded; a timeout sets the library's flag and the CTA drains.
#include "attn_umma.cuh"
#include "t3_lut.cuh"

namespace q27b {

extern __device__ int g_wait_timeout_flag;
#ifdef Q27_TRACE
// timing experiments only: cycles spent waiting, summed over CTAs, by (role, barrier)
__device__ unsigned long long g_umma_trace[16];
__device__ long long g_umma_ev[8][64];   // per-event timestamps of CTA (0,0,0), first 64 tiles
#define TRACE_EV(e, i) do { if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && (i) < 64) g_umma_ev[e][i] = clock64(); } while (0)
#define TRACE_T0() const long long t0__ = clock64()
#define TRACE_ADD(slot, cond) do { if (cond) atomicAdd(&g_umma_trace[slot], (unsigned long long)(clock64() - t0__)); } while (0)
#else
#define TRACE_T0()
#define TRACE_ADD(slot, cond)
#define TRACE_EV(e, i)
#endif

namespace {

constexpr int BM = 128;                 // Q rows per CTA (TMEM lanes)
constexpr int BN = 64;                  // keys per tile = one cache page
constexpr int TOK_PER_TILE = 21;        // 21 tokens x 6 heads = 126 rows
constexpr int KV_STAGES = 3;
constexpr int Q_BYTES = BM * HD * 2;            // 65536: 4 blocks of [128 rows][128 B]
constexpr int KT_BYTES = BN * HD * 2;           // 32768: 4 blocks of [64 rows][128 B]
constexpr int P_BYTES = BM * BN * 2;            // 16384: 1 block of [128 rows][128 B]
constexpr int STAGE_BYTES = 2 * KT_BYTES;       // K then V
constexpr int SMEM_BAR = 1024;                  // barriers + tmem slot, keeps tiles 1024-aligned
constexpr int UMMA_SMEM = SMEM_BAR + KV_STAGES * STAGE_BYTES + 1024;
constexpr int TMEM_COLS = 512;
// TMEM columns: two S buffers, O, and the Q tile itself (fp16 pairs, 8 columns per k-step):
// Q is the A operand of every S MMA, so keeping it in tensor memory takes its re-reads off
// the shared-memory port and leaves room for a third K/V stage
constexpr int COL_S0 = 0, COL_S1 = 64, COL_O = 128, COL_Q = 384;
constexpr float LOG2E_F = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;       // log2 units

constexpr int N_SOFTMAX_WARPS = 4, MMA_WARP = 4, PV_WARP = 5, FIRST_LOAD_WARP = 6, N_LOAD_WARPS = 8;
constexpr int UMMA_THREADS = (FIRST_LOAD_WARP + N_LOAD_WARPS) * 32;   // 448
constexpr int NPROD = N_LOAD_WARPS * 32;                              // 256 staging threads

// ---- small PTX wrappers -------------------------------------------------------------------
__device__ __forceinline__ uint32_t s32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void bar_init(uint32_t bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void bar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool bar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < (1 << 20); i++) {
        if (bar_try(bar, parity)) return true;
        if (i > 2048) __nanosleep(64);
    }
    atomicExch(&g_wait_timeout_flag, 2);
    return false;
}
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(bar) : "memory");
}
// A operand taken from tensor memory (row = lane, 16 fp16 of K per 8 columns)
__device__ __forceinline__ void tc_mma_f16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tc_ld32(uint32_t taddr, float* v) {
    uint32_t* r = reinterpret_cast<uint32_t*>(v);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,"
        "%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr) : "memory");
}
__device__ __forceinline__ void tc_st32(uint32_t taddr, const float* v) {
    const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,"
        "%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
          "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
          "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]),
          "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
          "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), descriptor version 1.
// lbo / sbo in bytes (see the canonical layouts in the header comment of make_desc users).
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
// Instruction descriptor, kind::f16: D fp32, A/B fp16, M x N, B optionally MN-major.
constexpr uint32_t make_idesc(int M, int N, bool b_mn_major) {
    return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}
// byte offset of (row, 16-byte chunk 0..7) inside a [rows][128 B] block, 128-byte swizzle
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
    return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ---- what a CTA works on -----------------------------------------------------------------
struct TileArgs {
    // prefill (mode 0)
    const float* qT;
    const void* const* ktab;
    const void* const* vtab;
    float* outT;
    int q_stride, q_row, out_row;
    int base_pos, t0, t_end;
    int n_kv;
    float scale;
};

struct RowInfo {        // one Q row of the tile, owned by one softmax thread
    const float* q;     // 256 floats, or nullptr for a padding row
    int bound;          // keys [0, bound) of the tables are visible to this row
    float* out;         // prefill: 256 normalised floats
    float* part;        // verify: {m, l, acc[256]} of this split
};

// MODE 0: prefill tile (TileArgs). MODE 1: verify, all lanes of one slot (DevBatch).
template <int MODE>
struct Problem {
    const TileArgs* ta;
    const DevBatch* vb;
    const DevSlot* slot;
    int kvh, tile_t0, lo, hi, sp;

    __device__ __forceinline__ RowInfo row(int r) const {
        RowInfo ri{nullptr, 0, nullptr, nullptr};
        const int tok = r / GQA, j = r % GQA;
        if (MODE == 0) {
            const int t = tile_t0 + tok;
            if (tok < TOK_PER_TILE && t < ta->t_end) {
                const int h = kvh * GQA + j;
                ri.q = ta->qT + (size_t)t * ta->q_row + (size_t)h * ta->q_stride;
                ri.bound = ta->base_pos + t + 1;
                ri.out = ta->outT + (size_t)t * ta->out_row + (size_t)h * HD;
            }
        } else {
            if (tok < slot->ntok) {
                const int h = kvh * GQA + j;
                ri.q = slot->q[tok] + (size_t)h * vb->q_stride;
                ri.bound = min(hi, local_len(__ldg(slot->pos[tok]), slot->row_base, slot->row_count));
                ri.part = slot->scratch + (((size_t)tok * vb->n_q + h) * vb->nsplit + sp) * PART;
            }
        }
        return ri;
    }
};

// Staging of one 64-key tile of K and V as fp16 into the swizzled operand layouts, in two
// halves: `load` pulls the raw bytes of the tile into registers (issued before the ring slot
// is free, so the global latency hides behind the tiles in flight), `store` converts and
// writes them once the slot has been released.
template <int KVK> struct RawTile;
template <> struct RawTile<Q27_KV_F16> { uint4 k[8], v[8]; };
template <> struct RawTile<Q27_KV_FP8> { uint2 k[8], v[8]; };
template <> struct RawTile<Q27_KV_T3> { uint32_t w[14]; };

template <int KVK>
__device__ __forceinline__ void tile_load(RawTile<KVK>& t, const uint8_t* kpage, const uint8_t* vpage,
                                          int nkeys, int n_kv, int kvh, int ptid) {
    if constexpr (KVK == Q27_KV_T3) {
        // one thread = one 50-byte block: (key, side, block). Block 1 starts 2 bytes past a
        // word boundary, so 14 words from the aligned address below it cover either block.
        const int key = ptid & 63, side = (ptid >> 6) & 1, blk = ptid >> 7;
#pragma unroll
        for (int i = 0; i < 14; i++) t.w[i] = 0;
        if (key < nkeys) {
            const uint32_t* src = reinterpret_cast<const uint32_t*>(
                (side ? vpage : kpage) + ((size_t)key * n_kv + kvh) * (2 * T3_BLK)) + 12 * blk;
#pragma unroll
            for (int i = 0; i < 13; i++) t.w[i] = __ldg(src + i);
        }
    } else {
        constexpr int CB = KVK == Q27_KV_F16 ? 16 : 8;      // bytes per 8-dim chunk
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const int q = ptid + NPROD * n;
            const int key = q >> 5, ch = q & 31;
            const size_t src = ((size_t)key * n_kv + kvh) * (HD * CB / 8) + (size_t)ch * CB;
            if constexpr (KVK == Q27_KV_F16) {
                t.k[n] = t.v[n] = make_uint4(0, 0, 0, 0);   // rows past the range: exact zeros
                if (key < nkeys) {
                    t.k[n] = __ldg(reinterpret_cast<const uint4*>(kpage + src));
                    t.v[n] = __ldg(reinterpret_cast<const uint4*>(vpage + src));
                }
            } else {
                t.k[n] = t.v[n] = make_uint2(0, 0);
                if (key < nkeys) {
                    t.k[n] = __ldg(reinterpret_cast<const uint2*>(kpage + src));
                    t.v[n] = __ldg(reinterpret_cast<const uint2*>(vpage + src));
                }
            }
        }
    }
}

// WHICH: 0 = the K half of the tile, 1 = the V half
template <int KVK, int WHICH>
__device__ __forceinline__ void tile_store(const RawTile<KVK>& t, uint8_t* dstK, int nkeys, int ptid) {
    uint8_t* dstV = dstK + KT_BYTES;
    if constexpr (KVK == Q27_KV_F16) {
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const int q = ptid + NPROD * n;
            const int key = q >> 5, ch = q & 31;
            const uint32_t off = (uint32_t)(ch >> 3) * (BN * 128) + sw128(key, ch & 7);
            if (WHICH == 0) *reinterpret_cast<uint4*>(dstK + off) = t.k[n];
            else *reinterpret_cast<uint4*>(dstV + off) = t.v[n];
        }
    } else if constexpr (KVK == Q27_KV_FP8) {
#pragma unroll
        for (int n = 0; n < 8; n++) {
            const int q = ptid + NPROD * n;
            const int key = q >> 5, ch = q & 31;
            const uint32_t off = (uint32_t)(ch >> 3) * (BN * 128) + sw128(key, ch & 7);
            auto cv = [](uint32_t two) {
                __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two, __NV_E4M3);
                return (uint32_t)h.x | ((uint32_t)h.y << 16);
            };
            if (WHICH == 0)
                *reinterpret_cast<uint4*>(dstK + off) = make_uint4(
                    cv(t.k[n].x & 0xffffu), cv(t.k[n].x >> 16), cv(t.k[n].y & 0xffffu), cv(t.k[n].y >> 16));
            else
                *reinterpret_cast<uint4*>(dstV + off) = make_uint4(
                    cv(t.v[n].x & 0xffffu), cv(t.v[n].x >> 16), cv(t.v[n].y & 0xffffu), cv(t.v[n].y >> 16));
        }
    } else {
        const int key = ptid & 63, side = (ptid >> 6) & 1, blk = ptid >> 7;
        if (side != WHICH) return;              // warp-uniform: a warp holds one side only
        uint8_t* dst = side ? dstV : dstK;
        const uint32_t* w = t.w;
        const T3Tab tab = t3_tables();
        // 32-bit little-endian word at byte `o` of the block (o even, compile time); block 1
        // sits 2 bytes into the loaded words, block 0 at byte 0 (blk is warp-uniform)
        auto word_at = [&](int o) {
            const uint32_t a0 = (o & 3) ? __funnelshift_r(w[o >> 2], w[(o >> 2) + 1], 16) : w[o >> 2];
            const int o1 = o + 2;
            const uint32_t a1 = (o1 & 3) ? __funnelshift_r(w[o1 >> 2], w[(o1 >> 2) + 1], 16) : w[o1 >> 2];
            return blk ? a1 : a0;
        };
        const __half nh = __ushort_as_half((unsigned short)(word_at(0) & 0xffffu));
        const __half2 n2 = key < nkeys ? __half2half2(nh) : __float2half2_rn(0.f);
#pragma unroll
        for (int g8 = 0; g8 < 8; g8++) {         // 16 dims per group
            const uint32_t Qw = word_at(2 + 4 * g8);
            const uint32_t S16 = (word_at(34 + 2 * (g8 & ~1)) >> (16 * (g8 & 1))) & 0xffffu;
            uint32_t ze, zo, e[4], o[4];
            t3_selectors(Qw, S16, ze, zo);
            t3_lookup(tab, ze, e);                // (0,2) (4,6) (8,10) (12,14)
            t3_lookup(tab, zo, o);                // (1,3) (5,7) (9,11) (13,15)
            uint32_t nat[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                nat[2 * i] = prmt(e[i], o[i], 0x5410u);      // dims 4i, 4i+1
                nat[2 * i + 1] = prmt(e[i], o[i], 0x7632u);  // dims 4i+2, 4i+3
            }
#pragma unroll
            for (int i = 0; i < 8; i++) {   // fp16 centroid x fp16 norm, rounded once
                __half2 h = __hmul2(*reinterpret_cast<__half2*>(&nat[i]), n2);
                nat[i] = *reinterpret_cast<uint32_t*>(&h);
            }
            const int ch = 16 * blk + 2 * g8;    // 8-dim chunk index within the head
            *reinterpret_cast<uint4*>(dst + (ch >> 3) * (BN * 128) + sw128(key, ch & 7)) =
                make_uint4(nat[0], nat[1], nat[2], nat[3]);
            *reinterpret_cast<uint4*>(dst + ((ch + 1) >> 3) * (BN * 128) + sw128(key, (ch + 1) & 7)) =
                make_uint4(nat[4], nat[5], nat[6], nat[7]);
        }
    }
}

template <int KVK, int MODE>
__device__ __forceinline__ void attn_tile(const Problem<MODE>& pb, const void* const* ktab,
                                          const void* const* vtab, int n_kv, float scale,
                                          uint8_t* smem_raw) {
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + 512);
    uint8_t* kv_sm = base + SMEM_BAR;
    // K and V slots are released separately: a K slot as soon as its S MMAs have run, a V
    // slot after its PV MMAs, so the next K tile lands while the current tile is in softmax
    const uint32_t k_full = s32(&bars[0]), k_empty = s32(&bars[4]), v_full = s32(&bars[8]),
                   v_empty = s32(&bars[12]), s_full = s32(&bars[16]), pvb = s32(&bars[18]),
                   p_full = s32(&bars[20]);
    // pvb[b] completes when the PV MMAs of a tile that used S/P buffer b have run: it frees the
    // buffer for S(i+2) and tells the softmax warps that O may be touched
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = (pb.hi - pb.lo + BN - 1) / BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < KV_STAGES; s++) {
            bar_init(k_full + 8 * s, N_LOAD_WARPS * 32);
            bar_init(k_empty + 8 * s, 1);
            bar_init(v_full + 8 * s, N_LOAD_WARPS * 32);
            bar_init(v_empty + 8 * s, 1);
        }
        for (int s = 0; s < 2; s++) {
            bar_init(s_full + 8 * s, 1);
            bar_init(pvb + 8 * s, 1);
        }
        bar_init(p_full, N_SOFTMAX_WARPS * 32);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(s32(tmem_slot)), "n"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (warp < N_SOFTMAX_WARPS) {
        // Q tile: fp32 -> fp16 pairs, row r into TMEM lane r, dims 2c, 2c+1 into column COL_Q + c
        const RowInfo rq = pb.row(threadIdx.x);
        const uint32_t qaddr = tmem + ((uint32_t)(warp * 32) << 16) + COL_Q;
#pragma unroll 1
        for (int c = 0; c < HD / 2; c += 32) {
            float packed[32];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
                if (rq.q) a = __ldg(reinterpret_cast<const float4*>(rq.q + 2 * (c + e)));
                __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
                packed[e] = __uint_as_float(*reinterpret_cast<uint32_t*>(&h0));
                packed[e + 1] = __uint_as_float(*reinterpret_cast<uint32_t*>(&h1));
            }
            tc_st32(qaddr + c, packed);
        }
        tc_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    if (warp < N_SOFTMAX_WARPS) {
        // ------------------------------ softmax: thread = row ------------------------------
        const int r = threadIdx.x;
        const RowInfo ri = pb.row(r);
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const float sc2 = scale * LOG2E_F;
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
#ifdef Q27_TRACE
        const long long tloop = clock64();
#endif
        for (int i = 0; i < ntiles && ok; i++) {
            const int bsel = i & 1;
            { TRACE_T0();
              ok = __all_sync(0xffffffffu, bar_wait(s_full + 8 * bsel, (uint32_t)((i >> 1) & 1)));
              TRACE_ADD(0, threadIdx.x == 0); }
            if (!ok) break;
            if (threadIdx.x == 0) TRACE_EV(4, i);
            tc_fence_after();
            float s[BN];
            tc_ld32(lane_base + (bsel ? COL_S1 : COL_S0), s);
            tc_ld32(lane_base + (bsel ? COL_S1 : COL_S0) + 32, s + 32);
            tc_wait_ld();
            const int k0 = pb.lo + i * BN;
            const int vis = ri.bound - k0;            // columns [0, vis) are visible
            float mx = -INFINITY;
            if (vis >= BN) {                          // the common case: nothing to mask
#pragma unroll
                for (int j = 0; j < BN; j++) {
                    s[j] *= sc2;
                    mx = fmaxf(mx, s[j]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < BN; j++) {
                    s[j] = j < vis ? s[j] * sc2 : -INFINITY;
                    mx = fmaxf(mx, s[j]);
                }
            }
            float alpha = 1.f;
            bool need = false;
            if (mx > m_ref + RESCALE_THRESHOLD || (m_ref == -INFINITY && mx > -INFINITY)) {
                alpha = m_ref == -INFINITY ? 0.f : ex2f(m_ref - mx);
                m_ref = mx;
                need = i > 0;                          // O holds nothing before the first PV
            }
            const float mu = m_ref == -INFINITY ? 0.f : m_ref;
            float sum = 0.f;
            uint32_t ph[BN / 2];
#pragma unroll
            for (int j = 0; j < BN; j += 2) {
                const float p0 = ex2f(s[j] - mu), p1 = ex2f(s[j + 1] - mu);
                sum += p0 + p1;
                __half2 h = __floats2half2_rn(p0, p1);
                ph[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
            }
            l = l * alpha + sum;
            if (threadIdx.x == 0) TRACE_EV(5, i);
            if (__any_sync(0xffffffffu, need)) {       // warp-collective TMEM round trip on O
                { TRACE_T0();
                  ok = __all_sync(0xffffffffu,
                                  bar_wait(pvb + 8 * ((i - 1) & 1), (uint32_t)(((i - 1) >> 1) & 1)));
                  TRACE_ADD(1, threadIdx.x == 0); }
                if (!ok) break;
                tc_fence_after();
#pragma unroll 1
                for (int c = 0; c < HD; c += 32) {
                    float o[32];
                    tc_ld32(lane_base + COL_O + c, o);
                    tc_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e++) o[e] *= alpha;
                    tc_st32(lane_base + COL_O + c, o);
                }
            }
            // P (fp16 pairs) over the first 32 columns of this tile's S buffer: the A operand
            // of the PV MMAs, straight from tensor memory
            tc_st32(lane_base + (bsel ? COL_S1 : COL_S0), reinterpret_cast<const float*>(ph));
            tc_wait_st();
            tc_fence_before();
            bar_arrive(p_full);
            if (threadIdx.x == 0) TRACE_EV(6, i);
        }
        if (ok) ok = bar_wait(pvb + 8 * ((ntiles - 1) & 1), (uint32_t)(((ntiles - 1) >> 1) & 1));
        ok = __all_sync(0xffffffffu, ok);
#ifdef Q27_TRACE
        if (threadIdx.x == 0) {
            atomicAdd(&g_umma_trace[7], (unsigned long long)(clock64() - tloop));
            atomicAdd(&g_umma_trace[8], (unsigned long long)ntiles);
        }
#endif
        tc_fence_after();
        if (ok) {
            const float inv = l > 0.f ? 1.f / l : 0.f;
            if (ri.part) {
                ri.part[0] = m_ref == -INFINITY ? NEG_SENTINEL : m_ref * 0.6931471805599453f;
                ri.part[1] = l;
            }
            // the TMEM loads are warp-collective: every lane runs them, padding rows just
            // drop what they read
#pragma unroll 1
            for (int c = 0; c < HD; c += 32) {
                float o[32];
                tc_ld32(lane_base + COL_O + c, o);
                tc_wait_ld();
                if (ri.out) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(ri.out + c + e) =
                            make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
                } else if (ri.part) {
#pragma unroll
                    for (int e = 0; e < 32; e++) ri.part[2 + c + e] = o[e];
                }
            }
        }
        tc_fence_before();
    } else if (warp == MMA_WARP) {
        // ------------------------------ S issue: one thread --------------------------------
        if (lane == 0) {
            constexpr uint32_t IDESC_S = make_idesc(BM, BN, false);
            const uint32_t kv_s = s32(kv_sm);
            bool ok = true;
            auto issue_s = [&](int i) {
                const int st = i % KV_STAGES, bsel = i & 1;
                { TRACE_T0();
                  ok = ok && bar_wait(k_full + 8 * st, (uint32_t)((i / KV_STAGES) & 1));
                  TRACE_ADD(2, true); }
                { TRACE_T0();
                  if (ok && i >= 2) ok = bar_wait(pvb + 8 * bsel, (uint32_t)(((i >> 1) - 1) & 1));
                  TRACE_ADD(3, true); }
                if (!ok) return;
                fence_async_smem();
                tc_fence_after();
                const uint32_t k_s = kv_s + st * STAGE_BYTES;
                TRACE_EV(0, i);
                TRACE_T0();
#pragma unroll
                for (int ks = 0; ks < HD / 16; ks++) {
                    const uint64_t db = make_desc(k_s + (ks >> 2) * (BN * 128) + (ks & 3) * 32, 0, 1024);
                    tc_mma_f16_ta(tmem + (bsel ? COL_S1 : COL_S0), tmem + COL_Q + 8 * ks, db, IDESC_S,
                                  ks > 0);
                }
                tc_commit(s_full + 8 * bsel);
                tc_commit(k_empty + 8 * st);
                TRACE_EV(1, i);
                TRACE_ADD(9, true);
            };
            for (int i = 0; i < ntiles && ok; i++) issue_s(i);
        }
        __syncwarp();
    } else if (warp == PV_WARP) {
        // ------------------------------ PV issue: one thread -------------------------------
        if (lane == 0) {
            constexpr uint32_t IDESC_O = make_idesc(BM, HD, true);
            const uint32_t kv_s = s32(kv_sm);
            bool ok = true;
            for (int i = 0; i < ntiles && ok; i++) {
                { TRACE_T0();
                  ok = bar_wait(p_full, (uint32_t)(i & 1));
                  TRACE_ADD(4, true); }
                if (!ok) break;
                const int st = i % KV_STAGES;
                ok = bar_wait(v_full + 8 * st, (uint32_t)((i / KV_STAGES) & 1));
                if (!ok) break;
                fence_async_smem();
                tc_fence_after();
                const uint32_t v_s = kv_s + st * STAGE_BYTES + KT_BYTES;
                TRACE_EV(2, i);
                TRACE_T0();
#pragma unroll
                for (int kk = 0; kk < BN / 16; kk++) {
                    const uint64_t db = make_desc(v_s + kk * 2048, BN * 128, 1024);
                    tc_mma_f16_ta(tmem + COL_O, tmem + ((i & 1) ? COL_S1 : COL_S0) + 8 * kk, db, IDESC_O,
                                  (i > 0 || kk > 0));
                }
                tc_commit(pvb + 8 * (i & 1));
                tc_commit(v_empty + 8 * st);
                TRACE_EV(3, i);
                TRACE_ADD(10, true);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------ K/V staging ----------------------------------------
        const int ptid = threadIdx.x - FIRST_LOAD_WARP * 32;
        RawTile<KVK> raw0, raw1;
        // a tile is exactly one cache page (its first key is a multiple of 64)
        auto load = [&](RawTile<KVK>& r, int i) {
            if (i < ntiles) {
                const int k0 = pb.lo + i * BN;
                tile_load<KVK>(r, static_cast<const uint8_t*>(ktab[k0 >> PAGE_SHIFT]),
                               static_cast<const uint8_t*>(vtab[k0 >> PAGE_SHIFT]),
                               min(BN, pb.hi - k0), n_kv, pb.kvh, ptid);
            }
        };
        auto store = [&](const RawTile<KVK>& r, int i) -> bool {
            const int st = i % KV_STAGES;
            const uint32_t par = (uint32_t)(((i / KV_STAGES) - 1) & 1);
            const int nk = min(BN, pb.hi - (pb.lo + i * BN));
            { TRACE_T0();
              if (i >= KV_STAGES && !bar_wait(k_empty + 8 * st, par)) return false;
              TRACE_ADD(5, ptid == 0); }
            { TRACE_T0();
              tile_store<KVK, 0>(r, kv_sm + st * STAGE_BYTES, nk, ptid);
              fence_async_smem();
              TRACE_ADD(6, ptid == 0); }
            bar_arrive(k_full + 8 * st);
            if (i >= KV_STAGES && !bar_wait(v_empty + 8 * st, par)) return false;
            tile_store<KVK, 1>(r, kv_sm + st * STAGE_BYTES, nk, ptid);
            fence_async_smem();
            bar_arrive(v_full + 8 * st);
            return true;
        };
        if constexpr (KVK == Q27_KV_F16) {
            // fp16 rows need no conversion: cp.async writes them straight into the swizzled
            // operand layout and the slot's barrier is armed to fire when this thread's
            // copies have landed, so the staging threads never wait for data
            (void)raw0; (void)raw1;
            auto copy_half = [&](int i, int which) -> bool {
                const int st = i % KV_STAGES;
                const uint32_t par = (uint32_t)(((i / KV_STAGES) - 1) & 1);
                const uint32_t empty = (which ? v_empty : k_empty) + 8 * st;
                const uint32_t full = (which ? v_full : k_full) + 8 * st;
                if (i >= KV_STAGES && !bar_wait(empty, par)) return false;
                const int k0 = pb.lo + i * BN, nk = min(BN, pb.hi - k0);
                const uint8_t* page = static_cast<const uint8_t*>((which ? vtab : ktab)[k0 >> PAGE_SHIFT]);
                uint8_t* dst = kv_sm + st * STAGE_BYTES + which * KT_BYTES;
#pragma unroll
                for (int n = 0; n < 8; n++) {
                    const int q = ptid + NPROD * n;
                    const int key = q >> 5, ch = q & 31;
                    const uint32_t off = (uint32_t)(ch >> 3) * (BN * 128) + sw128(key, ch & 7);
                    if (key < nk) {
                        const size_t src = ((size_t)key * n_kv + pb.kvh) * (HD * 2) + (size_t)ch * 16;
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                                     ::"r"(s32(dst + off)), "l"(page + src) : "memory");
                    } else {
                        *reinterpret_cast<uint4*>(dst + off) = make_uint4(0, 0, 0, 0);
                    }
                }
                asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(full) : "memory");
                return true;
            };
            for (int i = 0; i < ntiles; i++)
                if (!copy_half(i, 0) || !copy_half(i, 1)) break;
        } else {
            load(raw0, 0);
            load(raw1, 1);
            for (int i = 0; i < ntiles; i += 2) {
                if (!store(raw0, i)) break;
                load(raw0, i + 2);
                if (i + 1 < ntiles) {
                    if (!store(raw1, i + 1)) break;
                    load(raw1, i + 3);
                }
            }
        }
    }
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "n"(TMEM_COLS) : "memory");
    }
}

template <int KVK>
__global__ void __launch_bounds__(UMMA_THREADS, 1)
k_prefill_umma(const __grid_constant__ TileArgs a) {
    extern __shared__ uint8_t smem_raw[];
    Problem<0> pb;
    pb.ta = &a;
    pb.vb = nullptr;
    pb.slot = nullptr;
    pb.kvh = blockIdx.y;
    pb.tile_t0 = a.t0 + blockIdx.x * TOK_PER_TILE;
    pb.lo = 0;
    pb.hi = a.base_pos + min(pb.tile_t0 + TOK_PER_TILE, a.t_end);
    pb.sp = 0;
    attn_tile<KVK, 0>(pb, a.ktab, a.vtab, a.n_kv, a.scale, smem_raw);
}

template <int KVK>
__global__ void __launch_bounds__(UMMA_THREADS, 1)
k_verify_umma(const __grid_constant__ DevBatch b) {
    extern __shared__ uint8_t smem_raw[];
    const DevSlot& S = b.s[blockIdx.z];
    int max_len = 0;
    for (int u = 0; u < S.ntok; u++)
        max_len = max(max_len, local_len(__ldg(S.pos[u]), S.row_base, S.row_count));
    const int chunk = split_chunk(max_len, b.nsplit, b.unit);
    Problem<1> pb;
    pb.ta = nullptr;
    pb.vb = &b;
    pb.slot = &S;
    pb.kvh = blockIdx.y;
    pb.tile_t0 = 0;
    pb.sp = blockIdx.x;
    pb.lo = pb.sp * chunk;
    pb.hi = min(max_len, pb.lo + chunk);
    if (pb.lo >= pb.hi) { // nothing of this split is visible to any lane: sentinels only
        for (int r = threadIdx.x; r < S.ntok * GQA; r += blockDim.x) {
            float* d = S.scratch + (((size_t)(r / GQA) * b.n_q + pb.kvh * GQA + r % GQA) * b.nsplit + pb.sp) * PART;
            d[0] = NEG_SENTINEL;
            d[1] = 0.f;
        }
        return;
    }
    attn_tile<KVK, 1>(pb, S.ktab, S.vtab, b.n_kv, b.scale, smem_raw);
}

template <int KVK>
int set_attrs() {
    static bool done = false;
    if (!done) {
        Q27_CUDA_TRY(cudaFuncSetAttribute(k_prefill_umma<KVK>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, UMMA_SMEM));
        Q27_CUDA_TRY(cudaFuncSetAttribute(k_verify_umma<KVK>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, UMMA_SMEM));
        done = true;
    }
    return Q27_OK;
}

} // namespace

int launch_prefill_umma(const float* qT, int q_stride, int q_row, const void* const* ktab,
                        const void* const* vtab, float* outT, int out_row, int base_pos, int t0,
                        int SB, int n_q, int n_kv, float scale, cudaStream_t st, int kvk,
                        bool* done) {
    *done = false;
    (void)n_q;
    // float4 loads of Q rows and float4 stores of output rows
    if ((q_stride & 3) || (q_row & 3) || (out_row & 3) || ((uintptr_t)qT & 15) || ((uintptr_t)outT & 15))
        return Q27_OK;
    TileArgs a{qT, ktab, vtab, outT, q_stride, q_row, out_row, base_pos, t0, t0 + SB, n_kv, scale};
    dim3 grid((SB + TOK_PER_TILE - 1) / TOK_PER_TILE, n_kv);
    int rc;
    if (kvk == Q27_KV_F16) {
        if ((rc = set_attrs<Q27_KV_F16>())) return rc;
        k_prefill_umma<Q27_KV_F16><<<grid, UMMA_THREADS, UMMA_SMEM, st>>>(a);
    } else if (kvk == Q27_KV_FP8) {
        if ((rc = set_attrs<Q27_KV_FP8>())) return rc;
        k_prefill_umma<Q27_KV_FP8><<<grid, UMMA_THREADS, UMMA_SMEM, st>>>(a);
    } else if (kvk == Q27_KV_T3) {
        if ((rc = set_attrs<Q27_KV_T3>())) return rc;
        k_prefill_umma<Q27_KV_T3><<<grid, UMMA_THREADS, UMMA_SMEM, st>>>(a);
    } else {
        return Q27_ERR_UNSUPPORTED_KIND;
    }
    Q27_CUDA_TRY(cudaGetLastError());
    *done = true;
    return Q27_OK;
}

#ifdef Q27_TRACE
extern "C" int q27_debug_umma_trace(unsigned long long* out, int reset) {
    cudaMemcpyFromSymbol(out, g_umma_trace, sizeof(unsigned long long) * 16);
    if (reset) { unsigned long long z[16] = {0}; cudaMemcpyToSymbol(g_umma_trace, z, sizeof(z)); }
    return 0;
}
extern "C" int q27_debug_umma_events(long long* out) {
    cudaMemcpyFromSymbol(out, g_umma_ev, sizeof(long long) * 8 * 64);
    return 0;
}
#endif

int launch_verify_umma(DevBatch& b, int kvk, int sm_count, cudaStream_t st, bool* done) {
    *done = false;
    if (b.q_stride & 3) return Q27_OK;
    for (int i = 0; i < b.nslots; i++)
        for (int t = 0; t < b.s[i].ntok; t++)
            if ((uintptr_t)b.s[i].q[t] & 15) return Q27_OK;
    int ns = sm_count / (b.nslots * b.n_kv);
    b.nsplit = ns < 1 ? 1 : ns > Q27_MAX_SPLITS ? Q27_MAX_SPLITS : ns;
    b.unit = BN;
    dim3 grid(b.nsplit, b.n_kv, b.nslots);
    int rc;
    if (kvk == Q27_KV_F16) {
        if ((rc = set_attrs<Q27_KV_F16>())) return rc;
        k_verify_umma<Q27_KV_F16><<<grid, UMMA_THREADS, UMMA_SMEM, st>>>(b);
    } else if (kvk == Q27_KV_FP8) {
        if ((rc = set_attrs<Q27_KV_FP8>())) return rc;
        k_verify_umma<Q27_KV_FP8><<<grid, UMMA_THREADS, UMMA_SMEM, st>>>(b);
    } else if (kvk == Q27_KV_T3) {
        if ((rc = set_attrs<Q27_KV_T3>())) return rc;
        k_verify_umma<Q27_KV_T3><<<grid, UMMA_THREADS, UMMA_SMEM, st>>>(b);
    } else {
        return Q27_ERR_UNSUPPORTED_KIND;
    }
    Q27_CUDA_TRY(cudaGetLastError());
    *done = true;
    return Q27_OK;
}

} // namespace q27b
