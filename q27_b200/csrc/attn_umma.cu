// Attention on the 5th-generation tensor cores (tcgen05.mma, accumulators in tensor memory).
//
// One CTA = one Q tile of up to 128 rows against a range of cache rows of ONE kv head. The
// rows of the tile are (token, GQA head) pairs -- 21 tokens x 6 heads for prefill, ntok lanes
// x 6 heads for verify -- so every K/V tile that is staged serves all six heads (and, for
// verify, all draft lanes: one pass over the cache). Each row carries its own causal bound.
//
//   S  = Q . K^T   M=128 rows, N=64 keys, K=256 dims     -> TMEM (a ring of three S buffers)
//   O += P . V     M=128 rows, N=256 dims, K=64 keys      -> TMEM (256 columns)
//
// Q, K and V are fp16 in shared memory in the 128-byte-swizzled canonical layouts (Q and K
// K-major, V MN-major = its natural [key][dim] rows); P is written as fp16 over the S buffer
// it came from and is the A operand of the PV MMAs straight from tensor memory; accumulation
// is fp32. The S ring is three deep because the chain S -> softmax -> PV -> (buffer free) is
// several thousand cycles of mbarrier hops and MMA latency long: three tiles in flight keep
// the tensor pipe and the softmax warps busy through it.
// Warp roles: warps 0-3 softmax (thread = row = TMEM lane); warps 4-5 issue the S MMAs and warp
// 6 the PV MMAs (independent issue streams, ordered only by mbarriers); warps 7-10 stage
// K tiles and warps 11-14 V tiles (rings of three): cp.async for fp16 rows,
// registers + convert for fp8 / turbo3. The running max is only advanced when it grows by
// more than 2^8, so O in TMEM is rarely rescaled.
// Every mbarrier wait is bounded; a timeout sets the library's flag and the CTA drains.
#include "attn_umma.cuh"
#include "t3_lut.cuh"
#include "wht.cuh"

namespace q27b {

// without relocatable device code a __device__ variable is private to its translation unit:
// this file keeps its own timeout flag and the library's reader ORs them together
__device__ int g_umma_timeout_flag = 0;

namespace {

constexpr int BM = 128;                 // Q rows per CTA (TMEM lanes)
constexpr int BN = 64;                  // keys per tile = one cache page
constexpr int TOK_PER_TILE = 21;        // 21 tokens x 6 heads = 126 rows
constexpr int K_SLOTS = 3, V_SLOTS = 3;         // separate rings: K runs ahead with the S MMAs
constexpr int S_BUFS = 3;                       // S / P buffers in tensor memory
constexpr int Q_TMEM_DIMS = 128;                // dims 0..127 of Q live in tensor memory ...
constexpr int Q_BYTES = BM * (HD - Q_TMEM_DIMS) * 2;   // ... the rest in 2 blocks of [128 rows][128 B]
constexpr int KT_BYTES = BN * HD * 2;           // 32768: 4 blocks of [64 rows][128 B]
constexpr int SMEM_BAR = 1024;                  // barriers + tmem slot, keeps tiles 1024-aligned
constexpr int UMMA_SMEM = SMEM_BAR + Q_BYTES + (K_SLOTS + V_SLOTS) * KT_BYTES + 1024;
constexpr int TMEM_COLS = 512;
// TMEM columns: S buffer b at 64 b (its first 32 columns are reused for P), O behind them,
// then the first half of the Q tile as fp16 pairs (8 columns per k-step of 16 dims). Q is
// the A operand of every S MMA: each half kept out of shared memory takes 32 KB per K tile
// off the shared-memory port, which the operand reads of the MMAs and the staging writes
// otherwise saturate; all of Q does not fit beside three S buffers.
constexpr int COL_S = 0, COL_O = S_BUFS * BN, COL_Q = COL_O + HD;
static_assert(COL_Q + Q_TMEM_DIMS / 2 <= TMEM_COLS, "tensor memory columns");
constexpr float LOG2E_F = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;       // log2 units

constexpr int N_SOFTMAX_WARPS = 4, MMA_WARP = 4, N_S_WARPS = 2, PV_WARP = 6, FIRST_LOAD_WARP = 7,
              N_LOAD_WARPS = 8;
constexpr int UMMA_THREADS = (FIRST_LOAD_WARP + N_LOAD_WARPS) * 32;   // 480
constexpr int NPROD = N_LOAD_WARPS * 16;        // 128 staging threads per side (K or V)
// turbo3: the 128 threads of a side work as two teams of 64 that take alternate tiles, each
// with its own raw buffer. A tile costs a staging thread a fixed ~0.7 us of barrier round trips
// and shared-memory latency around the decode itself (~0.6 us for a 128th of a tile): one team
// of 128 on every tile published a tile every 1.45 us and set the pace of the whole loop; two
// teams of 64 decode twice as much per thread and tile, pay the fixed part once per two tiles
// and overlap each other (c5 -6 %). fp8 stays with one team of 128: its conversion runs on the
// 16-lane convert pipe, which two teams only crowd (+20 % measured).
constexpr int TEAM = NPROD / 2;
template <int KVK> constexpr int stagers() { return KVK == Q27_KV_T3 ? TEAM : NPROD; }   // threads that stage one tile

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
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok) : "r"(bar), "r"(parity), "r"(4000u) : "memory");   // suspend-time hint, ns
    return ok != 0;
}
// Bounded: ~2 s of polling, then the flag. (A tenth of that expired inside a profiler's
// instrumented replay pass, which slows the kernel a thousandfold.)
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
    for (int i = 0; i < (1 << 24); i++) {
        if (bar_try(bar, parity)) return true;
        if (i > 2048) __nanosleep(64);
    }
    atomicExch(&g_umma_timeout_flag, 2);
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
// tcgen05.mma kind::f16 with the accumulate flag known at compile time (no predicate set-up per
// MMA); _ta: the A operand taken from tensor memory (row = lane, 16 fp16 of K per 8 columns)
template <int ACC>
__device__ __forceinline__ void tc_mma_f16_ta_c(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "n"(ACC) : "memory");
}
template <int ACC>
__device__ __forceinline__ void tc_mma_f16_c(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "n"(ACC) : "memory");
}
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile("{\n .reg .pred p;\n elect.sync _|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}"
                 : "=r"(pred));
    return pred != 0;
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
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float y;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(y) : "f"(a), "f"(b), "f"(c));
    return y;
}
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
    // split of the items (Q tile x kv head) that do not fill a wave: items [0, n_full) run
    // whole; every later item is cut into `pieces` key ranges whose un-normalised results go
    // to part[((head * part_rows + (t - t0)) * PF_SPLIT_MAX + piece) * 258] for the fix-up
    float* part;
    int part_rows, nx, n_full, pieces;
    int wht;            // WHT_Q: rotate the Q rows as they are staged; WHT_OUT: un-rotate the output rows
};
constexpr int PF_SPLIT_MAX = 8;   // pieces a row's scratch has room for (src/prefill.cuh:88)

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
    int piece = -1;     // prefill: >= 0 when this CTA holds one key range of a split item

    // the Q head of row r alone (nullptr for a padding row): what the staging loops need, without
    // the bound (a load of the lane's position) and the output addresses of row()
    __device__ __forceinline__ const float* q_of(int r) const {
        const int tok = r / GQA, j = r % GQA;
        if (MODE == 0) {
            const int t = tile_t0 + tok;
            if (tok >= TOK_PER_TILE || t >= ta->t_end) return nullptr;
            return ta->qT + (size_t)t * ta->q_row + (size_t)(kvh * GQA + j) * ta->q_stride;
        }
        if (tok >= slot->ntok) return nullptr;
        return slot->q[tok] + (size_t)(kvh * GQA + j) * vb->q_stride;
    }

    // rows [0, live_rows()) of the tile carry a Q head, the rest is padding
    __device__ __forceinline__ int live_rows() const {
        if (MODE == 0) return max(0, min(TOK_PER_TILE, ta->t_end - tile_t0)) * GQA;
        return min(slot->ntok * GQA, BM);
    }

    __device__ __forceinline__ RowInfo row(int r) const {
        // a padding row (no q) sees everything: its lanes stay on the unmasked path of their
        // warp and what they compute from a zero Q row is dropped
        RowInfo ri{nullptr, 0x3fffffff, nullptr, nullptr};
        const int tok = r / GQA, j = r % GQA;
        if (MODE == 0) {
            const int t = tile_t0 + tok;
            if (tok < TOK_PER_TILE && t < ta->t_end) {
                const int h = kvh * GQA + j;
                ri.q = ta->qT + (size_t)t * ta->q_row + (size_t)h * ta->q_stride;
                ri.bound = ta->base_pos + t + 1;
                if (piece < 0)
                    ri.out = ta->outT + (size_t)t * ta->out_row + (size_t)h * HD;
                else
                    ri.part = ta->part + (((size_t)h * ta->part_rows + (t - ta->t0)) * PF_SPLIT_MAX +
                                          piece) * PART;
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

// Staging of one 64-key tile of ONE side (K or V) as fp16 into the swizzled operand layout
// by that side's 128 threads. fp16 rows go from global to shared memory with cp.async,
// straight into that layout. fp8 and turbo3 rows come in packed (coalesced asynchronous
// copies into raw shared-memory buffers); each thread then takes its share into registers
// (`RawHalf`) and `half_store` converts and writes it once the ring slot has been released.
template <int KVK> struct RawHalf;
template <> struct RawHalf<Q27_KV_F16> { };
template <> struct RawHalf<Q27_KV_FP8> { uint2 d[16]; };
template <> struct RawHalf<Q27_KV_T3> { uint32_t w[14]; };

// BLK (turbo3 only): which of the two blocks of a (key, kv head) the thread decodes; warp-uniform
template <int KVK, int BLK = 0>
__device__ __forceinline__ void half_store(const RawHalf<KVK>& t, uint8_t* dst, int nkeys, int p) {
    if constexpr (KVK == Q27_KV_FP8) {
#pragma unroll
        for (int n = 0; n < 16; n++) {
            const int q = p + NPROD * n;
            const int key = q >> 5, ch = q & 31;
            const uint32_t off = (uint32_t)(ch >> 3) * (BN * 128) + sw128(key, ch & 7);
            auto cv = [](uint32_t two) {
                __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two, __NV_E4M3);
                return (uint32_t)h.x | ((uint32_t)h.y << 16);
            };
            *reinterpret_cast<uint4*>(dst + off) = make_uint4(
                cv(t.d[n].x & 0xffffu), cv(t.d[n].x >> 16), cv(t.d[n].y & 0xffffu), cv(t.d[n].y >> 16));
        }
    } else if constexpr (KVK == Q27_KV_T3) {
        const int key = p & 63;
        const uint32_t* w = t.w;
        // 32-bit little-endian word at byte `o` of the block (o even, compile time); block 1
        // sits 2 bytes into the loaded words, block 0 at byte 0
        auto word_at = [&](int o) {
            const int ob = o + 2 * BLK;
            return (ob & 3) ? __funnelshift_r(w[ob >> 2], w[(ob >> 2) + 1], 16) : w[ob >> 2];
        };
        constexpr int blk = BLK;
        const __half nh = __ushort_as_half((unsigned short)(word_at(0) & 0xffffu));
        // one block, one norm: the pools hold centroid x norm (rows past the range: zeros)
        const T3Tab tab = t3_tables_scaled(key < nkeys ? __half2float(nh) : 0.f);
#pragma unroll
        for (int g8 = 0; g8 < 8; g8++) {         // 16 dims per group
            const uint32_t Qw = word_at(2 + 4 * g8);
            const uint32_t S16 = (word_at(34 + 2 * (g8 & ~1)) >> (16 * (g8 & 1))) & 0xffffu;
            uint32_t ze, zo, e[4], o[4];
            t3_selectors(Qw, S16, ze, zo);
            t3_lookup(tab, ze, e);                // (0,2) (4,6) (8,10) (12,14)
            t3_lookup(tab, zo, o);                // (1,3) (5,7) (9,11) (13,15)
            // The lookups give (even dims) and (odd dims) of the group. They are stored as they
            // are: positions 0..7 of a 16-dim group hold its even dims, 8..15 its odd dims.
            // Q is staged with the same permutation (a dot product does not care) and the
            // output columns are put back in order in the epilogue, so the eight PRMTs per
            // group that would interleave them are never spent.
            const int ch = 16 * blk + 2 * g8;    // 8-position chunk index within the head
            *reinterpret_cast<uint4*>(dst + (ch >> 3) * (BN * 128) + sw128(key, ch & 7)) =
                make_uint4(e[0], e[1], e[2], e[3]);
            *reinterpret_cast<uint4*>(dst + ((ch + 1) >> 3) * (BN * 128) + sw128(key, (ch + 1) & 7)) =
                make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

template <int KVK, int MODE>
__device__ __forceinline__ void attn_tile(const Problem<MODE>& pb, const void* const* ktab,
                                          const void* const* vtab, int n_kv, float scale,
                                          int wht, uint8_t* smem_raw) {
    uint8_t* base = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(base);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + 512);
    uint32_t* epi_bad = tmem_slot + 1;  // a softmax warp gave up waiting: no folded output rotation
    uint8_t* q_sm = base + SMEM_BAR;
    uint8_t* k_sm = q_sm + Q_BYTES;
    uint8_t* v_sm = k_sm + K_SLOTS * KT_BYTES;
    // turbo3 gives its third V slot to a raw staging area: the packed rows of a tile are
    // fetched with coalesced asynchronous copies and decoded from shared memory
    // (fp8: the third K slot and the third V slot each hold a side's two raw buffers)
    constexpr int VSL = KVK == Q27_KV_F16 ? V_SLOTS : 2;
    constexpr int KSL = KVK == Q27_KV_FP8 ? 2 : K_SLOTS;
    uint8_t* raw_sm = v_sm + 2 * KT_BYTES;
    // A K slot is released as soon as its S MMAs have run, a V slot after its PV MMAs.
    // pvb[b] completes when the PV MMAs of a tile that used S/P buffer b have run: it frees
    // the buffer for the S MMAs four tiles on and tells the softmax warps that O may be touched.
    const uint32_t k_full = s32(&bars[0]), k_empty = s32(&bars[4]), v_full = s32(&bars[8]),
                   v_empty = s32(&bars[12]), s_full = s32(&bars[16]), pvb = s32(&bars[20]),
                   p_full = s32(&bars[24]);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles = (pb.hi - pb.lo + BN - 1) / BN;

    if (threadIdx.x == 0) {
        *epi_bad = 0;
        constexpr int STAGERS = stagers<KVK>();
        for (int s = 0; s < KSL; s++) {
            bar_init(k_full + 8 * s, STAGERS);
            bar_init(k_empty + 8 * s, 1);
        }
        for (int s = 0; s < VSL; s++) {
            bar_init(v_full + 8 * s, STAGERS);
            bar_init(v_empty + 8 * s, 1);
        }
        for (int s = 0; s < S_BUFS; s++) {
            bar_init(s_full + 8 * s, 1);
            bar_init(pvb + 8 * s, 1);
            bar_init(p_full + 8 * s, N_SOFTMAX_WARPS * 32);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(s32(tmem_slot)), "n"(TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    // ---- what the staging warps know about their side (K or V), before the roles part ways ----
    // the first four staging warps feed the K ring, the other four the V ring; a tile is exactly
    // one cache page
    const bool is_load = warp >= FIRST_LOAD_WARP;
    const int side = is_load ? (warp - FIRST_LOAD_WARP) >> 2 : 0;                  // 0 = K, 1 = V
    const int p = is_load ? (int)threadIdx.x - (FIRST_LOAD_WARP + 4 * side) * 32 : 0;   // 0..127 within the side
    const void* const* tab = side ? vtab : ktab;
    auto page_of = [&](int i) {
        return static_cast<const uint8_t*>(tab[(pb.lo + i * BN) >> PAGE_SHIFT]);
    };
    auto nkeys_of = [&](int i) { return min(BN, pb.hi - (pb.lo + i * BN)); };
    // Packed rows (turbo3, fp8) come in with 16-byte asynchronous copies into two raw buffers per
    // side (tile i: buffer i & 1 -- for turbo3 that is the buffer of the team that takes the
    // tile). A warp copies exactly the rows it converts, so the buffers need no barrier: the
    // lanes wait for their own copies (cp.async groups) and meet in a __syncwarp.
    //   turbo3: a tile's rows of this kv head are 64 keys x 100 B, 400 B apart in the page; what
    //   is copied is the aligned 112-byte window that holds them (a row starts on a 16-byte
    //   boundary and kv head h sits at byte 100 h, so the window [100 h rounded down, + 112)
    //   never leaves the row): 448 copies per tile and side instead of 1600 four-byte ones (a
    //   block per thread straight from global memory costs one L1 wavefront per lane per load
    //   and bounded this path). The buffers live in the third V slot.
    //   fp8: 64 keys x 256 B, coalesced; the third K slot and the third V slot each hold a
    //   side's two buffers. (Holding two tiles of raw bytes in registers instead spilled and
    //   made this path the bottleneck of the fp8 kernels.)
    constexpr bool TEAMS = KVK == Q27_KV_T3;
    const int team = TEAMS ? p >> 6 : 0, q = TEAMS ? p & (TEAM - 1) : p;   // q: thread within the tile's stagers
    constexpr int RAW_ROW = 112;
    constexpr int RAW_BYTES = KVK == Q27_KV_T3 ? BN * RAW_ROW : BN * HD;
    static_assert(KVK != Q27_KV_T3 || 4 * RAW_BYTES <= KT_BYTES, "the raw buffers live in the third V slot");
    uint8_t* raw = KVK == Q27_KV_T3 ? raw_sm + side * 2 * RAW_BYTES : (side ? v_sm : k_sm) + 2 * KT_BYTES;
    const int win0 = (pb.kvh * 2 * T3_BLK) & ~15;        // turbo3: window start inside the row
    const int blk_off = pb.kvh * 2 * T3_BLK - win0;      // 0, 4, 8 or 12
    // turbo3: a warp copies the windows of the 32 keys it decodes itself (224 pieces, 7 per lane;
    // piece c = key 7 + 16-byte chunk; key and chunk are the same for every tile), so its raw
    // rows need no barrier: the lanes wait for their own copies (cp.async groups) and meet in a
    // __syncwarp. (With the team's two warps sharing the buffer through a pair of mbarriers, a
    // staging thread spent 0.3-0.9 us per tile between reading its rows and having the next
    // ones on their way.)
    int t3_key[7], t3_j[7];
    if constexpr (KVK == Q27_KV_T3) {
#pragma unroll
        for (int n = 0; n < 7; n++) {
            const int c = lane + 32 * n;
            t3_key[n] = (q & 32) + c / 7;
            t3_j[n] = c % 7;
        }
    }
    // by the threads that stage tile i
    auto issue_raw = [&](int i, const uint8_t* page) {
        const int buf = i & 1, nk = nkeys_of(i);
        if constexpr (KVK == Q27_KV_T3) {
            const uint32_t dst = s32(raw + buf * RAW_BYTES);
#pragma unroll
            for (int n = 0; n < 7; n++)
                if (t3_key[n] < nk)
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                                 ::"r"(dst + (uint32_t)(t3_key[n] * RAW_ROW + 16 * t3_j[n])),
                                   "l"(page + (size_t)(t3_key[n] * n_kv * (2 * T3_BLK) + win0 + 16 * t3_j[n]))
                                 : "memory");
        } else if constexpr (KVK == Q27_KV_FP8) {
            // a warp copies the 16 rows it converts itself (keys 4 k + its index in the side):
            // 256 16-byte chunks, 8 per lane
            uint8_t* dst = raw + buf * RAW_BYTES;
            const int wq = p >> 5;
#pragma unroll
            for (int n = 0; n < 8; n++) {
                const int c = lane + 32 * n;
                const int key = 4 * (c >> 4) + wq, c16 = c & 15;
                if (key < nk)
                    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                                 ::"r"(s32(dst + key * HD + c16 * 16)),
                                   "l"(page + ((size_t)key * n_kv + pb.kvh) * HD + c16 * 16)
                                 : "memory");
                else                                   // rows past the range: exact zeros
                    *reinterpret_cast<uint4*>(dst + key * HD + c16 * 16) = make_uint4(0, 0, 0, 0);
            }
        }
        // the lanes wait for their own copies (cp.async groups) and meet in a __syncwarp
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    // The first two tiles' packed rows are asked for before the Q tile is staged (the table
    // look-up and the trip to HBM overlap it) -- unless the folded rotation needs the buffers'
    // room for the fp32 Q tile first.
    const bool raw_early = KVK != Q27_KV_F16 && !(wht & WHT_Q);
    if (raw_early) {
        __syncthreads();                               // the barriers are initialised
        if (is_load) {
            if (TEAMS) {
                if (team < ntiles) issue_raw(team, page_of(team));
            } else {
                if (ntiles > 0) issue_raw(0, page_of(0));
                if (ntiles > 1) issue_raw(1, page_of(1));
            }
        }
    }
    {
        // Q tile, fp32 -> fp16, by ALL threads with coalesced loads: consecutive threads take
        // consecutive 16-byte pieces of a row (a thread walking its own row costs a dependent
        // chain of uncoalesced loads, ~20 us per CTA). Dims 128..255 go straight into row r
        // of two [128][128 B] swizzled blocks; dims 0..127 wait in the (still idle) K ring
        // for the thread that owns TMEM lane r.
        constexpr int QT_PITCH = 264;                       // bytes per row of the waiting half
        // Folded forward rotation (wht3 / wht_T on Q, src/spec3.cu:595-614,
        // src/prefill.cu:2598-2618): the tile's rows first land as fp32 in the idle third K slot
        // and V ring, every warp rotates its share of the 128-groups in place, and the loop
        // below converts from there instead of from global memory.
        const float4* q_rot4 = reinterpret_cast<const float4*>(k_sm + 2 * KT_BYTES);
        static_assert((K_SLOTS - 2 + V_SLOTS) * KT_BYTES >= BM * HD * 4, "room for the fp32 Q tile");
        static_assert(2 * KT_BYTES >= BM * QT_PITCH, "the waiting half stays clear of it");
        // Only the tile's live rows (lanes x 6 heads of a verify step: 36 of 128) are fetched and
        // converted; the rows behind them are zeroed without a trip to memory.
        const int live = pb.live_rows();
        const int pieces = live * (HD / 4);                 // 16-byte pieces of the live rows
        if (wht & WHT_Q) {
            float* q_rot = reinterpret_cast<float*>(k_sm + 2 * KT_BYTES);
            for (int i = threadIdx.x; i < pieces; i += UMMA_THREADS) {
                const float* rq = pb.q_of(i >> 6);
                if (rq) reinterpret_cast<float4*>(q_rot)[i] = __ldg(reinterpret_cast<const float4*>(rq) + (i & 63));
            }
            __syncthreads();
            for (int gi = warp; gi < 2 * live; gi += UMMA_THREADS / 32)
                if (pb.q_of(gi >> 1)) wht_group<false>(q_rot + gi * 128, lane);
            __syncthreads();
        }
        // loads in flight per thread: a verify step's rows (up to 6 lanes) in one pass
        constexpr int QU = MODE == 1 ? 5 : 9;              // prefill: 126 rows in two passes
        for (int base_i = 0; base_i < pieces; base_i += UMMA_THREADS * QU) {
            float4 v[QU];
            int idx[QU];
#pragma unroll
            for (int u = 0; u < QU; u++) {
                idx[u] = base_i + u * UMMA_THREADS + threadIdx.x;
                v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (idx[u] < pieces) {
                    const float* rq = pb.q_of(idx[u] >> 6);
                    if (rq)
                        v[u] = (wht & WHT_Q) ? q_rot4[idx[u]]
                                             : __ldg(reinterpret_cast<const float4*>(rq) + (idx[u] & 63));
                }
            }
#pragma unroll
            for (int u = 0; u < QU; u++) {
                if (idx[u] >= pieces) continue;
                const int row = idx[u] >> 6, d = (idx[u] & 63) * 4;
                // where the 16-bit value of operand position X of this row lives
                auto q_loc = [&](int X) -> uint8_t* {
                    if (X >= Q_TMEM_DIMS) {
                        const int c2 = (X - Q_TMEM_DIMS) >> 3;
                        return q_sm + (c2 >> 3) * (BM * 128) + sw128(row, c2 & 7) + (X & 7) * 2;
                    }
                    return k_sm + row * QT_PITCH + X * 2;
                };
                if constexpr (KVK == Q27_KV_T3) {
                    // turbo3 operand order (see half_store): evens of a 16-dim group, then odds
                    __half2 he = __floats2half2_rn(v[u].x, v[u].z), ho = __floats2half2_rn(v[u].y, v[u].w);
                    const int X = (d & ~15) + ((d & 15) >> 1);
                    *reinterpret_cast<uint32_t*>(q_loc(X)) = *reinterpret_cast<uint32_t*>(&he);
                    *reinterpret_cast<uint32_t*>(q_loc(X + 8)) = *reinterpret_cast<uint32_t*>(&ho);
                } else {
                    __half2 h0 = __floats2half2_rn(v[u].x, v[u].y), h1 = __floats2half2_rn(v[u].z, v[u].w);
                    *reinterpret_cast<uint2*>(q_loc(d)) =
                        make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
                }
            }
        }
        // the padding rows of the shared-memory half: whole 128-byte rows of both blocks (the
        // swizzle permutes 16-byte chunks inside a row); those of the tensor-memory half are
        // zeroed by their owners below
        for (int i = threadIdx.x; i < (BM - live) * 16; i += UMMA_THREADS) {
            const int row = live + (i >> 4), blk = (i >> 3) & 1, ch = i & 7;
            *reinterpret_cast<uint4*>(q_sm + blk * (BM * 128) + row * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (warp < N_SOFTMAX_WARPS) {
            // dims 0..127 of row r into TMEM lane r, dims 2c, 2c+1 into column COL_Q + c
            const uint32_t qaddr = (*tmem_slot) + ((uint32_t)(warp * 32) << 16) + COL_Q;
            const uint32_t* src = reinterpret_cast<const uint32_t*>(k_sm + threadIdx.x * QT_PITCH);
#pragma unroll 1
            for (int c = 0; c < Q_TMEM_DIMS / 2; c += 32) {
                float packed[32];
#pragma unroll
                for (int e = 0; e < 32; e++) packed[e] = (int)threadIdx.x < live ? __uint_as_float(src[c + e]) : 0.f;
                tc_st32(qaddr + c, packed);
            }
            tc_wait_st();
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < N_SOFTMAX_WARPS) {
        // ------------------------------ softmax: thread = row ------------------------------
        const int r = threadIdx.x;
        const RowInfo ri = pb.row(r);
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        const float sc2 = scale * LOG2E_F;      // > 0: the row max may be taken before scaling
        float m_ref = -INFINITY, l = 0.f;
        bool ok = true;
        const bool warp_has_rows = __any_sync(0xffffffffu, ri.q != nullptr);
        for (int i = 0; i < ntiles && ok; i++) {
            const int b = i % S_BUFS;
            const uint32_t s_col = lane_base + COL_S + b * BN;
            ok = __all_sync(0xffffffffu, bar_wait(s_full + 8 * b, (uint32_t)((i / S_BUFS) & 1)));
            if (!ok) break;
            if (!warp_has_rows) {
                // a warp of padding rows only (verify tiles use 6 rows per lane): it keeps
                // step with the barriers and leaves its issue slots to the staging warps;
                // whatever its S columns hold is multiplied into O rows nobody reads
                tc_fence_before();
                bar_arrive(p_full + 8 * b);
                continue;
            }
            tc_fence_after();
            float s[BN];
            tc_ld32(s_col, s);
            tc_ld32(s_col + 32, s + 32);
            tc_wait_ld();
            const int k0 = pb.lo + i * BN;
            const int vis = ri.bound - k0;            // columns [0, vis) are visible
            if (vis < BN) {                           // rare: the diagonal and the ragged tail
#pragma unroll
                for (int j = 0; j < BN; j++) s[j] = j < vis ? s[j] : -INFINITY;
            }
            float mx = fmaxf(s[0], s[1]);
#pragma unroll
            for (int j = 2; j < BN; j += 2) mx = max3f(mx, s[j], s[j + 1]);
            mx *= sc2;
            float alpha = 1.f;
            bool need = false;
            if (mx > m_ref + RESCALE_THRESHOLD || (m_ref == -INFINITY && mx > -INFINITY)) {
                alpha = m_ref == -INFINITY ? 0.f : ex2f(m_ref - mx);
                m_ref = mx;
                need = i > 0;                          // O holds nothing before the first PV
            }
            const float nmu = m_ref == -INFINITY ? 0.f : -m_ref;
            float sum0 = 0.f, sum1 = 0.f;
            uint32_t ph[BN / 2];
#pragma unroll
            for (int j = 0; j < BN; j += 2) {
                const float p0 = ex2f(fmaf(s[j], sc2, nmu)), p1 = ex2f(fmaf(s[j + 1], sc2, nmu));
                sum0 += p0;
                sum1 += p1;
                __half2 h = __floats2half2_rn(p0, p1);
                ph[j >> 1] = *reinterpret_cast<uint32_t*>(&h);
            }
            l = l * alpha + (sum0 + sum1);
            if (__any_sync(0xffffffffu, need)) {       // warp-collective TMEM round trip on O
                const int pi = i - 1;
                ok = __all_sync(0xffffffffu,
                                bar_wait(pvb + 8 * (pi % S_BUFS), (uint32_t)((pi / S_BUFS) & 1)));
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
            tc_st32(s_col, reinterpret_cast<const float*>(ph));
            tc_wait_st();
            tc_fence_before();
            bar_arrive(p_full + 8 * b);
        }
        if (ok) ok = bar_wait(pvb + 8 * ((ntiles - 1) % S_BUFS), (uint32_t)(((ntiles - 1) / S_BUFS) & 1));
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
        // The normalised rows of a prefill tile go to the idle rings instead of global memory, and
        // after the closing barrier every warp writes its share -- un-rotated first where the
        // inverse rotation is folded in (wht_T on the output rows). (Rows of a split item go to
        // the fix-up kernel, which rotates.)
        constexpr int OROT_PITCH = HD + 4;          // floats: float4-aligned, rows 4 banks apart
        static_assert((K_SLOTS + V_SLOTS) * KT_BYTES >= BM * OROT_PITCH * 4, "room for the fp32 O tile");
        float* o_rot = reinterpret_cast<float*>(k_sm);
        // Output rows of a prefill tile take the same road whether or not they are rotated on the
        // way: a row per thread straight to global memory is one 16-byte piece of 32 different
        // lines per store instruction (5.6 us of a prefill CTA's ~150).
        const bool rot_out = MODE == 0 && pb.piece < 0;
        // Partial records {m, l, acc[256]} (verify; a key range of a split prefill item) take the
        // same road: a thread owns a row, so storing it from here costs one 8-byte piece of 32
        // different lines per instruction (2.7 us of a verify step). The rows go to the idle rings
        // as {m, l, -, -, acc[256]} and every warp writes whole rows after the closing barrier.
        const bool part_rows = MODE == 1 || pb.piece >= 0;
        if (!ok && (rot_out || part_rows)) *epi_bad = 1;
        if (ok) {
            const float inv = l > 0.f ? 1.f / l : 0.f;
            float* stage = o_rot + (size_t)r * OROT_PITCH;
            if (ri.part) {
                stage[0] = m_ref == -INFINITY ? NEG_SENTINEL : m_ref * 0.6931471805599453f;
                stage[1] = l;
            }
            // the TMEM loads are warp-collective: every lane runs them, padding rows just
            // drop what they read
            if (warp_has_rows) {
#pragma unroll 1
                for (int c = 0; c < HD; c += 32) {
                    float o[32];
                    tc_ld32(lane_base + COL_O + c, o);
                    tc_wait_ld();
                    // register that holds natural column n of this 32-column chunk (turbo3
                    // operand order: evens of a 16-dim group, then odds)
                    auto reg = [](int n) {
                        return KVK == Q27_KV_T3 ? (n & 16) + ((n & 1) ? 8 + ((n & 15) >> 1) : ((n & 15) >> 1)) : n;
                    };
                    if (ri.out) {
                        float* dst = rot_out ? stage : ri.out;
#pragma unroll
                        for (int e = 0; e < 32; e += 4)
                            *reinterpret_cast<float4*>(dst + c + e) =
                                make_float4(o[reg(e)] * inv, o[reg(e + 1)] * inv, o[reg(e + 2)] * inv,
                                            o[reg(e + 3)] * inv);
                    } else if (ri.part) {
#pragma unroll
                        for (int e = 0; e < 32; e += 4)
                            *reinterpret_cast<float4*>(stage + 4 + c + e) =
                                make_float4(o[reg(e)], o[reg(e + 1)], o[reg(e + 2)], o[reg(e + 3)]);
                    }
                }
            }
        }
        tc_fence_before();
    } else if (warp < MMA_WARP + N_S_WARPS) {
        // ------------------------------ S issue ------------------------------------------
        // Two warps take alternate tiles: the waits and bookkeeping of one overlap the MMA issue
        // of the other (the S buffers, K slots and barriers of consecutive tiles are distinct).
        // The whole warp runs the loop (waits and address arithmetic stay warp-uniform, so the
        // descriptors live in uniform registers); one elected lane issues the MMAs.
        {
            constexpr uint32_t IDESC_S = make_idesc(BM, BN, false);
            const uint64_t qd0 = make_desc(s32(q_sm), 0, 1024);
            const uint64_t kd_base = make_desc(s32(k_sm), 0, 1024);
            bool ok = true;
            for (int i = warp - MMA_WARP; i < ntiles && ok; i += N_S_WARPS) {
                const int ks_ = i % KSL, b = i % S_BUFS;
                const uint32_t kpar = (uint32_t)((i / KSL) & 1);
                const uint32_t bpar = (uint32_t)(((i / S_BUFS) - 1) & 1);   // previous use of buffer b
                ok = bar_wait(k_full + 8 * ks_, kpar);
                if (ok && i >= S_BUFS) ok = bar_wait(pvb + 8 * b, bpar);
                if (!ok) break;
                fence_async_smem();
                tc_fence_after();
                const uint64_t kd0 = kd_base + (uint64_t)((ks_ * KT_BYTES) >> 4);
                const uint32_t d = tmem + COL_S + b * BN;
                if (elect_one()) {
#pragma unroll
                    for (int ks = 0; ks < HD / 16; ks++) {
                        const uint64_t db = kd0 + (uint64_t)(((ks >> 2) * (BN * 128) + (ks & 3) * 32) >> 4);
                        if (ks == 0) {
                            tc_mma_f16_ta_c<0>(d, tmem + COL_Q, db, IDESC_S);
                        } else if (ks < Q_TMEM_DIMS / 16) {
                            tc_mma_f16_ta_c<1>(d, tmem + COL_Q + 8 * ks, db, IDESC_S);
                        } else {
                            const int k2 = ks - Q_TMEM_DIMS / 16;
                            const uint64_t da = qd0 + (uint64_t)(((k2 >> 2) * (BM * 128) + (k2 & 3) * 32) >> 4);
                            tc_mma_f16_c<1>(d, da, db, IDESC_S);
                        }
                    }
                    tc_commit(s_full + 8 * b);
                    tc_commit(k_empty + 8 * ks_);
                }
                __syncwarp();
            }
        }
    } else if (warp == PV_WARP) {
        // ------------------------------ PV issue -----------------------------------------
        {
            constexpr uint32_t IDESC_O = make_idesc(BM, HD, true);
            const uint64_t vd_base = make_desc(s32(v_sm), BN * 128, 1024);
            bool ok = true;
            int vs_ = 0, b = 0;
            uint32_t vpar = 0, bpar = 0;
            for (int i = 0; i < ntiles && ok; i++) {
                ok = bar_wait(p_full + 8 * b, bpar);
                if (!ok) break;
                ok = bar_wait(v_full + 8 * vs_, vpar);
                if (!ok) break;
                fence_async_smem();
                tc_fence_after();
                const uint64_t vd0 = vd_base + (uint64_t)((vs_ * KT_BYTES) >> 4);
                const uint32_t pa = tmem + COL_S + b * BN;
                if (elect_one()) {
                    if (i > 0) tc_mma_f16_ta_c<1>(tmem + COL_O, pa, vd0, IDESC_O);
                    else tc_mma_f16_ta_c<0>(tmem + COL_O, pa, vd0, IDESC_O);
#pragma unroll
                    for (int kk = 1; kk < BN / 16; kk++)
                        tc_mma_f16_ta_c<1>(tmem + COL_O, pa + 8 * kk, vd0 + (uint64_t)((kk * 2048) >> 4), IDESC_O);
                    tc_commit(pvb + 8 * b);
                    tc_commit(v_empty + 8 * vs_);
                }
                __syncwarp();
                if (++vs_ == VSL) { vs_ = 0; vpar ^= 1; }
                if (++b == S_BUFS) { b = 0; bpar ^= 1; }
            }
        }
    } else {
        // ------------------------------ K / V staging --------------------------------------
        const int nslots = side ? VSL : KSL;
        const uint32_t full = side ? v_full : k_full, empty = side ? v_empty : k_empty;
        uint8_t* ring = side ? v_sm : k_sm;
        auto wait_slot = [&](int i) -> bool {
            bool okw = true;
            if (i >= nslots) okw = bar_wait(empty + 8 * (i % nslots), (uint32_t)(((i / nslots) - 1) & 1));
            return okw;
        };
        if constexpr (KVK == Q27_KV_F16) {
            // fp16 rows need no conversion: cp.async writes them straight into the swizzled
            // operand layout and the slot's barrier is arrived when the copies have landed
            for (int i = 0; i < ntiles; i++) {
                if (!wait_slot(i)) break;
                const int st = i % nslots, nk = nkeys_of(i);
                const uint8_t* page = page_of(i);
                uint8_t* dst = ring + st * KT_BYTES;
#pragma unroll
                for (int n = 0; n < 16; n++) {
                    const int q = p + NPROD * n;
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
                if (nk < BN) __threadfence_block();        // the zeros, before the arrival below
                asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];"
                             ::"r"(full + 8 * st) : "memory");
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
        } else if constexpr (KVK == Q27_KV_T3) {
            // each thread decodes the two 50-byte blocks of one key of its team's tiles from
            // shared memory
            if (!raw_early && team < ntiles) issue_raw(team, page_of(team));
            for (int i = team; i < ntiles; i += 2) {
                // the page of the tile after this one, looked up now: the refill below must not
                // wait for the table
                const uint8_t* next_page = i + 2 < ntiles ? page_of(i + 2) : nullptr;
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                __syncwarp();                              // the warp's rows of tile i have landed
                RawHalf<KVK> rw0, rw1;
                {
                    const uint32_t* src = reinterpret_cast<const uint32_t*>(raw + team * RAW_BYTES + q * RAW_ROW + blk_off);
#pragma unroll
                    for (int k = 0; k < 13; k++) {
                        rw0.w[k] = src[k];
                        rw1.w[k] = src[12 + k];            // block 1 starts 2 bytes into word 12
                    }
                    rw0.w[13] = rw1.w[13] = 0;
                }
                // The warp's raw rows are refilled as soon as its lanes have read them: the copies
                // then have the decode below to land in. (Asked for after the decode, they cost
                // a trip to memory per tile, 0.4-0.8 us.)
                __syncwarp();
                if (i + 2 < ntiles) issue_raw(i + 2, next_page);
                if (!wait_slot(i)) break;
                const int st = i % nslots;
                half_store<KVK, 0>(rw0, ring + st * KT_BYTES, nkeys_of(i), q);
                half_store<KVK, 1>(rw1, ring + st * KT_BYTES, nkeys_of(i), q);
                fence_async_smem();
                bar_arrive(full + 8 * st);
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
        } else {
            // fp8: each thread converts its sixteen 8-byte pieces of the tile (they lie in the 16
            // rows its warp copied) from shared memory
            if (!raw_early) {
                if (ntiles > 0) issue_raw(0, page_of(0));
                if (ntiles > 1) issue_raw(1, page_of(1));
            }
            for (int i = 0; i < ntiles; i++) {
                const int buf = i & 1;
                // the copies of tile i have landed; those of tile i + 1 may still be on their way
                if (i + 1 < ntiles) asm volatile("cp.async.wait_group 1;" ::: "memory");
                else asm volatile("cp.async.wait_group 0;" ::: "memory");
                __syncwarp();
                RawHalf<KVK> rw;
#pragma unroll
                for (int n = 0; n < 16; n++)
                    rw.d[n] = *reinterpret_cast<const uint2*>(raw + buf * RAW_BYTES + (p + NPROD * n) * 8);
                __syncwarp();                              // the warp's rows are read: refill them
                if (i + 2 < ntiles) issue_raw(i + 2, page_of(i + 2));
                if (!wait_slot(i)) break;
                const int st = i % nslots;
                half_store<KVK>(rw, ring + st * KT_BYTES, nkeys_of(i), p);
                fence_async_smem();
                bar_arrive(full + 8 * st);
            }
            asm volatile("cp.async.wait_all;" ::: "memory");
        }
    }
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "n"(TMEM_COLS) : "memory");
    }
    if ((MODE == 1 || pb.piece >= 0) && *epi_bad == 0) {
        // the partial records of the live rows, a warp per row, 8-byte pieces (a record starts on
        // an 8-byte boundary): whole lines
        constexpr int OROT_PITCH = HD + 4;
        const float* o_st = reinterpret_cast<const float*>(k_sm);
        const int live = pb.live_rows();
        for (int r = warp; r < live; r += UMMA_THREADS / 32) {
            float* part = pb.row(r).part;
            if (!part) continue;
            const float* src = o_st + (size_t)r * OROT_PITCH;
            for (int q = lane; q < PART / 2; q += 32)
                reinterpret_cast<float2*>(part)[q] =
                    q == 0 ? make_float2(src[0], src[1]) : *reinterpret_cast<const float2*>(src + 2 + 2 * q);
        }
    }
    if (MODE == 0 && pb.piece < 0 && *epi_bad == 0) {
        // the normalised rows, half a row (one 128-group of the rotation) per warp at a time:
        // un-rotated if asked, then 512 contiguous bytes per store instruction
        constexpr int OROT_PITCH = HD + 4;
        float* o_rot = reinterpret_cast<float*>(k_sm);
        for (int gi = warp; gi < 2 * BM; gi += UMMA_THREADS / 32) {
            const RowInfo ri = pb.row(gi >> 1);
            if (!ri.out) continue;
            float* x = o_rot + (size_t)(gi >> 1) * OROT_PITCH + (gi & 1) * 128;
            if (wht & WHT_OUT) wht_group<true>(x, lane);
            reinterpret_cast<float4*>(ri.out + (gi & 1) * 128)[lane] = reinterpret_cast<const float4*>(x)[lane];
        }
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
    pb.sp = 0;
    // items in launch order: Q tile fastest, then kv head; whole items first, then the pieces
    const int id = blockIdx.x;
    int item = id;
    if (id >= a.n_full) {
        const int j = id - a.n_full;
        item = a.n_full + j / a.pieces;
        pb.piece = j % a.pieces;
    }
    pb.kvh = item / a.nx;
    pb.tile_t0 = a.t0 + (item % a.nx) * TOK_PER_TILE;
    const int item_hi = a.base_pos + min(pb.tile_t0 + TOK_PER_TILE, a.t_end);
    pb.lo = 0;
    pb.hi = item_hi;
    if (pb.piece >= 0) {               // tile-aligned key range of this piece
        const int tiles = (item_hi + BN - 1) / BN;
        pb.lo = (int)((int64_t)pb.piece * tiles / a.pieces) * BN;
        pb.hi = min(item_hi, (int)((int64_t)(pb.piece + 1) * tiles / a.pieces) * BN);
        if (pb.lo >= pb.hi) {           // fewer tiles than pieces: an empty range
            for (int r = threadIdx.x; r < BM; r += blockDim.x) {
                const RowInfo ri = pb.row(r);
                if (ri.part) { ri.part[0] = NEG_SENTINEL; ri.part[1] = 0.f; }
            }
            return;
        }
    }
    attn_tile<KVK, 0>(pb, a.ktab, a.vtab, a.n_kv, a.scale, a.wht, smem_raw);
}

// Merge the pieces of the split items: one block per (item, token), thread = dim, six heads.
__global__ void __launch_bounds__(HD)
k_prefill_fixup(const __grid_constant__ TileArgs a) {
    __shared__ float s_o[HD];
    pdl_wait();
    const int item = a.n_full + blockIdx.y;
    const int kvh = item / a.nx;
    const int t = a.t0 + (item % a.nx) * TOK_PER_TILE + blockIdx.x;
    if (t >= a.t_end) return;
#pragma unroll
    for (int j = 0; j < GQA; j++) {
        const int h = kvh * GQA + j;
        const float* pp = a.part + (((size_t)h * a.part_rows + (t - a.t0)) * PF_SPLIT_MAX) * PART;
        float mg = NEG_SENTINEL;
        for (int p = 0; p < a.pieces; p++) mg = fmaxf(mg, pp[(size_t)p * PART]);
        float lg = 0.f, acc = 0.f;
        for (int p = 0; p < a.pieces; p++) {
            const float ms = pp[(size_t)p * PART];
            if (ms == NEG_SENTINEL) continue;          // its accumulator was never written
            const float w = expf(ms - mg);
            lg += pp[(size_t)p * PART + 1] * w;
            acc += pp[(size_t)p * PART + 2 + threadIdx.x] * w;
        }
        float o = lg > 0.f ? acc / lg : 0.f;
        if (a.wht & WHT_OUT) {                    // the folded inverse rotation of wht_T on this head
            __syncthreads();
            s_o[threadIdx.x] = o;
            __syncthreads();
            if (threadIdx.x < 64) wht_group<true>(s_o + (threadIdx.x >> 5) * 128, threadIdx.x & 31);
            __syncthreads();
            o = s_o[threadIdx.x];
        }
        a.outT[(size_t)t * a.out_row + (size_t)h * HD + threadIdx.x] = o;
    }
}

template <int KVK>
__global__ void __launch_bounds__(UMMA_THREADS, 1)
k_verify_umma(const __grid_constant__ DevBatch b) {
    extern __shared__ uint8_t smem_raw[];
    pdl_trigger();               // the combine kernel may be scheduled; it waits for this grid
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
    attn_tile<KVK, 1>(pb, S.ktab, S.vtab, b.n_kv, b.scale, b.wht, smem_raw);
}

template <int KVK>
int set_attrs() {
    static DeviceOnce once;      // the attribute belongs to a device, not to the process
    return device_once(once, []() -> int {
        Q27_CUDA_TRY(cudaFuncSetAttribute(k_prefill_umma<KVK>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, UMMA_SMEM));
        Q27_CUDA_TRY(cudaFuncSetAttribute(k_verify_umma<KVK>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, UMMA_SMEM));
        return Q27_OK;
    });
}

} // namespace

int launch_prefill_umma(const float* qT, int q_stride, int q_row, const void* const* ktab,
                        const void* const* vtab, float* outT, int out_row, float* part,
                        int base_pos, int t0, int SB, int n_q, int n_kv, float scale,
                        int sm_count, cudaStream_t st, int kvk, int wht, bool* done) {
    *done = false;
    if (kind_known(kvk) && !kind_has_tensor_path(kvk)) return Q27_OK;   // served by the fp32 family
    if (kvk == Q27_KV_T3 && (n_kv & 3)) return Q27_OK;   // turbo3 rows are copied in 16-byte pieces: 400 n_kv / 4 bytes per row
    (void)n_q;
    // float4 loads of Q rows and float4 stores of output rows
    if ((q_stride & 3) || (q_row & 3) || (out_row & 3) || ((uintptr_t)qT & 15) || ((uintptr_t)outT & 15))
        return Q27_OK;
    TileArgs a{qT, ktab, vtab, outT, q_stride, q_row, out_row, base_pos, t0, t0 + SB, n_kv, scale,
               part, (SB + 15) / 16 * 16, (SB + TOK_PER_TILE - 1) / TOK_PER_TILE, 0, 1, wht};
    // One CTA per SM: the items beyond the last full wave would hold the machine for a whole
    // item time at partial occupancy. They are cut into P key ranges each when that pays: a
    // piece costs its share of the item's tiles plus a fixed ~32 tile-times (measured: pipeline
    // fill and drain, Q staging, scattered partial stores), the fix-up kernel ~10 more, against one
    // item time for leaving the tail whole (a row's scratch has room for 8 pieces).
    const int items = a.nx * n_kv;
    a.n_full = items;
    const int tail = items % sm_count;
    if (part && ((uintptr_t)part & 15) == 0 && tail > 0) {
        const int min_tiles = (base_pos + t0 + min(TOK_PER_TILE, SB) + BN - 1) / BN;
        const double item_tiles = (base_pos + t0 + 0.5 * SB) / BN;
        int best = 1;
        double best_cost = 0.95 * (item_tiles + 6.0);
        for (int P = 2; P <= PF_SPLIT_MAX && P <= min_tiles; P++) {
            const int rounds = (tail * P + sm_count - 1) / sm_count;
            const double cost = rounds * (item_tiles / P + 32.0) + 10.0;
            if (cost < best_cost) { best_cost = cost; best = P; }
        }
        if (best > 1) {
            a.n_full = items - tail;
            a.pieces = best;
        }
    }
    const int ncta = a.n_full + (items - a.n_full) * a.pieces;
    int rc;
    if (kvk == Q27_KV_F16) {
        if ((rc = set_attrs<Q27_KV_F16>())) return rc;
        k_prefill_umma<Q27_KV_F16><<<ncta, UMMA_THREADS, UMMA_SMEM, st>>>(a);
    } else if (kvk == Q27_KV_FP8) {
        if ((rc = set_attrs<Q27_KV_FP8>())) return rc;
        k_prefill_umma<Q27_KV_FP8><<<ncta, UMMA_THREADS, UMMA_SMEM, st>>>(a);
    } else if (kvk == Q27_KV_T3) {
        if ((rc = set_attrs<Q27_KV_T3>())) return rc;
        k_prefill_umma<Q27_KV_T3><<<ncta, UMMA_THREADS, UMMA_SMEM, st>>>(a);
    } else {
        return Q27_ERR_UNSUPPORTED_KIND;
    }
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    if (a.pieces > 1)
        Q27_CUDA_TRY(launch_pdl(k_prefill_fixup, dim3(TOK_PER_TILE, items - a.n_full), dim3(HD),
                                0, st, a));
    *done = true;
    return Q27_OK;
}


int read_umma_timeout_flag(int* out) {
    Q27_CUDA_TRY(cudaMemcpyFromSymbol(out, g_umma_timeout_flag, sizeof(int)));
    return Q27_OK;
}

int launch_verify_umma(DevBatch& b, int kvk, int sm_count, cudaStream_t st, bool* done,
                       int force_nsplit) {
    *done = false;
    if (kind_known(kvk) && !kind_has_tensor_path(kvk)) return Q27_OK;   // served by the fp32 family
    if (kvk == Q27_KV_T3 && (b.n_kv & 3)) return Q27_OK;   // turbo3 rows are copied in 16-byte pieces: 400 n_kv / 4 bytes per row
    if (b.q_stride & 3) return Q27_OK;
    for (int i = 0; i < b.nslots; i++)
        for (int t = 0; t < b.s[i].ntok; t++)
            if ((uintptr_t)b.s[i].q[t] & 15) return Q27_OK;
    // One CTA per SM at a time. When the (slot, kv head) pairs do not divide the machine, a
    // single wave leaves SMs idle (8 slots x 4 heads x 4 splits = 128 CTAs on 148 SMs); finer
    // splits over several waves fill it: take the smallest split count whose last wave is
    // nearly full.
    const int pairs = b.nslots * b.n_kv;
    int ns = force_nsplit;
    if (ns <= 0) {
        ns = sm_count / pairs;
        if (ns < 1) ns = 1;
        auto fill = [&](int n) {
            const int ctas = pairs * n, waves = (ctas + sm_count - 1) / sm_count;
            return (double)ctas / ((double)waves * sm_count);
        };
        double best = fill(ns);
        for (int n = ns + 1; n <= Q27_MAX_SPLITS && n <= 4 * ns + 4 && best < 0.95; n++)
            if (fill(n) > best + 0.02) { best = fill(n); ns = n; }
    }
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
    Q27_COUNT_LAUNCH();
    *done = true;
    return Q27_OK;
}

} // namespace q27b
