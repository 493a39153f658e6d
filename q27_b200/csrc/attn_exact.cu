// Exact (fp32 scalar) attention family: tiled split-KV partials, the log-sum-exp combine /
// merge kernels, and a scalar causal prefill. These kernels decode every cache element with the
// bit-exact decoders of common.cuh and do all arithmetic in fp32 with expf, so they are the
// engine's tight-tolerance path (the class of the reference's k_attn_fd2, src/spec3.cu:804-921,
// and k_attn_prefill_T, src/prefill.cu:2293-2388). The tensor-core kernels are checked
// against them on the GPU and against the CPU oracle.
#include "common.cuh"
#include "finish.cuh"
#include "p2p_exchange.cuh"
#include "wht.cuh"

namespace q27b {

namespace {

// without relocatable device code a __device__ variable is private to its translation unit:
// the one-kernel exchange below keeps its own timeout flag, ORed into the library's by the reader
__device__ int g_xchg1_timeout_flag = 0;
__device__ __forceinline__ void xchg_note_timeout() { atomicExch(&g_xchg1_timeout_flag, 8); }

// Split-KV partial of one (split, kv head, slot-lane), fp32 throughout, as a tiled two-phase
// loop over blocks of 32 keys that lives in shared memory:
//   phase 1  the block's K rows are decoded (bit-exact element decoders) into shared memory;
//            thread (head j, key k) -- warp j holds the 32 keys of head j -- forms one whole
//            dot product in dimension order, the warp takes the block maximum and sum with
//            shuffles, and the block's probabilities go to shared memory;
//   phase 2  the block's V rows take the K rows' place; thread d owns output dimension d of
//            all six heads and adds the 32 weighted rows in key order.
// The running (m, l) of head j live in the registers of warp j, the accumulators of dimension
// d in thread d: one state per CTA, nothing to merge at the end, and every sum has a fixed
// order, so results are run-to-run identical. Tolerance class of the reference's scalar decode
// (src/spec3.cu:804-921): exact element decode, fp32 FMA, expf.
constexpr int EXK = 32;                  // keys per block
constexpr int EX_THREADS = 256;          // = head_dim: one output dimension per thread
constexpr int EX_PITCH = HD + 1;         // odd pitch: rows read by 32 keys at once hit 32 banks

template <int FMT>
__device__ __forceinline__ void stage_rows(float (*tile)[EX_PITCH], const void* const* tab,
                                           int row0, int nrows, int n_kv, int kvh) {
    for (int i = threadIdx.x; i < EXK * (HD / 8); i += EX_THREADS) {
        const int k = i / (HD / 8), d0 = (i % (HD / 8)) * 8;
        float v[8];
        if (k < nrows) {
            const int p = row0 + k;
            load8_exact<FMT>(static_cast<const uint8_t*>(tab[p >> PAGE_SHIFT]), p & (PAGE - 1), n_kv,
                             kvh, d0, v);
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = 0.f;   // past the window: weight 0, value finite
        }
#pragma unroll
        for (int e = 0; e < 8; e++) tile[k][d0 + e] = v[e];
    }
}

template <int KF, int VF>   // storage formats of the K and V sides
__global__ void __launch_bounds__(EX_THREADS)
k_exact_partial(const __grid_constant__ DevBatch b) {
    const int sp = blockIdx.x, kvh = blockIdx.y;
    const int slot = blockIdx.z / b.max_ntok, t = blockIdx.z % b.max_ntok;
    const DevSlot& S = b.s[slot];
    if (t >= S.ntok) return;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // slot-wide chunking from the longest lane (all lanes share split boundaries)
    int max_len = 0;
    for (int u = 0; u < S.ntok; u++)
        max_len = max(max_len, local_len(__ldg(S.pos[u]), S.row_base, S.row_count));
    const int my_len = local_len(__ldg(S.pos[t]), S.row_base, S.row_count);
    const int chunk = split_chunk(max_len, b.nsplit, b.unit);
    const int lo = sp * chunk, hi = min(my_len, lo + chunk);

    float* dst0 = S.scratch + (((size_t)t * b.n_q + kvh * GQA) * b.nsplit + sp) * PART;
    if (lo >= hi) { // empty window: stamp the sentinel so the combine can skip it
        if (tid < GQA) {
            float* d = dst0 + (size_t)tid * b.nsplit * PART;
            d[0] = NEG_SENTINEL;
            d[1] = 0.f;
        }
        return;
    }

    __shared__ float s_q[GQA][HD];
    __shared__ float s_tile[EXK][EX_PITCH];
    __shared__ float s_p[GQA][EXK];
    __shared__ float s_shrink[GQA];
    for (int i = tid; i < GQA * HD; i += EX_THREADS)
        s_q[i / HD][i % HD] = S.q[t][(size_t)(kvh * GQA + i / HD) * b.q_stride + (i % HD)];
    if (b.wht & WHT_Q) {                          // the forward rotation of wht3, in place
        __syncthreads();
        for (int gi = warp; gi < GQA * 2; gi += EX_THREADS / 32) wht_group<false>(&s_q[0][0] + gi * 128, lane);
    }

    float m_run = NEG_SENTINEL, l_run = 0.f;      // head `warp` (warps 0..5), same in every lane
    float acc[GQA];                               // dimension `tid` of every head
#pragma unroll
    for (int j = 0; j < GQA; j++) acc[j] = 0.f;

    for (int r0 = lo; r0 < hi; r0 += EXK) {
        const int nrows = min(EXK, hi - r0);
        __syncthreads();                          // the tile's previous user is done (and s_q is in)
        stage_rows<KF>(s_tile, S.ktab, r0, nrows, b.n_kv, kvh);
        __syncthreads();
        if (warp < GQA) {
            float dot = 0.f;
#pragma unroll 8
            for (int d = 0; d < HD; d++) dot = fmaf(s_q[warp][d], s_tile[lane][d], dot);
            const float sc = lane < nrows ? dot * b.scale : NEG_SENTINEL;
            float bm = sc;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
            const float m_new = fmaxf(m_run, bm);             // finite: the block has a live key
            const float pk = lane < nrows ? expf(sc - m_new) : 0.f;
            float ps = pk;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            const float shrink = m_run == NEG_SENTINEL ? 0.f : expf(m_run - m_new);
            l_run = l_run * shrink + ps;
            m_run = m_new;
            s_p[warp][lane] = pk;
            if (lane == 0) s_shrink[warp] = shrink;
        }
        __syncthreads();                          // scores are out of the tile
        stage_rows<VF>(s_tile, S.vtab, r0, nrows, b.n_kv, kvh);
        __syncthreads();
#pragma unroll
        for (int j = 0; j < GQA; j++) {
            float a = acc[j] * s_shrink[j];
#pragma unroll 8
            for (int k = 0; k < EXK; k++) a = fmaf(s_p[j][k], s_tile[k][tid], a);
            acc[j] = a;
        }
    }
#pragma unroll
    for (int j = 0; j < GQA; j++) dst0[(size_t)j * b.nsplit * PART + 2 + tid] = acc[j];
    if (warp < GQA && lane == 0) {
        float* d = dst0 + (size_t)warp * b.nsplit * PART;
        d[0] = m_run;
        d[1] = l_run;
    }
}

// Log-sum-exp merge of the nsplit partials {m, l, acc[256]} at pp (stride PART) by a block of
// COMBINE_THREADS threads. The kernel sits on the step's critical path behind the partial
// kernel, so it is built around ONE round trip to L2: warp 0 fetches {m, l} of every split
// and, in the same breath, every thread fetches the accumulator pieces it will weigh (four
// groups of 128 threads each own every fourth split, two dims per thread; the first 80 splits
// -- all of them in the usual one-CTA-per-SM launches -- are in flight together, which keeps the
// block at 64 registers so that it fits beside a CTA of the partial kernel when it is launched
// early); warp 0 then forms the global max, the weights
// e^{m_s - M} and l; the groups' sums are added in the order that csrc/finish.cuh lays down for
// every merge of split records (same bits every run, and the same as a self-finished launch).
// Splits with weight 0 (sentinels) hold undefined accumulators: selected, never added. On
// return threads 0..255 hold the merged accumulator of dim threadIdx.x; mg / lg are valid in
// every thread.
constexpr int COMBINE_THREADS = 512;
__device__ __forceinline__ float combine_core(const float* __restrict__ pp, int nsplit, float& mg,
                                              float& lg) {
    __shared__ float s_w[Q27_MAX_SPLITS];
    __shared__ float s_ml[2];
    __shared__ float s_red[4][HD];
    const int tid = threadIdx.x;
    const int grp = tid >> 7, c = tid & 127;
    constexpr int EARLY = 20;            // loads per thread issued before the weights are known
    float2 v[EARLY];
#pragma unroll
    for (int k = 0; k < EARLY; k++) {
        const int sp = grp + 4 * k;
        v[k] = sp < nsplit ? *reinterpret_cast<const float2*>(pp + (size_t)sp * PART + 2 + 2 * c)
                           : make_float2(0.f, 0.f);
    }
    if (tid < 32) {
        float m, l;
        split_weights(pp, nsplit, tid, s_w, m, l);
        if (tid == 0) { s_ml[0] = m; s_ml[1] = l; }
    }
    __syncthreads();
    mg = s_ml[0];
    lg = s_ml[1];
    float ax = 0.f, ay = 0.f;            // group grp is running sum grp of the merge order
#pragma unroll
    for (int k = 0; k < EARLY; k++) {
        const int sp = grp + 4 * k;
        const float w = sp < nsplit ? s_w[sp] : 0.f;
        split_add(ax, v[k].x, w);
        split_add(ay, v[k].y, w);
    }
    for (int sp = grp + 4 * EARLY; sp < nsplit; sp += 4) {
        const float w = s_w[sp];
        const float2 u = *reinterpret_cast<const float2*>(pp + (size_t)sp * PART + 2 + 2 * c);
        split_add(ax, u.x, w);
        split_add(ay, u.y, w);
    }
    s_red[grp][2 * c] = ax;
    s_red[grp][2 * c + 1] = ay;
    __syncthreads();
    float a = 0.f;
    if (tid < HD) a = split_total(s_red[0][tid], s_red[1][tid], s_red[2][tid], s_red[3][tid]);
    return a;
}

// The inverse rotation of wht3 on one output head held one dim per thread (threads 0..255 of a
// block, every thread of the block calls): through shared memory, two warps, one group each.
__device__ __forceinline__ float unrotate_head(float v) {
    __shared__ float s_o[HD];
    const int tid = threadIdx.x;
    if (tid < HD) s_o[tid] = v;
    __syncthreads();
    if (tid < 64) wht_group<true>(s_o + (tid >> 5) * 128, tid & 31);
    __syncthreads();
    return tid < HD ? s_o[tid] : 0.f;
}

// Merge the nsplit partials of one (slot, lane, head). NORMALISE: write out = acc / l to the
// lane's output row; otherwise write the merged {m, l, acc} for a cross-GPU merge.
template <bool NORMALISE>
__global__ void __launch_bounds__(COMBINE_THREADS, 2)
k_combine(const __grid_constant__ DevBatch b, float* __restrict__ partial_out, int lanes_stride) {
    pdl_wait();                  // the partials come from the kernel before this one
    const int h = blockIdx.x, t = blockIdx.y, slot = blockIdx.z;
    const DevSlot& S = b.s[slot];
    if (t >= S.ntok) {
        if (!NORMALISE && t < lanes_stride) { // keep padded lanes well-defined for collectives
            float* d = partial_out + (((size_t)slot * lanes_stride + t) * b.n_q + h) * PART;
            for (int i = threadIdx.x; i < PART; i += blockDim.x)
                d[i] = i == 0 ? NEG_SENTINEL : 0.f;
        }
        return;
    }
    float mg, lg;
    const float a = combine_core(S.scratch + ((size_t)t * b.n_q + h) * b.nsplit * PART, b.nsplit, mg, lg);
    float o = __fmul_rn(a, split_inv(lg));
    if (NORMALISE && (b.wht & WHT_OUT)) o = unrotate_head(o);
    if (threadIdx.x < HD) {
        if (NORMALISE) {
            S.out[t][(size_t)h * HD + threadIdx.x] = o;
        } else {
            float* d = partial_out + (((size_t)slot * lanes_stride + t) * b.n_q + h) * PART;
            d[2 + threadIdx.x] = a;
            if (threadIdx.x == 0) { d[0] = mg; d[1] = lg; }
        }
    }
}

// k_combine<false> with the exchange fused in: the merged {m, l, acc} row of (slot, lane,
// head) goes straight into slot `rank` of EVERY rank's mailbox (peer stores over NVLink),
// and the last block publishes the epoch. Padded lanes get sentinel rows like everyone else.
__global__ void __launch_bounds__(COMBINE_THREADS, 2)
k_combine_push(const __grid_constant__ DevBatch b, const __grid_constant__ Peers peers_in,
               int lanes_stride) {
    pdl_trigger();               // the merge kernel may be scheduled; it waits for this grid
    pdl_wait();                  // the partials come from the kernel before this one
    Peers peers = peers_in;
    peers.epoch = xchg_epoch(peers.box[peers.rank], peers.world, peers.npairs, peers_in.epoch);
    const int h = blockIdx.x, t = blockIdx.y, slot = blockIdx.z;
    const DevSlot& S = b.s[slot];
    const size_t row = peers.slot_floats() + (((size_t)slot * lanes_stride + t) * b.n_q + h) * PART;
    if (t >= S.ntok) {
        for (int i = threadIdx.x; i < PART; i += blockDim.x) {
            const float v = i == 0 ? NEG_SENTINEL : 0.f;
            for (int r = 0; r < peers.world; r++) reinterpret_cast<float*>(peers.box[r])[row + i] = v;
        }
    } else {
        float mg, lg;
        const float a = combine_core(S.scratch + ((size_t)t * b.n_q + h) * b.nsplit * PART, b.nsplit,
                                     mg, lg);
        if (threadIdx.x < HD)
            for (int r = 0; r < peers.world; r++) {
                float* d = reinterpret_cast<float*>(peers.box[r]) + row;
                d[2 + threadIdx.x] = a;
                if (threadIdx.x == 0) { d[0] = mg; d[1] = lg; }
            }
    }
    xchg_publish(peers, gridDim.x * gridDim.y * gridDim.z);
}

// The whole exchange in ONE kernel, for launches whose blocks are all resident at once: block
// (head, lane, slot) merges its splits and stores the row into slot `rank` of every OTHER rank's
// mailbox, each float in one 64-bit word together with the step's epoch; it then reads the same
// row of every other rank from its own mailbox, polling (bounded) each word until it carries the
// epoch, merges the `world` rows and writes the output head -- un-rotated if asked. No fence and
// no flag: a word that shows the epoch is that step's value. A block waits only for words that
// its peers store before they wait themselves, so with all blocks resident nobody can be in
// anybody's way. Parities and the step word are those of the two-kernel exchange
// (p2p_exchange.cu).
__global__ void __launch_bounds__(COMBINE_THREADS, 2)
k_combine_xchg(const __grid_constant__ DevBatch b, const __grid_constant__ Peers peers,
               int lanes_stride, float* __restrict__ out) {
    pdl_wait();                  // the partials come from the kernel before this one
    uint8_t* own = peers.box[peers.rank];
    const uint32_t epoch = xchg_epoch(own, peers.world, peers.npairs, peers.epoch);
    const int par = epoch & 1;
    const int h = blockIdx.x, t = blockIdx.y, slot = blockIdx.z, tid = threadIdx.x;
    const DevSlot& S = b.s[slot];
    const int64_t w = ((int64_t)slot * lanes_stride + t) * b.n_q + h;
    __shared__ int s_ok;
    __shared__ float s_m[Q27_MAX_RANKS], s_l[Q27_MAX_RANKS];
    float a = 0.f, mg = NEG_SENTINEL, lg = 0.f;
    if (t < S.ntok)
        a = combine_core(S.scratch + ((size_t)t * b.n_q + h) * b.nsplit * PART, b.nsplit, mg, lg);
    if (tid == 0) s_ok = 1;
    // this rank's row into every other mailbox: word 0 = m, 1 = l, 2 + d = acc[d]
    if (tid < HD)
        for (int r = 0; r < peers.world; r++) {
            if (r == peers.rank) continue;
            uint8_t* d = peers.box[r] + xchg_ll_word(peers.world, peers.npairs, par, peers.rank, w);
            xchg_ll_store(d + 8 * (2 + tid), a, epoch);
            if (tid == 0) {
                xchg_ll_store(d, mg, epoch);
                xchg_ll_store(d + 8, lg, epoch);
            }
        }
    __syncthreads();             // s_ok
    // {m, l} of every rank (two threads per rank), then every thread's own accumulator words
    if (tid < 2 * peers.world) {
        const int r = tid >> 1, which = tid & 1;
        float v = which ? lg : mg;
        if (r != peers.rank &&
            !xchg_ll_load(own + xchg_ll_word(peers.world, peers.npairs, par, r, w) + 8 * which, epoch, v)) {
            s_ok = 0;
            xchg_note_timeout();
        }
        (which ? s_l : s_m)[r] = v;
    }
    __syncthreads();
    float m = NEG_SENTINEL;
    for (int s = 0; s < peers.world; s++) m = fmaxf(m, s_m[s]);
    float l = 0.f, o = 0.f;
    bool mine_ok = true;
    for (int s = 0; s < peers.world; s++) {
        if (s_m[s] == NEG_SENTINEL) continue;       // an empty shard: its accumulator is never read
        const float e = expf(s_m[s] - m);
        l += s_l[s] * e;
        if (tid < HD) {
            float v = a;
            if (s != peers.rank)
                mine_ok = xchg_ll_load(own + xchg_ll_word(peers.world, peers.npairs, par, s, w) + 8 * (2 + tid),
                                       epoch, v) && mine_ok;
            o += v * e;
        }
    }
    if (!mine_ok) { s_ok = 0; xchg_note_timeout(); }
    __syncthreads();
    const bool ok = s_ok != 0;                   // the same in every thread of the block
    o *= l > 0.f ? 1.0f / l : 0.f;
    if (b.wht & WHT_OUT) o = unrotate_head(o);
    if (ok && tid < HD) out[(size_t)w * HD + tid] = o;
    // completion, as in the two-kernel exchange: every block counts itself, the last one
    // records the exchange as done only if nobody gave up
    __syncthreads();
    if (tid == 0) {
        unsigned* ctr = reinterpret_cast<unsigned*>(own + xchg_counter_offset(peers.world, peers.npairs) + XCHG_MERGE_CTR);
        __threadfence();
        const unsigned nblocks = gridDim.x * gridDim.y * gridDim.z;
        const unsigned seen = atomicAdd(ctr, ok ? 1u : 0x10001u) + (ok ? 1u : 0x10001u);
        if ((seen & 0xffffu) == nblocks) {
            *ctr = 0;
            if ((seen >> 16) == 0)
                *reinterpret_cast<volatile uint32_t*>(own + xchg_counter_offset(peers.world, peers.npairs) + XCHG_STEP) = epoch;
        }
    }
}

// parts: [nparts][npairs][258] -> out [npairs][256] normalised
__global__ void __launch_bounds__(256)
k_merge(const float* __restrict__ parts, int nparts, int64_t npairs, float* __restrict__ out,
        int wht) {
    const int64_t w = blockIdx.x;
    float mg = NEG_SENTINEL;
    for (int s = 0; s < nparts; s++) mg = fmaxf(mg, parts[((size_t)s * npairs + w) * PART]);
    float lg = 0.f;
    for (int s = 0; s < nparts; s++) {
        const float* pp = parts + ((size_t)s * npairs + w) * PART;
        if (pp[0] != NEG_SENTINEL) lg += pp[1] * expf(pp[0] - mg);
    }
    const float inv = lg > 0.f ? 1.0f / lg : 0.f;
    const int d = threadIdx.x;                    // blockDim.x == HD
    float a = 0.f;
    for (int s = 0; s < nparts; s++) {
        const float* pp = parts + ((size_t)s * npairs + w) * PART;
        if (pp[0] != NEG_SENTINEL) a += pp[2 + d] * expf(pp[0] - mg);
    }
    float o = a * inv;
    if (wht & WHT_OUT) o = unrotate_head(o);
    out[(size_t)w * HD + d] = o;
}

// Scalar causal prefill: one warp per (token, kv head), six heads per warp, rows read
// straight from the paged cache (neighbouring tokens share them through L1/L2).
constexpr int PFX_WARPS = 8;
template <int KF, int VF>
__global__ void __launch_bounds__(PFX_WARPS * 32)
k_prefill_exact(const float* __restrict__ qT, int q_stride, int q_row,
                const void* const* __restrict__ ktab, const void* const* __restrict__ vtab,
                float* __restrict__ outT, int out_row, int base_pos, int t0, int t_end, int n_kv,
                float scale, int wht) {
    __shared__ float s_rot[PFX_WARPS][HD];        // one head at a time, for the folded rotations
    const int kvh = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = t0 + blockIdx.y * PFX_WARPS + warp;
    if (t >= t_end) return;
    // a head's 256 values, 8 per lane, through the rotation of wht_T and back
    auto rotate8 = [&](float (&x)[8], bool inv) {
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; i++) s_rot[warp][8 * lane + i] = x[i];
        __syncwarp();
        if (inv) { wht_group<true>(s_rot[warp], lane); wht_group<true>(s_rot[warp] + 128, lane); }
        else { wht_group<false>(s_rot[warp], lane); wht_group<false>(s_rot[warp] + 128, lane); }
#pragma unroll
        for (int i = 0; i < 8; i++) x[i] = s_rot[warp][8 * lane + i];
    };
    const int bound = base_pos + t + 1;
    float qr[GQA][8], m[GQA], l[GQA], acc[GQA][8];
#pragma unroll
    for (int j = 0; j < GQA; j++) {
        m[j] = NEG_SENTINEL;
        l[j] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            acc[j][i] = 0.f;
            qr[j][i] = qT[(size_t)t * q_row + (size_t)(kvh * GQA + j) * q_stride + 8 * lane + i];
        }
        if (wht & WHT_Q) rotate8(qr[j], false);
    }
    for (int p = 0; p < bound;) {
        const int pg = p >> PAGE_SHIFT;
        const int pend = min(bound, (pg + 1) << PAGE_SHIFT);
        const uint8_t* kpage = static_cast<const uint8_t*>(ktab[pg]);
        const uint8_t* vpage = static_cast<const uint8_t*>(vtab[pg]);
        for (; p < pend; p++) {
            float kv[8], vv[8];
            load8_exact<KF>(kpage, p & (PAGE - 1), n_kv, kvh, 8 * lane, kv);
            load8_exact<VF>(vpage, p & (PAGE - 1), n_kv, kvh, 8 * lane, vv);
#pragma unroll
            for (int j = 0; j < GQA; j++) {
                float d = 0.f;
#pragma unroll
                for (int i = 0; i < 8; i++) d = fmaf(qr[j][i], kv[i], d);
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
                d *= scale;
                const float mn = fmaxf(m[j], d);
                const float so = expf(m[j] - mn), w = expf(d - mn);
                l[j] = l[j] * so + w;
                m[j] = mn;
#pragma unroll
                for (int i = 0; i < 8; i++) acc[j][i] = acc[j][i] * so + w * vv[i];
            }
        }
    }
#pragma unroll
    for (int j = 0; j < GQA; j++) {
        const float inv = 1.0f / l[j];
#pragma unroll
        for (int i = 0; i < 8; i++) acc[j][i] *= inv;
        if (wht & WHT_OUT) rotate8(acc[j], true);
#pragma unroll
        for (int i = 0; i < 8; i++)
            outT[(size_t)t * out_row + (size_t)(kvh * GQA + j) * HD + 8 * lane + i] = acc[j][i];
    }
}

} // namespace

int launch_exact_partials(const DevBatch& b, int kvk, cudaStream_t st) {
    dim3 grid(b.nsplit, b.n_kv, b.nslots * b.max_ntok);
#define Q27_LAUNCH(KF, VF) k_exact_partial<KF, VF><<<grid, EX_THREADS, 0, st>>>(b)
    Q27_FOR_KIND(kvk, Q27_LAUNCH, return Q27_ERR_UNSUPPORTED_KIND)
#undef Q27_LAUNCH
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

int launch_combine(const DevBatch& b, float* partial_out, int lanes_stride, cudaStream_t st) {
    if (partial_out) {
        dim3 grid(b.n_q, lanes_stride, b.nslots);
        Q27_CUDA_TRY(launch_pdl(k_combine<false>, grid, dim3(COMBINE_THREADS), 0, st, b, partial_out, lanes_stride));
    } else {
        dim3 grid(b.n_q, b.max_ntok, b.nslots);
        Q27_CUDA_TRY(launch_pdl(k_combine<true>, grid, dim3(COMBINE_THREADS), 0, st, b, (float*)nullptr, b.max_ntok));
    }
    Q27_CUDA_TRY(cudaGetLastError());
    return Q27_OK;
}

int launch_combine_push(const DevBatch& b, const Peers& peers, int lanes_stride, cudaStream_t st) {
    dim3 grid(b.n_q, lanes_stride, b.nslots);
    Q27_CUDA_TRY(launch_pdl(k_combine_push, grid, dim3(COMBINE_THREADS), 0, st, b, peers, lanes_stride));
    Q27_CUDA_TRY(cudaGetLastError());
    return Q27_OK;
}

// 0 = the launch does not fit the machine at once (the caller runs push + merge instead)
int launch_combine_xchg(const DevBatch& b, const Peers& peers, int lanes_stride, float* out,
                        int sm_count, cudaStream_t st, bool* done) {
    *done = false;
    static std::atomic<int> per_sm[MAX_DEVICES];
    int dev = 0;
    Q27_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= MAX_DEVICES) return Q27_ERR_INVALID_ARG;
    int nb = per_sm[dev].load(std::memory_order_relaxed);
    if (nb == 0) {
        Q27_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, k_combine_xchg, COMBINE_THREADS, 0));
        per_sm[dev].store(nb > 0 ? nb : -1, std::memory_order_relaxed);
    }
    const int64_t blocks = (int64_t)b.n_q * lanes_stride * b.nslots;
    if (nb <= 0 || blocks > (int64_t)nb * sm_count || blocks > 0xffff) return Q27_OK;
    dim3 grid(b.n_q, lanes_stride, b.nslots);
    Q27_CUDA_TRY(launch_pdl(k_combine_xchg, grid, dim3(COMBINE_THREADS), 0, st, b, peers, lanes_stride, out));
    Q27_CUDA_TRY(cudaGetLastError());
    *done = true;
    return Q27_OK;
}

int read_xchg1_timeout_flag(int* out) {
    Q27_CUDA_TRY(cudaMemcpyFromSymbol(out, g_xchg1_timeout_flag, sizeof(int)));
    return Q27_OK;
}

int launch_merge(const float* parts, int nparts, int64_t npairs, float* out, int wht,
                 cudaStream_t st) {
    k_merge<<<(unsigned)npairs, HD, 0, st>>>(parts, nparts, npairs, out, wht);
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

int launch_prefill_exact(const float* qT, int q_stride, int q_row, const void* const* ktab,
                         const void* const* vtab, float* outT, int out_row, int base_pos, int t0,
                         int SB, int n_q, int n_kv, float scale, cudaStream_t st, int kvk, int wht) {
    (void)n_q;
    dim3 grid(n_kv, (SB + PFX_WARPS - 1) / PFX_WARPS);
    const int te = t0 + SB;
#define Q27_LAUNCH(KF, VF)                                        \
    k_prefill_exact<KF, VF><<<grid, PFX_WARPS * 32, 0, st>>>(     \
        qT, q_stride, q_row, ktab, vtab, outT, out_row, base_pos, t0, te, n_kv, scale, wht)
    Q27_FOR_KIND(kvk, Q27_LAUNCH, return Q27_ERR_UNSUPPORTED_KIND)
#undef Q27_LAUNCH
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

} // namespace q27b
