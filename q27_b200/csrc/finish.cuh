// A launch that finishes itself: the CTAs that share a group of split-KV partials wait for one
// another once their partials are written (counters in the caller's scratch, a cooperative
// launch so that every CTA is resident, bounded waits) and share the log-sum-exp merge
// (k_attn_fd_combine, src/spec3.cu:706-739) of the group's outputs in units of half heads.
// Used by the decode kernel (csrc/decode_mma.cu). The verify kernel (csrc/attn_umma.cu) keeps its
// separate combine launch: finishing itself measured 0.5-4 us slower per step at every size tried
// (the combine is launched early and its blocks are resident by the time the partials land).
#pragma once
#include "common.cuh"
#include "wht.cuh"

namespace q27b {

constexpr int FINISH_MAX_SPLITS = 127;   // the group counters live behind the last split's partials

// The two counters (arrivals, departures) of group `g` of a slot whose partials use `nsplit`
// splits: behind the partials, in the room the scratch keeps for 128 splits.
__device__ __forceinline__ unsigned long long* group_counters(float* scratch, int ntok, int n_q,
                                                              int nsplit, int g) {
    return reinterpret_cast<unsigned long long*>(scratch + (size_t)ntok * n_q * nsplit * PART) + 2 * (size_t)g;
}
// Any time before the first arrival, by one thread of every CTA of the group: words that do not
// carry the tag yet (first use of this scratch, or another call's partials written over them)
// get a zero count.
__device__ __forceinline__ void group_arm(unsigned long long* ctr) {
    ticket_arm(ctr);
    ticket_arm(ctr + 1);
}
// By ONE thread, after a block barrier that follows the CTA's last partial store: count this CTA
// in and wait (bounded, ~0.1 s) for all n. false = gave up.
__device__ __forceinline__ bool group_wait(unsigned long long* ctr, unsigned n) {
    __threadfence();
    atomicAdd(ctr, 1ull);
    for (int i = 0; i < (1 << 20); i++) {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(ctr) : "memory");
        if ((unsigned)(v & 0xffffu) >= n) return true;
        if (i > 64) __nanosleep(64);
    }
    return false;
}
// By ONE thread, after the CTA's last read of the group's partials: the last CTA to leave clears
// both counters for the next launch.
__device__ __forceinline__ void group_leave(unsigned long long* ctr, unsigned n) {
    const unsigned long long prev = atomicAdd(ctr + 1, 1ull);
    if ((unsigned)(prev & 0xffffu) + 1 == n) {
        atomicExch(ctr, TICKET_TAG << 16);
        atomicExch(ctr + 1, TICKET_TAG << 16);
    }
}

// ---- the merge arithmetic, one order everywhere -----------------------------------------------
// Every kernel that merges split records (the combine kernels of csrc/attn_exact.cu and the
// self-finishing launches below) forms the same sums in the same order with roundings that the
// compiler cannot contract, so that a step gives the same bits whichever of them finished it:
//   weights   w_s = e^{m_s - M} (0 for a split that saw no key), l = sum of l_s w_s: lane j of one
//             warp adds its splits j, j + 32, ... in order, then the xor tree;
//   outputs   four running sums per output, split s into sum s & 3, ascending s; then
//             ((a0 + a1) + a2) + a3, times 1 / l (0 where l is 0).
// Splits of weight 0 hold undefined accumulators: selected, never added.

// By one warp: the weights of the first `used` (1..128) records at `rec` (stride PART) into
// s_w[0..used); M and l in every lane. Records are read past L1.
__device__ __forceinline__ void split_weights(const float* __restrict__ rec, int used, int lane,
                                              float* __restrict__ s_w, float& m_out, float& l_out) {
    float2 ml[4];
    bool live[4];
    float m = NEG_SENTINEL;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const int sp = lane + 32 * k;
        ml[k] = __ldcg(reinterpret_cast<const float2*>(rec + (size_t)min(sp, used - 1) * PART));
        live[k] = sp < used && ml[k].x != NEG_SENTINEL;
        m = fmaxf(m, live[k] ? ml[k].x : NEG_SENTINEL);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float l = 0.f;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float w = live[k] ? expf(ml[k].x - m) : 0.f;
        if (lane + 32 * k < used) s_w[lane + 32 * k] = w;
        l = live[k] ? __fadd_rn(l, __fmul_rn(ml[k].y, w)) : l;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l = __fadd_rn(l, __shfl_xor_sync(0xffffffffu, l, off));
    m_out = m;
    l_out = l;
}
__device__ __forceinline__ void split_add(float& a, float v, float w) {
    a = w != 0.f ? __fadd_rn(a, __fmul_rn(v, w)) : a;
}
__device__ __forceinline__ float split_total(float a0, float a1, float a2, float a3) {
    return __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
}
__device__ __forceinline__ float split_inv(float l) { return l > 0.f ? 1.0f / l : 0.f; }

// One half head (128 outputs) of one (lane, head) from the first `used` of its split records at
// `rec`: every thread of a block of >= 256 threads calls. Warp 0 forms the weights; two threads
// per output (even / odd splits, sixteen loads in flight each) hold two of the four running
// sums each; with WHT_OUT the 128 values -- one group of the rotation -- are un-rotated before
// they go to dst[0..127]. `sm`: FINISH_SMEM_FLOATS floats nobody else uses meanwhile.
constexpr int FINISH_SMEM_FLOATS = 3 * 128 + 4;
__device__ __forceinline__ void merge_half_head(const float* __restrict__ rec, int used, int half,
                                                float* __restrict__ dst, int wht, float* sm) {
    float* s_w = sm;
    float* s_odd = sm + 128;          // [2][128]: the odd thread's sums 1 and 3, then the outputs
    float& s_inv = sm[384];
    const int tid = threadIdx.x, lane = tid & 31;
    const int d = half * 128 + (tid & 127), par = tid >> 7;   // par 0, 1: summing; beyond: idle
    __syncthreads();                                        // the unit before is done with `sm`
    if (tid < 32 && used > 0) {
        float m, l;
        split_weights(rec, used, lane, s_w, m, l);
        if (lane == 0) s_inv = split_inv(l);
    }
    __syncthreads();
    // (asking for the first splits before the weights are known, to share one trip to L2, measured
    // 0.4 us slower on the 4096-row decode: the loads then queue ahead of warp 0's {m, l} loads)
    float a[2] = {0.f, 0.f};                                // sums par and par + 2
    if (par < 2 && used > 0) {
        for (int s0 = par; s0 < used; s0 += 32) {           // this thread's splits: s0, s0 + 2, ...
            float v[16], w[16];
#pragma unroll
            for (int u = 0; u < 16; u++) {                  // every load is issued before any is used
                const int sp = min(s0 + 2 * u, used - 1);
                v[u] = __ldcg(rec + (size_t)sp * PART + 2 + d);
                w[u] = s0 + 2 * u < used ? s_w[sp] : 0.f;
            }
#pragma unroll
            for (int u = 0; u < 16; u++) split_add(a[u & 1], v[u], w[u]);   // (s0 + 2u) & 3 = par + 2 (u & 1)
        }
    }
    if (par == 1) {
        s_odd[tid & 127] = a[0];
        s_odd[128 + (tid & 127)] = a[1];
    }
    __syncthreads();
    // nothing attended (an empty shard): zeros, rotated like the combine kernel's
    if (tid < 128)
        s_odd[tid] = used > 0 ? __fmul_rn(split_total(a[0], s_odd[tid], a[1], s_odd[128 + tid]), s_inv) : 0.f;
    if (wht & WHT_OUT) {
        __syncthreads();
        if (tid < 32) wht_group<true>(s_odd, lane);
    }
    __syncthreads();
    if (tid < 128) dst[tid] = s_odd[tid];
}

} // namespace q27b
