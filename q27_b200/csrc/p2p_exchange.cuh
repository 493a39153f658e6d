// Layout of a partial-exchange mailbox and what a kernel needs to publish into every rank's:
// [2 parities][world][npairs][258] floats, [2][world] release flags, two block counters, the
// step word (the number of exchanges completed on this rank, for callers that let the device
// count the epochs so that a step's launches have constant arguments and can sit in a CUDA
// graph) and the epoch-tagged copy of the rows that the one-kernel exchange uses.
#pragma once
#include "common.cuh"

namespace q27b {

constexpr int XCHG_FLAG_STRIDE = 32;   // bytes between flags

__host__ __device__ inline size_t xchg_data_floats(int world, int64_t npairs) {
    return (size_t)world * (size_t)npairs * PART;
}
__host__ __device__ inline size_t xchg_flags_offset(int world, int64_t npairs) {
    const size_t b = 2 * xchg_data_floats(world, npairs) * sizeof(float);
    return (b + 255) & ~(size_t)255;
}
__host__ __device__ inline size_t xchg_counter_offset(int world, int64_t npairs) {
    return xchg_flags_offset(world, npairs) + (size_t)2 * world * XCHG_FLAG_STRIDE;
}

// byte offsets from the first counter: push counter 0, merge counter 64, step word 128
constexpr int XCHG_MERGE_CTR = 64, XCHG_STEP = 128;
// Behind the counters: the rows once more for the one-kernel exchange, every float packed with
// the step's epoch into ONE 64-bit word, [2 parities][world][npairs][258] words. A 64-bit store
// is a single access, so a word whose upper half holds the epoch carries that step's value:
// the receiver polls the words it needs and no fence orders anything (a system-scope fence
// costs ~5 us on this part, measured).
__host__ __device__ inline size_t xchg_ll_offset(int world, int64_t npairs) {
    return xchg_counter_offset(world, npairs) + 256;
}
__host__ __device__ inline size_t xchg_ll_word(int world, int64_t npairs, int parity, int src,
                                               int64_t row) {
    return xchg_ll_offset(world, npairs) + ((((size_t)parity * world + src) * (size_t)npairs + row) * PART) * 8;
}
__device__ __forceinline__ void xchg_ll_store(uint8_t* word, float v, uint32_t epoch) {
    const unsigned long long x = ((unsigned long long)epoch << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(word), "l"(x) : "memory");
}
// bounded wait for the word to carry `epoch`; false = gave up
__device__ __forceinline__ bool xchg_ll_load(const uint8_t* word, uint32_t epoch, float& v) {
    for (int i = 0; i < (1 << 22); i++) {                  // about half a second, then give up
        unsigned long long x;
        asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(x) : "l"(word) : "memory");
        if ((uint32_t)(x >> 32) == epoch) { v = __uint_as_float((uint32_t)x); return true; }
        if (i > 64) __nanosleep(100);
    }
    return false;
}

struct Peers {
    uint8_t* box[Q27_MAX_RANKS];   // every rank's mailbox as mapped in this process
    int world, rank;
    int64_t npairs;
    uint32_t epoch;                // 0: take it from the own mailbox's step word (+1)
    // float offset of this rank's slot for this epoch (the same in every mailbox)
    __host__ __device__ size_t slot_floats() const {
        return ((size_t)(epoch & 1) * world + rank) * (size_t)npairs * PART;
    }
};

// The epoch of the exchange a kernel belongs to: given by the host, or one past the number
// of exchanges this rank has completed (the merge kernel advances that word when its last
// block is done, and launches are stream-ordered behind it).
__device__ __forceinline__ uint32_t xchg_epoch(const uint8_t* own_box, int world, int64_t npairs,
                                               uint32_t given) {
    if (given) return given;
    return *reinterpret_cast<const volatile uint32_t*>(
               own_box + xchg_counter_offset(world, npairs) + XCHG_STEP) + 1u;
}

// Called by every block of a kernel that has just stored its share of this rank's rows into
// all mailboxes: the last block to arrive publishes the epoch in every mailbox. Blocks count
// themselves with a release/acquire atomic at GPU scope (after the block barrier, so it
// covers every thread's stores); only the publishing block pays for a system-scope fence,
// once, before the flags. The chain rows -> block count -> last block -> fence -> flag ->
// the peer's acquire load orders the rows before whatever the peer reads after its flag.
__device__ __forceinline__ void xchg_publish(const Peers& p, unsigned nblocks) {
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* counter = reinterpret_cast<unsigned*>(
            p.box[p.rank] + xchg_counter_offset(p.world, p.npairs));
        unsigned old;
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
        if (old == nblocks - 1) {
            *counter = 0;
            asm volatile("fence.acq_rel.sys;" ::: "memory");
            for (int r = 0; r < p.world; r++)
                asm volatile("st.relaxed.sys.global.u32 [%0], %1;"
                             ::"l"(p.box[r] + xchg_flags_offset(p.world, p.npairs) +
                                   ((size_t)(p.epoch & 1) * p.world + p.rank) * XCHG_FLAG_STRIDE),
                               "r"(p.epoch) : "memory");
        }
    }
}
// acquire load of a flag (pairs with the release store above)
__device__ __forceinline__ uint32_t xchg_flag_acquire(const uint8_t* addr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}

} // namespace q27b
