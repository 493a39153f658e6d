// Layout of a partial-exchange mailbox and what a kernel needs to publish into every rank's:
// [2 parities][world][npairs][258] floats, [2][world] release flags, one block counter.
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

struct Peers {
    uint8_t* box[Q27_MAX_RANKS];   // every rank's mailbox as mapped in this process
    int world, rank;
    int64_t npairs;
    uint32_t epoch;
    // float offset of this rank's slot for this epoch (the same in every mailbox)
    __host__ __device__ size_t slot_floats() const {
        return ((size_t)(epoch & 1) * world + rank) * (size_t)npairs * PART;
    }
};

// Called by every block of a kernel that has just stored its share of this rank's rows into
// all mailboxes: the last block to arrive publishes the epoch in every mailbox. The stores
// of each block are fenced system-wide before its count, and the publishing block fences
// again before the flags, so a rank that sees the flag sees the rows.
__device__ __forceinline__ void xchg_publish(const Peers& p, unsigned nblocks) {
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* counter = reinterpret_cast<unsigned*>(
            p.box[p.rank] + xchg_counter_offset(p.world, p.npairs));
        if (atomicAdd(counter, 1u) == nblocks - 1) {
            *counter = 0;
            __threadfence_system();
            for (int r = 0; r < p.world; r++)
                *reinterpret_cast<volatile uint32_t*>(
                    p.box[r] + xchg_flags_offset(p.world, p.npairs) +
                    ((size_t)(p.epoch & 1) * p.world + p.rank) * XCHG_FLAG_STRIDE) = p.epoch;
        }
    }
}

} // namespace q27b
