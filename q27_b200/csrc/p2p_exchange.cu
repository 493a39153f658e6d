// Exchange of split-KV partials between the GPUs of one node through peer memory.
//
// Every rank owns a MAILBOX in its own HBM, mapped into the other ranks' processes with CUDA
// IPC: [2 parities][world][npairs][258] floats, then [2][world] release flags. A rank's
// combine kernel stores each merged partial row into slot `rank` of every mailbox with plain
// peer stores the moment it is formed and, once all rows are out, writes the step's epoch
// into its flag in every mailbox. The merge kernel of each rank waits (bounded) until all
// `world` flags of the step's parity hold the epoch and merges what its own memory then
// holds. Nothing but these 258-float rows ever crosses NVLink, there is no host involvement
// per step, and no collective library call. Two parities: a rank can be one step ahead of a
// slow peer (it cannot be two ahead: its own merge of step e+1 needs the peer's push of e+1,
// which the peer issues after its merge of step e).
#include "p2p_exchange.cuh"
#include "wht.cuh"

namespace q27b {

namespace {

__device__ int g_xchg_timeout_flag = 0;

// box: this rank's own mailbox. out [npairs][256] normalised.
__global__ void __launch_bounds__(256)
k_merge_pushed(uint8_t* __restrict__ box, int world, int64_t npairs, uint32_t epoch_given,
               float* __restrict__ out, int wht) {
    pdl_wait();                  // this rank's own rows come from the kernel before this one
    const uint32_t epoch = xchg_epoch(box, world, npairs, epoch_given);
    const int par = epoch & 1;
    __shared__ int s_ok;
    if (threadIdx.x == 0) s_ok = 1;
    __syncthreads();
    if (threadIdx.x < world) {
        const uint8_t* f =
            box + xchg_flags_offset(world, npairs) + ((size_t)par * world + threadIdx.x) * XCHG_FLAG_STRIDE;
        bool got = false;
        for (int i = 0; i < (1 << 21); i++) {          // about half a second, then give up
            if (xchg_flag_acquire(f) == epoch) { got = true; break; }
            __nanosleep(200);
        }
        if (!got) { s_ok = 0; atomicExch(&g_xchg_timeout_flag, 4); }
    }
    __syncthreads();
    const bool ok = s_ok != 0;                    // the same in every thread of the block
    const int64_t w = blockIdx.x;
    __shared__ float s_o[HD];
    if (ok) {
        const float* parts = reinterpret_cast<const float*>(box) + (size_t)par * xchg_data_floats(world, npairs);
        float mg = NEG_SENTINEL;
        for (int s = 0; s < world; s++) mg = fmaxf(mg, __ldcg(parts + ((size_t)s * npairs + w) * PART));
        float lg = 0.f;
        for (int s = 0; s < world; s++) {
            const float* pp = parts + ((size_t)s * npairs + w) * PART;
            const float ms = __ldcg(pp);
            if (ms != NEG_SENTINEL) lg += __ldcg(pp + 1) * expf(ms - mg);
        }
        const float inv = lg > 0.f ? 1.0f / lg : 0.f;
        const int d = threadIdx.x;                // blockDim.x == HD
        float a = 0.f;
        for (int s = 0; s < world; s++) {
            const float* pp = parts + ((size_t)s * npairs + w) * PART;
            const float ms = __ldcg(pp);
            if (ms != NEG_SENTINEL) a += __ldcg(pp + 2 + d) * expf(ms - mg);
        }
        float o = a * inv;
        if (wht & WHT_OUT) {                      // the inverse rotation of wht3 on this head
            s_o[d] = o;
            __syncthreads();
            if (d < 64) wht_group<true>(s_o + (d >> 5) * 128, d & 31);
            __syncthreads();
            o = s_o[d];
        }
        out[(size_t)w * HD + d] = o;
    }
    // Every block, timed out or not, counts itself (a block that gave up adds a mark in the
    // upper half), so the counter always returns to zero. The last block records the exchange
    // as completed only if nobody gave up: after a timeout the step word stays where it was,
    // `out` is untouched in the blocks that gave up, and the same epoch can be tried again.
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* ctr = reinterpret_cast<unsigned*>(box + xchg_counter_offset(world, npairs) + XCHG_MERGE_CTR);
        __threadfence();
        const unsigned seen = atomicAdd(ctr, ok ? 1u : 0x10001u) + (ok ? 1u : 0x10001u);
        if ((seen & 0xffffu) == gridDim.x) {
            *ctr = 0;
            if ((seen >> 16) == 0)
                *reinterpret_cast<volatile uint32_t*>(box + xchg_counter_offset(world, npairs) + XCHG_STEP) = epoch;
        }
    }
}

} // namespace

size_t xchg_mailbox_bytes(int world, int64_t npairs) {
    return xchg_ll_offset(world, npairs) + (size_t)2 * world * (size_t)npairs * PART * 8 + 256;
}

int launch_merge_pushed(void* box, int world, int64_t npairs, uint32_t epoch, float* out,
                        int wht, cudaStream_t st) {
    if (npairs > 0xffff) return Q27_ERR_TOO_LARGE;   // the block counter keeps 16 bits
    Q27_CUDA_TRY(launch_pdl(k_merge_pushed, dim3((unsigned)npairs), dim3(HD), 0, st,
                            static_cast<uint8_t*>(box), world, npairs, epoch, out, wht));
    return Q27_OK;
}

int read_xchg_timeout_flag(int* out) {
    Q27_CUDA_TRY(cudaMemcpyFromSymbol(out, g_xchg_timeout_flag, sizeof(int)));
    return Q27_OK;
}

} // namespace q27b
