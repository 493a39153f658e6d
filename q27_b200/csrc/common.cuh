// Shared definitions of the sm_100a attention engine: geometry, status plumbing, KV-format
// element decoders (bit-exact to the reference codec) and the per-launch argument bundles.
#pragma once
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <float.h>
#include <stdint.h>

#include <atomic>

#include "../../include/q27_b200.h"
#include "t3_tables.cuh"

namespace q27b {

constexpr int HD = Q27_HEAD_DIM;       // 256
constexpr int GQA = Q27_GQA;           // 6 query heads per KV head
constexpr int PAGE = Q27_KV_PAGE;      // 64 rows per page (src/cuda_common.h:70)
constexpr int PAGE_SHIFT = 6;
constexpr int PART = Q27_PART_STRIDE;  // 258 floats: m, l, acc[256]
constexpr int T3_BLK = Q27_T3_BLOCK_BYTES;
constexpr int T5_BLK = Q27_T5_BLOCK_BYTES;
constexpr int I8_BLK = Q27_I8_BLOCK_BYTES;

// Storage format of one side of a cache. The first three coincide with the KvKinds whose two
// sides are stored alike; from turbo3 up the V side is always turbo3 and only the K side
// varies (src/cuda_common.h:47-53).
enum RowFmt : int { RF_F16 = 0, RF_FP8 = 1, RF_T3 = 2, RF_T5 = 3, RF_I8 = 4 };
static_assert((int)RF_F16 == (int)Q27_KV_F16 && (int)RF_FP8 == (int)Q27_KV_FP8 && (int)RF_T3 == (int)Q27_KV_T3,
              "formats 0..2 are kinds 0..2");
__host__ __device__ constexpr int k_fmt(int kvk) {
    return kvk == Q27_KV_T3V ? RF_F16 : kvk == Q27_KV_T5K ? RF_T5 : kvk == Q27_KV_I8G64 ? RF_I8 : kvk;
}
__host__ __device__ constexpr int v_fmt(int kvk) { return kvk >= Q27_KV_T3 ? RF_T3 : kvk; }
__host__ __device__ constexpr int side_fmt(int kvk, bool is_v) { return is_v ? v_fmt(kvk) : k_fmt(kvk); }
inline bool kind_known(int kvk) { return kvk >= Q27_KV_F16 && kvk <= Q27_KV_I8G64; }
// kinds the tensor-core kernels read (both sides in one of the first three formats)
inline bool kind_has_tensor_path(int kvk) { return kvk >= Q27_KV_F16 && kvk <= Q27_KV_T3; }
constexpr float NEG_SENTINEL = -FLT_MAX; // "empty partial" marker (src/prefill.cu:1353-1362)

// Per-thread record of the last failing CUDA call (read by q27_last_cuda_error()).
extern thread_local int g_last_cuda_error;
// Kernels this library has launched from this thread (read by q27_launch_count()).
extern thread_local long long g_launch_count;
#define Q27_COUNT_LAUNCH() (++q27b::g_launch_count)

#define Q27_CUDA_TRY(expr)                                  \
    do {                                                    \
        cudaError_t e__ = (expr);                           \
        if (e__ != cudaSuccess) {                           \
            q27b::g_last_cuda_error = (int)e__;             \
            return Q27_ERR_CUDA;                            \
        }                                                   \
    } while (0)

// Per-device one-shot set-up (cudaFuncSetAttribute belongs to ONE device, so a process that
// drives several GPUs must repeat it on each). Threads that race on a device's first call all
// run `f`, which is idempotent, and publish the same flag: safe without a lock.
constexpr int MAX_DEVICES = 64;
struct DeviceOnce {
    std::atomic<unsigned char> done[MAX_DEVICES];
};
template <typename F>
inline int device_once(DeviceOnce& once, F&& f) {
    int dev = 0;
    Q27_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= MAX_DEVICES) return Q27_ERR_INVALID_ARG;
    if (once.done[dev].load(std::memory_order_acquire)) return Q27_OK;
    const int rc = f();
    if (rc == Q27_OK) once.done[dev].store(1, std::memory_order_release);
    return rc;
}

// One slot as the kernels see it (device-visible copy of q27_slot, passed by value as a
// __grid_constant__ parameter so no descriptor memory has to be allocated or copied).
struct DevSlot {
    const void* const* ktab;
    const void* const* vtab;
    const float* q[Q27_MAX_LANES];
    const int* pos[Q27_MAX_LANES];
    float* out[Q27_MAX_LANES];
    float* scratch;  // partials: [lane][head][nsplit][258]
    int ntok;
    int row_base;
    int row_count;
    int pad;
};
struct DevBatch {
    DevSlot s[Q27_MAX_SLOTS];
    int nslots;
    int nsplit;     // position splits per slot
    int max_ntok;   // widest slot (grid extent of the lane axis)
    int q_stride;
    int n_q;
    int n_kv;
    float scale;
    int unit;       // split granularity in rows (chunk is a multiple of it)
    int fuse;       // the partial kernel also merges the splits and writes the output rows
    int wht;        // rotation folded into the call (WHT_Q: Q heads as they are staged;
                    // WHT_OUT: output heads before they are written); 0 = the plain entries
};
static_assert(sizeof(DevBatch) <= 4000, "DevBatch must fit the kernel parameter space");

// Rows of the slot's tables a lane may read: [0, local_len). Lane t attends logical rows
// [0, pos_t]; the tables hold logical rows [row_base, row_base + row_count).
__host__ __device__ __forceinline__ int local_len(int pos, int row_base, int row_count) {
    long long n = (long long)pos + 1 - row_base;
    if (n < 0) n = 0;
    if (n > row_count) n = row_count;
    return (int)n;
}

// Split geometry shared by the partial kernels and the combine: the slot's longest lane
// decides the chunk; every lane uses the same chunk boundaries (one KV pass serves all).
__host__ __device__ __forceinline__ int split_chunk(int max_len, int nsplit, int unit) {
    int c = (max_len + nsplit - 1) / nsplit;
    c = (c + unit - 1) / unit * unit;
    return c < unit ? unit : c;
}

// Counters in caller scratch that nobody has to clear first: a 64-bit word carries a 48-bit
// tag above a 16-bit count. ticket_arm (any time before the first arrival, by every CTA that
// will use the word) gives a word without the tag a zero count; users count with atomicAdd and
// put the word back to the armed value when they are done with it.
constexpr unsigned long long TICKET_TAG = 0xD15C0A77E5B2ull;      // 48 bits
__device__ __forceinline__ void ticket_arm(unsigned long long* word) {
    const unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(word);
    if ((old >> 16) != TICKET_TAG) atomicCAS(word, old, TICKET_TAG << 16);   // losers change nothing
}

// ---- element decoders ---------------------------------------------------------------

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
    __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
    return __half2float(__half(hr));
}

// 8 consecutive elements (d0 multiple of 8) of one (row, kv head) slice as fp32.
// Bit-exact to kv2f (src/cuda_common.h:113-114), turbo3_deq_elem (src/turbo3.cuh:134),
// turbo5_deq_elem (src/turbo5.cuh:163-166) and i8g64_deq_elem (src/i8g64.cuh:68-72).
template <int FMT>
__device__ __forceinline__ void load8_exact(const uint8_t* __restrict__ page, int r, int n_kv,
                                            int kvh, int d0, float* o) {
    if constexpr (FMT == RF_F16) {
        const uint4 v = *reinterpret_cast<const uint4*>(
            page + ((size_t)(r * n_kv + kvh) * HD + d0) * 2);
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float2 f = __half22float2(h[i]);
            o[2 * i] = f.x;
            o[2 * i + 1] = f.y;
        }
    } else if constexpr (FMT == RF_FP8) {
        const uint2 v =
            *reinterpret_cast<const uint2*>(page + (size_t)(r * n_kv + kvh) * HD + d0);
        const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = e4m3_to_f32(b[i]);
    } else if constexpr (FMT == RF_T5) {
        // block = 82 B: fp16 norm @0, qs[64] @2 (low 4 bits, 2 per byte), hi[16] @66 (fifth bit)
        const uint8_t* blk = page + ((size_t)(r * n_kv + kvh) * 2 + (d0 >> 7)) * T5_BLK;
        const int j0 = d0 & 127;
        const float norm = __half2float(*reinterpret_cast<const __half*>(blk));
        const uint16_t* q16 = reinterpret_cast<const uint16_t*>(blk + 2 + (j0 >> 1));   // 2-aligned
        const uint32_t qs = (uint32_t)q16[0] | ((uint32_t)q16[1] << 16);
        const uint32_t hb = blk[66 + (j0 >> 3)];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int idx = ((qs >> (4 * i)) & 15) | (((hb >> i) & 1) << 4);
            o[i] = kT5Centroid[idx] * norm;
        }
    } else if constexpr (FMT == RF_I8) {
        // block = 132 B: int8 codes[128] @0, fp16 scale per 64 dims @128
        const uint8_t* blk = page + ((size_t)(r * n_kv + kvh) * 2 + (d0 >> 7)) * I8_BLK;
        const int j0 = d0 & 127;
        const float sc = __half2float(*reinterpret_cast<const __half*>(blk + 128 + 2 * (j0 >> 6)));
        const uint2 v = make_uint2(*reinterpret_cast<const uint32_t*>(blk + j0),
                                   *reinterpret_cast<const uint32_t*>(blk + j0 + 4));  // 4-aligned
        const int8_t* c = reinterpret_cast<const int8_t*>(&v);
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = (float)c[i] * sc;
    } else {
        static_assert(FMT == RF_T3, "unknown row format");
        // block = 50 B: fp16 norm @0, qs[32] @2 (2 bits/elem), signs[16] @34 (1 bit/elem)
        const uint8_t* blk = page + ((size_t)(r * n_kv + kvh) * 2 + (d0 >> 7)) * T3_BLK;
        const int j0 = d0 & 127;
        const float norm = __half2float(*reinterpret_cast<const __half*>(blk));
        const uint32_t qs = *reinterpret_cast<const uint16_t*>(blk + 2 + (j0 >> 2));
        const uint32_t sg = blk[34 + (j0 >> 3)];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            int idx = ((qs >> (2 * i)) & 3) | (((sg >> i) & 1) << 2);
            o[i] = kT3Centroid[idx] * norm;
        }
    }
}

// bytes per cache row of a storage format
__host__ __device__ __forceinline__ int row_bytes_of(int fmt, int n_kv) {
    return fmt == RF_F16 ? n_kv * HD * 2
         : fmt == RF_FP8 ? n_kv * HD
         : fmt == RF_T3  ? n_kv * 2 * T3_BLK
         : fmt == RF_T5  ? n_kv * 2 * T5_BLK
                         : n_kv * 2 * I8_BLK;
}

// Run CALL(KF, VF) with the storage formats of the K and V sides of a kind as compile-time
// constants; `otherwise` for a kind outside the enum.
#define Q27_FOR_KIND(kvk, CALL, otherwise)                      \
    switch (kvk) {                                              \
    case Q27_KV_F16: CALL(RF_F16, RF_F16); break;               \
    case Q27_KV_FP8: CALL(RF_FP8, RF_FP8); break;               \
    case Q27_KV_T3: CALL(RF_T3, RF_T3); break;                  \
    case Q27_KV_T3V: CALL(RF_F16, RF_T3); break;                \
    case Q27_KV_T5K: CALL(RF_T5, RF_T3); break;                 \
    case Q27_KV_I8G64: CALL(RF_I8, RF_T3); break;               \
    default: otherwise;                                         \
    }

// ---- launch entry points implemented per translation unit -----------------------------
// exact (fp32 scalar) family
int launch_exact_partials(const DevBatch& b, int kvk, cudaStream_t st);
// Programmatic dependent launch: the kernel may be scheduled while the kernel before it in
// the stream is still running (once all of that one's CTAs have called pdl_trigger or
// exited); it must call pdl_wait before it touches anything the earlier kernel writes.
// Hides the launch latency of the short combine / merge kernels behind the partial kernel.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    Q27_COUNT_LAUNCH();
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

int launch_combine(const DevBatch& b, float* partial_out, int lanes_stride, cudaStream_t st);
int launch_merge(const float* parts, int nparts, int64_t npairs, float* out, int wht,
                 cudaStream_t st);
// peer-memory exchange of partials (p2p_exchange.cu)
size_t xchg_mailbox_bytes(int world, int64_t npairs);
struct Peers;
int launch_combine_push(const DevBatch& b, const Peers& peers, int lanes_stride, cudaStream_t st);
int launch_merge_pushed(void* box, int world, int64_t npairs, uint32_t epoch, float* out,
                        int wht, cudaStream_t st);
int launch_combine_xchg(const DevBatch& b, const Peers& peers, int lanes_stride, float* out,
                        int sm_count, cudaStream_t st, bool* done);
int read_xchg_timeout_flag(int* out);
int read_xchg1_timeout_flag(int* out);
int read_umma_timeout_flag(int* out);
int launch_prefill_exact(const float* qT, int q_stride, int q_row, const void* const* ktab,
                         const void* const* vtab, float* outT, int out_row, int base_pos, int t0,
                         int SB, int n_q, int n_kv, float scale, cudaStream_t st, int kvk, int wht);
int launch_kv_dequant(const void* const* tab, int fmt, int row0, int nrows, int n_kv, float* out,
                      cudaStream_t st);
// [row_base, row_base + row_count): the logical rows the tables hold (rows outside are skipped)
int launch_kv_store_T(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                      int base_pos, int n_kv, int T, cudaStream_t st, int kvk, int row_base = 0,
                      int row_count = 0x7fffffff);
int launch_kv_store3(const float* const* k, const float* const* v, const int* const* pos,
                     void* const* ktab, void* const* vtab, int n_kv, int ntok, cudaStream_t st,
                     int kvk, int row_base = 0, int row_count = 0x7fffffff);
int launch_wht3(float* const* x, int n_heads, int stride, int ntok, bool inv, cudaStream_t st);
int launch_wht_T(float* x, int n_heads, int head_stride, int row_stride, int T, bool inv,
                 cudaStream_t st);
int launch_mk_tab(const void* base, size_t row_bytes, int rows, void** d_tab, cudaStream_t st);

} // namespace q27b
