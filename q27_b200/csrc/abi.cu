// The extern "C" surface: argument validation, split planning and dispatch. Nothing here
// allocates or synchronises; every call only enqueues kernels on the caller's stream.
#include <limits.h>
#include <stdio.h>
#include <string.h>

#include "common.cuh"
#include "p2p_exchange.cuh"
#include "attn_umma.cuh"
#include "decode_mma.cuh"
#include "wht.cuh"

namespace q27b {
thread_local int g_last_cuda_error = 0;
thread_local long long g_launch_count = 0;

namespace {

// Per-device caches below are filled on first use; threads that race on a device's first call
// compute and publish the same value (relaxed atomics), so concurrent first calls are safe.
int sm_count() {
    static std::atomic<int> cached[MAX_DEVICES];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return 148;
    int v = cached[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
            v = 148;
        cached[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

int check_geometry(int q_stride, int n_q, int n_kv, int head_dim, int kvk) {
    if (!kind_known(kvk)) return Q27_ERR_UNSUPPORTED_KIND;
    if (head_dim != HD || n_kv < 1 || n_kv > 8 || n_q != GQA * n_kv) return Q27_ERR_UNSUPPORTED_WIDTH;
    if (q_stride < HD) return Q27_ERR_INVALID_ARG;
    return Q27_OK;
}

// Copy and validate the caller's slot descriptors into the by-value kernel bundle.
int build_batch(const q27_slot* slots, int nslots, int q_stride, int n_q, int n_kv, int head_dim,
                float scale, int kvk, bool need_out, DevBatch& b) {
    int rc = check_geometry(q_stride, n_q, n_kv, head_dim, kvk);
    if (rc) return rc;
    if (!slots || nslots < 1) return Q27_ERR_INVALID_ARG;
    if (nslots > Q27_MAX_SLOTS) return Q27_ERR_UNSUPPORTED_WIDTH;
    b.nslots = nslots;
    b.max_ntok = 0;
    int total_lanes = 0;
    for (int i = 0; i < nslots; i++) {
        const q27_slot& s = slots[i];
        if (s.ntok < 1 || s.ntok > Q27_MAX_LANES) return Q27_ERR_UNSUPPORTED_WIDTH;
        if (!s.ktab || !s.vtab || !s.scratch || s.row_base < 0 || s.row_count < 0)
            return Q27_ERR_INVALID_ARG;
        DevSlot& d = b.s[i];
        d.ktab = s.ktab;
        d.vtab = s.vtab;
        d.scratch = s.scratch;
        d.ntok = s.ntok;
        d.row_base = s.row_base;
        d.row_count = s.row_count;
        d.pad = 0;
        for (int t = 0; t < Q27_MAX_LANES; t++) {
            const bool live = t < s.ntok;
            if (live && (!s.q.p[t] || !s.pos.p[t] || (need_out && !s.out.p[t])))
                return Q27_ERR_INVALID_ARG;
            d.q[t] = live ? s.q.p[t] : nullptr; // dead slots may hold garbage: never forwarded
            d.pos[t] = live ? s.pos.p[t] : nullptr;
            d.out[t] = live ? s.out.p[t] : nullptr;
        }
        b.max_ntok = s.ntok > b.max_ntok ? s.ntok : b.max_ntok;
        total_lanes += s.ntok;
    }
    for (int i = nslots; i < Q27_MAX_SLOTS; i++) b.s[i] = DevSlot{};
    b.q_stride = q_stride;
    b.n_q = n_q;
    b.n_kv = n_kv;
    b.scale = scale;
    b.unit = 32;
    b.fuse = 0;
    b.wht = 0;
    (void)total_lanes;
    return Q27_OK;
}

enum Family { FAM_AUTO = 0, FAM_EXACT = 1 };

// Optional measurement hook: when set, the split-KV partial kernel of every decode call
// made by this thread is bracketed by these two events on the launch stream.
thread_local cudaEvent_t g_ev_start = nullptr, g_ev_stop = nullptr;

int run_decode(const q27_slot* slots, int nslots, int lanes_stride, int q_stride, int n_q, int n_kv,
               int head_dim, float scale, float* partial_out, void* stream, int kvk, Family fam,
               const Peers* peers = nullptr, int wht = 0, float* xchg_out = nullptr) {
    DevBatch b;
    int rc = build_batch(slots, nslots, q_stride, n_q, n_kv, head_dim, scale, kvk,
                         partial_out == nullptr && peers == nullptr, b);
    if (rc) return rc;
    b.wht = wht;
    if ((partial_out || peers) && (lanes_stride < b.max_ntok || lanes_stride > Q27_MAX_LANES))
        return Q27_ERR_INVALID_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int sms = sm_count();
    bool done = false;
    if (g_ev_start) Q27_CUDA_TRY(cudaEventRecord(g_ev_start, st));
    if (fam == FAM_AUTO) {
        // two or more lanes: one pass over the cache for all of them (tcgen05 tile kernel);
        // a single lane: the mma.sync streaming kernel
        if (b.max_ntok >= 2) rc = launch_verify_umma(b, kvk, sms, st, &done);
        if (rc) return rc;
        if (!done) rc = launch_decode_mma(b, kvk, sms, partial_out == nullptr && peers == nullptr,
                                          st, &done);
        if (rc) return rc;
    }
    if (!done) {
        // exact family: one CTA per (split, kv head, lane)
        int lanes = b.nslots * b.max_ntok;
        int ns = (16 * sms) / (n_kv * lanes);
        b.nsplit = ns < 8 ? 8 : ns > Q27_MAX_SPLITS ? Q27_MAX_SPLITS : ns;
        b.unit = 32;
        rc = launch_exact_partials(b, kvk, st);
        if (rc) return rc;
    }
    if (g_ev_stop) Q27_CUDA_TRY(cudaEventRecord(g_ev_stop, st));
    if (peers && xchg_out) {
        // the whole exchange in one kernel when its blocks are all resident at once, else the
        // push kernel followed by the merge kernel
        bool one = false;
        rc = launch_combine_xchg(b, *peers, lanes_stride, xchg_out, sms, st, &one);
        if (rc || one) return rc;
        rc = launch_combine_push(b, *peers, lanes_stride, st);
        if (rc) return rc;
        return launch_merge_pushed(peers->box[peers->rank], peers->world, peers->npairs, peers->epoch,
                                   xchg_out, wht & WHT_OUT, st);
    }
    if (peers) return launch_combine_push(b, *peers, lanes_stride, st);
    if (b.fuse) return Q27_OK;       // the partial kernel has merged and normalised already
    return launch_combine(b, partial_out, partial_out ? lanes_stride : b.max_ntok, st);
}

q27_slot single_slot(const q27_CP3* q, const void* const* ktab, const void* const* vtab,
                     const q27_P3* out, float* scratch, const q27_IP3* pos, int ntok) {
    q27_slot s{};
    s.ktab = ktab;
    s.vtab = vtab;
    if (q) s.q = *q;
    if (pos) s.pos = *pos;
    if (out) s.out = *out;
    s.scratch = scratch;
    s.ntok = ntok;
    s.row_base = 0;
    s.row_count = INT_MAX;
    return s;
}

// ---- scratch that nobody has to allocate ---------------------------------------------------
// Split-KV partials for the no-allocation decode entry: Q27_NOALLOC_MAX_LANES lanes x 24
// heads x 128 splits x 258 floats. Lives in the library image: every GPU that loads the
// library holds these bytes until the process exits. In host code `g_noalloc_scratch` is
// only a handle; the device address comes from cudaGetSymbolAddress, once per device.
constexpr size_t NOALLOC_FLOATS =
    (size_t)Q27_NOALLOC_MAX_LANES * 24 * Q27_MAX_SPLITS * Q27_PART_STRIDE;
static __device__ __align__(256) float g_noalloc_scratch[NOALLOC_FLOATS];

// Device address of the static scratch on the current device (set up on first use).
int noalloc_scratch_ptr(float** out) {
    static std::atomic<float*> by_device[MAX_DEVICES];
    int dev = 0;
    Q27_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= MAX_DEVICES) return Q27_ERR_INVALID_ARG;
    float* p = by_device[dev].load(std::memory_order_relaxed);
    if (!p) {
        Q27_CUDA_TRY(cudaGetSymbolAddress((void**)&p, g_noalloc_scratch));
        by_device[dev].store(p, std::memory_order_relaxed);
    }
    *out = p;
    return Q27_OK;
}

} // namespace
} // namespace q27b

using namespace q27b;

extern "C" {

const char* q27_status_string(int status) {
    switch (status) {
    case Q27_OK: return "ok";
    case Q27_ERR_INVALID_ARG: return "invalid argument";
    case Q27_ERR_UNSUPPORTED_KIND: return "unsupported KV kind (refused, not mis-read)";
    case Q27_ERR_UNSUPPORTED_WIDTH: return "unsupported width or geometry";
    case Q27_ERR_CUDA: return "CUDA error (see q27_last_cuda_error)";
    case Q27_ERR_TOO_LARGE: return "size exceeds a fixed capacity";
    default: return "unknown status";
    }
}

int q27_last_cuda_error(void) { return g_last_cuda_error; }

long long q27_launch_count(void) { return g_launch_count; }

int q27_device_arch(void) {
    int dev = 0, mj = 0, mn = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&mj, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
    if (cudaDeviceGetAttribute(&mn, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return 0;
    return (mj == 10 && mn == 0) ? 1000 : 0; // the image holds sm_100a code only
}

int64_t q27_kv_row_bytes_side(int kvk, int n_kv_heads, int is_v) {
    if (!kind_known(kvk)) return -1;
    return row_bytes_of(side_fmt(kvk, is_v != 0), n_kv_heads);
}

int64_t q27_kv_row_bytes(int kvk, int n_kv_heads) { return q27_kv_row_bytes_side(kvk, n_kv_heads, 0); }

int64_t q27_decode_scratch_floats(int ntok, int n_q_heads) {
    return (int64_t)ntok * n_q_heads * Q27_MAX_SPLITS * Q27_PART_STRIDE;
}

int64_t q27_prefill_part_floats(int SB, int n_q_heads) {
    return (int64_t)n_q_heads * ((SB + 15) / 16 * 16) * Q27_PF_SPLIT_MAX * Q27_PART_STRIDE;
}

static int decode3(const q27_CP3* q, int q_stride, const void* const* ktab,
                   const void* const* vtab, const q27_P3* out, float* scratch, const q27_IP3* pos,
                   int n_q_heads, int n_kv_heads, int head_dim, float scale, void* stream, int ntok,
                   int kvk, int wht) {
    if (!q || !out || !pos) return Q27_ERR_INVALID_ARG;
    if (ntok < 1 || ntok > Q27_MAX_LANES) return Q27_ERR_UNSUPPORTED_WIDTH;
    q27_slot s = single_slot(q, ktab, vtab, out, scratch, pos, ntok);
    return run_decode(&s, 1, 0, q_stride, n_q_heads, n_kv_heads, head_dim, scale, nullptr, stream,
                      kvk, FAM_AUTO, nullptr, wht);
}

int q27_attn_decode3(const q27_CP3* q, int q_stride, const void* const* ktab,
                     const void* const* vtab, const q27_P3* out, float* scratch,
                     const q27_IP3* pos, int max_ctx, int n_q_heads, int n_kv_heads,
                     int head_dim, float scale, void* stream, int ntok, int kvk) {
    (void)max_ctx;
    return decode3(q, q_stride, ktab, vtab, out, scratch, pos, n_q_heads, n_kv_heads, head_dim,
                   scale, stream, ntok, kvk, 0);
}

int q27_attn_decode3_wht(const q27_CP3* q, int q_stride, const void* const* ktab,
                         const void* const* vtab, const q27_P3* out, float* scratch,
                         const q27_IP3* pos, int max_ctx, int n_q_heads, int n_kv_heads,
                         int head_dim, float scale, void* stream, int ntok, int kvk) {
    (void)max_ctx;
    return decode3(q, q_stride, ktab, vtab, out, scratch, pos, n_q_heads, n_kv_heads, head_dim,
                   scale, stream, ntok, kvk, wht_flags_for(kvk));
}

int q27_attn_decode(const float* q, int q_stride, const void* const* ktab,
                    const void* const* vtab, float* out, float* scratch, const int* d_pos,
                    int max_ctx, int n_q_heads, int n_kv_heads, int head_dim, float scale,
                    void* stream, int kvk) {
    q27_CP3 qp{};
    q27_P3 op{};
    q27_IP3 pp{};
    qp.p[0] = q;
    op.p[0] = out;
    pp.p[0] = d_pos;
    return q27_attn_decode3(&qp, q_stride, ktab, vtab, &op, scratch, &pp, max_ctx, n_q_heads,
                            n_kv_heads, head_dim, scale, stream, 1, kvk);
}

int q27_attn_verify_partials(const q27_CP3* q, int q_stride, const void* const* ktab,
                             const void* const* vtab, float* part, const q27_IP3* pos,
                             int n_kv_heads, int gqa, int head_dim, float scale, int ns, int ntok,
                             void* stream, int kvk) {
    if (!q || !pos || !part) return Q27_ERR_INVALID_ARG;
    if (gqa != GQA || ntok < 1 || ntok > Q27_MAX_LANES || ns < 1 || ns > Q27_MAX_SPLITS)
        return Q27_ERR_UNSUPPORTED_WIDTH;
    q27_slot s = single_slot(q, ktab, vtab, nullptr, part, pos, ntok);
    DevBatch b;
    int rc = build_batch(&s, 1, q_stride, gqa * n_kv_heads, n_kv_heads, head_dim, scale, kvk, false, b);
    if (rc) return rc;
    bool done = false;
    rc = launch_verify_umma(b, kvk, sm_count(), static_cast<cudaStream_t>(stream), &done, ns);
    if (rc) return rc;
    return done ? Q27_OK : Q27_ERR_UNSUPPORTED_WIDTH;
}

int q27_attn_decode3_noalloc(const q27_CP3* q, int q_stride, const void* const* ktab,
                             const void* const* vtab, const q27_P3* out, const q27_IP3* pos,
                             int n_q_heads, int n_kv_heads, int head_dim, float scale,
                             void* stream, int ntok, int kvk) {
    if (!q || !out || !pos) return Q27_ERR_INVALID_ARG;
    if (ntok < 1) return Q27_ERR_UNSUPPORTED_WIDTH;
    if (ntok > Q27_NOALLOC_MAX_LANES || n_q_heads > 24) return Q27_ERR_TOO_LARGE;
    float* scratch = nullptr;
    int rc = noalloc_scratch_ptr(&scratch);
    if (rc) return rc;
    q27_slot s = single_slot(q, ktab, vtab, out, scratch, pos, ntok);
    return run_decode(&s, 1, 0, q_stride, n_q_heads, n_kv_heads, head_dim, scale, nullptr, stream,
                      kvk, FAM_AUTO);
}

int q27_attn_decode_batched(const q27_slot* slots, int nslots, int q_stride, int n_q_heads,
                            int n_kv_heads, int head_dim, float scale, void* stream, int kvk) {
    return run_decode(slots, nslots, 0, q_stride, n_q_heads, n_kv_heads, head_dim, scale, nullptr,
                      stream, kvk, FAM_AUTO);
}

int q27_attn_decode_batched_wht(const q27_slot* slots, int nslots, int q_stride, int n_q_heads,
                                int n_kv_heads, int head_dim, float scale, void* stream, int kvk,
                                int exact) {
    return run_decode(slots, nslots, 0, q_stride, n_q_heads, n_kv_heads, head_dim, scale, nullptr,
                      stream, kvk, exact ? FAM_EXACT : FAM_AUTO, nullptr, wht_flags_for(kvk));
}

int q27_attn_decode_batched_exact(const q27_slot* slots, int nslots, int q_stride, int n_q_heads,
                                  int n_kv_heads, int head_dim, float scale, void* stream,
                                  int kvk) {
    return run_decode(slots, nslots, 0, q_stride, n_q_heads, n_kv_heads, head_dim, scale, nullptr,
                      stream, kvk, FAM_EXACT);
}

int q27_attn_decode_partial(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                            int n_q_heads, int n_kv_heads, int head_dim, float scale,
                            float* partial_out, void* stream, int kvk) {
    if (!partial_out) return Q27_ERR_INVALID_ARG;
    return run_decode(slots, nslots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim, scale,
                      partial_out, stream, kvk, FAM_AUTO);
}

int q27_attn_decode_partial_wht(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                                int n_q_heads, int n_kv_heads, int head_dim, float scale,
                                float* partial_out, void* stream, int kvk) {
    if (!partial_out) return Q27_ERR_INVALID_ARG;
    return run_decode(slots, nslots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim, scale,
                      partial_out, stream, kvk, FAM_AUTO, nullptr, wht_flags_for(kvk) & WHT_Q);
}

static int merge_partials(const float* parts, int nparts, int64_t npairs, float* out, void* stream,
                          int wht) {
    if (!parts || !out || nparts < 1 || npairs < 0) return Q27_ERR_INVALID_ARG;
    if (npairs == 0) return Q27_OK;
    if (npairs > INT_MAX) return Q27_ERR_TOO_LARGE;
    return launch_merge(parts, nparts, npairs, out, wht, static_cast<cudaStream_t>(stream));
}

int q27_attn_merge_partials(const float* parts, int nparts, int64_t npairs, float* out,
                            void* stream) {
    return merge_partials(parts, nparts, npairs, out, stream, 0);
}

int q27_attn_merge_partials_wht(const float* parts, int nparts, int64_t npairs, float* out,
                                void* stream, int kvk) {
    if (!kind_known(kvk)) return Q27_ERR_UNSUPPORTED_KIND;
    return merge_partials(parts, nparts, npairs, out, stream, wht_flags_for(kvk) & WHT_OUT);
}

static int prefill_T(const float* qT, int q_stride, int q_row, const void* const* ktab,
                     const void* const* vtab, float* outT, int out_row, float* part, int base_pos,
                     int t0, int SB, int n_q_heads, int n_kv_heads, int head_dim, float scale,
                     void* stream, int kvk, bool exact, int wht) {
    int rc = check_geometry(q_stride, n_q_heads, n_kv_heads, head_dim, kvk);
    if (rc) return rc;
    if (!qT || !ktab || !vtab || !outT || base_pos < 0 || t0 < 0 || SB < 0 ||
        q_row < n_q_heads * HD || out_row < n_q_heads * HD)
        return Q27_ERR_INVALID_ARG;
    if (SB == 0) return Q27_OK;
    if (!exact) {
        bool done = false;
        rc = launch_prefill_umma(qT, q_stride, q_row, ktab, vtab, outT, out_row, part, base_pos, t0,
                                 SB, n_q_heads, n_kv_heads, scale, sm_count(),
                                 static_cast<cudaStream_t>(stream), kvk, wht, &done);
        if (rc || done) return rc;
    }
    return launch_prefill_exact(qT, q_stride, q_row, ktab, vtab, outT, out_row, base_pos, t0, SB,
                                n_q_heads, n_kv_heads, scale, static_cast<cudaStream_t>(stream),
                                kvk, wht);
}

int q27_attn_prefill_T_exact(const float* qT, int q_stride, int q_row, const void* const* ktab,
                             const void* const* vtab, float* outT, int out_row, float* part,
                             int base_pos, int t0, int SB, int n_q_heads, int n_kv_heads,
                             int head_dim, float scale, void* stream, int kvk) {
    return prefill_T(qT, q_stride, q_row, ktab, vtab, outT, out_row, part, base_pos, t0, SB,
                     n_q_heads, n_kv_heads, head_dim, scale, stream, kvk, true, 0);
}

int q27_attn_prefill_T(const float* qT, int q_stride, int q_row, const void* const* ktab,
                       const void* const* vtab, float* outT, int out_row, float* part,
                       int base_pos, int t0, int SB, int n_q_heads, int n_kv_heads,
                       int head_dim, float scale, void* stream, int kvk) {
    return prefill_T(qT, q_stride, q_row, ktab, vtab, outT, out_row, part, base_pos, t0, SB,
                     n_q_heads, n_kv_heads, head_dim, scale, stream, kvk, false, 0);
}

int q27_attn_prefill_T_wht(const float* qT, int q_stride, int q_row, const void* const* ktab,
                           const void* const* vtab, float* outT, int out_row, float* part,
                           int base_pos, int t0, int SB, int n_q_heads, int n_kv_heads,
                           int head_dim, float scale, void* stream, int kvk, int exact) {
    return prefill_T(qT, q_stride, q_row, ktab, vtab, outT, out_row, part, base_pos, t0, SB,
                     n_q_heads, n_kv_heads, head_dim, scale, stream, kvk, exact != 0,
                     wht_flags_for(kvk));
}

int q27_set_kernel_events(void* ev_start, void* ev_stop) {
    g_ev_start = static_cast<cudaEvent_t>(ev_start);
    g_ev_stop = static_cast<cudaEvent_t>(ev_stop);
    return Q27_OK;
}

int q27_wait_timeout_flag(int* out) {
    if (!out) return Q27_ERR_INVALID_ARG;
    int a = 0, b = 0, c = 0, d = 0, rc;
    if ((rc = read_wait_timeout_flag(&a))) return rc;
    if ((rc = read_umma_timeout_flag(&b))) return rc;
    if ((rc = read_xchg_timeout_flag(&c))) return rc;
    if ((rc = read_xchg1_timeout_flag(&d))) return rc;
    *out = a | b | c | d;
    return Q27_OK;
}

int q27_xchg_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || bytes == 0) return Q27_ERR_INVALID_ARG;
    static_assert(sizeof(cudaIpcMemHandle_t) == Q27_XCHG_HANDLE_BYTES, "IPC handle size");
    void* p = nullptr;
    Q27_CUDA_TRY(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess && handle) {
        cudaIpcMemHandle_t h;
        e = cudaIpcGetMemHandle(&h, p);
        if (e == cudaSuccess) memcpy(handle, &h, sizeof(h));
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        fprintf(stderr, "q27_b200: %s at %s:%d\n", cudaGetErrorString(e), __FILE__, __LINE__);
        return Q27_ERR_CUDA;
    }
    *ptr = p;
    return Q27_OK;
}

int q27_xchg_open(const void* handle, void** ptr) {
    if (!handle || !ptr) return Q27_ERR_INVALID_ARG;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    Q27_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return Q27_OK;
}

int q27_xchg_close(void* ptr) {
    if (!ptr) return Q27_ERR_INVALID_ARG;
    Q27_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return Q27_OK;
}

int q27_xchg_free(void* ptr) {
    if (!ptr) return Q27_ERR_INVALID_ARG;
    Q27_CUDA_TRY(cudaFree(ptr));
    return Q27_OK;
}

size_t q27_xchg_mailbox_bytes(int world, int64_t npairs) {
    if (world < 1 || world > Q27_MAX_RANKS || npairs < 1) return 0;
    return xchg_mailbox_bytes(world, npairs);
}

static int partial_push(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                        int n_q_heads, int n_kv_heads, int head_dim, float scale,
                        void* const* mailboxes, int world, int rank, unsigned epoch, void* stream,
                        int kvk, int wht, float* xchg_out = nullptr) {
    if (!mailboxes || world < 1 || world > Q27_MAX_RANKS || rank < 0 || rank >= world)
        return Q27_ERR_INVALID_ARG;
    for (int r = 0; r < world; r++)
        if (!mailboxes[r] || ((uintptr_t)mailboxes[r] & 255)) return Q27_ERR_INVALID_ARG;
    if (nslots < 1 || lanes_stride < 1 || n_q_heads < 1 || ((n_q_heads * lanes_stride * nslots) & 1))
        return Q27_ERR_INVALID_ARG;
    Peers p{};
    for (int r = 0; r < world; r++) p.box[r] = static_cast<uint8_t*>(mailboxes[r]);
    p.world = world;
    p.rank = rank;
    p.npairs = (int64_t)nslots * lanes_stride * n_q_heads;
    p.epoch = epoch;
    if (xchg_out && p.npairs > INT_MAX) return Q27_ERR_TOO_LARGE;
    return run_decode(slots, nslots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim, scale,
                      nullptr, stream, kvk, FAM_AUTO, &p, wht, xchg_out);
}

int q27_attn_decode_exchange(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                             int n_q_heads, int n_kv_heads, int head_dim, float scale,
                             void* const* mailboxes, int world, int rank, unsigned epoch,
                             float* out, void* stream, int kvk, int wht) {
    if (!out) return Q27_ERR_INVALID_ARG;
    return partial_push(slots, nslots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim,
                        scale, mailboxes, world, rank, epoch, stream, kvk,
                        wht ? wht_flags_for(kvk) : 0, out);
}

int q27_attn_decode_partial_push(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                                 int n_q_heads, int n_kv_heads, int head_dim, float scale,
                                 void* const* mailboxes, int world, int rank, unsigned epoch,
                                 void* stream, int kvk) {
    return partial_push(slots, nslots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim,
                        scale, mailboxes, world, rank, epoch, stream, kvk, 0);
}

int q27_attn_decode_partial_push_wht(const q27_slot* slots, int nslots, int lanes_stride,
                                     int q_stride, int n_q_heads, int n_kv_heads, int head_dim,
                                     float scale, void* const* mailboxes, int world, int rank,
                                     unsigned epoch, void* stream, int kvk) {
    return partial_push(slots, nslots, lanes_stride, q_stride, n_q_heads, n_kv_heads, head_dim,
                        scale, mailboxes, world, rank, epoch, stream, kvk,
                        wht_flags_for(kvk) & WHT_Q);
}

static int merge_pushed(void* mailbox, int world, int64_t npairs, unsigned epoch, float* out,
                        void* stream, int wht) {
    if (!mailbox || !out || world < 1 || world > Q27_MAX_RANKS || npairs < 1 || (npairs & 1))
        return Q27_ERR_INVALID_ARG;
    if (npairs > INT_MAX) return Q27_ERR_TOO_LARGE;
    return launch_merge_pushed(mailbox, world, npairs, epoch, out, wht,
                               static_cast<cudaStream_t>(stream));
}

int q27_attn_merge_pushed(void* mailbox, int world, int64_t npairs, unsigned epoch, float* out,
                          void* stream) {
    return merge_pushed(mailbox, world, npairs, epoch, out, stream, 0);
}

int q27_attn_merge_pushed_wht(void* mailbox, int world, int64_t npairs, unsigned epoch, float* out,
                              void* stream, int kvk) {
    if (!kind_known(kvk)) return Q27_ERR_UNSUPPORTED_KIND;
    return merge_pushed(mailbox, world, npairs, epoch, out, stream, wht_flags_for(kvk) & WHT_OUT);
}

int q27_kv_dequant_side(const void* const* tab, int kvk, int is_v, int row0, int nrows,
                        int n_kv_heads, float* out, void* stream) {
    if (!kind_known(kvk)) return Q27_ERR_UNSUPPORTED_KIND;
    if (!tab || !out || row0 < 0 || nrows < 0 || n_kv_heads < 1) return Q27_ERR_INVALID_ARG;
    return launch_kv_dequant(tab, side_fmt(kvk, is_v != 0), row0, nrows, n_kv_heads, out,
                             static_cast<cudaStream_t>(stream));
}

int q27_kv_dequant(const void* const* tab, int kvk, int row0, int nrows, int n_kv_heads,
                   float* out, void* stream) {
    return q27_kv_dequant_side(tab, kvk, 0, row0, nrows, n_kv_heads, out, stream);
}

int q27_kv_store_T(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                   int base_pos, int rowlen, int T, void* stream, int fp8) {
    if (!kT || !vT || !ktab || !vtab || base_pos < 0 || T < 0 || rowlen <= 0 || rowlen % HD)
        return Q27_ERR_INVALID_ARG;
    return launch_kv_store_T(kT, vT, ktab, vtab, base_pos, rowlen / HD, T,
                             static_cast<cudaStream_t>(stream), fp8 ? Q27_KV_FP8 : Q27_KV_F16);
}

int q27_kv_store_T_t3(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                      int base_pos, int n_kv_heads, int head_dim, int T, void* stream, int kvk) {
    if (kvk < Q27_KV_T3 || !kind_known(kvk)) return Q27_ERR_UNSUPPORTED_KIND;
    if (head_dim != HD || n_kv_heads < 1) return Q27_ERR_UNSUPPORTED_WIDTH;
    if (!kT || !vT || !ktab || !vtab || base_pos < 0 || T < 0) return Q27_ERR_INVALID_ARG;
    return launch_kv_store_T(kT, vT, ktab, vtab, base_pos, n_kv_heads, T,
                             static_cast<cudaStream_t>(stream), kvk);
}

int q27_wht_T(float* x, int n_heads, int head_dim, int head_stride, int row_stride, int T, int inv,
              void* stream) {
    if (head_dim != HD) return Q27_ERR_UNSUPPORTED_WIDTH;
    if (!x || n_heads < 0 || T < 0 || head_stride < HD) return Q27_ERR_INVALID_ARG;
    return launch_wht_T(x, n_heads, head_stride, row_stride, T, inv != 0,
                        static_cast<cudaStream_t>(stream));
}

int q27_kv_store3(const q27_CP3* k, const q27_CP3* v, void* const* ktab, void* const* vtab,
                  const q27_IP3* pos, int rowlen, void* stream, int ntok, int fp8) {
    if (!k || !v || !pos || !ktab || !vtab || ntok < 0 || ntok > Q27_MAX_LANES || rowlen < HD ||
        rowlen % HD)
        return Q27_ERR_INVALID_ARG;
    for (int t = 0; t < ntok; t++)
        if (!k->p[t] || !v->p[t] || !pos->p[t]) return Q27_ERR_INVALID_ARG;
    return launch_kv_store3(k->p, v->p, pos->p, ktab, vtab, rowlen / HD, ntok,
                            static_cast<cudaStream_t>(stream), fp8 ? Q27_KV_FP8 : Q27_KV_F16);
}

int q27_kv_store_t3(const q27_CP3* k, const q27_CP3* v, void* const* ktab, void* const* vtab,
                    const q27_IP3* pos, int n_kv_heads, int head_dim, void* stream, int ntok,
                    int kvk) {
    if (kvk < Q27_KV_T3 || !kind_known(kvk)) return Q27_ERR_UNSUPPORTED_KIND;
    if (head_dim != HD || n_kv_heads < 1) return Q27_ERR_UNSUPPORTED_WIDTH;
    if (!k || !v || !pos || !ktab || !vtab || ntok < 0 || ntok > Q27_MAX_LANES)
        return Q27_ERR_INVALID_ARG;
    for (int t = 0; t < ntok; t++)
        if (!k->p[t] || !v->p[t] || !pos->p[t]) return Q27_ERR_INVALID_ARG;
    return launch_kv_store3(k->p, v->p, pos->p, ktab, vtab, n_kv_heads, ntok,
                            static_cast<cudaStream_t>(stream), kvk);
}

int q27_kv_store_lanes_shard(const q27_CP3* k, const q27_CP3* v, void* const* ktab,
                             void* const* vtab, const q27_IP3* pos, int n_kv_heads, int head_dim,
                             void* stream, int ntok, int kvk, int row_base, int row_count) {
    if (!kind_known(kvk)) return Q27_ERR_UNSUPPORTED_KIND;
    if (head_dim != HD || n_kv_heads < 1) return Q27_ERR_UNSUPPORTED_WIDTH;
    if (!k || !v || !pos || !ktab || !vtab || ntok < 0 || ntok > Q27_MAX_LANES || row_base < 0 ||
        row_count < 0)
        return Q27_ERR_INVALID_ARG;
    for (int t = 0; t < ntok; t++)
        if (!k->p[t] || !v->p[t] || !pos->p[t]) return Q27_ERR_INVALID_ARG;
    return launch_kv_store3(k->p, v->p, pos->p, ktab, vtab, n_kv_heads, ntok,
                            static_cast<cudaStream_t>(stream), kvk, row_base, row_count);
}

int q27_kv_store_rows_shard(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                            int base_pos, int n_kv_heads, int head_dim, int T, void* stream,
                            int kvk, int row_base, int row_count) {
    if (!kind_known(kvk)) return Q27_ERR_UNSUPPORTED_KIND;
    if (head_dim != HD || n_kv_heads < 1) return Q27_ERR_UNSUPPORTED_WIDTH;
    if (!kT || !vT || !ktab || !vtab || base_pos < 0 || T < 0 || row_base < 0 || row_count < 0)
        return Q27_ERR_INVALID_ARG;
    return launch_kv_store_T(kT, vT, ktab, vtab, base_pos, n_kv_heads, T,
                             static_cast<cudaStream_t>(stream), kvk, row_base, row_count);
}

int q27_wht3(const q27_P3* x, int n_heads, int head_dim, int stride, int inv, void* stream,
             int ntok) {
    if (head_dim != HD) return Q27_ERR_UNSUPPORTED_WIDTH;
    if (!x || n_heads < 0 || ntok < 0 || ntok > Q27_MAX_LANES || stride < HD)
        return Q27_ERR_INVALID_ARG;
    for (int t = 0; t < ntok; t++)
        if (!x->p[t]) return Q27_ERR_INVALID_ARG;
    return launch_wht3(x->p, n_heads, stride, ntok, inv != 0, static_cast<cudaStream_t>(stream));
}

int q27_mk_tab(const void* base, size_t row_bytes, int rows, void** d_tab, void* stream) {
    if (!base || !d_tab || row_bytes == 0 || rows < 0) return Q27_ERR_INVALID_ARG;
    return launch_mk_tab(base, row_bytes, rows, d_tab, static_cast<cudaStream_t>(stream));
}

} // extern "C"
