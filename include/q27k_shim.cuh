// q27k_shim.cuh -- the reference's own launch functions, by name and signature, over the C
// ABI of q27_b200. A translation unit of the reference that includes this header instead of
// the attention declarations of blocks.cuh / spec3.cuh / prefill.cuh (and links
// libq27_b200.so) calls the B200 engine unchanged:
//
//   q27k::attn_decode      src/blocks.cuh:39-42     -> q27_attn_decode
//   q27k::attn_decode3     src/spec3.cuh:139-143    -> q27_attn_decode3
//   q27k::attn_decode3_fd2 src/spec3.cuh:144-147    -> q27_attn_decode_batched_exact
//   q27k::attn_prefill_T   src/prefill.cuh:95-98    -> q27_attn_prefill_T
//   q27k::kv_store_T       src/blocks.cuh:56-57     -> q27_kv_store_T
//   q27k::kv_store_T_t3    src/blocks.cuh:63-65     -> q27_kv_store_T_t3
//   q27k::wht_T            src/blocks.cuh:76-81     -> q27_wht_T
//   q27k::kv_store3        src/spec3.cuh:87-88      -> q27_kv_store3
//   q27k::kv_store_t3      src/spec3.cuh:98-99      -> q27_kv_store_t3
//   q27k::wht3             src/spec3.cuh:106-107    -> q27_wht3
//   q27k::kv_store         src/blocks.cuh:45-46     -> q27_kv_store3 (one lane)
//   fdmma::launch_fdmma     src/fdmma.cuh:460-463   -> q27_attn_verify_partials
//   fdmma::launch_fdmma_h16 src/fdmma.cuh:808-810   -> q27_attn_verify_partials
//
// Error behaviour is the reference's: the q27k:: functions return void and a failure is fatal
// (message + exit(1), CUDA_CHECK in src/cuda_common.h:8-16); the two fdmma:: launchers return
// `false` for a width they do not cover, and the caller must then fall through to another path
// (src/fdmma.cuh:497), any other failure being fatal as well. All six KvKinds are read; a value
// outside the enum is fatal here rather than silently mis-read. The kinds whose K side differs
// (turbo3v, turbo5k, int8-g64) are served by the fp32 kernels behind the q27k:: entries, and
// the fdmma:: launchers return `false` for them, which sends the caller to attn_decode3_fd2
// as the reference does for the kinds its tensor-core verify does not cover
// (src/spec3.cu:1118-1135).
#pragma once
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "q27_b200.h"

#ifndef Q27K_SHIM_NO_TYPES
// The reference's lane bundles (src/kernels.cuh:67-68, src/spec3.cuh:13) and KvKind
// (src/cuda_common.h:53). Define Q27K_SHIM_NO_TYPES when the reference's own headers are
// included before this one.
enum KvKind : int { KV_F16 = 0, KV_FP8 = 1, KV_T3 = 2, KV_T3V = 3, KV_T5K = 4, KV_I8G64 = 5 };
namespace q27k {
struct P3 { float* p[16]; };
struct CP3 { const float* p[16]; };
struct IP3 { const int* p[16]; };
} // namespace q27k
#endif

namespace q27k {

static_assert(sizeof(P3) == sizeof(q27_P3) && sizeof(CP3) == sizeof(q27_CP3) &&
                  sizeof(IP3) == sizeof(q27_IP3),
              "lane bundles must stay layout-compatible with the C ABI");

inline void q27_shim_check(int rc, const char* what) {
    if (rc != Q27_OK) {
        std::fprintf(stderr, "q27_b200: %s failed: %s (cudaError %d)\n", what,
                     q27_status_string(rc), q27_last_cuda_error());
        std::exit(1);
    }
}

inline void attn_decode(const float* q, int q_stride, const void* const* ktab,
                        const void* const* vtab, float* out, float* scratch, const int* d_pos,
                        int max_ctx, int n_q_heads, int n_kv_heads, int head_dim, float scale,
                        cudaStream_t st = 0, int kvk = KV_F16) {
    q27_shim_check(q27_attn_decode(q, q_stride, ktab, vtab, out, scratch, d_pos, max_ctx,
                                   n_q_heads, n_kv_heads, head_dim, scale, st, kvk),
                   "attn_decode");
}

inline void attn_decode3(CP3 q, int q_stride, const void* const* ktab, const void* const* vtab,
                         P3 out, float* scratch, IP3 pos, int max_ctx, int n_q_heads,
                         int n_kv_heads, int head_dim, float scale, cudaStream_t st = 0,
                         int ntok = 3, int kvk = KV_F16) {
    q27_shim_check(q27_attn_decode3(reinterpret_cast<const q27_CP3*>(&q), q_stride, ktab, vtab,
                                    reinterpret_cast<const q27_P3*>(&out), scratch,
                                    reinterpret_cast<const q27_IP3*>(&pos), max_ctx, n_q_heads,
                                    n_kv_heads, head_dim, scale, st, ntok, kvk),
                   "attn_decode3");
}

// Extensions (no counterpart in the reference): attn_decode3 / attn_prefill_T with the two
// rotation launches around them folded in. A call site of the form
//     if (kv_k_rotated(kvk)) wht3(q, ..., false);  attn_decode3(q, ...);  if (kvk >= KV_T3) wht3(out, ..., true);
// (src/engine.cuh:1482-1506) becomes one call with the UN-rotated q;
// the q||gate buffer is left untouched and the output is bit for bit what the three calls give.
inline void attn_decode3_wht(CP3 q, int q_stride, const void* const* ktab, const void* const* vtab,
                             P3 out, float* scratch, IP3 pos, int max_ctx, int n_q_heads,
                             int n_kv_heads, int head_dim, float scale, cudaStream_t st = 0,
                             int ntok = 3, int kvk = KV_T3) {
    q27_shim_check(q27_attn_decode3_wht(reinterpret_cast<const q27_CP3*>(&q), q_stride, ktab, vtab,
                                        reinterpret_cast<const q27_P3*>(&out), scratch,
                                        reinterpret_cast<const q27_IP3*>(&pos), max_ctx, n_q_heads,
                                        n_kv_heads, head_dim, scale, st, ntok, kvk),
                   "attn_decode3_wht");
}
inline void attn_prefill_T_wht(const float* qT, int q_stride, int q_row, const void* const* ktab,
                               const void* const* vtab, float* outT, int out_row, float* part,
                               int base_pos, int t0, int SB, int n_q_heads, int n_kv_heads,
                               int head_dim, float scale, cudaStream_t st, int kvk = KV_T3) {
    q27_shim_check(q27_attn_prefill_T_wht(qT, q_stride, q_row, ktab, vtab, outT, out_row, part,
                                          base_pos, t0, SB, n_q_heads, n_kv_heads, head_dim, scale,
                                          st, kvk, 0),
                   "attn_prefill_T_wht");
}

// the explicit fp32 entry the reference's unit gate compares the default dispatch against
inline void attn_decode3_fd2(CP3 q, int q_stride, const void* const* ktab,
                             const void* const* vtab, P3 out, float* scratch, IP3 pos,
                             int max_ctx, int n_q_heads, int n_kv_heads, int head_dim,
                             float scale, cudaStream_t st = 0, int ntok = 3, int kvk = KV_F16) {
    (void)max_ctx;
    q27_slot s{};
    s.ktab = ktab;
    s.vtab = vtab;
    s.scratch = scratch;
    s.ntok = ntok;
    s.row_base = 0;
    s.row_count = 0x7fffffff;
    for (int t = 0; t < ntok && t < 16; t++) { s.q.p[t] = q.p[t]; s.pos.p[t] = pos.p[t]; s.out.p[t] = out.p[t]; }
    q27_shim_check(q27_attn_decode_batched_exact(&s, 1, q_stride, n_q_heads, n_kv_heads, head_dim,
                                                 scale, st, kvk),
                   "attn_decode3_fd2");
}

inline void attn_prefill_T(const float* qT, int q_stride, int q_row, const void* const* ktab,
                           const void* const* vtab, float* outT, int out_row, float* part,
                           int base_pos, int t0, int SB, int n_q_heads, int n_kv_heads,
                           int head_dim, float scale, cudaStream_t st, int kvk = KV_F16) {
    q27_shim_check(q27_attn_prefill_T(qT, q_stride, q_row, ktab, vtab, outT, out_row, part,
                                      base_pos, t0, SB, n_q_heads, n_kv_heads, head_dim, scale, st,
                                      kvk),
                   "attn_prefill_T");
}

inline void kv_store_T(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                       int base_pos, int rowlen, int T, cudaStream_t st, bool fp8 = false) {
    q27_shim_check(q27_kv_store_T(kT, vT, ktab, vtab, base_pos, rowlen, T, st, fp8 ? 1 : 0),
                   "kv_store_T");
}

inline void kv_store_T_t3(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                          int base_pos, int n_kv_heads, int head_dim, int T, cudaStream_t st,
                          int kvk = KV_T3) {
    q27_shim_check(q27_kv_store_T_t3(kT, vT, ktab, vtab, base_pos, n_kv_heads, head_dim, T, st,
                                     kvk),
                   "kv_store_T_t3");
}

inline void wht_T(float* x, int n_heads, int head_dim, int head_stride, int row_stride, int T,
                  bool inv, cudaStream_t st) {
    q27_shim_check(q27_wht_T(x, n_heads, head_dim, head_stride, row_stride, T, inv ? 1 : 0, st),
                   "wht_T");
}

inline void kv_store3(CP3 k, CP3 v, void* const* ktab, void* const* vtab, IP3 pos, int rowlen,
                      cudaStream_t st = 0, int ntok = 3, bool fp8 = false) {
    q27_shim_check(q27_kv_store3(reinterpret_cast<const q27_CP3*>(&k),
                                 reinterpret_cast<const q27_CP3*>(&v), ktab, vtab,
                                 reinterpret_cast<const q27_IP3*>(&pos), rowlen, st, ntok,
                                 fp8 ? 1 : 0),
                   "kv_store3");
}

inline void kv_store_t3(CP3 k, CP3 v, void* const* ktab, void* const* vtab, IP3 pos,
                        int n_kv_heads, int head_dim, cudaStream_t st = 0, int ntok = 3,
                        int kvk = KV_T3) {
    q27_shim_check(q27_kv_store_t3(reinterpret_cast<const q27_CP3*>(&k),
                                   reinterpret_cast<const q27_CP3*>(&v), ktab, vtab,
                                   reinterpret_cast<const q27_IP3*>(&pos), n_kv_heads, head_dim, st,
                                   ntok, kvk),
                   "kv_store_t3");
}

inline void wht3(P3 x, int n_heads, int head_dim, int stride, bool inv, cudaStream_t st = 0,
                 int ntok = 3) {
    q27_shim_check(q27_wht3(reinterpret_cast<const q27_P3*>(&x), n_heads, head_dim, stride,
                            inv ? 1 : 0, st, ntok),
                   "wht3");
}

// the single-token store of the plain decode step: row *d_pos of the pair's tables
inline void kv_store(const float* kbuf, const float* vbuf, void* const* ktab, void* const* vtab,
                     const int* d_pos, int rowlen, cudaStream_t st = 0, bool fp8 = false) {
    q27_CP3 k{}, v{};
    q27_IP3 p{};
    k.p[0] = kbuf;
    v.p[0] = vbuf;
    p.p[0] = d_pos;
    q27_shim_check(q27_kv_store3(&k, &v, ktab, vtab, &p, rowlen, st, 1, fp8 ? 1 : 0), "kv_store");
}

} // namespace q27k

// The reference's shared-KV verify launchers (src/fdmma.cuh): partials only, the caller runs
// its own combine with the same `ns`. `stages` is a staging choice of the reference's kernel
// and has no meaning here.
namespace fdmma {
#ifndef Q27K_SHIM_NO_TYPES
struct FCP3 { const float* p[16]; };
struct FIP3 { const int* p[16]; };
#endif

inline bool q27_shim_partials(FCP3 qp, int q_stride, const void* const* ktab,
                              const void* const* vtab, float* part, FIP3 pos, int n_kv_heads,
                              int gqa, int head_dim, float scale, int ns, int ntok, cudaStream_t st,
                              int kvk, const char* what) {
    static_assert(sizeof(FCP3) == sizeof(q27_CP3) && sizeof(FIP3) == sizeof(q27_IP3),
                  "lane bundles must stay layout-compatible with the C ABI");
    const int rc = q27_attn_verify_partials(reinterpret_cast<const q27_CP3*>(&qp), q_stride, ktab,
                                            vtab, part, reinterpret_cast<const q27_IP3*>(&pos),
                                            n_kv_heads, gqa, head_dim, scale, ns, ntok, st, kvk);
    if (rc == Q27_ERR_UNSUPPORTED_WIDTH) return false;
    q27k::q27_shim_check(rc, what);
    return true;
}

inline bool launch_fdmma(FCP3 qp, int q_stride, const void* const* ktab, const void* const* vtab,
                         float* part, FIP3 pos, int n_kv_heads, int gqa, int head_dim, float scale,
                         int ns, int ntok, cudaStream_t st, int stages = 2, bool t3 = false) {
    (void)stages;
    if (ntok < 4 || ntok > 16) return false;       // the widths the reference instantiates
    return q27_shim_partials(qp, q_stride, ktab, vtab, part, pos, n_kv_heads, gqa, head_dim, scale,
                             ns, ntok, st, t3 ? KV_T3 : KV_FP8, "launch_fdmma");
}

// fmt 0 = fp16, 1 = fp8, 2 = turbo3 rows (3 = turbo5k: no tensor-core verify here -> false)
inline bool launch_fdmma_h16(FCP3 qp, int q_stride, const void* const* ktab,
                             const void* const* vtab, float* part, FIP3 pos, int n_kv_heads,
                             int gqa, int head_dim, float scale, int ns, int ntok, int fmt,
                             cudaStream_t st) {
    if (ntok < 4 || ntok > 8 || fmt < 0 || fmt > 2) return false;
    return q27_shim_partials(qp, q_stride, ktab, vtab, part, pos, n_kv_heads, gqa, head_dim, scale,
                             ns, ntok, st, fmt, "launch_fdmma_h16");
}
} // namespace fdmma
