// extern "C" doorway to the reference's own attention launch functions, compiled for
// sm_100a straight from the reference tree by oracle/Makefile (spec3.cu + prefill.cu are
// compiled where they lie; nothing of them is copied). TEST INFRASTRUCTURE: the GPU tests
// use it as a second comparator ("the reference itself, run on this box") and the
// benchmark may time it as the same-box baseline. It is never loaded by the product path.
#include <cuda_runtime.h>

#include "spec3.cuh"   // q27k::attn_decode3, attn_decode3_fd2, kv_store_t3, wht3
#include "prefill.cuh" // q27k::attn_prefill_T, kv_store_T_t3, wht_T
#include "blocks.cuh"

extern "C" {

// src/spec3.cuh:139-147. fd2_only != 0 calls the explicit fd2 entry.
void q27ref_attn_decode3(const float* const* q, int q_stride, const void* const* ktab,
                         const void* const* vtab, float* const* out, float* scratch,
                         const int* const* pos, int n_q, int n_kv, int hd, float scale,
                         void* stream, int ntok, int kvk, int fd2_only) {
    q27k::CP3 qp{};
    q27k::P3 op{};
    q27k::IP3 pp{};
    for (int t = 0; t < ntok && t < 16; t++) { qp.p[t] = q[t]; op.p[t] = out[t]; pp.p[t] = pos[t]; }
    if (fd2_only)
        q27k::attn_decode3_fd2(qp, q_stride, ktab, vtab, op, scratch, pp, 0, n_q, n_kv, hd, scale,
                               (cudaStream_t)stream, ntok, kvk);
    else
        q27k::attn_decode3(qp, q_stride, ktab, vtab, op, scratch, pp, 0, n_q, n_kv, hd, scale,
                           (cudaStream_t)stream, ntok, kvk);
}

// src/prefill.cuh:95-98
void q27ref_attn_prefill_T(const float* qT, int q_stride, int q_row, const void* const* ktab,
                           const void* const* vtab, float* outT, int out_row, float* part,
                           int base_pos, int t0, int SB, int n_q, int n_kv, int hd, float scale,
                           void* stream, int kvk) {
    q27k::attn_prefill_T(qT, q_stride, q_row, ktab, vtab, outT, out_row, part, base_pos, t0, SB,
                         n_q, n_kv, hd, scale, (cudaStream_t)stream, kvk);
}

// src/prefill.cuh:61-69: the reference's device turbo3 encoder over T rows
void q27ref_kv_store_T_t3(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                          int base_pos, int n_kv, int hd, int T, void* stream, int kvk) {
    q27k::kv_store_T_t3(kT, vT, ktab, vtab, base_pos, n_kv, hd, T, (cudaStream_t)stream, kvk);
}

// src/prefill.cuh:76-81
void q27ref_wht_T(float* x, int n_heads, int hd, int head_stride, int row_stride, int T, int inv,
                  void* stream) {
    q27k::wht_T(x, n_heads, hd, head_stride, row_stride, T, inv != 0, (cudaStream_t)stream);
}

// src/blocks.cuh:56-57
void q27ref_kv_store_T(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                       int base_pos, int rowlen, int T, void* stream, int fp8) {
    q27k::kv_store_T(kT, vT, ktab, vtab, base_pos, rowlen, T, (cudaStream_t)stream, fp8 != 0);
}
}
