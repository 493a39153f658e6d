// tcgen05 / TMEM attention tile kernel: causal GQA prefill over a reused prefix and the
// one-pass shared-KV verify step. Launchers set *done = false when the shape is not covered.
#pragma once
#include "common.cuh"

namespace q27b {

// part: the caller's prefill scratch (24 * roundup16(SB) * 8 * 258 floats) or NULL.
int launch_prefill_umma(const float* qT, int q_stride, int q_row, const void* const* ktab,
                        const void* const* vtab, float* outT, int out_row, float* part,
                        int base_pos, int t0, int SB, int n_q, int n_kv, float scale,
                        int sm_count, cudaStream_t st, int kvk, int wht, bool* done);

// Writes split-KV partials for every lane of every slot in ONE pass over the cache per
// (slot, kv head, split); fills b.nsplit / b.unit for the combine. force_nsplit > 0 fixes the
// split count (a caller that merges the partials itself chose the stride).
int launch_verify_umma(DevBatch& b, int kvk, int sm_count, cudaStream_t st, bool* done,
                       int force_nsplit = 0);

} // namespace q27b
