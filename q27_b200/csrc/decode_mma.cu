#include "decode_mma.cuh"

namespace q27b {
int launch_decode_mma(DevBatch& b, int kvk, int sm_count, cudaStream_t st, bool* done) {
    (void)b; (void)kvk; (void)sm_count; (void)st;
    *done = false;
    return Q27_OK;
}
}
