// Tensor-core decode family (split-KV partials through an mbarrier-guarded shared-memory
// ring fed by bulk async copies). launch_decode_mma sets *done = true when it has written
// the partials for the batch (and the split geometry in `b`); false means the shape is not
// covered and the caller must run the exact family. With may_fuse the kernel may also merge
// the splits and write the normalised output rows itself; it says so in b.fuse, and the
// caller then launches no combine.
#pragma once
#include "common.cuh"

namespace q27b {
int launch_decode_mma(DevBatch& b, int kvk, int sm_count, bool may_fuse, cudaStream_t st,
                      bool* done);
// Reads (synchronously) the flag a kernel sets when one of its bounded waits ran out.
int read_wait_timeout_flag(int* out);
}
