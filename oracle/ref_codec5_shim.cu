// Builds the reference's own CPU turbo5 codec (the oracle half of tools/turbo5_test.cu:36-89)
// and its table header (src/turbo5.cuh:63-107) into oracle/_ref/libq27ref_codec.so, straight
// from the reference tree, so that the oracle restatement of the 5-bit K format can be checked
// against it and golden fixtures generated from it. TEST INFRASTRUCTURE: nothing of the
// reference is copied here -- the file is #included where it lies, the test program's main()
// is renamed and its file-static functions are re-exported below.
#define main q27ref_turbo5_test_main
#define fails q27ref_turbo5_test_fails   // a global the test programs share by name
#include "tools/turbo5_test.cu"
#undef main
#undef fails

extern "C" {
// tree != 0: the reduction order of the reference's device encoder (its bit-for-bit gate)
void q27ref_cpu_quant5(const float* x, void* blk, int tree) {
    cpu_quant5(x, (block_turbo5*)blk, tree != 0);
}
void q27ref_cpu_dequant5(const void* blk, float* y) { cpu_dequant5((const block_turbo5*)blk, y); }
int q27ref_cpu5_nearest(float v) { return cpu5_nearest(v); }
int q27ref_hdr5_nearest(float v) { return q27turbo::turbo5_nearest(v); }
const float* q27ref_hdr5_centroids() { return q27turbo::TURBO_CENTROIDS_5BIT_HOST; }
const float* q27ref_hdr5_thresholds() { return q27turbo::TURBO_THRESH_5BIT_HOST; }
int q27ref_block5_bytes() { return (int)sizeof(q27turbo::block_turbo5); }
}
