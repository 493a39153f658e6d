// Builds the reference's own CPU turbo3 codec (the fork-verbatim copy it keeps in
// tools/turbo3_test.cu:17-58) and its shared table header (src/turbo3.cuh:38-66) into a
// small library, straight from the reference tree, so that the oracle restatement can be
// checked against it and golden fixtures can be generated from it. TEST INFRASTRUCTURE:
// nothing of the reference is copied here -- the two files are #included where they lie
// (REF_ROOT is given by oracle/Makefile), the test program's main() is renamed, and its
// file-static functions are re-exported below. The fp16 / e4m3 converters exported here
// are the CUDA toolkit's host implementations, the ones the reference's host checks use
// (src/test_kernels.cu:751-754).
#define main q27ref_turbo3_test_main
#include "tools/turbo3_test.cu"
#undef main
#include <cuda_fp8.h>

extern "C" {
void q27ref_cpu_quant(const float* x, void* blk) { cpu_quant(x, (block_turbo3*)blk); }
void q27ref_cpu_dequant(const void* blk, float* y) { cpu_dequant((const block_turbo3*)blk, y); }
void q27ref_cpu_fwht(float* x) { cpu_fwht(x); }
void q27ref_cpu_fwht_inv(float* x) { cpu_fwht_inv(x); }
int q27ref_cpu_nearest(float v) { return cpu_nearest(v); }
// header copies (src/turbo3.cuh): host mirrors of the device tables
const float* q27ref_hdr_centroids() { return q27turbo::TURBO_CENTROIDS_HOST; }
const float* q27ref_hdr_s1() { return q27turbo::TURBO_S1_HOST; }
const float* q27ref_hdr_s2() { return q27turbo::TURBO_S2_HOST; }
int q27ref_hdr_nearest(float v) { return q27turbo::turbo3_nearest(v); }
int q27ref_block_bytes() { return (int)sizeof(q27turbo::block_turbo3); }
// CUDA host-side converters
unsigned short q27ref_float_to_half(float f) { __half h = __float2half_rn(f); return *(unsigned short*)&h; }
float q27ref_half_to_float(unsigned short u) { __half h; *(unsigned short*)&h = u; return __half2float(h); }
unsigned char q27ref_float_to_e4m3(float f) { __nv_fp8_e4m3 e(f); return e.__x; }
float q27ref_e4m3_to_float(unsigned char b) { __nv_fp8_e4m3 e; e.__x = b; return float(e); }
}
