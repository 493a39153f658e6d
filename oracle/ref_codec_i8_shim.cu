// Builds the reference's own CPU int8-g64 codec (the oracle half of tools/i8g64_test.cu:29-50)
// into oracle/_ref/libq27ref_codec.so, straight from the reference tree, so that the oracle
// restatement of the int8 group-64 K format can be checked against it code for code.
// TEST INFRASTRUCTURE: nothing of the reference is copied here -- the file is #included where
// it lies, the test program's main() is renamed and its file-static functions re-exported.
#define main q27ref_i8g64_test_main
#define fails q27ref_i8g64_test_fails   // a global the test programs share by name
#include "tools/i8g64_test.cu"
#undef main
#undef fails

extern "C" {
void q27ref_i8_quant(const float* x, void* blk) { oracle_quant(x, (block_i8g64*)blk); }
// one 256-dim head row stored as a pair of blocks
void q27ref_i8_dequant_row(const void* blk2, float* y256) {
    for (int d = 0; d < 256; d++) y256[d] = oracle_deq((const block_i8g64*)blk2, d);
}
int q27ref_block_i8_bytes() { return (int)sizeof(q27turbo::block_i8g64); }
}
