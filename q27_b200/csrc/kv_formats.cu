// KV-format utilities: the bit-exact dequantisation kernel (the "dequantised KV" parity
// target) and the identity page-table builder.
#include "common.cuh"

namespace q27b {
namespace {

// One thread per 8 elements: out[row][kvh][d0..d0+7].
template <int FMT>
__global__ void __launch_bounds__(256)
k_kv_dequant(const void* const* __restrict__ tab, int row0, int nrows, int n_kv,
             float* __restrict__ out) {
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)nrows * n_kv * (HD / 8);
    if (gid >= total) return;
    const int c = (int)(gid % (HD / 8));
    const int kvh = (int)((gid / (HD / 8)) % n_kv);
    const int r = (int)(gid / ((int64_t)(HD / 8) * n_kv));
    const int p = row0 + r;
    const uint8_t* page = static_cast<const uint8_t*>(tab[p >> PAGE_SHIFT]);
    float v[8];
    load8_exact<FMT>(page, p & (PAGE - 1), n_kv, kvh, 8 * c, v);
    float4* o = reinterpret_cast<float4*>(out + ((size_t)r * n_kv + kvh) * HD + 8 * c);
    o[0] = make_float4(v[0], v[1], v[2], v[3]);
    o[1] = make_float4(v[4], v[5], v[6], v[7]);
}

__global__ void k_mk_tab(const char* base, size_t page_bytes, int npages, void** tab) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < npages) tab[i] = const_cast<char*>(base) + (size_t)i * page_bytes;
}

} // namespace

int launch_kv_dequant(const void* const* tab, int fmt, int row0, int nrows, int n_kv, float* out,
                      cudaStream_t st) {
    const int64_t total = (int64_t)nrows * n_kv * (HD / 8);
    if (total == 0) return Q27_OK;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    if (fmt == RF_F16) k_kv_dequant<RF_F16><<<blocks, 256, 0, st>>>(tab, row0, nrows, n_kv, out);
    else if (fmt == RF_FP8) k_kv_dequant<RF_FP8><<<blocks, 256, 0, st>>>(tab, row0, nrows, n_kv, out);
    else if (fmt == RF_T3) k_kv_dequant<RF_T3><<<blocks, 256, 0, st>>>(tab, row0, nrows, n_kv, out);
    else if (fmt == RF_T5) k_kv_dequant<RF_T5><<<blocks, 256, 0, st>>>(tab, row0, nrows, n_kv, out);
    else if (fmt == RF_I8) k_kv_dequant<RF_I8><<<blocks, 256, 0, st>>>(tab, row0, nrows, n_kv, out);
    else return Q27_ERR_UNSUPPORTED_KIND;
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

int launch_mk_tab(const void* base, size_t row_bytes, int rows, void** d_tab, cudaStream_t st) {
    const int np = (rows + PAGE - 1) / PAGE;
    if (np == 0) return Q27_OK;
    k_mk_tab<<<(np + 255) / 256, 256, 0, st>>>(static_cast<const char*>(base),
                                               (size_t)PAGE * row_bytes, np, d_tab);
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

} // namespace q27b
