// Compiles against include/q27k_shim.cuh exactly as a translation unit of the reference would
// (same names, same argument lists as src/blocks.cuh / src/spec3.cuh / src/prefill.cuh) and
// links libq27_b200.so. Run on a GPU it performs one attn_decode3 call over an fp16 cache with
// an identity page table and prints the checksum of the output; tests/test_shim_gpu.py
// compares the default entry with the explicit fp32 one. Mode "fdmma" drives the reference's
// verify launchers (fdmma::launch_fdmma_h16: partials only, merged here on the host the way
// k_attn_fd_combine does, src/spec3.cu:706-739) and the single-token q27k::kv_store.
#include <cfloat>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "q27k_shim.cuh"

int main(int argc, char** argv) {
    const int rows = 300, ntok = 4, NQ = 24, NKV = 4, HD = 256, QS = 512;
    std::vector<unsigned short> kv((size_t)rows * NKV * HD);
    unsigned s = 12345u;
    for (auto& h : kv) { s = s * 1664525u + 1013904223u; h = (unsigned short)(0x3000u | ((s >> 9) & 0x0fffu) | ((s >> 3) & 0x8000u)); }
    std::vector<float> q((size_t)ntok * NQ * QS);
    for (auto& f : q) { s = s * 1664525u + 1013904223u; f = ((s >> 8) & 0xffff) / 65536.f - 0.5f; }
    unsigned short *dk, *dv;
    float *dq, *dout, *dscr;
    int* dpos;
    void** dtab_k;
    void** dtab_v;
    const int npages = (rows + Q27_KV_PAGE - 1) / Q27_KV_PAGE;
    const size_t page_elems = (size_t)Q27_KV_PAGE * NKV * HD;
    if (cudaMalloc(&dk, npages * page_elems * 2) != cudaSuccess) { std::printf("no device\n"); return 2; }
    cudaMalloc(&dv, npages * page_elems * 2);
    cudaMemset(dk, 0, npages * page_elems * 2);
    cudaMemset(dv, 0, npages * page_elems * 2);
    cudaMemcpy(dk, kv.data(), kv.size() * 2, cudaMemcpyHostToDevice);
    cudaMemcpy(dv, kv.data(), kv.size() * 2, cudaMemcpyHostToDevice);
    cudaMalloc(&dq, q.size() * 4);
    cudaMemcpy(dq, q.data(), q.size() * 4, cudaMemcpyHostToDevice);
    cudaMalloc(&dout, (size_t)ntok * NQ * HD * 4);
    cudaMalloc(&dscr, (size_t)q27_decode_scratch_floats(ntok, NQ) * 4);
    cudaMalloc(&dpos, ntok * 4);
    int hpos[4] = {rows - 4, rows - 3, rows - 2, rows - 1};
    cudaMemcpy(dpos, hpos, sizeof(hpos), cudaMemcpyHostToDevice);
    cudaMalloc(&dtab_k, npages * sizeof(void*));
    cudaMalloc(&dtab_v, npages * sizeof(void*));
    q27_mk_tab(dk, (size_t)NKV * HD * 2, rows, dtab_k, 0);
    q27_mk_tab(dv, (size_t)NKV * HD * 2, rows, dtab_v, 0);

    q27k::CP3 qp{};
    q27k::P3 op{};
    q27k::IP3 pp{};
    for (int t = 0; t < ntok; t++) { qp.p[t] = dq + (size_t)t * NQ * QS; op.p[t] = dout + (size_t)t * NQ * HD; pp.p[t] = dpos + t; }
    const bool exact = argc > 1 && !std::strcmp(argv[1], "fd2");
    if (argc > 1 && !std::strcmp(argv[1], "fdmma")) {
        // the reference's call pattern (src/spec3.cu:1224-1268): partials with a split count of
        // the caller's choosing, then the caller's own combine with the same count
        q27k::attn_decode3(qp, QS, dtab_k, dtab_v, op, dscr, pp, 0, NQ, NKV, HD, 0.0625f, 0, ntok, KV_F16);
        std::vector<float> want((size_t)ntok * NQ * HD);
        cudaMemcpy(want.data(), dout, want.size() * 4, cudaMemcpyDeviceToHost);
        fdmma::FCP3 fq{};
        fdmma::FIP3 fp{};
        for (int t = 0; t < ntok; t++) { fq.p[t] = qp.p[t]; fp.p[t] = pp.p[t]; }
        const int ns = 16, ST = Q27_PART_STRIDE;
        const bool narrow = fdmma::launch_fdmma_h16(fq, QS, dtab_k, dtab_v, dscr, fp, NKV, 6, HD, 0.0625f, ns, 3, 0, 0);
        const bool wide = fdmma::launch_fdmma_h16(fq, QS, dtab_k, dtab_v, dscr, fp, NKV, 6, HD, 0.0625f, ns, ntok, 0, 0);
        std::vector<float> part((size_t)ntok * NQ * ns * ST);
        if (cudaMemcpy(part.data(), dscr, part.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
        double maxdiff = 0;
        for (int r = 0; r < ntok * NQ; r++) {
            const float* pr = part.data() + (size_t)r * ns * ST;
            float mg = -FLT_MAX;
            for (int sp = 0; sp < ns; sp++) mg = std::fmax(mg, pr[sp * ST]);
            double lg = 0;
            std::vector<double> acc(HD, 0.0);
            for (int sp = 0; sp < ns; sp++) {
                if (pr[sp * ST] == -FLT_MAX) continue;
                const double w = std::exp((double)pr[sp * ST] - mg);
                lg += pr[sp * ST + 1] * w;
                for (int d = 0; d < HD; d++) acc[d] += pr[sp * ST + 2 + d] * w;
            }
            for (int d = 0; d < HD; d++)
                maxdiff = std::fmax(maxdiff, std::fabs(acc[d] / lg - want[(size_t)r * HD + d]));
        }
        // q27k::kv_store: overwrite row 7 of both sides with one token's K / V row
        int* d7;
        cudaMalloc(&d7, 4);
        const int seven = 7;
        cudaMemcpy(d7, &seven, 4, cudaMemcpyHostToDevice);
        q27k::kv_store(dq, dq + NKV * HD, dtab_k, dtab_v, d7, NKV * HD, 0, false);
        unsigned short h0 = 0;
        cudaMemcpy(&h0, dk + (size_t)7 * NKV * HD, 2, cudaMemcpyDeviceToHost);
        std::printf("shim_smoke fdmma narrow %d wide %d maxdiff %.3e stored %04x\n", (int)narrow, (int)wide,
                    maxdiff, (unsigned)h0);
        return 0;
    }
    if (exact)
        q27k::attn_decode3_fd2(qp, QS, dtab_k, dtab_v, op, dscr, pp, 0, NQ, NKV, HD, 0.0625f, 0, ntok, KV_F16);
    else
        q27k::attn_decode3(qp, QS, dtab_k, dtab_v, op, dscr, pp, 0, NQ, NKV, HD, 0.0625f, 0, ntok, KV_F16);
    std::vector<float> out((size_t)ntok * NQ * HD);
    if (cudaMemcpy(out.data(), dout, out.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 1;
    double sum = 0, asum = 0;
    for (float f : out) { sum += f; asum += f < 0 ? -f : f; }
    std::printf("shim_smoke %s sum %.6f abs %.6f\n", exact ? "fd2" : "default", sum, asum);
    return 0;
}
