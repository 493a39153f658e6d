// Process-wide paged KV pool: the host-side mirror of the reference's KvPool
// (src/kv_pool.h:24-72). Two device allocations, one per side, carved into 64-row pages;
// LIFO free lists with high indices pushed first so early grants get low addresses; a page
// is identified by its index and lives at base + idx * page_bytes. No lock (the caller
// serialises reserve/release), and the only allocation happens at creation.
#include <vector>

#include "common.cuh"

struct q27_kvpool {
    char* base[2] = {nullptr, nullptr};
    size_t page_bytes[2] = {0, 0};
    int npages[2] = {0, 0};
    std::vector<int> free_list[2];
};

extern "C" {

q27_kvpool* q27_kvpool_create(size_t k_bytes, size_t v_bytes, size_t k_row, size_t v_row) {
    if (k_row == 0 || v_row == 0) return nullptr;
    q27_kvpool* p = new q27_kvpool();
    p->page_bytes[0] = (size_t)Q27_KV_PAGE * k_row;
    p->page_bytes[1] = (size_t)Q27_KV_PAGE * v_row;
    for (int s = 0; s < 2; s++) {
        const size_t want = s ? v_bytes : k_bytes;
        p->npages[s] = (int)(want / p->page_bytes[s]); // rounded DOWN to whole pages
        if (p->npages[s] <= 0) { delete p; return nullptr; }
    }
    for (int s = 0; s < 2; s++) {
        cudaError_t e = cudaMalloc((void**)&p->base[s], (size_t)p->npages[s] * p->page_bytes[s]);
        if (e != cudaSuccess) {
            q27b::g_last_cuda_error = (int)e;
            if (s == 1) cudaFree(p->base[0]);
            delete p;
            return nullptr;
        }
        p->free_list[s].reserve(p->npages[s]);
        for (int j = p->npages[s] - 1; j >= 0; j--) p->free_list[s].push_back(j);
    }
    return p;
}

void q27_kvpool_destroy(q27_kvpool* p) {
    if (!p) return;
    for (int s = 0; s < 2; s++)
        if (p->base[s]) cudaFree(p->base[s]);
    delete p;
}

int q27_kvpool_npages(const q27_kvpool* p, int side) { return p && (side == 0 || side == 1) ? p->npages[side] : 0; }
int q27_kvpool_free_pages(const q27_kvpool* p, int side) {
    return p && (side == 0 || side == 1) ? (int)p->free_list[side].size() : 0;
}
size_t q27_kvpool_page_bytes(const q27_kvpool* p, int side) {
    return p && (side == 0 || side == 1) ? p->page_bytes[side] : 0;
}
void* q27_kvpool_page_ptr(const q27_kvpool* p, int side, int idx) {
    if (!p || (side != 0 && side != 1) || idx < 0 || idx >= p->npages[side]) return nullptr;
    return p->base[side] + (size_t)idx * p->page_bytes[side];
}
int q27_kvpool_reserve(q27_kvpool* p, int side, int n, int* out_idx) {
    if (!p || (side != 0 && side != 1) || n < 0 || (n > 0 && !out_idx)) return 0;
    if ((int)p->free_list[side].size() < n) return 0; // pops nothing
    for (int i = 0; i < n; i++) {
        out_idx[i] = p->free_list[side].back();
        p->free_list[side].pop_back();
    }
    return 1;
}
void q27_kvpool_release(q27_kvpool* p, int side, const int* idx, int n) {
    if (!p || (side != 0 && side != 1)) return;
    for (int i = 0; i < n; i++) p->free_list[side].push_back(idx[i]);
}

} // extern "C"
