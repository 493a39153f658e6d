// Page ownership of one conversation ("lineage") on one GPU, and the row-ordered snapshot of
// its caches: the host-side mirror of the reference's pooled mapping (kv_entitle,
// kv_release_for_takeover, kv_row_host: src/engine.cuh:781-845) and of the KV section of its
// prefix snapshots (pfx_export / pfx_import, src/engine.cuh:3786-3857).
//
// A lineage owns, per side and per cache pair (one pair per attention layer, plus whatever
// extra pair the caller keeps, e.g. the draft head's), a list of pool pages; its device table
// [2 sides][pairs][npages] holds the page pointers in logical order, entries past the last
// owned page aliasing the pair's first page (never read below the causal bound, but always a
// valid address). Growing a lineage reserves whole pages for every pair or nothing at all.
// On a KV-sequence-sharded cache every GPU runs one lineage over ITS rows of the conversation.
//
// The snapshot is the reference's blob: for each pair, the K rows [0, n) then the V rows
// [0, n) in logical order, n = rows + extra[pair] (the draft head's pair carries one row
// more, src/engine.cuh:3689-3695). Rows live in scattered pages, so export gathers and
// import scatters page by page -- here as ONE kernel over all sections instead of
// ceil(rows/64) copies per buffer; both ends of a copy are 16-byte pieces of whole rows.
#include <vector>

#include "common.cuh"

struct q27_kvpool;
extern "C" {
void* q27_kvpool_page_ptr(const q27_kvpool* p, int side, int idx);
int q27_kvpool_free_pages(const q27_kvpool* p, int side);
size_t q27_kvpool_page_bytes(const q27_kvpool* p, int side);
int q27_kvpool_reserve(q27_kvpool* p, int side, int n, int* out_idx);
void q27_kvpool_release(q27_kvpool* p, int side, const int* idx, int n);
}

struct q27_kvlineage {
    q27_kvpool* pool = nullptr;
    int pairs = 0, npages = 0, rows = 0;
    std::vector<std::vector<int>> pages[2];   // [side][pair] -> pool page indices, logical order
    void** h_tab = nullptr;                   // pinned mirror of the device table
    void** d_tab = nullptr;
};

namespace q27b {
namespace {

constexpr int SNAP_MAX_SECTIONS = 2 * Q27_SNAPSHOT_MAX_PAIRS;
struct SnapSections {
    const void* const* tab[SNAP_MAX_SECTIONS];   // page table of the section's (pair, side)
    unsigned long long blob_off[SNAP_MAX_SECTIONS + 1];   // in 16-byte pieces, prefix sums
    int row_pieces[SNAP_MAX_SECTIONS];            // 16-byte pieces per row
    int n;
    int row0;                                     // first cache row of every section
};
static_assert(sizeof(SnapSections) <= 4000, "passed as a kernel parameter");

// TO_BLOB: cache rows -> blob (export); otherwise blob -> cache rows (import). grid.y = section;
// a section's pieces are walked with 32-bit arithmetic (its size is checked on the host).
template <bool TO_BLOB>
__global__ void __launch_bounds__(256)
k_snapshot_copy(const __grid_constant__ SnapSections S, uint4* __restrict__ blob) {
    const int s = blockIdx.y;
    const unsigned n = (unsigned)(S.blob_off[s + 1] - S.blob_off[s]);
    const unsigned rp = (unsigned)S.row_pieces[s];
    const void* const* tab = S.tab[s];
    uint4* sec = blob + S.blob_off[s];
    for (unsigned j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        const unsigned rr = j / rp, c = j - rr * rp;
        const int r = S.row0 + (int)rr;
        uint4* cell = reinterpret_cast<uint4*>(const_cast<void*>(tab[r >> PAGE_SHIFT])) +
                      (size_t)(r & (PAGE - 1)) * rp + c;
        if (TO_BLOB) sec[j] = *cell;
        else *cell = sec[j];
    }
}

int snapshot_sections(const q27_kvlineage* l, int row0, int nrows, const int* extra, size_t k_row,
                      size_t v_row, SnapSections& S, size_t* bytes) {
    if (!l || row0 < 0 || nrows < 0 || (k_row & 15) || (v_row & 15) || k_row == 0 || v_row == 0)
        return Q27_ERR_INVALID_ARG;
    if (l->pairs > Q27_SNAPSHOT_MAX_PAIRS) return Q27_ERR_TOO_LARGE;
    S.n = 2 * l->pairs;
    S.row0 = row0;
    unsigned long long off = 0;
    for (int c = 0; c < l->pairs; c++) {
        const int n = nrows + (extra ? extra[c] : 0);
        if (n < 0 || row0 + n > l->npages * PAGE) return Q27_ERR_INVALID_ARG;
        for (int side = 0; side < 2; side++) {
            const int s = 2 * c + side;
            S.tab[s] = l->d_tab + ((size_t)side * l->pairs + c) * l->npages;
            S.row_pieces[s] = (int)((side ? v_row : k_row) / 16);
            S.blob_off[s] = off;
            if ((unsigned long long)n * S.row_pieces[s] > 0xffffffffull) return Q27_ERR_TOO_LARGE;
            off += (unsigned long long)n * S.row_pieces[s];
        }
    }
    S.blob_off[S.n] = off;
    *bytes = (size_t)off * 16;
    return Q27_OK;
}

} // namespace
} // namespace q27b

static_assert(sizeof(q27_pfx_hdr) == 64, "the snapshot header is 64 bytes (src/prefix_cache.h:66-80)");

using namespace q27b;

extern "C" {

q27_kvlineage* q27_kvlineage_create(q27_kvpool* pool, int pairs, int max_rows) {
    if (!pool || pairs < 1 || max_rows < 1) return nullptr;
    q27_kvlineage* l = new q27_kvlineage();
    l->pool = pool;
    l->pairs = pairs;
    l->npages = (max_rows + PAGE - 1) / PAGE;
    for (int s = 0; s < 2; s++) l->pages[s].resize(pairs);
    const size_t n = (size_t)2 * pairs * l->npages;
    cudaError_t e = cudaMallocHost((void**)&l->h_tab, n * sizeof(void*));
    if (e == cudaSuccess) e = cudaMalloc((void**)&l->d_tab, n * sizeof(void*));
    if (e != cudaSuccess) {
        g_last_cuda_error = (int)e;
        if (l->h_tab) cudaFreeHost(l->h_tab);
        delete l;
        return nullptr;
    }
    // until pages are mapped every entry points at page 0 of its side: a valid address
    for (int s = 0; s < 2; s++)
        for (size_t i = 0; i < (size_t)pairs * l->npages; i++)
            l->h_tab[(size_t)s * pairs * l->npages + i] = q27_kvpool_page_ptr(pool, s, 0);
    cudaMemcpy(l->d_tab, l->h_tab, n * sizeof(void*), cudaMemcpyHostToDevice);
    return l;
}

void q27_kvlineage_release(q27_kvlineage* l) {
    if (!l) return;
    for (int s = 0; s < 2; s++)
        for (auto& pg : l->pages[s]) {
            q27_kvpool_release(l->pool, s, pg.data(), (int)pg.size());
            pg.clear();
        }
    l->rows = 0;
}

void q27_kvlineage_destroy(q27_kvlineage* l) {
    if (!l) return;
    q27_kvlineage_release(l);
    if (l->h_tab) cudaFreeHost(l->h_tab);
    if (l->d_tab) cudaFree(l->d_tab);
    delete l;
}

int q27_kvlineage_entitle(q27_kvlineage* l, int rows, const int* extra, void* stream) {
    if (!l || rows < 0) return -1;
    std::vector<int> want(l->pairs);
    int need[2] = {0, 0};
    for (int c = 0; c < l->pairs; c++) {
        const int n = rows + (extra ? extra[c] : 0);
        if (n < 0 || n > l->npages * PAGE) return -1;
        want[c] = (n + PAGE - 1) / PAGE;
        for (int s = 0; s < 2; s++) {
            const int have = (int)l->pages[s][c].size();
            if (want[c] > have) need[s] += want[c] - have;
        }
    }
    if (q27_kvpool_free_pages(l->pool, 0) < need[0] || q27_kvpool_free_pages(l->pool, 1) < need[1])
        return 0;                                  // all or nothing: no page was taken
    for (int s = 0; s < 2; s++)
        for (int c = 0; c < l->pairs; c++) {
            auto& pg = l->pages[s][c];
            while ((int)pg.size() < want[c]) {
                int idx = -1;
                q27_kvpool_reserve(l->pool, s, 1, &idx);
                pg.push_back(idx);
            }
            void** row = l->h_tab + ((size_t)s * l->pairs + c) * l->npages;
            const int have = (int)pg.size();
            for (int j = 0; j < l->npages; j++)
                row[j] = have ? q27_kvpool_page_ptr(l->pool, s, pg[j < have ? j : 0])
                              : q27_kvpool_page_ptr(l->pool, s, 0);
        }
    if (rows > l->rows) l->rows = rows;
    cudaError_t e = cudaMemcpyAsync(l->d_tab, l->h_tab, (size_t)2 * l->pairs * l->npages * sizeof(void*),
                                    cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) { g_last_cuda_error = (int)e; return -1; }
    return 1;
}

int q27_kvlineage_rows(const q27_kvlineage* l) { return l ? l->rows : 0; }
int q27_kvlineage_npages(const q27_kvlineage* l) { return l ? l->npages : 0; }
int q27_kvlineage_pages_of(const q27_kvlineage* l, int side, int pair) {
    if (!l || (side != 0 && side != 1) || pair < 0 || pair >= l->pairs) return 0;
    return (int)l->pages[side][pair].size();
}

const void* const* q27_kvlineage_tab(const q27_kvlineage* l, int side, int pair) {
    if (!l || (side != 0 && side != 1) || pair < 0 || pair >= l->pairs) return nullptr;
    return l->d_tab + ((size_t)side * l->pairs + pair) * l->npages;
}

void* q27_kvlineage_row(const q27_kvlineage* l, int side, int pair, int r) {
    if (!l || (side != 0 && side != 1) || pair < 0 || pair >= l->pairs || r < 0 ||
        r >= l->npages * PAGE)
        return nullptr;
    char* pg = static_cast<char*>(l->h_tab[((size_t)side * l->pairs + pair) * l->npages + (r >> PAGE_SHIFT)]);
    return pg + (size_t)(r & (PAGE - 1)) * (q27_kvpool_page_bytes(l->pool, side) / PAGE);
}

int64_t q27_kv_snapshot_bytes(int pairs, int nrows, const int* extra, size_t k_row, size_t v_row) {
    if (pairs < 1 || nrows < 0) return -1;
    int64_t n = 0;
    for (int c = 0; c < pairs; c++) {
        const int r = nrows + (extra ? extra[c] : 0);
        if (r < 0) return -1;
        n += (int64_t)r * (int64_t)(k_row + v_row);
    }
    return n;
}

static int snapshot_copy(const q27_kvlineage* l, int row0, int nrows, const int* extra, void* blob,
                         void* stream, bool to_blob) {
    if (!blob || ((uintptr_t)blob & 15)) return Q27_ERR_INVALID_ARG;
    if (!l) return Q27_ERR_INVALID_ARG;
    SnapSections S;
    size_t bytes = 0;
    const size_t k_row = q27_kvpool_page_bytes(l->pool, 0) / PAGE, v_row = q27_kvpool_page_bytes(l->pool, 1) / PAGE;
    int rc = snapshot_sections(l, row0, nrows, extra, k_row, v_row, S, &bytes);
    if (rc) return rc;
    if (bytes == 0) return Q27_OK;
    // the largest section decides the x extent; every section gets the same number of blocks
    unsigned long long widest = 0;
    for (int s = 0; s < S.n; s++)
        widest = S.blob_off[s + 1] - S.blob_off[s] > widest ? S.blob_off[s + 1] - S.blob_off[s] : widest;
    unsigned bx = (unsigned)((widest + 255) / 256);
    const unsigned cap = (148u * 8 + S.n - 1) / S.n;          // about eight blocks per SM in all
    bx = bx < 1 ? 1 : bx > cap ? cap : bx;
    const dim3 grid(bx, S.n);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (to_blob) k_snapshot_copy<true><<<grid, 256, 0, st>>>(S, static_cast<uint4*>(blob));
    else k_snapshot_copy<false><<<grid, 256, 0, st>>>(S, static_cast<uint4*>(blob));
    Q27_CUDA_TRY(cudaGetLastError());
    Q27_COUNT_LAUNCH();
    return Q27_OK;
}

int q27_kv_snapshot_export(const q27_kvlineage* l, int row0, int nrows, const int* extra,
                           void* blob, void* stream) {
    return snapshot_copy(l, row0, nrows, extra, blob, stream, true);
}

int q27_kv_snapshot_import(q27_kvlineage* l, int row0, int nrows, const int* extra,
                           const void* blob, void* stream) {
    return snapshot_copy(l, row0, nrows, extra, const_cast<void*>(blob), stream, false);
}

// ---- snapshot identity (src/prefix_cache.h:44-82): host-only ------------------------------

uint64_t q27_pfx_fnv1a64(const void* p, size_t n, uint64_t h) {
    const unsigned char* b = static_cast<const unsigned char*>(p);
    for (size_t i = 0; i < n; i++) {
        h ^= b[i];
        h *= 1099511628211ULL;
    }
    return h;
}

uint64_t q27_pfx_compat_hash(const char* model_path, uint64_t model_bytes, int n_layer, int n_kv,
                             int head_dim, int gdn_heads, int gdn_dim, int gdn_ch, int kv_kind,
                             int format_version) {
    size_t len = 0;
    while (model_path && model_path[len]) len++;
    uint64_t h = q27_pfx_fnv1a64(model_path, len, Q27_PFX_FNV_SEED);
    const int64_t v[] = {(int64_t)model_bytes, n_layer, n_kv, head_dim, gdn_heads,
                         gdn_dim, gdn_ch, kv_kind, format_version};
    return q27_pfx_fnv1a64(v, sizeof v, h);
}

} // extern "C"
