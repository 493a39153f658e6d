// Builds the reference's own snapshot-identity code (src/prefix_cache.h:44-82: pfx_fnv1a64,
// pfx_compat_hash, PfxHdr and its constants; a host-only header) into
// oracle/_ref/libq27ref_codec.so, straight from the reference tree, so that the restatements in
// oracle/snapshot_oracle.py and in the engine can be checked against it and golden fixtures
// generated from it. TEST INFRASTRUCTURE: the header is #included where it lies.
#include <cerrno>
#include <ctime>

#include "src/prefix_cache.h"

extern "C" {
unsigned long long q27ref_pfx_fnv1a64(const void* p, size_t n) { return q27::pfx_fnv1a64(p, n); }
unsigned long long q27ref_pfx_fnv1a64_seed(const void* p, size_t n, unsigned long long h) {
    return q27::pfx_fnv1a64(p, n, h);
}
unsigned long long q27ref_pfx_compat_hash(const char* path, unsigned long long model_bytes,
                                          int n_layer, int n_kv, int head_dim, int gdn_heads,
                                          int gdn_dim, int gdn_ch, int kv_kind, int version) {
    return q27::pfx_compat_hash(path, model_bytes, n_layer, n_kv, head_dim, gdn_heads, gdn_dim, gdn_ch,
                                kv_kind, version);
}
int q27ref_pfx_hdr_bytes() { return (int)sizeof(q27::PfxHdr); }
unsigned q27ref_pfx_magic() { return q27::PFX_MAGIC; }
unsigned q27ref_pfx_version() { return q27::PFX_VERSION; }
// a header as PrefixCache::write fills it (src/prefix_cache.h:241-248)
void q27ref_pfx_fill_hdr(void* out64, unsigned long long compat, const int* toks, int L,
                         unsigned long long gdn_n, unsigned long long kv_n) {
    q27::PfxHdr h{};
    h.magic = q27::PFX_MAGIC;
    h.version = q27::PFX_VERSION;
    h.compat = compat;
    h.tok_hash = q27::pfx_fnv1a64(toks, (size_t)L * sizeof(int));
    h.L = L;
    h.gdn_bytes = gdn_n;
    h.kv_bytes = kv_n;
    memcpy(out64, &h, sizeof h);
}
}
