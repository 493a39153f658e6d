/*
 * q27_b200.h -- C ABI of the B200 (sm_100a) attention engine that slots in behind the
 * kernel-launch surface of signalnine/q27's full-attention layers.
 *
 * Every entry point takes plain pointers and sizes, returns an int status (0 = ok) and
 * never exits the process or throws. Pointers named d_* / tables / Q / out / scratch are
 * DEVICE pointers owned by the caller; small descriptor structs are HOST memory read
 * during the call. All work is enqueued on the caller's stream; nothing is allocated and
 * nothing synchronises, so every entry point may be called under stream capture (the
 * reference captures its rounds into CUDA graphs, src/engine.cuh:2515) -- with one proviso:
 * the first call that reaches a kernel family on a device opts that kernel into its
 * shared-memory size (cudaFuncSetAttribute) and loads its module, so make one call per entry
 * point and KV kind on each device before the first capture (the reference's own launchers
 * latch the same attribute the same way, src/fdmma.cuh:795-800). The per-device caches behind
 * this are filled with atomics: first calls may race across host threads.
 *
 * Fixed geometry of the path (src/engine.cuh:45, docs/SPEC.md:17): head_dim 256,
 * n_q_heads = 6 * n_kv_heads (24 / 4), 64-row KV pages (src/cuda_common.h:70-105).
 */
#ifndef Q27_B200_H
#define Q27_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------ */
enum {
    Q27_OK = 0,
    Q27_ERR_INVALID_ARG = 1,      /* null pointer, bad stride, misaligned page, ... */
    Q27_ERR_UNSUPPORTED_KIND = 2, /* a KvKind outside the enum below (refused, never
                                     mis-read: src/spec3.cu:1109-1122) */
    Q27_ERR_UNSUPPORTED_WIDTH = 3,/* ntok / geometry outside the instantiated range
                                     (the reference's `bool false`, src/fdmma.cuh:497) */
    Q27_ERR_CUDA = 4,             /* a CUDA call failed; see q27_last_cuda_error() */
    Q27_ERR_TOO_LARGE = 5         /* exceeds a fixed capacity (no-allocation entry) */
};

/* KvKind, src/cuda_common.h:53. From turbo3 up the V side is always turbo3 blocks and only
 * the K side varies: turbo3v keeps K as fp16 rows, turbo5k as 82-byte 5-bit blocks
 * (src/turbo5.cuh), int8-g64 as 132-byte int8 blocks with one fp16 scale per 64 dims
 * (src/i8g64.cuh). Q must arrive rotated for turbo3 and turbo5k only (kv_k_rotated,
 * src/cuda_common.h:59). Kinds 3..5 are served by the fp32 family of kernels (as the reference
 * serves them with its scalar kernel, src/spec3.cu:1080-1088); the tensor-core kernels cover
 * kinds 0..2. */
enum { Q27_KV_F16 = 0, Q27_KV_FP8 = 1, Q27_KV_T3 = 2, Q27_KV_T3V = 3, Q27_KV_T5K = 4,
       Q27_KV_I8G64 = 5 };

#define Q27_KV_PAGE 64        /* rows per page, src/cuda_common.h:70 */
#define Q27_HEAD_DIM 256
#define Q27_GQA 6
#define Q27_MAX_LANES 16      /* lane-pointer bundles carry p[16], src/kernels.cuh:67-68 */
#define Q27_MAX_SPLITS 128    /* FD_MAXNS, src/spec3.cuh:126 */
#define Q27_PART_STRIDE 258   /* {m, l, acc[256]}: FD_ST src/spec3.cuh:127, PF_PART_STRIDE */
#define Q27_PF_SPLIT_MAX 8    /* src/prefill.cuh:88 */
#define Q27_T3_BLOCK_BYTES 50 /* sizeof(block_turbo3), src/turbo3.cuh:26-32 */
#define Q27_T5_BLOCK_BYTES 82 /* sizeof(block_turbo5), src/turbo5.cuh:41-47 */
#define Q27_I8_BLOCK_BYTES 132 /* sizeof(block_i8g64), src/i8g64.cuh:36-41 */
#define Q27_MAX_SLOTS 8       /* slots per batched launch */
#define Q27_MAX_RANKS 8       /* GPUs of one node that share a KV-sequence split */
#define Q27_XCHG_HANDLE_BYTES 64

/* Lane pointer bundles: P3 / CP3 (src/kernels.cuh:67-68) and IP3 (src/spec3.cuh:13).
 * Slots >= ntok may hold garbage and are never dereferenced. */
typedef struct { float* p[Q27_MAX_LANES]; } q27_P3;
typedef struct { const float* p[Q27_MAX_LANES]; } q27_CP3;
typedef struct { const int* p[Q27_MAX_LANES]; } q27_IP3;

const char* q27_status_string(int status);
/* cudaError_t of the most recent failing CUDA call made by this library on this thread */
int q27_last_cuda_error(void);
/* compiled-for architecture, e.g. 1000 for sm_100a; 0 if the image cannot run here */
int q27_device_arch(void);
/* Diagnostics: how many kernels this library has launched from the calling thread so far
 * (a difference of two readings counts the launches of the calls in between). */
long long q27_launch_count(void);

/* Diagnostics: every device-side wait in this library is bounded; a kernel whose wait ran
 * out sets a device flag and returns early. This reads the flag (synchronous copy; do
 * not call under stream capture). 0 = no wait has ever timed out in this process. */
int q27_wait_timeout_flag(int* out);

/* Measurement hook: when both events (cudaEvent_t) are non-NULL, every decode / verify
 * call made by this thread records ev_start before and ev_stop after its split-KV partial
 * kernel, on the call's stream, so that the dominant kernel can be timed apart from the
 * combine. Pass NULLs to switch it off. Not for use under stream capture. */
int q27_set_kernel_events(void* ev_start, void* ev_stop);

/* bytes per cache row: fp16 n_kv*512, fp8 n_kv*256, turbo3 n_kv*100; -1 = refused kind.
 * For a kind whose sides differ this is the K side (turbo3v n_kv*512, turbo5k n_kv*164,
 * int8-g64 n_kv*264); q27_kv_row_bytes_side gives either side (is_v != 0: the V side, turbo3
 * for every kind from Q27_KV_T3 up). Engine::kv_bytes(is_v), src/engine.cuh:868-876. */
int64_t q27_kv_row_bytes(int kvk, int n_kv_heads);
int64_t q27_kv_row_bytes_side(int kvk, int n_kv_heads, int is_v);
/* floats the caller must provide as `scratch` for ntok lanes:
 * ntok * n_q_heads * Q27_MAX_SPLITS * Q27_PART_STRIDE (src/spec3.cuh:109-111) */
int64_t q27_decode_scratch_floats(int ntok, int n_q_heads);
/* floats for `part` of q27_attn_prefill_T: n_q_heads * round_up(SB,16) * 8 * 258
 * (src/prefill.cuh:86-88) */
int64_t q27_prefill_part_floats(int SB, int n_q_heads);

/* ---- decode / verify --------------------------------------------------------------- */

/* Replaces q27k::attn_decode (src/blocks.cuh:39-42, src/spec3.cu:1291-1299): one query
 * token attends cache rows [0, *d_pos]. q: head h at q + h*q_stride (first 256 floats of
 * each head; the gate half is not touched). out: [n_q_heads][256] fp32. For Q27_KV_T3, q
 * is already WHT-rotated and out is left in the rotated basis. max_ctx is unused, as in
 * the reference. */
int q27_attn_decode(const float* q, int q_stride, const void* const* ktab,
                    const void* const* vtab, float* out, float* scratch, const int* d_pos,
                    int max_ctx, int n_q_heads, int n_kv_heads, int head_dim, float scale,
                    void* stream, int kvk);

/* Replaces q27k::attn_decode3 and attn_decode3_fd2 (src/spec3.cuh:139-147,
 * src/spec3.cu:1066-1288): ntok lanes (1..16) against ONE pass over the cache; lane t
 * attends rows [0, *pos->p[t]], which makes draft lanes causal among themselves
 * (src/engine.cuh:2124-2125). This is also the shared-KV verify step that the reference
 * reaches through fdmma::launch_fdmma / launch_fdmma_h16 (src/fdmma.cuh:460,808). */
int q27_attn_decode3(const q27_CP3* q, int q_stride, const void* const* ktab,
                     const void* const* vtab, const q27_P3* out, float* scratch,
                     const q27_IP3* pos, int max_ctx, int n_q_heads, int n_kv_heads,
                     int head_dim, float scale, void* stream, int ntok, int kvk);

/* Replaces fdmma::launch_fdmma and fdmma::launch_fdmma_h16 (src/fdmma.cuh:460-463,808-810), the
 * reference's shared-KV verify step WITHOUT its combine: ntok lanes against one pass over the
 * cache, un-normalised split partials {m, l, acc[256]} written at
 * part + ((t*n_q + h)*ns + sp)*258 with exactly the ns splits the caller names (its own
 * k_attn_fd_combine then merges them with the same ns, src/spec3.cu:1224-1235). Splits that
 * hold no row are stamped {-FLT_MAX, 0}, which that combine skips (src/spec3.cu:722). gqa must
 * be 6, ns 1..128. Q27_ERR_UNSUPPORTED_WIDTH is the reference's `false`: the caller must fall
 * through to another path (src/fdmma.cuh:497). Operands are fp16 with fp32 accumulation for
 * every kind (the class of launch_fdmma_h16; tighter than launch_fdmma's e4m3). */
int q27_attn_verify_partials(const q27_CP3* q, int q_stride, const void* const* ktab,
                             const void* const* vtab, float* part, const q27_IP3* pos,
                             int n_kv_heads, int gqa, int head_dim, float scale, int ns, int ntok,
                             void* stream, int kvk);

/* Has no counterpart in the reference. For callers that are not able to hand over scratch
 * memory: code running where device allocation is off limits (a CUDA graph being captured in
 * global mode forbids cudaMalloc from every thread, which is why the reference allocates
 * everything before serving, src/kv_pool.h:8-10), plugin hosts that own no allocator, or a
 * thin binding that only forwards the tensors it was given. Same semantics as
 * q27_attn_decode3 without the `scratch` argument: the split partials go to an array that
 * is part of the library image, sized for Q27_NOALLOC_MAX_LANES lanes (4 lanes x 24 heads
 * x 128 splits x 258 floats = 12.1 MiB, held by every GPU that loads the library until the
 * process exits). ntok above that limit (or more than 24 query heads) is refused with
 * Q27_ERR_TOO_LARGE. The call itself allocates nothing and frees nothing.
 *   - The first call on each device looks the array's device address up; make that first
 *     call outside any stream capture.
 *   - All calls share the one array. Nothing in it has to be cleared between calls (every
 *     cell that is read was written by the same call), but two calls that overlap on the
 *     GPU -- different streams, or graph branches that run side by side -- race on it. */
#define Q27_NOALLOC_MAX_LANES 4
int q27_attn_decode3_noalloc(const q27_CP3* q, int q_stride, const void* const* ktab,
                             const void* const* vtab, const q27_P3* out, const q27_IP3* pos,
                             int n_q_heads, int n_kv_heads, int head_dim, float scale,
                             void* stream, int ntok, int kvk);

/* One slot of a batched launch. The reference runs one attn_decode3 per slot on its own
 * stream (src/conductor.h:681-694); here all slots ride one launch.
 * row_base / row_count describe which logical rows the tables hold (KV-sequence
 * sharding): table row r is logical row row_base + r, for 0 <= r < row_count. An
 * unsharded cache passes row_base = 0, row_count = INT32_MAX. */
typedef struct {
    const void* const* ktab;
    const void* const* vtab;
    q27_CP3 q;
    q27_IP3 pos;
    q27_P3 out;       /* normalised output rows; used by q27_attn_decode_batched */
    float* scratch;   /* ntok * n_q_heads * 128 * 258 floats, private to the slot */
    int ntok;
    int row_base;
    int row_count;
    int reserved;
} q27_slot;

/* Additive (no reference counterpart as a single call): nslots (1..8) independent slots
 * in one launch, same per-slot semantics as q27_attn_decode3. */
int q27_attn_decode_batched(const q27_slot* slots, int nslots, int q_stride, int n_q_heads,
                            int n_kv_heads, int head_dim, float scale, void* stream, int kvk);

/* Additive: the fp32-scalar ("exact") kernel family behind the same arguments, the
 * counterpart of the reference's explicit attn_decode3_fd2 entry (src/spec3.cuh:144-147),
 * which its unit gate compares the default dispatch against. */
int q27_attn_decode_batched_exact(const q27_slot* slots, int nslots, int q_stride,
                                  int n_q_heads, int n_kv_heads, int head_dim, float scale,
                                  void* stream, int kvk);

/* Additive, for KV-sequence sharding across GPUs: like q27_attn_decode_batched but each
 * lane's rows are clipped to the slot's [row_base, row_base+row_count) window and the
 * result is left UN-normalised: partial_out receives, per (slot, lane, head), the
 * merged {m, l, acc[256]} (258 floats) at ((slot*lanes_stride + lane)*n_q_heads + h)*258.
 * A lane whose window is empty gets {-FLT_MAX, 0, 0...} (src/prefill.cu:1353-1362). */
int q27_attn_decode_partial(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                            int n_q_heads, int n_kv_heads, int head_dim, float scale,
                            float* partial_out, void* stream, int kvk);

/* Additive: log-sum-exp merge of nparts partial sets (k_attn_fd_combine,
 * src/spec3.cu:706-739, applied across GPUs instead of across splits).
 * parts: [nparts][npairs][258]; out: [npairs][256] normalised. */
int q27_attn_merge_partials(const float* parts, int nparts, int64_t npairs, float* out,
                            void* stream);

/* ---- exchange of partials through peer memory (no reference counterpart: the reference
 * is single-GPU). One MAILBOX per rank, in that rank's HBM, mapped into the other ranks'
 * processes (one process per GPU) with CUDA IPC. ------------------------------------- */

/* cudaMalloc'ed, zero-filled device buffer that other processes of this node can map;
 * handle (Q27_XCHG_HANDLE_BYTES bytes, may be NULL) is what they pass to q27_xchg_open. */
int q27_xchg_alloc(size_t bytes, void** ptr, void* handle);
int q27_xchg_open(const void* handle, void** ptr);
int q27_xchg_close(void* ptr);   /* a pointer from q27_xchg_open */
int q27_xchg_free(void* ptr);    /* a pointer from q27_xchg_alloc */
/* bytes of a mailbox for `world` ranks x npairs (slot, lane, head) partials */
size_t q27_xchg_mailbox_bytes(int world, int64_t npairs);

/* q27_attn_decode_partial whose result goes to slot `rank` of EVERY rank's mailbox
 * (mailboxes[r] = rank r's mailbox as mapped here; mailboxes[rank] = the own one) with peer
 * stores, followed by a release flag carrying `epoch`. epoch starts at 1 and grows by one
 * per exchange on every rank; or pass 0 in every push and merge on a mailbox and the device
 * counts the exchanges itself (the merge advances a step word in the mailbox), so that a
 * step's launches have constant arguments and can be captured in a CUDA graph.
 * npairs = nslots * lanes_stride * n_q_heads. */
int q27_attn_decode_partial_push(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                                 int n_q_heads, int n_kv_heads, int head_dim, float scale,
                                 void* const* mailboxes, int world, int rank, unsigned epoch,
                                 void* stream, int kvk);

/* Waits on the device (bounded; a timeout sets the flag q27_wait_timeout_flag reads and
 * leaves `out` untouched) until all `world` ranks have pushed `epoch` into this rank's own
 * mailbox, then log-sum-exp merges them: out [npairs][256] normalised. After a timeout the
 * mailbox stays usable: the exchange is not recorded as completed, so the same epoch may be
 * merged again once the missing ranks have pushed. npairs <= 65535. */
int q27_attn_merge_pushed(void* mailbox, int world, int64_t npairs, unsigned epoch, float* out,
                          void* stream);

/* One sharded decode / verify step in one call: q27_attn_decode_partial_push followed by
 * q27_attn_merge_pushed on this rank's own mailbox (mailboxes[rank]); `out` [npairs][256]
 * normalised on every rank. When all (slot, lane, head) rows of the call fit the GPU at once
 * the combine, the peer stores, the wait and the merge run as ONE kernel in which every float
 * travels in a 64-bit word together with the step's epoch and is polled for on its own (no
 * fence, no flag); otherwise as the two kernels above.
 * wht != 0: the rotation of the kind folded in (see the _wht entries below). */
int q27_attn_decode_exchange(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                             int n_q_heads, int n_kv_heads, int head_dim, float scale,
                             void* const* mailboxes, int world, int rank, unsigned epoch,
                             float* out, void* stream, int kvk, int wht);

/* ---- prefill ----------------------------------------------------------------------- */

/* Replaces q27k::attn_prefill_T (src/prefill.cuh:95-98, src/prefill.cu:2620-2655):
 * causal GQA attention for SB tokens t0..t0+SB-1 of a chunk whose first token sits at
 * cache row base_pos; token t attends rows [0, base_pos + t + 1) -- the reused prefix
 * fully, the chunk causally. qT: [T][q_row] fp32, head h at h*q_stride; outT:
 * [T][out_row], head h at h*256. part: caller scratch (may be NULL). */
int q27_attn_prefill_T(const float* qT, int q_stride, int q_row, const void* const* ktab,
                       const void* const* vtab, float* outT, int out_row, float* part,
                       int base_pos, int t0, int SB, int n_q_heads, int n_kv_heads,
                       int head_dim, float scale, void* stream, int kvk);

/* The scalar fp32 prefill (the reference's "lite" k_attn_prefill_T, src/prefill.cu:2293-2388,
 * its in-repo exact GPU reference), same arguments. */
int q27_attn_prefill_T_exact(const float* qT, int q_stride, int q_row,
                             const void* const* ktab, const void* const* vtab, float* outT,
                             int out_row, float* part, int base_pos, int t0, int SB,
                             int n_q_heads, int n_kv_heads, int head_dim, float scale,
                             void* stream, int kvk);

/* ---- attention with the rotation folded in ---------------------------------------------
 * For the kinds from Q27_KV_T3 up the reference brackets every attention call with two
 * launches of its own: wht3 / wht_T forward on Q where the K side is rotated (turbo3, turbo5k:
 * kv_k_rotated, src/cuda_common.h:59) and wht3 / wht_T inverse on the output wherever V is
 * turbo3 (src/engine.cuh:1482-1506, src/spec3.cu:595-614, src/prefill.cu:2598-2618). The
 * entries below take the UN-rotated Q and write the UN-rotated output: the forward rotation
 * runs on the Q heads as the attention kernel stages them (the caller's Q buffer, its gate
 * half included, is left as it was), the inverse on each output head in the kernel that
 * normalises it (combine, fused finish, merge, prefill epilogue / fix-up). Each rotation is
 * the same sequence of rounded operations as q27_wht3 / q27_wht_T, so the result equals the
 * three-launch sequence bit for bit. For Q27_KV_F16 / Q27_KV_FP8 they are the plain entries.
 * Arguments as for the entry each one is named after. */
int q27_attn_decode3_wht(const q27_CP3* q, int q_stride, const void* const* ktab,
                         const void* const* vtab, const q27_P3* out, float* scratch,
                         const q27_IP3* pos, int max_ctx, int n_q_heads, int n_kv_heads,
                         int head_dim, float scale, void* stream, int ntok, int kvk);
/* exact != 0: the fp32 family (q27_attn_decode_batched_exact) */
int q27_attn_decode_batched_wht(const q27_slot* slots, int nslots, int q_stride, int n_q_heads,
                                int n_kv_heads, int head_dim, float scale, void* stream, int kvk,
                                int exact);
/* exact != 0: the scalar fp32 prefill (q27_attn_prefill_T_exact) */
int q27_attn_prefill_T_wht(const float* qT, int q_stride, int q_row, const void* const* ktab,
                           const void* const* vtab, float* outT, int out_row, float* part,
                           int base_pos, int t0, int SB, int n_q_heads, int n_kv_heads,
                           int head_dim, float scale, void* stream, int kvk, int exact);
/* KV-sequence split: the partial side rotates Q, the merge side un-rotates the output */
int q27_attn_decode_partial_wht(const q27_slot* slots, int nslots, int lanes_stride, int q_stride,
                                int n_q_heads, int n_kv_heads, int head_dim, float scale,
                                float* partial_out, void* stream, int kvk);
int q27_attn_merge_partials_wht(const float* parts, int nparts, int64_t npairs, float* out,
                                void* stream, int kvk);
int q27_attn_decode_partial_push_wht(const q27_slot* slots, int nslots, int lanes_stride,
                                     int q_stride, int n_q_heads, int n_kv_heads, int head_dim,
                                     float scale, void* const* mailboxes, int world, int rank,
                                     unsigned epoch, void* stream, int kvk);
int q27_attn_merge_pushed_wht(void* mailbox, int world, int64_t npairs, unsigned epoch, float* out,
                              void* stream, int kvk);

/* ---- KV formats -------------------------------------------------------------------- */

/* Bit-exact dequantisation of cache rows [row0, row0+nrows) through a page table to fp32
 * [nrows][n_kv_heads][256]: half2float / float(e4m3) / CENTROIDS[idx]*half2float(norm)
 * (kv2f src/cuda_common.h:113-114, turbo3_deq_elem src/turbo3.cuh:134-137). For a kind whose
 * sides differ this form reads the table as K rows. */
int q27_kv_dequant(const void* const* tab, int kvk, int row0, int nrows, int n_kv_heads,
                   float* out, void* stream);
/* The same for one side of a kind (is_v: 0 = the table holds K rows, 1 = V rows): turbo5
 * CENTROIDS5[idx]*norm (turbo5_deq_elem, src/turbo5.cuh:163-166), int8-g64 code*scale
 * (i8g64_deq_elem, src/i8g64.cuh:68-72). */
int q27_kv_dequant_side(const void* const* tab, int kvk, int is_v, int row0, int nrows,
                        int n_kv_heads, float* out, void* stream);

/* Replaces q27k::kv_store_T (src/blocks.cuh:56-57, src/prefill.cu:1221-1243): store T
 * tokens' K and V rows (fp32 [T][rowlen], rowlen = n_kv_heads*256) into cache rows
 * base_pos .. base_pos+T-1 as fp16 (round to nearest even) or saturating e4m3. */
int q27_kv_store_T(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                   int base_pos, int rowlen, int T, void* stream, int fp8);

/* Replaces q27k::kv_store_T_t3 (src/blocks.cuh:63-65, src/prefill.cu:2556-2596) for kinds
 * Q27_KV_T3 .. Q27_KV_I8G64. turbo3 (V of every kind, K of Q27_KV_T3): per 128-element group
 * L2 norm -> forward WHT -> nearest of 8 centroids -> pack -> corrected fp16 norm, written
 * block-addressed; byte-identical to the reference's serial CPU codec (t3_quant,
 * src/test_kernels.cu:1089-1103). K legs of the other kinds: turbo3v plain fp16 rows;
 * turbo5k the same pipeline over 32 centroids with the two norms summed in the halving-tree
 * order of the reference's device encoder (turbo5_quant_group, src/turbo5.cuh:129-162), so
 * the blocks equal that encoder's and its CPU oracle's tree mode byte for byte; int8-g64
 * per-64 absmax, fp16 scale, codes from the reciprocal of the ROUNDED scale
 * (i8g64_quant_group, src/i8g64.cuh:48-64), exact. K must already be rope'd. */
int q27_kv_store_T_t3(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                      int base_pos, int n_kv_heads, int head_dim, int T, void* stream, int kvk);

/* Replaces q27k::wht_T (src/blocks.cuh:76-81, src/prefill.cu:2598-2618): per-128-group
 * signed Walsh-Hadamard rotation in place over a flat [T][row_stride] buffer; forward on Q
 * after rope (inv = 0), inverse on the attention output (inv = 1). Only the first 256
 * floats of each head are touched (head_stride = 512 for the q||gate layout). T = ntok
 * rows cover the decode-time wht3 (src/spec3.cuh:103-105) when lanes are contiguous. */
int q27_wht_T(float* x, int n_heads, int head_dim, int head_stride, int row_stride, int T, int inv,
              void* stream);

/* Lane forms of the three calls above, for the draft tokens of a decode / verify round:
 * lane t's rows come from k->p[t] / v->p[t] (fp32 [n_kv_heads*256]) and go to cache row
 * *pos->p[t] (read on the device), or x->p[t] is rotated in place.
 * Replaces q27k::kv_store3 (src/spec3.cuh:87-88, src/spec3.cu:512-535). */
int q27_kv_store3(const q27_CP3* k, const q27_CP3* v, void* const* ktab, void* const* vtab,
                  const q27_IP3* pos, int rowlen, void* stream, int ntok, int fp8);
/* Replaces q27k::kv_store_t3 (src/spec3.cuh:98-99, src/spec3.cu:556-588) for kinds
 * Q27_KV_T3 .. Q27_KV_I8G64; encoders and byte-level guarantees as for q27_kv_store_T_t3. */
int q27_kv_store_t3(const q27_CP3* k, const q27_CP3* v, void* const* ktab, void* const* vtab,
                    const q27_IP3* pos, int n_kv_heads, int head_dim, void* stream, int ntok,
                    int kvk);
/* Replaces q27k::wht3 (src/spec3.cuh:106-107, src/spec3.cu:595-614): per-128-group rotation
 * of the first head_dim floats of each of n_heads heads (stride floats apart), bitwise equal
 * to the CPU t3_fwht / t3_fwht_inv. */
int q27_wht3(const q27_P3* x, int n_heads, int head_dim, int stride, int inv, void* stream,
             int ntok);

/* The stores above on a cache split by rows over several GPUs (any kind): every GPU runs the
 * same call on the same lanes / chunk rows with its own tables and its own range of logical
 * rows [row_base, row_base + row_count); a row is encoded and written by the GPU that owns it
 * (at row - row_base of its tables) and skipped by the others, the decision taken on the
 * device from the positions the lanes point at. No row crosses a link. */
int q27_kv_store_lanes_shard(const q27_CP3* k, const q27_CP3* v, void* const* ktab,
                             void* const* vtab, const q27_IP3* pos, int n_kv_heads, int head_dim,
                             void* stream, int ntok, int kvk, int row_base, int row_count);
int q27_kv_store_rows_shard(const float* kT, const float* vT, void* const* ktab, void* const* vtab,
                            int base_pos, int n_kv_heads, int head_dim, int T, void* stream,
                            int kvk, int row_base, int row_count);

/* mk_tab (src/test_kernels.cu:27-36): fill a DEVICE table of ceil(rows/64) entries with
 * identity page pointers over a contiguous buffer. d_tab is caller-allocated. */
int q27_mk_tab(const void* base, size_t row_bytes, int rows, void** d_tab, void* stream);

/* ---- KvPool (src/kv_pool.h:24-72) ---------------------------------------------------
 * Two device allocations (K side, V side) carved into 64-row pages, LIFO free lists,
 * page address = base + idx*page_bytes. No lock of its own (caller's mutex), allocation
 * happens once at creation. */
typedef struct q27_kvpool q27_kvpool;
/* returns NULL if either side would get zero pages (pool disabled) or allocation fails */
q27_kvpool* q27_kvpool_create(size_t k_bytes, size_t v_bytes, size_t k_row, size_t v_row);
void q27_kvpool_destroy(q27_kvpool* pool);
int q27_kvpool_npages(const q27_kvpool* pool, int side);
int q27_kvpool_free_pages(const q27_kvpool* pool, int side);
size_t q27_kvpool_page_bytes(const q27_kvpool* pool, int side);
void* q27_kvpool_page_ptr(const q27_kvpool* pool, int side, int idx);
/* pops n page indices into out_idx; returns 0 (and pops nothing) if fewer are free */
int q27_kvpool_reserve(q27_kvpool* pool, int side, int n, int* out_idx);
void q27_kvpool_release(q27_kvpool* pool, int side, const int* idx, int n);

/* ---- lineages: pooled pages of one conversation (src/engine.cuh:781-845) ---------------
 * A lineage owns pool pages per side and per cache pair (one pair per attention layer plus
 * any extra pair of the caller's, e.g. the draft head's) and keeps the device page tables
 * [2][pairs][ceil(max_rows/64)] the attention and store entries read. On a cache sharded by
 * rows over several GPUs each GPU runs one lineage over its own rows. Allocation happens at
 * creation only; entitle / release just move page indices and rewrite table entries (the
 * table POINTERS stay fixed, so captured graphs that hold them stay valid). */
typedef struct q27_kvlineage q27_kvlineage;
q27_kvlineage* q27_kvlineage_create(q27_kvpool* pool, int pairs, int max_rows);
void q27_kvlineage_destroy(q27_kvlineage* l);          /* returns its pages to the pool */
/* kv_entitle: make rows [0, rows + extra[pair]) of every pair addressable (extra may be NULL).
 * All or nothing: 1 = mapped (table upload enqueued on `stream`), 0 = the pool lacks pages
 * and nothing changed, -1 = invalid argument. Entries past the last owned page alias the
 * pair's first page. Never shrinks. */
int q27_kvlineage_entitle(q27_kvlineage* l, int rows, const int* extra, void* stream);
/* kv_release_for_takeover: every page back to the pool; the tables keep stale but valid
 * addresses until the next entitle. */
void q27_kvlineage_release(q27_kvlineage* l);
int q27_kvlineage_rows(const q27_kvlineage* l);
int q27_kvlineage_npages(const q27_kvlineage* l);
int q27_kvlineage_pages_of(const q27_kvlineage* l, int side, int pair);
/* device page table of one (side, pair): what ktab / vtab of the attention entries take */
const void* const* q27_kvlineage_tab(const q27_kvlineage* l, int side, int pair);
/* kv_row_host (src/engine.cuh:840-845): device address of row r, from the host mirror */
void* q27_kvlineage_row(const q27_kvlineage* l, int side, int pair, int r);

/* ---- KV section of a prefix snapshot (pfx_export / pfx_import, src/engine.cuh:3786-3857) --
 * Blob layout: for each pair in order, K rows [0, n) then V rows [0, n), n = nrows +
 * extra[pair], rows in logical order whatever pages they live in -- so a blob is portable
 * across pool geometries, page scatter and the number of GPUs a cache is sharded over. Export
 * reads rows [row0, row0 + n) of this lineage (its local rows); `blob` is device-accessible
 * memory, 16-byte aligned, q27_kv_snapshot_bytes long. One kernel per call. */
#define Q27_SNAPSHOT_MAX_PAIRS 64
int64_t q27_kv_snapshot_bytes(int pairs, int nrows, const int* extra, size_t k_row, size_t v_row);
int q27_kv_snapshot_export(const q27_kvlineage* l, int row0, int nrows, const int* extra,
                           void* blob, void* stream);
int q27_kv_snapshot_import(q27_kvlineage* l, int row0, int nrows, const int* extra,
                           const void* blob, void* stream);

/* Identity of a snapshot (src/prefix_cache.h:44-82): FNV-1a over bytes (seed = the FNV offset
 * basis for a fresh hash), the compatibility hash over model path / size / geometry / KV kind
 * / format version, and the fixed 64-byte file header that precedes the L tokens and the
 * state bytes. Host-only. */
#define Q27_PFX_FNV_SEED 1469598103934665603ULL
#define Q27_PFX_MAGIC 0x50373251u   /* 'Q27P' little-endian */
#define Q27_PFX_VERSION 1u
#pragma pack(push, 1)
typedef struct {
    uint32_t magic, version;
    uint64_t compat, tok_hash;
    int32_t L, pad;
    uint64_t gdn_bytes, kv_bytes;
    uint64_t reserved[2];
} q27_pfx_hdr;
#pragma pack(pop)
uint64_t q27_pfx_fnv1a64(const void* p, size_t n, uint64_t seed);
uint64_t q27_pfx_compat_hash(const char* model_path, uint64_t model_bytes, int n_layer, int n_kv,
                             int head_dim, int gdn_heads, int gdn_dim, int gdn_ch, int kv_kind,
                             int format_version);

#ifdef __cplusplus
}
#endif
#endif
