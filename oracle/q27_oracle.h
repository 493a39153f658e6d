/*
 * q27_oracle.h -- CPU restatement of the q27 attention hot path. TEST INFRASTRUCTURE ONLY.
 *
 * This library is the checker, never the product: the only things allowed to load it are
 * the test-suite, the smoke check and the CPU-baseline leg of the benchmark. Nothing in
 * q27_b200/ imports it, and the CUDA path has no fallback onto it.
 *
 * Every function restates, in plain C with double accumulation, a piece of the reference
 * (signalnine/q27); the reference file:line each follows is given beside its prototype.
 * Parity pin: the turbo3 codec and its tables are checked against the reference's own
 * fork-verbatim CPU codec (tools/turbo3_test.cu:17-58, compiled from the reference tree by
 * oracle/Makefile into oracle/_ref/) and against the committed fixtures in tests/golden/.
 * The attention references follow lambdas that live inside the reference's test binary and
 * cannot be linked; they are pinned against the reference's own fd2 GPU kernels compiled
 * from the reference tree (oracle/_ref/, GPU tests) and its known-answer properties.
 */
#ifndef Q27_ORACLE_H
#define Q27_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* KvKind, src/cuda_common.h:53. From turbo3 up the V side is always turbo3 blocks; only the
 * K side varies: turbo3v = fp16 rows, turbo5k = 82-byte 5-bit blocks, int8-g64 = 132-byte
 * int8 blocks with one fp16 scale per 64 dims. */
enum { Q27O_KV_F16 = 0, Q27O_KV_FP8 = 1, Q27O_KV_T3 = 2, Q27O_KV_T3V = 3, Q27O_KV_T5K = 4,
       Q27O_KV_I8G64 = 5 };
#define Q27O_HD 256      /* head_dim, src/engine.cuh:45 */
#define Q27O_FD_ST 258   /* partial stride {m, l, acc[256]}, src/spec3.cuh:127 */
#define Q27O_T3_BLOCK 50 /* sizeof(block_turbo3), src/turbo3.cuh:26-32 */
#define Q27O_T5_BLOCK 82 /* sizeof(block_turbo5), src/turbo5.cuh:41-47 */
#define Q27O_I8_BLOCK 132 /* sizeof(block_i8g64), src/i8g64.cuh:36-41 */

/* ---- element conversions (src/cuda_common.h:110-121 use the CUDA intrinsics) ------- */
/* __half2float */
float q27o_half_to_float(uint16_t h);
/* __float2half_rn: round to nearest even, overflow to inf */
uint16_t q27o_float_to_half(float f);
/* float(__nv_fp8_e4m3) */
float q27o_e4m3_to_float(uint8_t v);
/* __nv_fp8_e4m3(float): round to nearest even, saturate to +-448, NaN -> 0x7f */
uint8_t q27o_float_to_e4m3(float f);
/* round a float to bf16 precision (nearest even) and return it as float */
float q27o_round_bf16(float f);
/* array forms of the above */
void q27o_float_to_half_n(const float* x, int64_t n, uint16_t* out);
void q27o_float_to_e4m3_n(const float* x, int64_t n, uint8_t* out);
void q27o_round_bf16_n(float* x, int64_t n);

/* ---- turbo3 codec (src/test_kernels.cu:1058-1107, tools/turbo3_test.cu:17-58) ------ */
const float* q27o_t3_centroids(void);          /* 8 values,  src/turbo3.cuh:38-40 */
const float* q27o_t3_s1(void);                 /* 128 signs, src/turbo3.cuh:42 */
const float* q27o_t3_s2(void);                 /* 128 signs, src/turbo3.cuh:43 */
int q27o_t3_nearest(float v);                  /* src/turbo3.cuh:57-66 */
void q27o_t3_fwht(float* x128);                /* t3_fwht,     test_kernels.cu:1065 */
void q27o_t3_fwht_inv(float* x128);            /* t3_fwht_inv, test_kernels.cu:1077 */
void q27o_t3_quant(const float* x128, uint8_t* blk50);   /* t3_quant,   :1089 */
void q27o_t3_dequant(const uint8_t* blk50, float* y128); /* t3_dequant, :1105 */

/* ---- turbo5 codec, the 5-bit K side (src/turbo5.cuh, tools/turbo5_test.cu:36-89) ---- */
const float* q27o_t5_centroids(void);          /* 32 values, src/turbo5.cuh:63-71 */
const float* q27o_t5_thresholds(void);         /* 31 values, src/turbo5.cuh:72-80 */
int q27o_t5_nearest(float v);                  /* #{i : v >= T[i]}, src/turbo5.cuh:95-107 */
/* cpu_quant5 (tools/turbo5_test.cu:67-84): turbo3's normalise -> rotate -> nearest -> norm
 * correction with the 32-level table; low 4 bits two per byte at +2, fifth bit eight per
 * byte at +66. tree != 0 sums the two norms in the order of the reference's device encoder
 * (r[j] += r[j+s], s = 64..1; turbo5_quant_group, src/turbo5.cuh:129-162) and is bit-equal
 * to it; tree == 0 sums serially (near-boundary ties against the device possible). */
void q27o_t5_quant(const float* x128, uint8_t* blk82, int tree);
void q27o_t5_dequant(const uint8_t* blk82, float* y128);   /* cpu_dequant5, :85-89 */
/* ---- int8-g64 codec (src/i8g64.cuh:48-72, tools/i8g64_test.cu:29-50) ----------------- */
/* oracle_quant: per 64 dims absmax; scale = fp16_rn(absmax / 127); codes = rint(x / the
 * ROUNDED scale) clamped to +-127; a zero scale stores zero codes. No rotation. */
void q27o_i8_quant(const float* x128, uint8_t* blk132);
void q27o_i8_dequant(const uint8_t* blk132, float* y128);  /* code * scale, oracle_deq */

/* rows helpers: ngroups consecutive 128-float groups <-> ngroups 50-byte blocks */
void q27o_t3_quant_groups(const float* x, int64_t ngroups, uint8_t* blocks, int nthreads);
void q27o_wht_groups(float* x, int64_t ngroups, int inverse, int nthreads);
void q27o_t5_quant_groups(const float* x, int64_t ngroups, uint8_t* blocks, int tree,
                          int nthreads);
void q27o_i8_quant_groups(const float* x, int64_t ngroups, uint8_t* blocks, int nthreads);

/* Dequantise `rows` cache rows of n_kv heads x 256 dims to fp32 [rows][n_kv][256].
 * fp16: half2float; fp8: float(e4m3); turbo3: CENTROIDS[idx] * half2float(norm) as an
 * fp32 product (src/turbo3.cuh:69-73) -- the bit-exact dequant target. */
int q27o_kv_dequant(const void* cache, int kvk, int64_t rows, int n_kv, float* out,
                    int nthreads);
/* the same for one side of a kind whose K and V rows differ (is_v: 0 = K rows, 1 = V rows):
 * turbo5 CENTROIDS5[idx]*norm (src/turbo5.cuh:111-115), int8-g64 code*scale
 * (src/i8g64.cuh:68-72) */
int q27o_kv_dequant_side(const void* cache, int kvk, int is_v, int64_t rows, int n_kv,
                         float* out, int nthreads);
/* bytes per cache row for a kind (fp16 2*n_kv*256, fp8 n_kv*256, turbo3 n_kv*2*50); the
 * plain form gives the K side. Engine::kv_bytes, src/engine.cuh:868-876 */
int64_t q27o_row_bytes(int kvk, int n_kv);
int64_t q27o_row_bytes_side(int kvk, int n_kv, int is_v);

/* ---- attention --------------------------------------------------------------------- */
/* Exact decode/verify reference: host_ref (src/test_kernels.cu:898-928) and the inner
 * part of host_ref_t3 (:1422-1473) without the WHT steps (the kernels take Q already
 * rotated and leave the output rotated, src/spec3.cu:930-934).
 * q: lane t, head h at q + t*q_lane_stride + h*q_stride (first 256 floats used).
 * cache: contiguous rows in logical order. Lane t attends rows [0, pos[t]].
 * out: [ntok][n_q*256]. */
int q27o_attn_decode(const float* q, int64_t q_lane_stride, int q_stride, const void* kcache,
                     const void* vcache, int kvk, const int* pos, int ntok, int n_q, int n_kv,
                     float scale, float* out, int nthreads);

/* Un-normalised partial over the row window [lo, hi) clipped to [0, pos[t]]: writes
 * {m, l, acc[256]} per (lane, head) at part + (t*n_q + h)*258. An empty window writes
 * {-FLT_MAX, 0, 0...} (the prefill convention, src/prefill.cu:1353-1362). The softmax
 * weights are exp(s - m) with m the window max, as k_attn_fd2 leaves them
 * (src/spec3.cu:908-920). */
int q27o_attn_partial(const float* q, int64_t q_lane_stride, int q_stride, const void* kcache,
                      const void* vcache, int kvk, const int* pos, int ntok, int n_q, int n_kv,
                      float scale, int64_t lo, int64_t hi, float* part, int nthreads);

/* LSE merge of nparts partial sets, k_attn_fd_combine (src/spec3.cu:706-739):
 * out = sum acc_s e^{m_s-mg} / sum l_s e^{m_s-mg}, skipping m == -FLT_MAX.
 * parts: [nparts][npairs][258]; out: [npairs][256]. If normalise == 0 the merged
 * {m, l, acc} is written instead ([npairs][258]). */
int q27o_merge_partials(const float* parts, int nparts, int64_t npairs, float* out,
                        int normalise);

/* Causal prefill reference, href (src/test_kernels.cu:2113-2165) without the WHT steps:
 * token t (t0 <= t < t0+SB) attends rows [0, base_pos + t + 1).
 * qT: [T][q_row], head h at h*q_stride; outT: [T][out_row], head h at h*256.
 * Only rows t0..t0+SB-1 of outT are written. */
int q27o_attn_prefill(const float* qT, int q_stride, int q_row, const void* kcache,
                      const void* vcache, int kvk, int base_pos, int t0, int SB, int n_q,
                      int n_kv, float scale, float* outT, int out_row, int nthreads);

/* ---- seeded synthetic data (own counter-based generator; the reference draws from
 * std::mt19937 + std::normal_distribution, src/test_kernels.cu:63-69, whose stream is
 * implementation-defined, so it is not reproduced) ------------------------------------ */
/* n iid N(0,1) floats: splitmix64(seed, counter) -> Box-Muller */
void q27o_randn(float* out, int64_t n, uint64_t seed, int nthreads);
uint64_t q27o_splitmix64(uint64_t x);

int q27o_version(void);

#ifdef __cplusplus
}
#endif
#endif
