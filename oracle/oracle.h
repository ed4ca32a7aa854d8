/* oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of libnnc's CPU attention path (ZacWalk/libllmcpu),
 * used as the checker for the CUDA path in libllmcpu_b200. Nothing in the
 * product links this: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg load it.
 *
 * Every function names the reference file:line it restates (paths relative
 * to the reference project root). The restatement is pinned against the
 * reference's own compiled kernels (oracle/_ref, built by oracle/Makefile)
 * and against the golden vectors in tests/golden/.
 *
 * Layout is the reference's: a K/V buffer is token-major, position p at row
 * p % rows, each row n_kv * head_dim elements (src/libnnc/model.h:231-242).
 */
#ifndef NNCU_ORACLE_H
#define NNCU_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORC_ATTN_BLOCK 256          /* MODEL_ATTN_BLOCK, src/libnnc/model.h:229 */
#define ORC_ATTN_PART(hd) ((hd) + 2) /* NNC_ATTN_PART, src/libnnc/nn_ops.h:45 */

enum { ORC_KV_BF16 = 0, ORC_KV_F32 = 1, ORC_KV_F16 = 2 };
enum { ORC_ROPE_NEOX = 0, ORC_ROPE_NORM = 1 };

/* Element conversions (src/libnnc/runtime.h:97-113; f16 is an extension). */
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t v);
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t v);
void orc_round_f32(float* x, size_t n, int kv_type); /* x <- widen(narrow(x)) */

/* src/libnnc/model.cpp:2300-2316 */
void orc_attn_span(int causal, int window, int pos, int n_seq, int* first, int* last);

/* src/libnnc/nn_ops.cpp:558-588 and :590-632 */
void orc_rmsnorm_f32(float* y, const float* x, size_t n, float eps);
void orc_rmsnorm_gamma_multi_f32(float* y, const float* x, size_t n_groups, size_t dim,
                                 const float* gamma, float eps);

/* src/libnnc/nn_ops.cpp:1830-1873 */
void orc_rope_f32(float* x, uint32_t n_heads, uint32_t head_dim, uint32_t n_rot, float pos,
                  float freq_base, int mode, const float* freq_factors);

/* src/libnnc/nn_ops.cpp:1877-1882 */
void orc_softcap_f32(float* y, const float* x, size_t n, float cap);

/* src/libnnc/nn_ops.cpp:372-459 (softcap: extension, 0 = off) */
void orc_attn_block(const float* q, size_t q_stride, const void* K, const void* V, int kv_type,
                    size_t kv_stride, size_t n_keys, size_t head_dim, size_t n_heads, float scale,
                    float softcap, float* scores, float* part);
/* src/libnnc/nn_ops.cpp:461-482 */
void orc_attn_merge(float* acc, const float* part, size_t head_dim, size_t n_heads);
/* src/libnnc/nn_ops.cpp:484-499 */
void orc_attn_finish(float* out, size_t out_stride, const float* acc, size_t head_dim, size_t n_heads);

/* The part of attention_forward (src/libnnc/model.cpp:1616-1757) after the
 * Q/K/V projections: per-head norms, RoPE, K/V append, blocked attention. */
typedef struct orc_attn_params
{
	int32_t n_tok, pos0, n_seq;     /* queries at pos0.., keys visible in [0, n_seq) */
	int32_t n_head, n_kv, head_dim, n_rot, rope_mode;
	float freq_base, rope_scale;    /* rpos = (pos0 + t) * rope_scale */
	const float* freq_factors;      /* n_rot/2 or NULL */
	const float* q_gamma;           /* head_dim or NULL: no Q norm */
	const float* k_gamma;           /* head_dim or NULL: no K norm */
	int32_t v_rmsnorm;              /* Gemma 4: plain RMSNorm of V rows */
	float eps, scale, softcap;
	int32_t causal, window, reuse_kv;
	const float* gate;              /* [n_tok][n_head*head_dim] or NULL: Qwen3.5 output gate */
} orc_attn_params;

/* q [n_tok][n_head*head_dim], k/v [n_tok][n_kv*head_dim] are modified in
 * place (normed, rotated) as the reference does. Kc/Vc are the layer's
 * buffers of `rows` rows, kv_type elements. out [n_tok][n_head*head_dim]. */
int orc_attention_forward(const orc_attn_params* p, float* q, float* k, float* v, void* Kc, void* Vc,
                          int kv_type, int rows, float* out);

/* Only the attend step (model.cpp:1251-1302 serial path): the cache already
 * holds every key; q is already normed and rotated. */
int orc_attend(const orc_attn_params* p, const float* q, const void* Kc, const void* Vc, int kv_type,
               int rows, float* out);

/* The projections' gemvs (src/libnnc/nn_ops.h:89-170), batched: n_batch
 * vectors x_stride floats apart in, y_stride apart out; sums in double (the
 * reference's own tests' scalar checks, tests.cpp:819-880). BF16 weights
 * (nn_ops.cpp:1000-1047); Q8_0: int8 quants, BF16 scale per 32-block
 * (nn_ops.cpp:1352-1377); Q4_S: nibbles, byte k of a block holding element k
 * low and k + 16 high, BF16 scale and bias per block, the bias term through
 * the vectors' block sums xsum (nn_ops.cpp:1252-1288, 1422-1446). */
void orc_gemv_bf16w(const uint16_t* W, const float* X, size_t x_stride, float* Y, size_t y_stride, uint32_t rows,
                    uint32_t cols, uint32_t n_batch);
void orc_gemv_q8_0(const int8_t* qs, const uint16_t* scales, const float* X, size_t x_stride, float* Y,
                   size_t y_stride, uint32_t rows, uint32_t cols, uint32_t n_batch);
void orc_gemv_q4_s(const uint8_t* qs, const uint16_t* scales, const uint16_t* biases, const float* X, size_t x_stride,
                   const float* XSUM, size_t xsum_stride, float* Y, size_t y_stride, uint32_t rows, uint32_t cols,
                   uint32_t n_batch);
/* nnc_block_sums_f32 (nn_ops.cpp:1305-1316). */
void orc_block_sums(const float* x, float* out, size_t n);
/* nnc_gemv_bf16w_argmax_f32x (nn_ops.cpp:1055-1197): the first index of the
 * largest y[r]. */
int orc_gemv_bf16w_argmax(const uint16_t* W, const float* x, uint32_t rows, uint32_t cols);
/* argmax of session.cpp:128-134 over each of n_rows rows of n floats. */
void orc_argmax_rows(const float* x, size_t x_stride, int n_rows, uint32_t n, int32_t* out);

/* Sliding-ring sizing of model_kv_init (src/libnnc/model.cpp:1934-1955). */
int orc_ring_rows(int window, int n_batch);

/* Seeded N(mean, std) floats from std::mt19937 + std::normal_distribution
 * <float>, the generator the reference's tests use (tests.cpp:2452-2453).
 * One stream per handle so q, k, v, gamma can be drawn in order. */
void* orc_rng_new(uint32_t seed);
void orc_rng_normal(void* rng, float* out, size_t n, float mean, float stddev);
void orc_rng_uniform(void* rng, float* out, size_t n, float lo, float hi);
void orc_rng_free(void* rng);

#ifdef __cplusplus
}
#endif
#endif
