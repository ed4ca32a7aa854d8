/* nncu.h -- C ABI of libllmcpu_b200 (libnncu.so): libnnc's attention hot path
 * on NVIDIA B200 (sm_100a).
 *
 * libnnc (ZacWalk/libllmcpu) runs attention on the CPU inside
 * attention_forward (src/libnnc/model.cpp:1559-1771), over a K/V cache held
 * in host vectors (model_kv_cache, src/libnnc/model.h:252-326). This library
 * replaces the part of attention_forward after the Q/K/V projections -- the
 * per-head Q/K RMSNorm, RoPE, the K/V append and the blocked attention
 * (model.cpp:1616-1757) -- and moves the K/V cache to HBM; on device memory it
 * also runs the whole attention_forward with its projections
 * (nncu_attention_forward_dev) and the verify logits with their argmax. nnc.h
 * and everything else in libnnc stay as they are.
 *
 * Conventions, all of them libnnc's:
 *  - Every entry point returns an int holding an nnc_status value
 *    (src/libnnc/nnc.h:50-61); NNCU_OK is 0. On failure the detail is kept per
 *    thread and read with nncu_last_error(), as nnc_last_error() does.
 *  - Nothing throws across this boundary, and nothing here prints.
 *  - A cache belongs to one caller thread at a time (nnc.h:27-32).
 *  - `stream` arguments are cudaStream_t values passed as void* (NULL = the
 *    legacy default stream); *_dev entry points take device pointers and are
 *    asynchronous on that stream. Entry points without a stream take host
 *    pointers and return when the result is in host memory.
 */
#ifndef NNCU_H
#define NNCU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NNCU_ATTN_BLOCK 256           /* MODEL_ATTN_BLOCK, src/libnnc/model.h:229 */
#define NNCU_ATTN_PART(hd) ((hd) + 2) /* NNC_ATTN_PART, src/libnnc/nn_ops.h:45 */

/* nnc_status values (src/libnnc/nnc.h:50-61), plus two for the device. */
enum
{
	NNCU_OK = 0,
	NNCU_ERR_INVALID_ARGUMENT = 1,
	NNCU_ERR_UNSUPPORTED = 2,     /* no usable sm_100 device (nnc: NNC_ERR_UNSUPPORTED_CPU) */
	NNCU_ERR_OUT_OF_MEMORY = 6,   /* HBM or pinned host memory exhausted */
	NNCU_ERR_CONTEXT_FULL = 7,
	NNCU_ERR_DEVICE = 20,         /* a CUDA call failed; nncu_last_error() has its text */
	NNCU_ERR_TIMEOUT = 21         /* a bounded wait on a peer ran out */
};

/* nnc_kv_type values (src/libnnc/nnc.h:199-203) plus F16. */
typedef enum nncu_kv_type
{
	NNCU_KV_BF16 = 0,
	NNCU_KV_F32 = 1,
	NNCU_KV_F16 = 2
} nncu_kv_type;

/* nnc_rope_mode (src/libnnc/nn_ops.h:286-290). */
typedef enum nncu_rope_mode
{
	NNCU_ROPE_NEOX = 0,
	NNCU_ROPE_NORM = 1
} nncu_rope_mode;

const char* nncu_status_string(int status);
/* Detail of the most recent failure on the calling thread; never NULL.
 * Replaces nnc_last_error() (nnc.h:66-69) for this library's calls. */
const char* nncu_last_error(void);
int nncu_last_status(void);
void nncu_clear_error(void);
/* The library's version string and the device it would use. */
const char* nncu_version(void);
int nncu_device_check(int device);

/* ---- spans ----------------------------------------------------------------
 * The keys [*first, *last] the query at `pos` attends to in a sequence whose
 * keys fill [0, n_seq). Replaces model_attn_span (model.cpp:2300-2316;
 * declared model.h:358-364). Host-only. */
void nncu_attn_span(int causal, int window, int pos, int n_seq, int* first, int* last);

/* ---- unit seam: nn_ops.h:31-61 and :79-81, :283-312, on device pointers ----
 * Same argument meaning as the reference's; every pointer is a device pointer
 * and the call is asynchronous on `stream`. */

/* nnc_attn_block (nn_ops.h:53-55): one block of n_keys keys (any count) for
 * n_heads query heads sharing one KV head. K/V rows are kv_stride elements
 * apart, of kv_type. No scores scratch: the scores never leave the chip.
 * softcap > 0 applies cap*tanh(s/cap) to the scaled scores (0 = off). */
int nncu_attn_block_dev(const float* q, size_t q_stride, const void* K, const void* V, int kv_type, size_t kv_stride,
                        size_t n_keys, size_t head_dim, size_t n_heads, float scale, float softcap, float* part,
                        void* stream);
/* nnc_attn_merge (nn_ops.h:58). */
int nncu_attn_merge_dev(float* acc, const float* part, size_t head_dim, size_t n_heads, void* stream);
/* nnc_attn_finish (nn_ops.h:61). */
int nncu_attn_finish_dev(float* out, size_t out_stride, const float* acc, size_t head_dim, size_t n_heads,
                         void* stream);
/* nnc_rmsnorm_gamma_multi_f32 (nn_ops.h:79-81). */
int nncu_rmsnorm_gamma_multi_dev(float* y, const float* x, size_t n_groups, size_t dim, const float* gamma, float eps,
                                 void* stream);
/* nnc_rmsnorm_f32 (nn_ops.h:73) over n_groups rows of dim. */
int nncu_rmsnorm_dev(float* y, const float* x, size_t n_groups, size_t dim, float eps, void* stream);
/* nnc_rope_f32 (nn_ops.h:292-294) for n_tok tokens at positions
 * (pos0 + t) * pos_scale, each token n_heads * head_dim floats. */
int nncu_rope_dev(float* x, uint32_t n_tok, uint32_t n_heads, uint32_t head_dim, uint32_t n_rot, int32_t pos0,
                  float pos_scale, float freq_base, int mode, const float* freq_factors, void* stream);
/* nnc_softcap_f32 (nn_ops.h:312). */
int nncu_softcap_dev(float* y, const float* x, size_t n, float cap, void* stream);

/* ---- the projections' gemvs (src/libnnc/nn_ops.h:89-170), device pointers --
 * n_batch vectors of cols floats x_stride apart in X, n_batch outputs of rows
 * floats y_stride apart in Y (n_batch 1 is the single-vector call); fp32
 * accumulation, asynchronous on `stream`. */
/* nnc_gemv_bf16w_f32x_batch (nn_ops.h:155-157): W BF16 [rows][cols]. */
int nncu_gemv_bf16w_f32x_batch_dev(const void* W, const float* X, size_t x_stride, float* Y, size_t y_stride,
                                   uint32_t rows, uint32_t cols, uint32_t n_batch, void* stream);
/* nnc_gemv_q8_0_f32x_batch (nn_ops.h:159-162): qs int8 [rows][cols] (16-byte
 * aligned), scales BF16 [rows][cols / 32]; cols a multiple of 32. */
int nncu_gemv_q8_0_f32x_batch_dev(const int8_t* qs, const uint16_t* scales, const float* X, size_t x_stride,
                                  float* Y, size_t y_stride, uint32_t rows, uint32_t cols, uint32_t n_batch,
                                  void* stream);
/* nnc_gemv_q4_s_f32x_batch (nn_ops.h:166-170): qs packed nibbles [rows][cols
 * / 2] (16-byte aligned; byte k of a 32-block holds element k low and k + 16
 * high), scales and biases BF16 [rows][cols / 32], XSUM the vectors' block
 * sums (nncu_block_sums_dev) xsum_stride apart; cols a multiple of 32. */
int nncu_gemv_q4_s_f32x_batch_dev(const uint8_t* qs, const uint16_t* scales, const uint16_t* biases,
                                  const float* X, size_t x_stride, const float* XSUM, size_t xsum_stride, float* Y,
                                  size_t y_stride, uint32_t rows, uint32_t cols, uint32_t n_batch, void* stream);
/* nnc_block_sums_f32 (nn_ops.h:142): out[b] = sum of x[32 b .. 32 b + 31]. */
int nncu_block_sums_dev(const float* x, float* out, size_t n, void* stream);
/* nnc_gemv_bf16w_argmax_f32x (nn_ops.h:98-115), the greedy lm_head: writes to
 * *out_index (device) the first index of the largest y[r] = W[r] . x without
 * writing y; `scratch` is 8 bytes of device memory the call uses (cleared on
 * the stream first), so calls sharing one scratch must not overlap. */
int nncu_gemv_bf16w_argmax_dev(const void* W, const float* x, uint32_t rows, uint32_t cols,
                               unsigned long long* scratch, int32_t* out_index, void* stream);

/* ---- the HBM K/V cache ------------------------------------------------------
 * Replaces model_kv_buffer / model_kv_cache storage (model.h:231-326),
 * model_kv_init (model.cpp:1891-2040) and model_kv_rewind (model.cpp:
 * 2137-2143). Sizing follows model_kv_init exactly: one buffer per
 * cache-owning layer, a causal sliding layer kept as a ring of
 * round_up(window + n_batch, 256) rows when that is smaller than n_ctx and
 * no global layer reads it, max_rewind = min over rings of rows - window, and
 * a bidirectional model shares one n_ctx-row buffer among all layers.
 *
 * Device layout (per buffer): [n_seq][n_kv][rows][head_dim] elements of the
 * cache type -- head-major, so one KV head's keys are one contiguous stream
 * -- K and V in separate 256-byte-aligned allocations. Position p of a
 * sequence is row p % rows. */

typedef struct nncu_kv nncu_kv;

typedef struct nncu_layer_desc
{
	int32_t n_kv;     /* KV heads */
	int32_t head_dim;
	int32_t window;   /* sliding window in keys; 0 = global */
	int32_t kv_layer; /* layer whose cache it reads; == its own index when it owns one */
} nncu_layer_desc;

typedef struct nncu_kv_params
{
	int32_t n_ctx;   /* most positions (model_kv_init n_ctx) */
	int32_t n_batch; /* most tokens one call appends (model_kv_init n_batch) */
	int32_t n_seq;   /* independent sequences held side by side (1 for a session) */
	int32_t kv_type; /* nncu_kv_type */
	int32_t causal;  /* 0: a bidirectional (embedding) model */
	int32_t device;  /* CUDA device ordinal */
} nncu_kv_params;

typedef struct nncu_kv_layer_info
{
	int32_t buffer;   /* the layer buffer it reads (its kv_layer) */
	int32_t rows;
	int32_t window;   /* a ring's window; 0 for a full buffer */
	int32_t n_kv, head_dim, kv_type;
	size_t head_bytes; /* bytes between KV heads: rows * head_dim * esize */
	size_t seq_bytes;  /* bytes between sequences: n_kv * head_bytes */
	void* k;           /* device pointers */
	void* v;
} nncu_kv_layer_info;

typedef struct nncu_kv_state
{
	int32_t cur_pos;    /* next position to fill (model_kv_cache::cur_pos) */
	int32_t kv_written; /* highest position written since 0, plus one */
	int32_t max_rewind; /* INT32_MAX without rings */
	int32_t n_ctx;
	size_t bytes;       /* K/V storage in HBM, all sequences */
} nncu_kv_state;

/* Per-layer sizing, as nncu_kv_create would allocate it (rows, window,
 * buffer per layer; max_rewind; total HBM bytes), without touching a device:
 * model_kv_init's rules (model.cpp:1929-1962) on their own. `per_layer` has
 * n_layer entries; its k and v pointers are left NULL. */
int nncu_kv_plan(const nncu_layer_desc* layers, int32_t n_layer, const nncu_kv_params* params,
                 nncu_kv_layer_info* per_layer, int32_t* max_rewind, size_t* bytes);
int nncu_kv_create(const nncu_layer_desc* layers, int32_t n_layer, const nncu_kv_params* params, nncu_kv** out);
void nncu_kv_free(nncu_kv* kv);
/* Decode and verify on a 16-bit (f16, bf16) cache with three or more query
 * rows per KV head (grouped heads x new tokens) and head_dim 64, 128 or 256
 * run on the tensor cores by default (tcgen05; q and the softmax weights
 * split into high and low 16-bit halves, so the products keep fp32
 * accuracy). enabled = 0 keeps those launches on the CUDA-core kernel, as
 * f32 caches and one- or two-row launches always are. No reference
 * counterpart (the reference has one CPU kernel). */
int nncu_kv_set_tensor_cores(nncu_kv* kv, int enabled);
int nncu_kv_layer(const nncu_kv* kv, int32_t layer, nncu_kv_layer_info* out);
int nncu_kv_get_state(const nncu_kv* kv, int32_t seq, nncu_kv_state* out);
/* model_kv_rewind: pos in [0, cur_pos]; refused (NNCU_ERR_INVALID_ARGUMENT,
 * nothing changed) when pos > 0 and kv_written - pos > max_rewind. */
int nncu_kv_rewind(nncu_kv* kv, int32_t seq, int32_t pos);
/* The bookkeeping model_forward does after its layers (model.cpp:2130-2133):
 * cur_pos = pos0 + n_tok; kv_written = max(pos0 == 0 ? 0 : kv_written, cur_pos). */
int nncu_kv_commit(nncu_kv* kv, int32_t seq, int32_t pos0, int32_t n_tok);
/* Copy rows into / out of a layer's cache (reference row layout
 * [n][n_kv * head_dim] of the cache type's bits; host or device memory), at
 * positions pos0 .. pos0+n-1 (row p % rows). For loading or inspecting a
 * cache; synchronous. */
int nncu_kv_write_rows(nncu_kv* kv, int32_t layer, int32_t seq, int32_t pos0, int32_t n, const void* k_rows,
                       const void* v_rows);
int nncu_kv_read_rows(const nncu_kv* kv, int32_t layer, int32_t seq, int32_t pos0, int32_t n, void* k_rows,
                      void* v_rows);

/* ---- the attention op --------------------------------------------------------
 * One layer's attention for a batch of n_tok query tokens at positions
 * pos0 .. pos0+n_tok-1: the body of attention_forward from the per-head norms
 * to the attention output (model.cpp:1616-1757). The parameters are what
 * attention_forward reads from the model and the cache. */
typedef struct nncu_attn_params
{
	int32_t n_tok, pos0, n_seq; /* n_seq: keys visible in [0, n_seq); pos0 + n_tok normally */
	int32_t n_head, n_kv, head_dim, n_rot, rope_mode;
	float freq_base, rope_scale;  /* rope position = (pos0 + t) * rope_scale */
	const float* freq_factors;    /* n_rot/2 floats or NULL (Llama 3 / Gemma 4 scaling) */
	const float* q_gamma;         /* head_dim floats, or NULL: no Q norm */
	const float* k_gamma;         /* head_dim floats, or NULL: no K norm */
	int32_t v_rmsnorm;            /* Gemma 4: RMS-normalise V rows, no gamma */
	float eps, scale, softcap;    /* softcap > 0: cap*tanh(s/cap) on scaled scores */
	int32_t causal, window, reuse_kv; /* reuse_kv: read another layer's cache, append nothing */
	/* Qwen3.5's output gate (model.cpp:1759-1760, nnc_mul_sigmoid_f32): the
	 * attention output is multiplied, element by element, by sigmoid(gate);
	 * gate is [n_tok][n_head*head_dim] like the output, or NULL (no gate). */
	const float* gate;
} nncu_attn_params;

/* The drop-in call for attention_forward: q [n_tok][n_head*head_dim] and
 * k, v [n_tok][n_kv*head_dim] are host fp32 rows straight from the
 * projections (k, v ignored when reuse_kv); out [n_tok][n_head*head_dim] host.
 * The pointer fields of `p` are host pointers. Synchronous. */
int nncu_attention(nncu_kv* kv, int32_t layer, int32_t seq, const nncu_attn_params* p, const float* q,
                   const float* k, const float* v, float* out);

/* Many layers and/or sequences in one submission. Each job is one
 * nncu_attention's worth of work. In nncu_attention_batch every pointer is a
 * host pointer and the call is synchronous (one host->device copy of all
 * inputs, one device->host copy of all outputs). In nncu_attention_batch_dev
 * every pointer is a device pointer and the call is asynchronous on `stream`;
 * the kernels bulk-copy q, k, v and the gains and write out with 16-byte
 * stores, so each of those must be 16-byte aligned (a misaligned one is
 * refused with NNCU_ERR_INVALID_ARGUMENT before anything runs).
 * Jobs of one submission must not append to a cache another of its jobs
 * reads. */
typedef struct nncu_attn_job
{
	int32_t layer, seq;
	nncu_attn_params p;
	const float* q;
	const float* k;
	const float* v;
	float* out;
} nncu_attn_job;

int nncu_attention_batch(nncu_kv* kv, const nncu_attn_job* jobs, int32_t n_jobs);

/* Pin [p, p + bytes) of the caller's host memory for the host-pointer calls
 * (cudaHostRegister, mapped and portable). A call of nncu_attention /
 * nncu_attention_batch whose every host buffer (q, k, v, the gains, the
 * frequency factors, the gate and out) lies inside registered ranges, with
 * 128 KiB or more moved in all, has one kernel read its inputs through the
 * GPU's mapping of that memory and another write its outputs back, instead
 * of copying them through the library's pinned staging block on the host
 * (the host copies of a verify step of a batch take longer than its kernels).
 * No counterpart in libnnc, which holds its activations in ordinary host
 * memory; the drop-in would register the session's scratch buffers, which
 * live as long as the session. Ranges may not overlap (registration pins
 * whole pages: keep small buffers inside one registered arena); unregister a
 * range (by its start) before its memory is freed. */
int nncu_host_register(void* p, size_t bytes);
int nncu_host_unregister(void* p);
int nncu_attention_batch_dev(nncu_kv* kv, const nncu_attn_job* jobs, int32_t n_jobs, void* stream);

/* ---- attention_forward on the device (model.cpp:1559-1768) -----------------
 * A weight matrix as the reference's gemv_batch (model.cpp:1181-1206) sees an
 * nnc_tensor: `type` NNCU_W_BF16 (data BF16 [rows][cols]), NNCU_W_Q8_0 (data
 * int8 quants [rows][cols], scales BF16 [rows][cols / 32]) or NNCU_W_Q4_S
 * (data packed nibbles [rows][cols / 2], scales and biases BF16 [rows][cols /
 * 32]); quants 16-byte aligned, cols a multiple of 32 for the quantised
 * types. Device pointers. */
enum
{
	NNCU_W_BF16 = 0,
	NNCU_W_Q8_0 = 1,
	NNCU_W_Q4_S = 2,
};

typedef struct nncu_weight
{
	int32_t type;
	uint32_t rows, cols;
	const void* data;
	const uint16_t* scales;
	const uint16_t* biases;
} nncu_weight;

/* One layer's attention weights (model_layer's attn_* tensors, model.h).
 * q: rows n_head * head_dim, or 2 * n_head * head_dim when `gated` (Qwen3.5:
 * each head's rows are its query, then its output gate). k, v: rows n_kv *
 * head_dim; v.data NULL means V is the raw K projection (Gemma 4 global
 * layers without v_proj). o: rows n_embd, cols n_head * head_dim. The q, k,
 * v biases (Qwen2) are fp32 device vectors of the projections' output length
 * or NULL. Every projection's cols is n_embd. */
typedef struct nncu_attn_weights
{
	nncu_weight q, k, v, o;
	const float* q_bias;
	const float* k_bias;
	const float* v_bias;
	int32_t gated;
} nncu_attn_weights;

/* attention_forward for n_tok tokens of one sequence, on device pointers:
 * x [n_tok][n_embd] are the normed hidden states (the reference's s.normed),
 * y [n_tok][n_embd] receives the output projection. The q / k / v gemvs
 * (with the gate split and the biases), the attention of
 * nncu_attention_batch_dev (Q / K norms, RoPE, append, attend, the gate's
 * sigmoid multiply), then the o gemv, all asynchronous on `stream`; k and v
 * are not projected when p->reuse_kv. p->gate must be NULL: the gate comes
 * from the q projection when w->gated. The pointer fields of `p` are device
 * pointers. The q, k, v and attention rows live in a scratch array of the
 * cache, grown (cudaMalloc) on a call that needs more than any before it;
 * calls on one cache are ordered on the device whatever their streams. x and
 * y must not overlap. */
int nncu_attention_forward_dev(nncu_kv* kv, int32_t layer, int32_t seq, const nncu_attn_params* p,
                               const nncu_attn_weights* w, const float* x, float* y, void* stream);

/* attention_forward for n_seqs sequences of one layer in one call (a serving
 * batch): sequence seqs[i] takes params[i] (the layer's heads the same for
 * all; n_tok, pos0, n_seq each its own) and its rows of x and y, the
 * sequences' tokens one after another. The q / k / v / o gemvs run over all
 * the tokens together (one pass over the weights for the batch), the
 * attention is one job per sequence. A sequence may appear once. */
int nncu_attention_forward_batch_dev(nncu_kv* kv, int32_t layer, int32_t n_seqs, const int32_t* seqs,
                                     const nncu_attn_params* params, const nncu_attn_weights* w, const float* x,
                                     float* y, void* stream);

/* model_logits_batch (model.cpp:2198-2208): logits [n][lm_head->rows] of n
 * hidden rows [n][lm_head->cols] (the verify rows of speculate, session.cpp:
 * 545), then final_softcap > 0 applies cap * tanh(x / cap) to each
 * (nnc_softcap_f32, nn_ops.cpp:1877-1882; the reference skips it for greedy
 * verify). For a Q4_S lm_head `xsum` (n * cols / 32 floats, the reference's
 * cache.sxsum) receives the block sums first; NULL lets the gemv form them
 * itself. Device pointers, asynchronous on `stream`. */
int nncu_logits_batch_dev(const nncu_weight* lm_head, const float* hidden, int32_t n, float* logits,
                          float final_softcap, float* xsum, void* stream);

/* Greedy verify's argmax of each of n_rows rows of n floats, x_stride apart
 * (session.cpp:128-134, 552): out[r] = the first index of the largest value
 * under >, so -0 and +0 tie, a NaN never replaces the best and a NaN in the
 * first place is the answer. Device pointers, asynchronous on `stream`. */
int nncu_argmax_rows_dev(const float* x, size_t x_stride, int32_t n_rows, uint32_t n, int32_t* out, void* stream);

/* One layer's decode / verify attention that allocates nothing: the same
 * K1 + K2 kernels as nncu_attention_batch_dev for one job, with every buffer
 * the caller's. No counterpart in the reference, whose CPU path never
 * allocates device memory: this is for callers that cannot let a library call
 * cudaMalloc -- hosts whose device memory all belongs to their own arena or
 * caching allocator, and latency-critical loops that must not stall on the
 * allocator's device synchronisation.
 *
 * q, k, v, out and the pointer fields of `p` are device pointers; k_cache and
 * v_cache are the caller's cache for this layer and sequence, laid out
 * [n_kv][rows][head_dim] of kv_type, position p at row p % rows, rows a
 * multiple of 256. Asynchronous on `stream`. It serves decode and verify:
 * n_tok is at most NNCU_NOALLOC_MAX_TOKENS, and a larger call fails with
 * NNCU_ERR_INVALID_ARGUMENT before anything runs. The kernels' scratch is one
 * 4 MiB device array inside the library, shared by every call: calls that
 * overlap on the GPU race on it (order them on one stream); a call that would
 * need more fails with NNCU_ERR_INVALID_ARGUMENT and a message. The first call
 * on each device looks the array's device address up (cudaGetSymbolAddress)
 * with that device current; make that first call during set-up. Every pointer
 * (q, k, v, out, the gains, freq_factors, k_cache, v_cache) must be 16-byte
 * aligned; a misaligned one is refused before anything runs.
 *
 * A kernel whose bounded wait runs out leaves an error word in the shared
 * array, which later calls keep; nncu_noalloc_check (below) reads it. */
/* ---- One sequence split over the GPUs of a node ----
 *
 * No counterpart in the reference (one CPU, one process). Its equivalent is
 * attend_blocks (model.cpp:1296-1319) merging 256-key blocks in order with
 * nnc_attn_merge (nn_ops.cpp:461-482): here GPU r holds and reads keys
 * [key_lo, key_hi) of the sequence, and the partials of all GPUs are merged
 * in rank order on every GPU: the attention kernel stores each GPU's partial
 * straight into every GPU's receive buffer over NVLink, and a kernel at the
 * end of the call merges, on each GPU, the partials that landed in its own
 * memory. One process per GPU; every rank makes the same calls in the same
 * order.
 *
 * nncu_group_create allocates this GPU's shared block (receive buffers,
 * counters, and the output: max_rows rows of head_dim floats, the jobs'
 * n_tok * n_head rows one after another). Exchange the handles out of band
 * (nncu_group_handle on each rank, nncu_group_open with every peer's) before
 * the first call. nncu_attention_split_dev runs the jobs over this GPU's keys
 * [key_lo, key_hi) (key_lo a multiple of 256; the new tokens are appended
 * only by the GPU whose range holds them) and leaves the merged attention in
 * nncu_group_output() of every GPU when `stream` reaches the end of the call.
 * A rank that does not take part makes the others' calls end with
 * NNCU_ERR_TIMEOUT (reported by nncu_sync) after 2 s (nncu_group_set_timeout)
 * instead of hanging.
 *
 * After a timeout the group is poisoned on the GPU that saw it: a late
 * partial may still be counted there, so every later split call on that GPU
 * fails with NNCU_ERR_TIMEOUT rather than merge stale partials. To recover,
 * every rank waits for its own calls (nncu_sync), the ranks meet on the host
 * (a barrier), each calls nncu_group_reset, and they meet again before the
 * next call: the counters of both parities are cleared and the call count
 * restarts in step on every rank. */
typedef struct nncu_group nncu_group;
#define NNCU_GROUP_HANDLE_BYTES 64
int nncu_group_create(int32_t device, int32_t rank, int32_t world, int32_t max_rows, int32_t head_dim,
                      nncu_group** out);
int nncu_group_handle(const nncu_group* g, void* handle);
int nncu_group_open(nncu_group* g, int32_t peer, const void* handle);
float* nncu_group_output(const nncu_group* g);
/* Copy the first n_floats of this GPU's merged output to dst (host or device
 * memory), ordered on `stream` after the split calls before it. */
int nncu_group_copy_output(const nncu_group* g, float* dst, size_t n_floats, void* stream);
void nncu_group_free(nncu_group* g);
/* The bounded wait of each GPU's end-of-call merge, in milliseconds (1 to
 * 60000; 2000 by default). */
int nncu_group_set_timeout(nncu_group* g, uint32_t ms);
/* Clear this GPU's counters and poison word and restart its call count; only
 * at a step boundary that every rank has reached with no call in flight
 * (see above). Waits for this GPU to be idle. */
int nncu_group_reset(nncu_group* g);
/* Failure injection for tests: this rank's next n_calls split calls store
 * their partials but never count them, so every GPU's merge of those calls
 * runs out of time (NNCU_ERR_TIMEOUT) -- a message dropped on the host's
 * side, with no fault on the device. */
int nncu_group_inject_drop(nncu_group* g, int32_t n_calls);
int nncu_attention_split_dev(nncu_kv* kv, nncu_group* group, const nncu_attn_job* jobs, int32_t n_jobs,
                             int32_t key_lo, int32_t key_hi, void* stream);

#define NNCU_NOALLOC_MAX_TOKENS 64
int nncu_attention_noalloc(const nncu_attn_params* p, const float* q, const float* k, const float* v, float* out,
                           void* k_cache, void* v_cache, int32_t kv_type, int32_t rows, void* stream);
/* Wait for `stream` and report whether a no-allocation call on the current
 * device since the last check had a kernel whose bounded wait ran out
 * (NNCU_ERR_TIMEOUT: the outputs of those calls are void); the word is then
 * cleared. Allocates nothing. No reference counterpart. */
int nncu_noalloc_check(void* stream);

/* Wait for `stream` (the asynchronous calls' completion) and report a kernel
 * whose bounded wait ran out (NNCU_ERR_TIMEOUT: the outputs are void). The
 * synchronous calls make this check themselves. No reference counterpart:
 * libnnc's calls are all synchronous. */
int nncu_sync(nncu_kv* kv, void* stream);

/* ---- profiling ----------------------------------------------------------------
 * The phase profiler of nnc_perf_enable / nnc_perf_reset / nnc_perf_report
 * (nnc.h:404-415; slots NNC_PERF_ATTN_ROPE and NNC_PERF_ATTN_CORE,
 * runtime.h:147-168) for this path: attn_rope is K1 (per-head norms, RoPE,
 * append), attn_core is K2+K3 (attention and its merge). Device time comes
 * from CUDA events recorded around the launches on their stream; bytes are
 * the algorithmic traffic (K/V of every key attended, q in, output out). Off
 * by default and free when off; process-wide, meant for one caller at a time. */
enum
{
	NNCU_PERF_ATTN_ROPE = 0,
	NNCU_PERF_ATTN_CORE = 1,
	NNCU_PERF_COUNT = 2
};

typedef struct nncu_perf_phase
{
	double ms;      /* device time */
	int64_t calls;  /* launches */
	uint64_t bytes; /* algorithmic bytes moved */
} nncu_perf_phase;

void nncu_perf_enable(int enabled);
void nncu_perf_reset(void);
/* Wait for the launches recorded so far and fill out[NNCU_PERF_COUNT]. */
int nncu_perf_read(nncu_perf_phase* out);
/* A text table like nnc_perf_report's: ms, share, calls, us/call, GB/s. */
const char* nncu_perf_report(const char* title, int32_t n_tokens);
/* Kernels this library has launched since it was loaded (all threads). */
uint64_t nncu_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif
