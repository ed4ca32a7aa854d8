// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C-callable face for the reference's OWN compiled attention kernels, so
// the checker and the CPU baseline run the reference's arithmetic rather than
// a restatement of it. oracle/Makefile compiles this file against the
// reference's headers and links it with the reference's libnnc objects
// (built from the reference's sources with its own compiler flags) into
// oracle/_ref/libnnc_ref.so. Nothing of the reference is copied here.
//
// The reference keeps its attention dispatch (attend_block, attend_token,
// attend_chunks, attend_blocks: src/libnnc/model.cpp:1251-1319, and the
// choice between them at :1696-1757) in an anonymous namespace, so it cannot
// be linked. ref_attention_forward() below re-expresses that dispatch around
// the exported kernels nnc_attn_block / nnc_attn_merge / nnc_attn_finish,
// nnc_rmsnorm_gamma_multi_f32, nnc_rmsnorm_f32, nnc_rope_f32 and
// nnc_f32_to_bf16, and parallelises it through the reference's own worker
// pool (nnc_parallel_for, sized by nnc_set_num_threads).
#include "model.h"
#include "nn_ops.h"
#include "runtime.h"

#include "oracle.h"

#include <algorithm>
#include <cstring>
#include <vector>

namespace
{
	// One attention call, as the pool's workers see it.
	struct ref_call
	{
		const orc_attn_params* p;
		const float* q;
		float* out;
		const uint8_t* K;
		const uint8_t* V;
		size_t esize;
		int rows;
		float* slots;    // n_slots x slot floats: block scores, then two partials
		size_t slot;
		float* parts;    // decode: one partial per (KV head, block)
		int n_chunks;
		int blk0, n_blk; // decode: the blocks of the single query's span
	};

	size_t group_of(const orc_attn_params* p) { return static_cast<size_t>(p->n_head / p->n_kv); }

	// Block b of token t's span for KV head kv_h, into `part`.
	void one_block(const ref_call& c, int t, int kv_h, int first, int last, int b, float* scores, float* part)
	{
		const orc_attn_params* p = c.p;
		const int lo = std::max(first, b * MODEL_ATTN_BLOCK);
		const int hi = std::min(last, (b + 1) * MODEL_ATTN_BLOCK - 1);
		const size_t hd = static_cast<size_t>(p->head_dim);
		const size_t kv_dim = static_cast<size_t>(p->n_kv) * hd;
		const size_t g = group_of(p);
		const size_t byte_off = (static_cast<size_t>(lo % c.rows) * kv_dim + kv_h * hd) * c.esize;
		const float* qh = c.q + static_cast<size_t>(t) * p->n_head * hd + kv_h * g * hd;
		nnc_attn_block(qh, hd, c.K + byte_off, c.V + byte_off, c.esize == 2, kv_dim, static_cast<size_t>(hi + 1 - lo),
		               hd, g, p->scale, scores, part);
	}

	// Every KV head of token t: its blocks in increasing order, merged as they come.
	void one_token(const ref_call& c, int t, float* slot)
	{
		const orc_attn_params* p = c.p;
		int first, last;
		model_attn_span(p->causal != 0, p->window, p->pos0 + t, p->n_seq, &first, &last);
		const size_t hd = static_cast<size_t>(p->head_dim);
		const size_t g = group_of(p);
		float* scores = slot;
		float* acc = slot + g * MODEL_ATTN_BLOCK;
		float* tmp = acc + g * NNC_ATTN_PART(hd);
		float* out_t = c.out + static_cast<size_t>(t) * p->n_head * hd;
		for (int kv_h = 0; kv_h < p->n_kv; ++kv_h)
		{
			const int b_first = first / MODEL_ATTN_BLOCK, b_last = last / MODEL_ATTN_BLOCK;
			for (int b = b_first; b <= b_last; ++b)
			{
				one_block(c, t, kv_h, first, last, b, scores, b == b_first ? acc : tmp);
				if (b != b_first) nnc_attn_merge(acc, tmp, hd, g);
			}
			nnc_attn_finish(out_t + kv_h * g * hd, hd, acc, hd, g);
		}
	}

	// A batch: chunk k takes tokens k, k + n_chunks, ... with its own slot.
	void token_chunks(uint32_t k0, uint32_t k1, void* user)
	{
		const auto& c = *static_cast<const ref_call*>(user);
		for (uint32_t k = k0; k < k1; ++k)
			for (int t = static_cast<int>(k); t < c.p->n_tok; t += c.n_chunks) one_token(c, t, c.slots + k * c.slot);
	}

	// Decode: the (KV head, block) items of the one query, item i into parts[i].
	void block_chunks(uint32_t k0, uint32_t k1, void* user)
	{
		const auto& c = *static_cast<const ref_call*>(user);
		int first, last;
		model_attn_span(c.p->causal != 0, c.p->window, c.p->pos0, c.p->n_seq, &first, &last);
		const size_t pw = group_of(c.p) * NNC_ATTN_PART(static_cast<size_t>(c.p->head_dim));
		const int n_items = c.p->n_kv * c.n_blk;
		for (uint32_t k = k0; k < k1; ++k)
			for (int i = static_cast<int>(k); i < n_items; i += c.n_chunks)
				one_block(c, 0, i / c.n_blk, first, last, c.blk0 + i % c.n_blk, c.slots + k * c.slot,
				          c.parts + static_cast<size_t>(i) * pw);
	}

	std::vector<float> g_slots, g_parts;
}

extern "C" {

void ref_set_num_threads(int n) { nnc_set_num_threads_avx(n); }
int ref_num_threads(void) { return nnc_num_threads_avx(); }

void ref_attn_span(int causal, int window, int pos, int n_seq, int* first, int* last)
{
	model_attn_span(causal != 0, window, pos, n_seq, first, last);
}

uint16_t ref_f32_to_bf16(float f) { return nnc_f32_to_bf16(f); }

// The projections' gemvs and their helpers, the reference's own (nn_ops.h:89-183).
void ref_gemv_bf16w(const void* W, const float* X, size_t x_stride, float* Y, size_t y_stride, uint32_t rows,
                    uint32_t cols, uint32_t n_batch)
{
	nnc_gemv_bf16w_f32x_batch(W, X, x_stride, Y, y_stride, rows, cols, n_batch);
}
void ref_gemv_q8_0(const int8_t* qs, const uint16_t* scales, const float* X, size_t x_stride, float* Y,
                   size_t y_stride, uint32_t rows, uint32_t cols, uint32_t n_batch)
{
	nnc_gemv_q8_0_f32x_batch(qs, scales, X, x_stride, Y, y_stride, rows, cols, n_batch);
}
void ref_gemv_q4_s(const uint8_t* qs, const uint16_t* scales, const uint16_t* biases, const float* X, size_t x_stride,
                   const float* XSUM, size_t xsum_stride, float* Y, size_t y_stride, uint32_t rows, uint32_t cols,
                   uint32_t n_batch)
{
	nnc_gemv_q4_s_f32x_batch(qs, scales, biases, X, x_stride, XSUM, xsum_stride, Y, y_stride, rows, cols, n_batch);
}
void ref_block_sums(const float* x, float* out, size_t n) { nnc_block_sums_f32(x, out, n); }
int ref_gemv_bf16w_argmax(const void* W, const float* x, uint32_t rows, uint32_t cols)
{
	return nnc_gemv_bf16w_argmax_f32x(W, x, rows, cols);
}
void ref_quantize_f32_to_q4_s(const float* src, uint8_t* qs, uint16_t* scales, uint16_t* biases, size_t n)
{
	nnc_quantize_f32_to_q4_s(src, qs, scales, biases, n);
}

void ref_rmsnorm_f32(float* y, const float* x, size_t n, float eps) { nnc_rmsnorm_f32(y, x, n, eps); }

void ref_rmsnorm_gamma_multi_f32(float* y, const float* x, size_t n_groups, size_t dim, const float* gamma, float eps)
{
	nnc_rmsnorm_gamma_multi_f32(y, x, n_groups, dim, gamma, eps);
}

void ref_rope_f32(float* x, uint32_t n_heads, uint32_t head_dim, uint32_t n_rot, float pos, float freq_base, int mode,
                  const float* freq_factors)
{
	nnc_rope_f32(x, n_heads, head_dim, n_rot, pos, freq_base, static_cast<nnc_rope_mode>(mode), freq_factors);
}

void ref_softcap_f32(float* y, const float* x, size_t n, float cap) { nnc_softcap_f32(y, x, n, cap); }

void ref_attn_block(const float* q, size_t q_stride, const void* K, const void* V, int kv_bf16, size_t kv_stride,
                    size_t n_keys, size_t head_dim, size_t n_heads, float scale, float* scores, float* part)
{
	nnc_attn_block(q, q_stride, K, V, kv_bf16 != 0, kv_stride, n_keys, head_dim, n_heads, scale, scores, part);
}

void ref_attn_merge(float* acc, const float* part, size_t head_dim, size_t n_heads)
{
	nnc_attn_merge(acc, part, head_dim, n_heads);
}

void ref_attn_finish(float* out, size_t out_stride, const float* acc, size_t head_dim, size_t n_heads)
{
	nnc_attn_finish(out, out_stride, acc, head_dim, n_heads);
}

// The attend step only (cache already filled, q already normed and rotated),
// with the reference's choice of serial / per-token / per-block dispatch.
// kv_type: ORC_KV_BF16 or ORC_KV_F32 (the reference has no F16 cache).
// Returns 0, or 1 for arguments the reference cannot take.
int ref_attend(const orc_attn_params* p, const float* q, const void* Kc, const void* Vc, int kv_type, int rows,
               float* out)
{
	if (kv_type != ORC_KV_BF16 && kv_type != ORC_KV_F32) return 1;
	if (p->softcap > 0.0f || p->n_kv <= 0 || p->n_head % p->n_kv != 0 || rows <= 0) return 1;
	const size_t hd = static_cast<size_t>(p->head_dim);
	const size_t g = group_of(p);
	const size_t pw = g * NNC_ATTN_PART(hd);
	const size_t kv_dim = static_cast<size_t>(p->n_kv) * hd;
	const int n_slots = std::max(1, std::min(nnc_num_threads_avx(), 64));

	ref_call c{};
	c.p = p;
	c.q = q;
	c.out = out;
	c.K = static_cast<const uint8_t*>(Kc);
	c.V = static_cast<const uint8_t*>(Vc);
	c.esize = kv_type == ORC_KV_BF16 ? 2 : 4;
	c.rows = rows;
	c.slot = g * MODEL_ATTN_BLOCK + 2 * pw;
	if (g_slots.size() < c.slot * n_slots) g_slots.resize(c.slot * n_slots);
	c.slots = g_slots.data();

	uint64_t bytes = 0;
	for (int t = 0; t < p->n_tok; ++t)
	{
		int first, last;
		model_attn_span(p->causal != 0, p->window, p->pos0 + t, p->n_seq, &first, &last);
		bytes += 2ull * static_cast<uint64_t>(last + 1 - first) * kv_dim * c.esize;
	}
	constexpr uint64_t parallel_bytes = 256u << 10; // the reference's threshold
	if (p->n_tok == 1 && bytes >= parallel_bytes && n_slots > 1)
	{
		int first, last;
		model_attn_span(p->causal != 0, p->window, p->pos0, p->n_seq, &first, &last);
		c.blk0 = first / MODEL_ATTN_BLOCK;
		c.n_blk = last / MODEL_ATTN_BLOCK + 1 - c.blk0;
		const int n_items = p->n_kv * c.n_blk;
		c.n_chunks = std::min(n_items, n_slots);
		if (g_parts.size() < pw * n_items) g_parts.resize(pw * n_items);
		c.parts = g_parts.data();
		nnc_parallel_for(static_cast<uint32_t>(c.n_chunks), block_chunks, &c);
		for (int kv_h = 0; kv_h < p->n_kv; ++kv_h)
		{
			float* acc = c.parts + static_cast<size_t>(kv_h) * c.n_blk * pw;
			for (int b = 1; b < c.n_blk; ++b) nnc_attn_merge(acc, acc + b * pw, hd, g);
			nnc_attn_finish(out + kv_h * g * hd, hd, acc, hd, g);
		}
	}
	else
	{
		c.n_chunks = std::min(p->n_tok, n_slots);
		if (c.n_chunks > 1 && bytes >= parallel_bytes)
			nnc_parallel_for(static_cast<uint32_t>(c.n_chunks), token_chunks, &c);
		else
			for (int t = 0; t < p->n_tok; ++t) one_token(c, t, c.slots);
	}
	return 0;
}

// Norms, RoPE, append and attend: the reference's attention_forward from the
// Q/K norm onward (model.cpp:1616-1757), on the reference's kernels.
int ref_attention_forward(const orc_attn_params* p, float* q, float* k, float* v, void* Kc, void* Vc, int kv_type,
                          int rows, float* out)
{
	if (kv_type != ORC_KV_BF16 && kv_type != ORC_KV_F32) return 1;
	const int hd = p->head_dim;
	const size_t q_dim = static_cast<size_t>(p->n_head) * hd;
	const size_t kv_dim = static_cast<size_t>(p->n_kv) * hd;
	if (p->q_gamma) nnc_rmsnorm_gamma_multi_f32(q, q, static_cast<size_t>(p->n_tok) * p->n_head, hd, p->q_gamma, p->eps);
	if (!p->reuse_kv)
	{
		if (p->k_gamma)
			nnc_rmsnorm_gamma_multi_f32(k, k, static_cast<size_t>(p->n_tok) * p->n_kv, hd, p->k_gamma, p->eps);
		if (p->v_rmsnorm)
			for (int i = 0; i < p->n_tok * p->n_kv; ++i)
				nnc_rmsnorm_f32(v + static_cast<size_t>(i) * hd, v + static_cast<size_t>(i) * hd, hd, p->eps);
	}
	for (int t = 0; t < p->n_tok; ++t)
	{
		const float rpos = static_cast<float>(p->pos0 + t) * p->rope_scale;
		const auto mode = static_cast<nnc_rope_mode>(p->rope_mode);
		nnc_rope_f32(q + t * q_dim, p->n_head, hd, p->n_rot, rpos, p->freq_base, mode, p->freq_factors);
		if (!p->reuse_kv) nnc_rope_f32(k + t * kv_dim, p->n_kv, hd, p->n_rot, rpos, p->freq_base, mode, p->freq_factors);
	}
	if (!p->reuse_kv)
		for (int t = 0; t < p->n_tok; ++t)
		{
			const size_t row = static_cast<size_t>((p->pos0 + t) % rows) * kv_dim;
			const float* kt = k + t * kv_dim;
			const float* vt = v + t * kv_dim;
			if (kv_type == ORC_KV_BF16)
			{
				auto* Kd = static_cast<nnc_bf16_t*>(Kc) + row;
				auto* Vd = static_cast<nnc_bf16_t*>(Vc) + row;
				for (size_t i = 0; i < kv_dim; ++i)
				{
					Kd[i] = nnc_f32_to_bf16(kt[i]);
					Vd[i] = nnc_f32_to_bf16(vt[i]);
				}
			}
			else
			{
				std::memcpy(static_cast<float*>(Kc) + row, kt, kv_dim * sizeof(float));
				std::memcpy(static_cast<float*>(Vc) + row, vt, kv_dim * sizeof(float));
			}
		}
	const int rc = ref_attend(p, q, Kc, Vc, kv_type, rows, out);
	// Qwen3.5's gate, the reference's own kernel (model.cpp:1759-1760)
	if (rc == 0 && p->gate) nnc_mul_sigmoid_f32(out, p->gate, static_cast<size_t>(p->n_tok) * q_dim);
	return rc;
}

} // extern "C"
