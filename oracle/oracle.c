/* oracle.c -- TEST INFRASTRUCTURE ONLY: the CPU restatement of libnnc's
 * attention path that the CUDA path is checked against. Not linked by the
 * product. Each function cites the reference file:line it restates.
 *
 * The arithmetic follows the reference's order where that order is part of
 * the algorithm (8-lane partial sums for the q.k dot, keys in increasing
 * order, blocks of 256 keys aligned to absolute positions, partials merged
 * in block order). It uses libm's expf where the reference uses its AVX2
 * polynomial (nn_ops.cpp:57-97, relative error ~3e-7): the restatement is
 * therefore within a few ulp of the reference, which tests/test_oracle.py
 * checks against the reference's own compiled kernels.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---- element conversions: runtime.h:97-113 ------------------------------ */

uint16_t orc_f32_to_bf16(float f)
{
	uint32_t u;
	memcpy(&u, &f, 4);
	/* round to nearest, ties to even, on the upper 16 bits */
	u += 0x7fffu + ((u >> 16) & 1u);
	return (uint16_t)(u >> 16);
}

float orc_bf16_to_f32(uint16_t v)
{
	const uint32_t u = (uint32_t)v << 16;
	float f;
	memcpy(&f, &u, 4);
	return f;
}

uint16_t orc_f32_to_f16(float f)
{
	const _Float16 h = (_Float16)f; /* IEEE round to nearest even */
	uint16_t u;
	memcpy(&u, &h, 2);
	return u;
}

float orc_f16_to_f32(uint16_t v)
{
	_Float16 h;
	memcpy(&h, &v, 2);
	return (float)h;
}

void orc_round_f32(float* x, size_t n, int kv_type)
{
	for (size_t i = 0; i < n; ++i)
	{
		if (kv_type == ORC_KV_BF16) x[i] = orc_bf16_to_f32(orc_f32_to_bf16(x[i]));
		else if (kv_type == ORC_KV_F16) x[i] = orc_f16_to_f32(orc_f32_to_f16(x[i]));
	}
}

static inline float kv_load(const void* base, size_t i, int kv_type)
{
	switch (kv_type)
	{
	case ORC_KV_BF16: return orc_bf16_to_f32(((const uint16_t*)base)[i]);
	case ORC_KV_F16: return orc_f16_to_f32(((const uint16_t*)base)[i]);
	default: return ((const float*)base)[i];
	}
}

static inline size_t kv_esize(int kv_type) { return kv_type == ORC_KV_F32 ? 4 : 2; }

/* ---- spans: model.cpp:2300-2316 ------------------------------------------ */

void orc_attn_span(int causal, int window, int pos, int n_seq, int* first, int* last)
{
	if (causal)
	{
		/* the last `window` positions up to pos (all of them without a window) */
		*first = (window > 0 && pos + 1 > window) ? pos + 1 - window : 0;
		*last = pos < n_seq - 1 ? pos : n_seq - 1;
		return;
	}
	/* bidirectional: everything, or |key - pos| <= window / 2 */
	int f = 0, l = n_seq - 1;
	if (window > 0)
	{
		const int half = window / 2;
		f = pos - half > 0 ? pos - half : 0;
		l = pos + half < n_seq - 1 ? pos + half : n_seq - 1;
	}
	*first = f;
	*last = l;
}

int orc_ring_rows(int window, int n_batch)
{
	/* model.cpp:1934: round_up(window + n_batch, MODEL_ATTN_BLOCK) */
	const int nb = n_batch > 0 ? n_batch : 1;
	return (window + nb + ORC_ATTN_BLOCK - 1) / ORC_ATTN_BLOCK * ORC_ATTN_BLOCK;
}

/* ---- norms: nn_ops.cpp:558-632 ------------------------------------------- */

/* Sum of squares as the reference forms it: 8 fused partial sums over the
 * 8-aligned prefix, folded (lo+hi, then pairwise), widened to double, then
 * the tail added in double. */
static double sum_squares(const float* x, size_t n)
{
	size_t i = 0;
	double s = 0.0;
	if (n >= 8)
	{
		float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
		for (; i + 8 <= n; i += 8)
			for (int j = 0; j < 8; ++j) acc[j] = fmaf(x[i + j], x[i + j], acc[j]);
		const float a0 = acc[0] + acc[4], a1 = acc[1] + acc[5], a2 = acc[2] + acc[6], a3 = acc[3] + acc[7];
		s = (double)((a0 + a1) + (a2 + a3));
	}
	for (; i < n; ++i) s += (double)x[i] * x[i];
	return s;
}

void orc_rmsnorm_f32(float* y, const float* x, size_t n, float eps)
{
	if (n == 0) return;
	const double s2 = sum_squares(x, n);
	const float scale = (float)(1.0 / sqrt(s2 / (double)n + eps));
	for (size_t i = 0; i < n; ++i) y[i] = x[i] * scale;
}

void orc_rmsnorm_gamma_multi_f32(float* y, const float* x, size_t n_groups, size_t dim, const float* gamma,
                                 float eps)
{
	if (n_groups == 0 || dim == 0) return;
	const float inv_dim = 1.0f / (float)dim;
	for (size_t g = 0; g < n_groups; ++g)
	{
		const float* xg = x + g * dim;
		float* yg = y + g * dim;
		const double s2 = sum_squares(xg, dim);
		const float scale = (float)(1.0 / sqrt(s2 * inv_dim + eps));
		for (size_t i = 0; i < dim; ++i) yg[i] = xg[i] * scale * gamma[i];
	}
}

/* ---- RoPE: nn_ops.cpp:1830-1873 ------------------------------------------ */

void orc_rope_f32(float* x, uint32_t n_heads, uint32_t head_dim, uint32_t n_rot, float pos, float freq_base,
                  int mode, const float* freq_factors)
{
	if (n_rot == 0) return;
	const uint32_t half = n_rot / 2;
	float* cs = (float*)malloc(sizeof(float) * half);
	float* sn = (float*)malloc(sizeof(float) * half);
	/* The inverse frequencies come from the fp32 recurrence inv *= base^(-2/n_rot),
	 * not from a pow per lane: at positions near 1e5 the angle's rounding is part
	 * of the answer, so it is formed exactly as the reference forms it. */
	const float ratio = powf(freq_base, -2.0f / (float)n_rot);
	float inv = 1.0f;
	for (uint32_t i = 0; i < half; ++i)
	{
		float theta = pos * inv;
		if (freq_factors) theta /= freq_factors[i];
		cs[i] = cosf(theta);
		sn[i] = sinf(theta);
		inv *= ratio;
	}
	const uint32_t step = mode == ORC_ROPE_NEOX ? 1 : 2;   /* lane of pair i */
	const uint32_t other = mode == ORC_ROPE_NEOX ? half : 1; /* its partner's offset */
	for (uint32_t h = 0; h < n_heads; ++h)
	{
		float* xh = x + (size_t)h * head_dim;
		for (uint32_t i = 0; i < half; ++i)
		{
			float* p = xh + i * step;
			const float a = p[0], b = p[other];
			p[0] = cs[i] * a - sn[i] * b;
			p[other] = sn[i] * a + cs[i] * b;
		}
	}
	free(cs);
	free(sn);
}

/* ---- soft-cap: nn_ops.cpp:1877-1882 -------------------------------------- */

void orc_softcap_f32(float* y, const float* x, size_t n, float cap)
{
	const float inv = 1.0f / cap;
	for (size_t i = 0; i < n; ++i) y[i] = tanhf(x[i] * inv) * cap;
}

/* ---- blocked attention: nn_ops.cpp:351-499 ------------------------------- */

/* q.k with the reference's lane order: 8 fused partial sums, folded, then the tail. */
static float dot_kv(const float* q, const void* K, size_t koff, size_t hd, int kv_type)
{
	float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
	const size_t hd8 = hd & ~(size_t)7;
	for (size_t i = 0; i < hd8; i += 8)
		for (int j = 0; j < 8; ++j) acc[j] = fmaf(q[i + j], kv_load(K, koff + i + j, kv_type), acc[j]);
	const float a0 = acc[0] + acc[4], a1 = acc[1] + acc[5], a2 = acc[2] + acc[6], a3 = acc[3] + acc[7];
	float s = (a0 + a1) + (a2 + a3);
	for (size_t i = hd8; i < hd; ++i) s += q[i] * kv_load(K, koff + i, kv_type);
	return s;
}

void orc_attn_block(const float* q, size_t q_stride, const void* K, const void* V, int kv_type, size_t kv_stride,
                    size_t n_keys, size_t head_dim, size_t n_heads, float scale, float softcap, float* scores,
                    float* part)
{
	if (n_keys == 0 || n_heads == 0) return;
	const size_t pw = ORC_ATTN_PART(head_dim);
	/* scores[h][t] = scale * q_h . k_t, each K row read once for every head */
	for (size_t t = 0; t < n_keys; ++t)
		for (size_t h = 0; h < n_heads; ++h)
			scores[h * n_keys + t] = dot_kv(q + h * q_stride, K, t * kv_stride, head_dim, kv_type) * scale;
	if (softcap > 0.0f)
		for (size_t h = 0; h < n_heads; ++h) orc_softcap_f32(scores + h * n_keys, scores + h * n_keys, n_keys, softcap);
	/* per head: the block's own max m, weights exp(s - m), their sum l */
	for (size_t h = 0; h < n_heads; ++h)
	{
		float* s = scores + h * n_keys;
		float m = s[0];
		for (size_t t = 1; t < n_keys; ++t) m = s[t] > m ? s[t] : m;
		float l = 0.0f;
		for (size_t t = 0; t < n_keys; ++t)
		{
			s[t] = expf(s[t] - m);
			l += s[t];
		}
		part[h * pw + head_dim] = m;
		part[h * pw + head_dim + 1] = l;
	}
	/* o_h = sum_t w_ht * v_t, keys outermost: the first row writes, the rest accumulate */
	for (size_t t = 0; t < n_keys; ++t)
		for (size_t h = 0; h < n_heads; ++h)
		{
			const float w = scores[h * n_keys + t];
			float* o = part + h * pw;
			for (size_t i = 0; i < head_dim; ++i)
			{
				const float vi = kv_load(V, t * kv_stride + i, kv_type);
				o[i] = t == 0 ? w * vi : fmaf(w, vi, o[i]);
			}
		}
}

void orc_attn_merge(float* acc, const float* part, size_t head_dim, size_t n_heads)
{
	const size_t pw = ORC_ATTN_PART(head_dim);
	for (size_t h = 0; h < n_heads; ++h)
	{
		float* a = acc + h * pw;
		const float* b = part + h * pw;
		const float m = a[head_dim] > b[head_dim] ? a[head_dim] : b[head_dim];
		const float ca = expf(a[head_dim] - m), cb = expf(b[head_dim] - m);
		for (size_t i = 0; i < head_dim; ++i) a[i] = fmaf(b[i], cb, a[i] * ca);
		a[head_dim] = m;
		a[head_dim + 1] = a[head_dim + 1] * ca + b[head_dim + 1] * cb;
	}
}

void orc_attn_finish(float* out, size_t out_stride, const float* acc, size_t head_dim, size_t n_heads)
{
	const size_t pw = ORC_ATTN_PART(head_dim);
	for (size_t h = 0; h < n_heads; ++h)
	{
		const float* a = acc + h * pw;
		const float l = a[head_dim + 1];
		const float inv = l > 0.0f ? 1.0f / l : 0.0f;
		for (size_t i = 0; i < head_dim; ++i) out[h * out_stride + i] = a[i] * inv;
	}
}

/* ---- dispatch: model.cpp:1251-1302 (serial path) -------------------------- */

int orc_attend(const orc_attn_params* p, const float* q, const void* Kc, const void* Vc, int kv_type, int rows,
               float* out)
{
	if (p->n_kv <= 0 || p->n_head % p->n_kv != 0 || rows <= 0) return 1;
	const size_t hd = (size_t)p->head_dim;
	const size_t kv_dim = (size_t)p->n_kv * hd;
	const size_t q_dim = (size_t)p->n_head * hd;
	const size_t group = (size_t)(p->n_head / p->n_kv);
	const size_t pw = group * ORC_ATTN_PART(hd);
	const size_t es = kv_esize(kv_type);
	float* scores = (float*)malloc(sizeof(float) * group * ORC_ATTN_BLOCK);
	float* acc = (float*)malloc(sizeof(float) * pw);
	float* tmp = (float*)malloc(sizeof(float) * pw);
	for (int t = 0; t < p->n_tok; ++t)
	{
		int first, last;
		orc_attn_span(p->causal, p->window, p->pos0 + t, p->n_seq, &first, &last);
		for (int kv_h = 0; kv_h < p->n_kv; ++kv_h)
		{
			const float* qh = q + (size_t)t * q_dim + (size_t)kv_h * group * hd;
			/* blocks aligned to absolute multiples of 256 keys, merged in order */
			for (int b = first / ORC_ATTN_BLOCK; b <= last / ORC_ATTN_BLOCK; ++b)
			{
				const int k0 = first > b * ORC_ATTN_BLOCK ? first : b * ORC_ATTN_BLOCK;
				const int k1e = b * ORC_ATTN_BLOCK + ORC_ATTN_BLOCK - 1;
				const int k1 = last < k1e ? last : k1e;
				const size_t off = ((size_t)(k0 % rows) * kv_dim + (size_t)kv_h * hd) * es;
				const int first_block = b == first / ORC_ATTN_BLOCK;
				orc_attn_block(qh, hd, (const char*)Kc + off, (const char*)Vc + off, kv_type, kv_dim,
				               (size_t)(k1 + 1 - k0), hd, group, p->scale, p->softcap, scores,
				               first_block ? acc : tmp);
				if (!first_block) orc_attn_merge(acc, tmp, hd, group);
			}
			orc_attn_finish(out + (size_t)t * q_dim + (size_t)kv_h * group * hd, hd, acc, hd, group);
		}
	}
	free(scores);
	free(acc);
	free(tmp);
	return 0;
}

/* ---- attention_forward after the projections: model.cpp:1616-1757 --------- */

int orc_attention_forward(const orc_attn_params* p, float* q, float* k, float* v, void* Kc, void* Vc, int kv_type,
                          int rows, float* out)
{
	const int hd = p->head_dim;
	const size_t q_dim = (size_t)p->n_head * hd;
	const size_t kv_dim = (size_t)p->n_kv * hd;
	/* per-head Q/K norms over every (token, head) group; Gemma 4's plain V norm */
	if (p->q_gamma) orc_rmsnorm_gamma_multi_f32(q, q, (size_t)p->n_tok * p->n_head, hd, p->q_gamma, p->eps);
	if (!p->reuse_kv)
	{
		if (p->k_gamma) orc_rmsnorm_gamma_multi_f32(k, k, (size_t)p->n_tok * p->n_kv, hd, p->k_gamma, p->eps);
		if (p->v_rmsnorm)
			for (int g = 0; g < p->n_tok * p->n_kv; ++g) orc_rmsnorm_f32(v + (size_t)g * hd, v + (size_t)g * hd, hd, p->eps);
	}
	/* RoPE on Q always, on K when it is fresh (cached K is already rotated) */
	for (int t = 0; t < p->n_tok; ++t)
	{
		const float rpos = (float)(p->pos0 + t) * p->rope_scale;
		orc_rope_f32(q + (size_t)t * q_dim, p->n_head, hd, p->n_rot, rpos, p->freq_base, p->rope_mode, p->freq_factors);
		if (!p->reuse_kv)
			orc_rope_f32(k + (size_t)t * kv_dim, p->n_kv, hd, p->n_rot, rpos, p->freq_base, p->rope_mode,
			             p->freq_factors);
	}
	/* append at row pos % rows, rounded to the cache's element type */
	if (!p->reuse_kv)
	{
		for (int t = 0; t < p->n_tok; ++t)
		{
			const size_t row = (size_t)((p->pos0 + t) % rows) * kv_dim;
			for (size_t i = 0; i < kv_dim; ++i)
			{
				const float kf = k[(size_t)t * kv_dim + i], vf = v[(size_t)t * kv_dim + i];
				if (kv_type == ORC_KV_F32)
				{
					((float*)Kc)[row + i] = kf;
					((float*)Vc)[row + i] = vf;
				}
				else
				{
					uint16_t (*narrow)(float) = kv_type == ORC_KV_BF16 ? orc_f32_to_bf16 : orc_f32_to_f16;
					((uint16_t*)Kc)[row + i] = narrow(kf);
					((uint16_t*)Vc)[row + i] = narrow(vf);
				}
			}
		}
	}
	const int rc = orc_attend(p, q, Kc, Vc, kv_type, rows, out);
	/* Qwen3.5 scales each head's output by its gate (model.cpp:1759-1760):
	 * y /= 1 + exp(-g), the scalar form of nnc_mul_sigmoid_f32 (nn_ops.cpp:1731-1742) */
	if (rc == 0 && p->gate)
		for (size_t i = 0; i < (size_t)p->n_tok * q_dim; ++i) out[i] /= 1.0f + expf(-p->gate[i]);
	return rc;
}

/* ---- the projections' gemvs (src/libnnc/nn_ops.h:89-170) ---- */

void orc_gemv_bf16w(const uint16_t* W, const float* X, size_t x_stride, float* Y, size_t y_stride, uint32_t rows,
                    uint32_t cols, uint32_t n_batch)
{
	for (uint32_t v = 0; v < n_batch; ++v)
		for (uint32_t r = 0; r < rows; ++r)
		{
			const uint16_t* row = W + (size_t)r * cols;
			const float* x = X + (size_t)v * x_stride;
			double s = 0.0;
			for (uint32_t k = 0; k < cols; ++k) s += (double)orc_bf16_to_f32(row[k]) * x[k];
			Y[(size_t)v * y_stride + r] = (float)s;
		}
}

void orc_gemv_q8_0(const int8_t* qs, const uint16_t* scales, const float* X, size_t x_stride, float* Y,
                   size_t y_stride, uint32_t rows, uint32_t cols, uint32_t n_batch)
{
	const uint32_t nb = cols / 32;
	for (uint32_t v = 0; v < n_batch; ++v)
		for (uint32_t r = 0; r < rows; ++r)
		{
			const float* x = X + (size_t)v * x_stride;
			double s = 0.0;
			for (uint32_t b = 0; b < nb; ++b)
			{
				double d = 0.0;
				for (uint32_t k = 0; k < 32; ++k) d += (double)qs[(size_t)r * cols + b * 32 + k] * x[b * 32 + k];
				s += (double)orc_bf16_to_f32(scales[(size_t)r * nb + b]) * d;
			}
			Y[(size_t)v * y_stride + r] = (float)s;
		}
}

void orc_gemv_q4_s(const uint8_t* qs, const uint16_t* scales, const uint16_t* biases, const float* X, size_t x_stride,
                   const float* XSUM, size_t xsum_stride, float* Y, size_t y_stride, uint32_t rows, uint32_t cols,
                   uint32_t n_batch)
{
	const uint32_t nb = cols / 32;
	for (uint32_t v = 0; v < n_batch; ++v)
		for (uint32_t r = 0; r < rows; ++r)
		{
			const float* x = X + (size_t)v * x_stride;
			const float* xs = XSUM + (size_t)v * xsum_stride;
			double s = 0.0;
			for (uint32_t b = 0; b < nb; ++b)
			{
				const uint8_t* blk = qs + (size_t)r * (cols / 2) + b * 16;
				double d = 0.0;
				for (uint32_t k = 0; k < 16; ++k)
				{
					d += (double)(blk[k] & 0x0F) * x[b * 32 + k];
					d += (double)(blk[k] >> 4) * x[b * 32 + k + 16];
				}
				s += (double)orc_bf16_to_f32(scales[(size_t)r * nb + b]) * d +
				     (double)orc_bf16_to_f32(biases[(size_t)r * nb + b]) * xs[b];
			}
			Y[(size_t)v * y_stride + r] = (float)s;
		}
}

void orc_block_sums(const float* x, float* out, size_t n)
{
	for (size_t b = 0; b < n / 32; ++b)
	{
		double s = 0.0;
		for (size_t k = 0; k < 32; ++k) s += x[b * 32 + k];
		out[b] = (float)s;
	}
}

/* Greedy verify's argmax of a logits row (session.cpp:128-134): the best
 * index moves only to a value comparing greater, so the first maximum wins,
 * -0 and +0 tie, a NaN never replaces the best and a NaN in the first place
 * stays the answer. */
void orc_argmax_rows(const float* x, size_t x_stride, int n_rows, uint32_t n, int32_t* out)
{
	for (int r = 0; r < n_rows; ++r)
	{
		const float* v = x + (size_t)r * x_stride;
		int32_t best = 0;
		for (uint32_t i = 1; i < n; ++i)
			if (v[i] > v[best]) best = (int32_t)i;
		out[r] = best;
	}
}

int orc_gemv_bf16w_argmax(const uint16_t* W, const float* x, uint32_t rows, uint32_t cols)
{
	int best = -1;
	float bv = 0.0f;
	for (uint32_t r = 0; r < rows; ++r)
	{
		float y;
		orc_gemv_bf16w(W + (size_t)r * cols, x, cols, &y, 1, 1, cols, 1);
		if (best < 0 || y > bv)
		{
			bv = y;
			best = (int)r;
		}
	}
	return best;
}
