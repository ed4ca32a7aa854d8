// noalloc.cu -- one layer's decode / verify attention without any allocation.
//
// Who needs this. The allocating entry points (nncu_kv_create and the
// attention calls on its cache) grow their scratch with cudaMalloc on first
// use. Some callers cannot have that: a host whose device memory is all
// handed out by its own arena or by a framework's caching allocator (an
// allocation behind its back breaks its accounting and can fail when the
// arena owns the whole device), and a latency-critical decode loop that must
// not stall on cudaMalloc / cudaFree, which may synchronise the whole device.
// nncu_attention_noalloc serves them: the caller passes every input, the
// output and its own K/V cache (allocated up front, by whatever means it
// uses), and the kernels' scratch -- the job descriptor and per-CTA starts,
// the RoPE table, the per-piece partials and their counters -- lives in one
// file-scope device array of fixed size.
//
// What sharing one array means:
//  * every GPU that loads the library holds the array (NOALLOC_SCRATCH_BYTES)
//    until the process exits;
//  * all calls use the same array: two calls whose kernels overlap on the GPU
//    (different streams, or different host threads, without ordering between
//    them) race on it and give wrong results; order them on one stream;
//  * a call leaves its scratch behind for the next one, which clears the
//    parts that must start at zero (the piece counters);
//  * the device error word (a kernel's bounded wait that ran out) stays set
//    across calls until nncu_noalloc_check reads and clears it, so a timeout
//    is never erased by the next call;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any use where even such a lookup is unwelcome.
//
// The kernels are the allocating path's own K1 (k_prep.cu) and K2 (the
// decode kernel, k_decode.cu), planned by the same planner (plan.cpp) for a
// single job.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "nncu.h"

namespace nncu
{
namespace
{

// The scratch of every no-allocation call on a device: 4 MiB, enough for one
// layer's decode or verify at the shapes of the benchmark configurations
// (e.g. 32 query heads of 64 or 8 of 256, a few tokens, 148 CTAs of partials).
constexpr size_t NOALLOC_SCRATCH_BYTES = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[MAX_DEVICES];

// Once per device, with that device current: the array's device address
// (host code cannot use the symbol itself as a device pointer).
int scratch_on_device(int dev, unsigned char** out)
{
	if (dev < 0 || dev >= MAX_DEVICES) return set_error(NNCU_ERR_INVALID_ARGUMENT, "device ordinal out of range");
	std::lock_guard<std::mutex> lk(g_setup_mu);
	if (!g_scratch_addr[dev])
	{
		void* p = nullptr;
		const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
		if (e != cudaSuccess) return set_cuda_error((int)e, "no-allocation scratch: cudaGetSymbolAddress");
		g_scratch_addr[dev] = p;
	}
	*out = static_cast<unsigned char*>(g_scratch_addr[dev]);
	return NNCU_OK;
}

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// Where the scratch keeps the device error word (first) and the rest.
constexpr size_t OFF_ERR = 0;
constexpr size_t OFF_ROPE = 256;

// Host staging for the job descriptor, the CTA starts and the RoPE table:
// static storage, so building them allocates nothing either.
constexpr int MAX_CTAS = 256;
struct alignas(16) HostHead
{
	DevJob job;
	CtaStart starts[MAX_CTAS];
	float rope[256];
};
thread_local HostHead t_head;

} // namespace
} // namespace nncu

using namespace nncu;

extern "C" int nncu_attention_noalloc(const nncu_attn_params* p, const float* q, const float* k, const float* v,
                                      float* out, void* k_cache, void* v_cache, int32_t kv_type, int32_t rows,
                                      void* stream)
{
	// ---- arguments (the allocating path's rules, for a caller-owned cache) ----
	if (!p || !q || !out || !k_cache || !v_cache) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL argument");
	if (!p->reuse_kv && (!k || !v)) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL k or v projections");
	if (kv_type != KV_F32 && kv_type != KV_BF16 && kv_type != KV_F16)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "unknown K/V type");
	const int D = p->head_dim;
	if (!decode_supported(D, kv_type))
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "head_dim must be 64, 128, 256 or 512");
	if (p->n_kv <= 0 || p->n_head <= 0 || p->n_head % p->n_kv)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "n_head must be a positive multiple of n_kv");
	if (p->n_tok <= 0 || p->pos0 < 0 || p->n_seq <= 0)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "n_tok, pos0 and n_seq must be positive");
	if (p->n_tok > NNCU_NOALLOC_MAX_TOKENS)
		return set_error(NNCU_ERR_INVALID_ARGUMENT,
		                 "the no-allocation entry point takes at most NNCU_NOALLOC_MAX_TOKENS tokens (decode and "
		                 "verify); use nncu_attention for more");
	if (rows <= 0 || rows % ATTN_BLOCK)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "the cache's rows must be a positive multiple of 256");
	if (p->n_rot < 0 || p->n_rot > D || (p->n_rot & 1) || p->n_rot > 512)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "n_rot must be even and at most head_dim");
	if (p->rope_mode != NNCU_ROPE_NEOX && p->rope_mode != NNCU_ROPE_NORM)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "unknown rope mode");
	if (p->window < 0 || p->softcap < 0.0f) return set_error(NNCU_ERR_INVALID_ARGUMENT, "negative window or softcap");
	if (p->freq_factors && p->n_rot % 8)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "freq_factors need n_rot to be a multiple of 8");
	JobPointers jp{};
	jp.q = q;
	jp.k = p->reuse_kv ? nullptr : k;
	jp.v = p->reuse_kv ? nullptr : v;
	jp.out = out;
	jp.q_gamma = p->q_gamma;
	jp.k_gamma = p->k_gamma;
	jp.freq_factors = p->freq_factors;
	jp.k_cache = k_cache;
	jp.v_cache = v_cache;
	int rc = check_alignment(jp, 0, "nncu_attention_noalloc");
	if (rc != NNCU_OK) return rc;
	// every key a query sees must still be in the caller's `rows` rows
	const bool windowed = p->causal && p->window > 0;
	if (windowed ? p->window + p->n_tok > rows : (p->pos0 + p->n_tok > rows || p->n_seq > rows))
		return set_error(NNCU_ERR_CONTEXT_FULL, "the cache's rows cannot hold every key these queries see");

	int dev = 0;
	cudaError_t ce = cudaGetDevice(&dev);
	if (ce != cudaSuccess) return set_cuda_error((int)ce, "cudaGetDevice");
	unsigned char* scratch = nullptr;
	rc = scratch_on_device(dev, &scratch);
	if (rc != NNCU_OK) return rc;
	int n_sms = 148;
	cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, dev);

	// ---- the job, then the plan (the allocating path's planner, for one job) ----
	const size_t es = kv_esize(kv_type);
	HostHead& hh = t_head;
	std::memset(&hh.job, 0, sizeof hh.job);
	DevJob& j = hh.job;
	const size_t off_rope = OFF_ROPE; // scratch: [error | rope | job | starts | partials | counters]
	j.q = q;
	j.k = k;
	j.v = v;
	j.out = out;
	j.q_gamma = p->q_gamma;
	j.k_gamma = p->k_gamma;
	j.freq_factors = p->freq_factors;
	j.gate = p->gate;
	j.rope_inv = reinterpret_cast<const float*>(scratch + off_rope);
	j.K = static_cast<char*>(k_cache);
	j.V = static_cast<char*>(v_cache);
	j.head_bytes = (long long)rows * D * (long long)es;
	j.rows = rows;
	j.n_tok = p->n_tok;
	j.pos0 = p->pos0;
	j.n_seq = p->n_seq;
	j.n_head = p->n_head;
	j.n_kv = p->n_kv;
	j.D = D;
	j.n_rot = p->n_rot;
	j.rope_mode = p->rope_mode;
	j.causal = p->causal != 0;
	j.window = p->window;
	j.reuse_kv = p->reuse_kv != 0;
	j.v_rmsnorm = p->v_rmsnorm != 0;
	j.rope_scale = p->rope_scale;
	j.eps = p->eps;
	j.scale = p->scale;
	j.softcap = p->softcap;
	j.key_lo = 0;
	j.key_hi = INT_MAX;
	DecodePlan P{};
	// whole chunks: the partial slots stay within the fixed scratch
	rc = plan_launch(&j, 1, kv_type, std::min(n_sms, MAX_CTAS), P, hh.starts, MAX_CTAS, false);
	if (rc != NNCU_OK) return rc;

	const size_t off_job = OFF_ROPE + up256(256 * sizeof(float));
	const size_t off_starts = off_job + up256(sizeof(DevJob));
	const size_t off_parts = off_starts + up256((size_t)MAX_CTAS * sizeof(CtaStart));
	const size_t off_count =
		off_parts + up256((size_t)std::max<long long>(P.n_parts, 1) * P.RM * (D + 4) * sizeof(float));
	const size_t need = off_count + up256((size_t)P.n_segments * sizeof(int));
	if (need > NOALLOC_SCRATCH_BYTES)
	{
		char msg[200];
		std::snprintf(msg, sizeof msg,
		              "this call needs %zu bytes of scratch; the no-allocation entry point has %zu (fewer tokens or "
		              "heads per call, or use nncu_attention)",
		              need, NOALLOC_SCRATCH_BYTES);
		return set_error(NNCU_ERR_INVALID_ARGUMENT, msg);
	}
	// nnc_rope_f32's inverse frequencies (nn_ops.cpp:1844-1856), the fp32 recurrence
	const int half = p->n_rot / 2;
	if (half > 0)
	{
		const float ratio = std::pow(p->freq_base, -2.0f / static_cast<float>(p->n_rot));
		float inv = 1.0f;
		for (int i = 0; i < half; ++i)
		{
			hh.rope[i] = inv;
			inv *= ratio;
		}
	}

	// ---- upload the job, the starts and the RoPE table, clear what must start at zero, run K1 and K2 ----
	auto st = static_cast<cudaStream_t>(stream);
	// copies from pageable host memory: each returns once its source is consumed
	ce = cudaMemcpyAsync(scratch + off_job, &hh.job, sizeof(DevJob), cudaMemcpyHostToDevice, st);
	if (ce == cudaSuccess && P.n_ctas > 0)
		ce = cudaMemcpyAsync(scratch + off_starts, hh.starts, (size_t)P.n_ctas * sizeof(CtaStart),
		                     cudaMemcpyHostToDevice, st);
	if (ce == cudaSuccess && half > 0)
	{
		for (int i = half; i < ((half + 3) & ~3); ++i) hh.rope[i] = 0.0f; // whole 16-byte pieces
		ce = cudaMemcpyAsync(scratch + off_rope, hh.rope, (size_t)((half + 3) & ~3) * sizeof(float),
		                     cudaMemcpyHostToDevice, st);
	}
	// the piece counters start at zero; the error word is cleared by nncu_noalloc_check
	if (ce == cudaSuccess) ce = cudaMemsetAsync(scratch + off_count, 0, need - off_count, st);
	if (ce == cudaSuccess && j.n_tiles == 0)
		ce = cudaMemsetAsync(out, 0, (size_t)p->n_tok * p->n_head * D * sizeof(float), st);
	if (ce != cudaSuccess) return set_cuda_error((int)ce, "no-allocation call: staging");

	P.jobs = reinterpret_cast<const DevJob*>(scratch + off_job);
	P.cta_start = reinterpret_cast<const CtaStart*>(scratch + off_starts);
	P.parts = reinterpret_cast<float*>(scratch + off_parts);
	P.counters = reinterpret_cast<int*>(scratch + off_count);
	P.err = reinterpret_cast<int*>(scratch + OFF_ERR);
	int e = P.fused ? 0 : launch_prep(P, st); // K2 appends itself when it can
	if (e) return set_cuda_error(e, "K1 (norm, RoPE, append) launch");
	if (!P.fused) note_launches(1);
	if (P.n_ctas > 0)
	{
		e = launch_decode(P, st);
		if (e) return set_cuda_error(e, "K2 (attention) launch");
		note_launches(1);
	}
	return NNCU_OK;
}

extern "C" int nncu_noalloc_check(void* stream)
{
	int dev = 0;
	cudaError_t ce = cudaGetDevice(&dev);
	if (ce != cudaSuccess) return set_cuda_error((int)ce, "cudaGetDevice");
	unsigned char* scratch = nullptr;
	int rc = scratch_on_device(dev, &scratch);
	if (rc != NNCU_OK) return rc;
	ce = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
	if (ce != cudaSuccess) return set_cuda_error((int)ce, "no-allocation check: stream");
	int word = 0;
	// into this stack variable: a plain copy, nothing allocated
	ce = cudaMemcpy(&word, scratch + OFF_ERR, sizeof word, cudaMemcpyDeviceToHost);
	if (ce == cudaSuccess && word != 0) ce = cudaMemset(scratch + OFF_ERR, 0, sizeof word);
	if (ce != cudaSuccess) return set_cuda_error((int)ce, "no-allocation check: error word");
	if (word != 0)
	{
		char msg[160];
		std::snprintf(msg, sizeof msg,
		              "a no-allocation call's bounded wait timed out (code %d); the outputs since the last check are void",
		              word);
		return set_error(NNCU_ERR_TIMEOUT, msg);
	}
	return NNCU_OK;
}
