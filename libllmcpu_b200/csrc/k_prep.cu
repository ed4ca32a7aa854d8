// k_prep.cu -- K1: the K/V half of the per-head work attention_forward does
// between the projections and the attention proper (src/libnnc/model.cpp:
// 1616-1694): K RMSNorm with gamma (nnc_rmsnorm_gamma_multi_f32, nn_ops.cpp:
// 590-632), Gemma 4's plain V RMSNorm (nn_ops.cpp:558-588), RoPE on the fresh
// k (nnc_rope_f32, nn_ops.cpp:1830-1873), and the append of k, v at row
// pos % rows in the cache's element type. The q half runs inside the decode
// kernel. One launch covers every token of every job; a warp takes one
// (token, head) vector at a time.
//
// Also the unit-seam kernels for nnc_rmsnorm*, nnc_rope_f32 and
// nnc_softcap_f32 on device pointers.
#include <cuda_runtime.h>

#include "common.cuh"

namespace nncu
{
namespace
{

constexpr int PREP_WARPS = 8;
constexpr int PREP_MAX_D = 512;

// Token t of job j (one CTA).
template <typename KV>
__device__ __forceinline__ void prep_token(const DevJob& j, int t)
{
	using T = typename KV::T;
	// The attention kernel that follows may start now: it streams the K/V
	// tiles that do not hold this kernel's rows and waits for it only before
	// the ones that do.
	griddep_launch_dependents();
	__shared__ float bufs[PREP_WARPS][PREP_MAX_D];
	__shared__ float s_kg[PREP_MAX_D], s_inv[PREP_MAX_D / 2], s_ff[PREP_MAX_D / 2];
	// block (t, job): token t of job blockIdx.y
	if (t >= j.n_tok || j.pos0 + t < j.key_lo || j.pos0 + t >= j.key_hi) return; // not this launch's row
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int D = j.D, half = j.n_rot / 2;
	float* buf = bufs[warp];
	const int n_kv = j.reuse_kv ? 0 : j.n_kv; // tasks: k heads, then v heads
	const int n_tasks = 2 * n_kv;
	if (n_tasks == 0) return;
	const float rpos = (float)(j.pos0 + t) * j.rope_scale;
	const int row = (j.pos0 + t) % j.rows;
	auto task_src = [&](int task) {
		return (task < n_kv ? j.k : j.v) + ((size_t)t * j.n_kv + task % n_kv) * D;
	};
	// one round of loads: this warp's first head vector, and the gains and
	// RoPE tables staged once for every head of the token
	HeadRegs x;
	if (warp < n_tasks) load_head(x, task_src(warp), D);
	const float* kg = j.k_gamma;
	const float* ff = j.freq_factors;
	for (int i = threadIdx.x; i < D; i += blockDim.x)
	{
		const float b = kg ? kg[i] : 0.0f;
		const float c = i < half ? j.rope_inv[i] : 0.0f, d = (ff && i < half) ? ff[i] : 0.0f;
		s_kg[i] = b;
		if (i < half)
		{
			s_inv[i] = c;
			s_ff[i] = d;
		}
	}
	__syncthreads();
	for (int task = warp; task < n_tasks; task += PREP_WARPS)
	{
		if (task != warp) load_head(x, task_src(task), D);
		const bool is_k = task < n_kv;
		const int h = task % n_kv;
		const float* gamma = is_k && kg ? s_kg : nullptr;
		prep_head(buf, x, D, gamma, !is_k && j.v_rmsnorm, j.eps, is_k, j.n_rot, j.rope_mode, rpos, s_inv,
		          ff ? s_ff : nullptr);
		char* base = (is_k ? j.K : j.V) + (size_t)h * j.head_bytes;
		T* dst = reinterpret_cast<T*>(base) + (size_t)row * D;
		for (int i = lane; i < D; i += 32) store_elem(dst + i, buf[i]);
		__syncwarp();
	}
}

template <typename KV>
__global__ void __launch_bounds__(PREP_WARPS * 32) prep_kernel(const DevJob* __restrict__ jobs)
{
	prep_token<KV>(jobs[blockIdx.y], blockIdx.x); // block (t, job)
}

// ---- unit seam ---------------------------------------------------------------

__global__ void rmsnorm_kernel(float* y, const float* x, size_t n_groups, size_t dim, const float* gamma, float eps)
{
	const size_t g = (size_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
	if (g >= n_groups) return;
	const int lane = threadIdx.x & 31;
	const float* xg = x + g * dim;
	float ss = 0.0f;
	for (size_t i = lane; i < dim; i += 32) ss = fmaf(xg[i], xg[i], ss);
	ss = warp_sum(ss);
	const double mean = gamma ? (double)ss * (double)(1.0f / (float)dim) : (double)ss / (double)dim;
	const float sc = (float)(1.0 / sqrt(mean + (double)eps));
	float* yg = y + g * dim;
	for (size_t i = lane; i < dim; i += 32) yg[i] = gamma ? xg[i] * sc * gamma[i] : xg[i] * sc;
}

__global__ void rope_kernel(float* x, uint32_t n_tok, uint32_t n_heads, uint32_t head_dim, uint32_t n_rot,
                            int32_t pos0, float pos_scale, const float* inv, int mode, const float* ff)
{
	extern __shared__ float sbuf[];
	const uint32_t w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
	if (w >= n_tok * n_heads) return;
	const uint32_t t = w / n_heads;
	float* xh = x + (size_t)w * head_dim;
	float* buf = sbuf + (threadIdx.x >> 5) * head_dim;
	for (uint32_t i = threadIdx.x & 31; i < head_dim; i += 32) buf[i] = xh[i];
	__syncwarp();
	rope_vec(buf, (int)n_rot, mode, (float)(pos0 + (int32_t)t) * pos_scale, inv, ff);
	__syncwarp();
	for (uint32_t i = threadIdx.x & 31; i < head_dim; i += 32) xh[i] = buf[i];
}

__global__ void softcap_kernel(float* y, const float* x, size_t n, float cap)
{
	const float inv = 1.0f / cap;
	for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
		y[i] = tanhf(x[i] * inv) * cap;
}

} // namespace

int launch_prep(const DecodePlan& P, void* stream)
{
	if (P.D > PREP_MAX_D || P.n_jobs > 65535) return (int)cudaErrorInvalidValue;
	if (P.max_tok == 0 || P.n_jobs == 0) return 0;
	auto st = static_cast<cudaStream_t>(stream);
	const dim3 grid((unsigned)P.max_tok, (unsigned)P.n_jobs);
	switch (P.kv_type)
	{
	case KV_F32: prep_kernel<kv_f32><<<grid, PREP_WARPS * 32, 0, st>>>(P.jobs); break;
	case KV_BF16: prep_kernel<kv_bf16><<<grid, PREP_WARPS * 32, 0, st>>>(P.jobs); break;
	default: prep_kernel<kv_f16><<<grid, PREP_WARPS * 32, 0, st>>>(P.jobs); break;
	}
	return (int)cudaGetLastError();
}

int launch_rmsnorm(float* y, const float* x, size_t n_groups, size_t dim, const float* gamma, float eps,
                   void* stream)
{
	if (n_groups == 0 || dim == 0) return 0;
	const unsigned blocks = (unsigned)((n_groups + 7) / 8);
	rmsnorm_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, x, n_groups, dim, gamma, eps);
	return (int)cudaGetLastError();
}

int launch_rope(float* x, uint32_t n_tok, uint32_t n_heads, uint32_t head_dim, uint32_t n_rot, int32_t pos0,
                float pos_scale, const float* rope_inv, int mode, const float* freq_factors, void* stream)
{
	if (n_rot == 0 || n_tok == 0 || n_heads == 0) return 0;
	const uint32_t warps = n_tok * n_heads;
	const unsigned blocks = (warps + 7) / 8;
	const size_t smem = (size_t)8 * head_dim * sizeof(float);
	rope_kernel<<<blocks, 256, smem, static_cast<cudaStream_t>(stream)>>>(x, n_tok, n_heads, head_dim, n_rot, pos0,
	                                                                      pos_scale, rope_inv, mode, freq_factors);
	return (int)cudaGetLastError();
}

int launch_softcap(float* y, const float* x, size_t n, float cap, void* stream)
{
	if (n == 0) return 0;
	const unsigned blocks = (unsigned)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096);
	softcap_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, x, n, cap);
	return (int)cudaGetLastError();
}

// One CTA per COPY_CHUNK piece of a copy list's entries: 16-byte loads and
// stores where both addresses are 16-byte aligned, 4-byte ones otherwise
// (every buffer here holds floats). Reads or writes through the mapping of
// registered host memory cross PCIe; each thread keeps four loads in flight.
__global__ void __launch_bounds__(256) copy_list_kernel(const __grid_constant__ CopyList L)
{
	int k = 0; // the entry whose pieces hold this CTA (entries in order of cta0)
	while (k + 1 < L.n && L.e[k + 1].cta0 <= blockIdx.x) ++k;
	CopyEntry e = L.e[k];
	const uint64_t off = (uint64_t)(blockIdx.x - e.cta0) * COPY_CHUNK;
	e.src = static_cast<const char*>(e.src) + off;
	e.dst = static_cast<char*>(e.dst) + off;
	e.bytes = e.bytes - off < COPY_CHUNK ? e.bytes - off : COPY_CHUNK;
	const bool wide = ((reinterpret_cast<uintptr_t>(e.src) | reinterpret_cast<uintptr_t>(e.dst)) & 15u) == 0;
	size_t done = 0;
	if (wide)
	{
		const uint4* s = static_cast<const uint4*>(e.src);
		uint4* d = static_cast<uint4*>(e.dst);
		const size_t n = e.bytes / 16;
		size_t i = threadIdx.x;
		for (; i + 3 * 256 < n; i += 4 * 256)
		{
			const uint4 a = s[i], b = s[i + 256], c = s[i + 512], f = s[i + 768];
			d[i] = a;
			d[i + 256] = b;
			d[i + 512] = c;
			d[i + 768] = f;
		}
		for (; i < n; i += 256) d[i] = s[i];
		done = n * 16;
	}
	const uint32_t* s4 = static_cast<const uint32_t*>(e.src);
	uint32_t* d4 = static_cast<uint32_t*>(e.dst);
	for (size_t i = done / 4 + threadIdx.x; i < e.bytes / 4; i += 256) d4[i] = s4[i];
}

int launch_copy_list(CopyList& l, void* stream)
{
	if (l.n <= 0) return 0;
	if (l.n > COPY_LIST_MAX) return (int)cudaErrorInvalidValue;
	uint64_t ctas = 0;
	for (int i = 0; i < l.n; ++i)
	{
		l.e[i].cta0 = (uint32_t)ctas;
		ctas += (l.e[i].bytes + COPY_CHUNK - 1) / COPY_CHUNK;
	}
	if (ctas == 0) return 0;
	if (ctas > 0x7fffffffu) return (int)cudaErrorInvalidValue;
	copy_list_kernel<<<(unsigned)ctas, 256, 0, static_cast<cudaStream_t>(stream)>>>(l);
	note_launches(1);
	return (int)cudaGetLastError();
}

} // namespace nncu
