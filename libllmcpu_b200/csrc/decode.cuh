// decode.cuh -- device code shared by the two decode kernels (k_decode.cu on
// the CUDA cores, k_decode_tc.cu on the tensor cores): the arrival counters
// and the in-order merge of a segment's pieces (nnc_attn_merge, nn_ops.cpp:
// 461-482, over the pieces of a split segment).
#pragma once

#include <math_constants.h>

#include "common.cuh"

namespace nncu
{

// The CTA's walk over its run of the launch's tiles: (job, segment within
// the job, tile within the segment), advanced one tile at a time.
struct Cursor
{
	int job = 0, seg = 0, tis = 0;
	int n_tiles = 1, n_segs = 1;
};

// `jobs`: the job table in global memory, or (INL) in the kernel's
// parameters.
template <bool INL>
__device__ __forceinline__ void cursor_load(const DevJob* jobs, int n_jobs, Cursor& c)
{
	const DevJob& J = jobs[c.job];
	c.n_tiles = J.n_tiles;
	c.n_segs = J.n_kv * J.n_rowgroups;
	if (!INL && c.job + 1 < n_jobs)
	{
		// the next job's descriptor into L1 ahead of the job change
		const char* nx = reinterpret_cast<const char*>(jobs + c.job + 1);
		for (int b = 0; b < (int)sizeof(DevJob); b += 128) asm volatile("prefetch.global.L1 [%0];" ::"l"(nx + b));
	}
}

// On to the first tile of the next segment.
template <bool INL>
__device__ __forceinline__ void cursor_next_segment(const DevJob* jobs, int n_jobs, Cursor& c)
{
	c.tis = 0;
	if (++c.seg < c.n_segs) return;
	c.seg = 0;
	do
		++c.job;
	while (c.job < n_jobs && jobs[c.job].n_tiles == 0);
	if (c.job < n_jobs) cursor_load<INL>(jobs, n_jobs, c);
}

// Whether tiles [tis, tis + n) of a job's segment hold keys appended in this
// launch: its new tokens within its key range (while K1 appends, they must
// wait for K1; earlier keys need not).
__device__ __forceinline__ bool holds_new_rows(const DevJob& J, int tis, int n, int T)
{
	const int lo = max(J.pos0, J.key_lo), hi = min(J.pos0 + J.n_tok, J.key_hi);
	return !J.reuse_kv && lo < hi && (J.tile_lo + tis) * T <= hi - 1 && (J.tile_lo + tis + n) * T - 1 >= lo;
}

// atom.add with acquire-release semantics at GPU scope: the arriving CTA's
// partial (written before it, ordered by the CTA barrier) is visible to the
// CTA that sees the final count.
__device__ __forceinline__ int atomic_add_acq_rel(int* p, int v)
{
	int old;
	asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
	return old;
}

__device__ __forceinline__ int atomic_add_relaxed_sys(int* p, int v)
{
	int old;
	asm volatile("atom.relaxed.sys.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
	return old;
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ int ld_acquire_sys(const int* p)
{
	int v;
	asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
	return v;
}

// Merge np partials of a segment's rows in order (nnc_attn_merge, piece 0
// first): piece c of row R is o[D], m, l at base + c * stride + R * PW, m in
// log2 units. A thread owns 4 columns of a row and merges online, FB pieces'
// worth of independent 16-byte loads at a time; `emit(R, d, acc, M, L)` gets
// the merged (o, m, l) of columns d .. d+3 (o relative to 2^M). Rows R >=
// rows_valid are padding and skipped.
template <int D, int RM, typename Emit>
__device__ __forceinline__ void merge_pieces(const float* base, size_t stride, int np, int rows_valid, int tid,
                                             int nthreads, Emit emit)
{
	constexpr int PW = D + 4;
	constexpr int FB = RM <= 4 && D == 256 ? 20 : 16; // as many as the registers allow without spills
	for (int idx = tid; idx < RM * (D / 4); idx += nthreads)
	{
		const int R = idx / (D / 4), d = 4 * (idx % (D / 4));
		if (R >= rows_valid) continue;
		const float* col = base + R * PW + d;
		const float* mlp = base + R * PW + D;
		float M = -CUDART_INF_F, L = 0.0f;
		float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
		for (int c0 = 0; c0 < np; c0 += FB)
		{
			float4 v[FB];
			float2 ml[FB];
#pragma unroll
			for (int u = 0; u < FB; ++u)
			{
				const bool ok = c0 + u < np;
				v[u] = ok ? __ldcg(reinterpret_cast<const float4*>(col + (size_t)(c0 + u) * stride))
				          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
				ml[u] = ok ? __ldcg(reinterpret_cast<const float2*>(mlp + (size_t)(c0 + u) * stride))
				           : make_float2(-CUDART_INF_F, 0.0f);
			}
			float mx = M;
#pragma unroll
			for (int u = 0; u < FB; ++u) mx = fmaxf(mx, ml[u].x);
			if (mx == -CUDART_INF_F) continue; // nothing seen yet
			const float sc = M == -CUDART_INF_F ? 0.0f : ex2(M - mx);
			acc.x *= sc;
			acc.y *= sc;
			acc.z *= sc;
			acc.w *= sc;
			L *= sc;
#pragma unroll
			for (int u = 0; u < FB; ++u)
			{
				const float w = ml[u].x == -CUDART_INF_F ? 0.0f : ex2(ml[u].x - mx);
				acc.x = fmaf(v[u].x, w, acc.x);
				acc.y = fmaf(v[u].y, w, acc.y);
				acc.z = fmaf(v[u].z, w, acc.z);
				acc.w = fmaf(v[u].w, w, acc.w);
				L = fmaf(ml[u].y, w, L);
			}
			M = mx;
		}
		emit(R, d, acc, M, L);
	}
}

// The rows of a segment that exist (the last row group may be short).
__device__ __forceinline__ int seg_rows(const DevJob& J, int rg, int RM)
{
	return min(RM, (J.n_head / J.n_kv) * J.n_tok - rg * RM);
}


} // namespace nncu
