// common.cuh -- device helpers shared by the kernels: element types, warp
// reductions, and the sm_90+/sm_100 asynchronous-copy primitives (mbarrier,
// cp.async.bulk) written as inline PTX.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "internal.h"

namespace nncu
{

// ---- element types --------------------------------------------------------

struct kv_f32
{
	using T = float;
	static constexpr int esize = 4;
	static constexpr int id = KV_F32;
};
struct kv_bf16
{
	using T = __nv_bfloat16;
	static constexpr int esize = 2;
	static constexpr int id = KV_BF16;
};
struct kv_f16
{
	using T = __half;
	static constexpr int esize = 2;
	static constexpr int id = KV_F16;
};

// fp32 -> stored element, round to nearest even (libnnc's nnc_f32_to_bf16,
// runtime.h:106-113, is RNE on the upper 16 bits, as __float2bfloat16_rn is).
__device__ __forceinline__ void store_elem(float* p, float x) { *p = x; }
__device__ __forceinline__ void store_elem(__nv_bfloat16* p, float x) { *p = __float2bfloat16_rn(x); }
__device__ __forceinline__ void store_elem(__half* p, float x) { *p = __float2half_rn(x); }

__device__ __forceinline__ float load_elem(const float* p) { return *p; }
__device__ __forceinline__ float load_elem(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load_elem(const __half* p) { return __half2float(*p); }

// A lane's share of a D-element row spread over LK lanes (32: the whole
// warp; fewer: the warp holds 32/LK rows side by side): E = D/LK elements,
// taken as chunks of VEC consecutive elements (16 bytes, or all E if fewer)
// with the lanes' chunks side by side, so each load instruction of a warp
// reads contiguous runs of shared memory (no bank conflicts). Element e of
// lane j (0 <= j < LK) is row[lane_elem<E, VEC, LK>(j, e)].
template <int E, int ESIZE>
struct LaneVec
{
	static constexpr int VEC = (16 / ESIZE) < E ? (16 / ESIZE) : E;
	static_assert(E % VEC == 0, "chunking");
};

template <int E, int VEC, int LK = 32>
__device__ __forceinline__ int lane_elem(int lane, int e)
{
	return (e / VEC) * LK * VEC + lane * VEC + (e % VEC);
}

__device__ __forceinline__ float2 widen2(uint32_t w, const __half*)
{
	return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
__device__ __forceinline__ float2 widen2(uint32_t w, const __nv_bfloat16*)
{
	return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}

// Load lane `lane`'s E elements of `row` (shared or global) as floats.
template <int E, int LK = 32>
__device__ __forceinline__ void load_lane(const float* row, int lane, float (&v)[E])
{
	constexpr int VEC = LaneVec<E, 4>::VEC;
#pragma unroll
	for (int c = 0; c < E / VEC; ++c)
	{
		const float* p = row + c * LK * VEC + lane * VEC;
		if constexpr (VEC == 4)
		{
			const float4 x = *reinterpret_cast<const float4*>(p);
			v[c * 4] = x.x, v[c * 4 + 1] = x.y, v[c * 4 + 2] = x.z, v[c * 4 + 3] = x.w;
		}
		else if constexpr (VEC == 2)
		{
			const float2 x = *reinterpret_cast<const float2*>(p);
			v[c * 2] = x.x, v[c * 2 + 1] = x.y;
		}
		else
		{
#pragma unroll
			for (int j = 0; j < VEC; ++j) v[c * VEC + j] = p[j];
		}
	}
}

// fp32 rows read with another element type's lane mapping (VEC per chunk).
template <int E, int VEC, int LK = 32>
__device__ __forceinline__ void load_lane_f(const float* row, int lane, float (&v)[E])
{
#pragma unroll
	for (int c = 0; c < E / VEC; ++c)
	{
		const float* p = row + c * LK * VEC + lane * VEC;
		if constexpr (VEC % 4 == 0)
		{
#pragma unroll
			for (int j = 0; j < VEC; j += 4)
			{
				const float4 x = *reinterpret_cast<const float4*>(p + j);
				v[c * VEC + j] = x.x, v[c * VEC + j + 1] = x.y, v[c * VEC + j + 2] = x.z, v[c * VEC + j + 3] = x.w;
			}
		}
		else if constexpr (VEC % 2 == 0)
		{
#pragma unroll
			for (int j = 0; j < VEC; j += 2)
			{
				const float2 x = *reinterpret_cast<const float2*>(p + j);
				v[c * VEC + j] = x.x, v[c * VEC + j + 1] = x.y;
			}
		}
		else
		{
#pragma unroll
			for (int j = 0; j < VEC; ++j) v[c * VEC + j] = p[j];
		}
	}
}

template <int E, int LK, typename H>
__device__ __forceinline__ void load_lane_h(const H* row, int lane, float (&v)[E])
{
	constexpr int VEC = LaneVec<E, 2>::VEC;
#pragma unroll
	for (int c = 0; c < E / VEC; ++c)
	{
		const H* p = row + c * LK * VEC + lane * VEC;
		if constexpr (VEC == 8)
		{
			const uint4 x = *reinterpret_cast<const uint4*>(p);
			const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
			for (int j = 0; j < 4; ++j)
			{
				const float2 f = widen2(w[j], p);
				v[c * 8 + 2 * j] = f.x, v[c * 8 + 2 * j + 1] = f.y;
			}
		}
		else if constexpr (VEC == 4)
		{
			const uint2 x = *reinterpret_cast<const uint2*>(p);
			const float2 f0 = widen2(x.x, p), f1 = widen2(x.y, p);
			v[c * 4] = f0.x, v[c * 4 + 1] = f0.y, v[c * 4 + 2] = f1.x, v[c * 4 + 3] = f1.y;
		}
		else if constexpr (VEC == 2)
		{
			const float2 f = widen2(*reinterpret_cast<const uint32_t*>(p), p);
			v[c * 2] = f.x, v[c * 2 + 1] = f.y;
		}
		else
		{
#pragma unroll
			for (int j = 0; j < VEC; ++j) v[c * VEC + j] = load_elem(p + j);
		}
	}
}

template <int E, int LK = 32>
__device__ __forceinline__ void load_lane(const __half* row, int lane, float (&v)[E])
{
	load_lane_h<E, LK>(row, lane, v);
}
template <int E, int LK = 32>
__device__ __forceinline__ void load_lane(const __nv_bfloat16* row, int lane, float (&v)[E])
{
	load_lane_h<E, LK>(row, lane, v);
}

// ---- warp helpers ---------------------------------------------------------

__device__ __forceinline__ float warp_sum(float x)
{
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
	return x;
}

__device__ __forceinline__ float warp_max(float x)
{
#pragma unroll
	for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
	return x;
}

// One exchange round of transpose_reduce: lanes whose MASK bit is set keep
// the upper half of their values and send the lower half to the partner,
// the others the reverse; each kept value gains the partner's copy.
template <int N, int MASK>
__device__ __forceinline__ float transpose_reduce_step(const float (&v)[N], int lane)
{
	if constexpr (N == 1)
	{
		float x = v[0];
#pragma unroll
		for (int o = MASK; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
		return x;
	}
	else
	{
		constexpr int H = N / 2;
		const bool upper = (lane & MASK) != 0;
		float keep[H];
#pragma unroll
		for (int i = 0; i < H; ++i)
		{
			const float send = upper ? v[i] : v[i + H];
			const float mine = upper ? v[i + H] : v[i];
			keep[i] = mine + __shfl_xor_sync(0xffffffffu, send, MASK);
		}
		return transpose_reduce_step<H, MASK / 2>(keep, lane);
	}
}

// Sum N per-lane values over each aligned group of LK lanes (the whole warp
// for LK = 32), leaving each lane with ONE full sum: lane l holds the sum
// of value index ((l % LK) >> (log2 LK - log2 N)) of its group. Each
// exchange round hands half of the remaining values to the partner lane and
// keeps the other half, so N values cost about N shuffles instead of log2 LK
// per value.
template <int N, int LK = 32>
__device__ __forceinline__ float transpose_reduce(const float (&v)[N], int lane)
{
	static_assert(N >= 1 && N <= LK && (N & (N - 1)) == 0, "N: power of two up to LK");
	static_assert(LK >= 2 && LK <= 32 && (LK & (LK - 1)) == 0, "LK: power of two up to 32");
	return transpose_reduce_step<N, LK / 2>(v, lane);
}

// ---- asynchronous copies and barriers (PTX ISA 8.x, sm_90+) ----------------

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
	return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
	asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init()
{
	asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
	asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
	             : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
	asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity)
{
	uint32_t ok;
	asm volatile(
		"{\n\t.reg .pred p;\n\t"
		"mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
		"selp.u32 %0, 1, 0, p;\n\t}"
		: "=r"(ok)
		: "r"(smem_u32(bar)), "r"(parity)
		: "memory");
	return ok != 0;
}

// Whether phase `parity` of `bar` has completed, without waiting (test_wait
// never suspends the thread, unlike try_wait): for a loop that polls several
// barriers in turn.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity)
{
	uint32_t ok;
	asm volatile(
		"{\n\t.reg .pred p;\n\t"
		"mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
		"selp.u32 %0, 1, 0, p;\n\t}"
		: "=r"(ok)
		: "r"(smem_u32(bar)), "r"(parity)
		: "memory");
	return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
	uint64_t t;
	asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
	return t;
}

// Wait for phase `parity` of `bar`, giving up after WAIT_LIMIT_NS. Returns
// false on timeout, after recording `code` in the device error word.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err, int code)
{
	if (mbar_try_wait(bar, parity)) return true;
	const uint64_t t0 = globaltimer_ns();
	for (uint32_t it = 0;; ++it)
	{
		if (mbar_try_wait(bar, parity)) return true;
		if ((it & 255u) == 255u && globaltimer_ns() - t0 > WAIT_LIMIT_NS)
		{
			if (err) atomicCAS(err, 0, code);
			return false;
		}
	}
}

// One contiguous global -> shared copy, completing on `bar` (bytes counted
// against its expect_tx). Addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar)
{
	asm volatile(
		"cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
			smem_u32(smem_dst)),
		"l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
		: "memory");
}

// Programmatic dependent launch (sm_90+): a primary kernel lets its dependent
// grid start early; the dependent waits, where it needs the primary's
// results, for the primary grid to complete and its writes to be visible.
__device__ __forceinline__ void griddep_launch_dependents()
{
	asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier over `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int count)
{
	asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// The same barrier, returning whether `pred` held on any of the threads: the
// one answer every thread gets, so a decision to leave a loop of named
// barriers is taken by all of them together (a flag read after a plain
// barrier may change between two threads' reads).
__device__ __forceinline__ bool named_sync_or(int id, int count, bool pred)
{
	uint32_t r;
	asm volatile(
		"{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
		: "=r"(r)
		: "r"((uint32_t)pred), "r"(id), "r"(count)
		: "memory");
	return r != 0;
}

__device__ __forceinline__ float ex2(float x)
{
	float y;
	asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
	return y;
}

// Qwen3.5's output gate (model.cpp:1759-1760, nnc_mul_sigmoid_f32): an
// attention output element times sigmoid(g), as y / (1 + exp(-g)).
__device__ __forceinline__ float gated(float y, const float* gate, size_t i)
{
	return gate ? y / (1.0f + expf(-gate[i])) : y;
}
__device__ __forceinline__ float4 gated4(float4 y, const float* gate, size_t i)
{
	if (!gate) return y;
	return make_float4(y.x / (1.0f + expf(-gate[i])), y.y / (1.0f + expf(-gate[i + 1])),
	                   y.z / (1.0f + expf(-gate[i + 2])), y.w / (1.0f + expf(-gate[i + 3])));
}

// The keys [first, last] the query at `pos` sees (model.cpp:2300-2316).
__device__ __forceinline__ void span_of(int causal, int window, int pos, int n_seq, int& first, int& last)
{
	if (causal)
	{
		first = (window > 0 && pos + 1 > window) ? pos + 1 - window : 0;
		last = min(pos, n_seq - 1);
	}
	else
	{
		first = 0;
		last = n_seq - 1;
		if (window > 0)
		{
			const int half = window / 2;
			first = max(0, pos - half);
			last = min(n_seq - 1, pos + half);
		}
	}
}

// Two floats to bf16 with round-to-nearest-even, packed (lo in the low half),
// on the integer pipe: the conversion instruction runs on the transcendental
// unit, which the softmax's exponentials already saturate. Exact RNE for
// every finite value and for infinities (the values rounded here are finite).
__device__ __forceinline__ uint32_t bf16_rne_bits(float f)
{
	const uint32_t u = __float_as_uint(f);
	return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
	return bf16_rne_bits(lo) | (bf16_rne_bits(hi) << 16);
}

// ---- per-head preparation (norms and RoPE) on a warp ------------------------

// RMS scale of a D-vector held in shared `buf`, the reference's form:
// 1 / sqrt(sum(x^2) * (1/D) + eps) in double (nnc_rmsnorm_gamma_multi_f32,
// nn_ops.cpp:590-632), or sum / D for the plain nnc_rmsnorm_f32 (:558-588).
__device__ __forceinline__ float rms_scale(const float* buf, int D, float eps, bool gamma_form)
{
	float ss = 0.0f;
	for (int i = threadIdx.x & 31; i < D; i += 32) ss = fmaf(buf[i], buf[i], ss);
	ss = warp_sum(ss);
	const double mean = gamma_form ? (double)ss * (double)(1.0f / (float)D) : (double)ss / (double)D;
	return (float)(1.0 / sqrt(mean + (double)eps));
}

// Rotate the first n_rot lanes of the vector in shared `buf` for position
// rpos (nnc_rope_f32, nn_ops.cpp:1830-1873): theta_i = rpos * inv[i]
// (/ freq_factors[i]); NEOX pairs i and i + n_rot/2, NORM pairs 2i and 2i+1.
__device__ __forceinline__ void rope_vec(float* buf, int n_rot, int mode, float rpos, const float* inv, const float* ff)
{
	const int half = n_rot / 2;
	const int step = mode == 0 ? 1 : 2;
	const int other = mode == 0 ? half : 1;
	for (int i = threadIdx.x & 31; i < half; i += 32)
	{
		float theta = rpos * inv[i];
		if (ff) theta = __fdiv_rn(theta, ff[i]);
		float sn, cs;
		sincosf(theta, &sn, &cs);
		float* p = buf + i * step;
		const float a = p[0], b = p[other];
		p[0] = cs * a - sn * b;
		p[other] = sn * a + cs * b;
	}
}

// The same rotation with the angles' cosines and sines computed beforehand
// (cs[i], sn[i] for pair i, as rope_vec forms them): the table depends only on
// the token's position, so one table serves every head of the token.
__device__ __forceinline__ void rope_apply(float* buf, int n_rot, int mode, const float* cs, const float* sn)
{
	const int half = n_rot / 2;
	const int step = mode == 0 ? 1 : 2;
	const int other = mode == 0 ? half : 1;
	for (int i = threadIdx.x & 31; i < half; i += 32)
	{
		float* p = buf + i * step;
		const float a = p[0], b = p[other];
		p[0] = cs[i] * a - sn[i] * b;
		p[other] = sn[i] * a + cs[i] * b;
	}
}

// A head vector of up to 512 floats held by a warp, lane-strided: element
// lane + 32 k in slot k. Loading all of it into registers before writing any
// of it to shared memory lets the loads overlap (through generic pointers the
// compiler could not otherwise move a load past the previous store).
struct HeadRegs
{
	float x[16];
};

__device__ __forceinline__ void load_head(HeadRegs& r, const float* __restrict__ src, int D)
{
	const int lane = threadIdx.x & 31;
#pragma unroll
	for (int k = 0; k < 16; ++k)
	{
		const int i = lane + 32 * k;
		r.x[k] = i < D ? src[i] : 0.0f;
	}
}

// One head vector in shared `buf` through attention_forward's per-head steps
// (model.cpp:1616-1660), in place: RMSNorm with `gamma` (or the plain norm
// when plain_norm), then RoPE when rotate. Warp-cooperative; buf holds the
// result, visible to the whole warp, on return.
__device__ __forceinline__ void prep_buf(float* buf, int D, const float* gamma, bool plain_norm, float eps,
                                         bool rotate, int n_rot, int mode, float rpos, const float* inv,
                                         const float* ff)
{
	const int lane = threadIdx.x & 31;
	if (gamma)
	{
		const float sc = rms_scale(buf, D, eps, true);
		for (int i = lane; i < D; i += 32) buf[i] = buf[i] * sc * gamma[i];
	}
	else if (plain_norm)
	{
		const float sc = rms_scale(buf, D, eps, false);
		for (int i = lane; i < D; i += 32) buf[i] = buf[i] * sc;
	}
	__syncwarp();
	if (rotate && n_rot > 0) rope_vec(buf, n_rot, mode, rpos, inv, ff);
	__syncwarp();
}

// The same from registers: the vector goes into `buf` first.
__device__ __forceinline__ void prep_head(float* buf, const HeadRegs& r, int D, const float* gamma, bool plain_norm,
                                          float eps, bool rotate, int n_rot, int mode, float rpos, const float* inv,
                                          const float* ff)
{
	const int lane = threadIdx.x & 31;
#pragma unroll
	for (int k = 0; k < 16; ++k)
	{
		const int i = lane + 32 * k;
		if (i < D) buf[i] = r.x[k];
	}
	__syncwarp();
	prep_buf(buf, D, gamma, plain_norm, eps, rotate, n_rot, mode, rpos, inv, ff);
}

// Narrow a D-vector of floats in shared `buf` to the cache's element type in
// place (element i at ((T*)buf)[i]); warp-cooperative, D <= 512.
template <typename KV>
__device__ __forceinline__ void narrow_buf(float* buf, int D)
{
	using T = typename KV::T;
	if constexpr (KV::esize == 4) return;
	const int lane = threadIdx.x & 31;
	float x[16];
#pragma unroll
	for (int k = 0; k < 16; ++k)
	{
		const int i = lane + 32 * k;
		x[k] = i < D ? buf[i] : 0.0f;
	}
	__syncwarp();
	T* out = reinterpret_cast<T*>(buf);
#pragma unroll
	for (int k = 0; k < 16; ++k)
	{
		const int i = lane + 32 * k;
		if (i < D) store_elem(out + i, x[k]);
	}
	__syncwarp();
}

} // namespace nncu
