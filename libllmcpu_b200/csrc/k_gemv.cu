// k_gemv.cu -- the projections' gemvs on the device: libnnc's weight formats
// (nn_ops.h:89-174) times fp32 activations, one vector or a batch of them.
//
//   BF16   y[r] = sum_k bf16(W[r, k]) x[k]                      (nnc_gemv_bf16w_f32x)
//   Q8_0   y[r] = sum_b scale[r, b] sum_{k in b} q[r, k] x[k]   (nnc_gemv_q8_0_f32x)
//   Q4_S   y[r] = sum_b scale[r, b] sum_{k in b} q[r, k] x[k]
//                 + sum_b bias[r, b] xsum[b]                    (nnc_gemv_q4_s_f32x)
//
// with 32-element blocks b, int8 q for Q8_0, and for Q4_S unsigned nibbles,
// byte k of a block holding element k (low nibble) and element k + 16 (high)
// (nnc_quantize_f32_to_q4_s, nn_ops.cpp:1252-1288); scales and biases are
// BF16, row-major [rows][cols / 32]. The batched forms (nn_ops.h:146-170)
// take n_batch vectors x_stride floats apart and write n_batch outputs
// y_stride floats apart. Also the streaming gemv + argmax of the greedy
// lm_head (nnc_gemv_bf16w_argmax_f32x, nn_ops.h:98-115): the index of the
// largest y[r], the first one on ties, without writing y.
//
// The work is the weight stream: one warp per row at a time, each lane
// taking 16 bytes of the row per step (8 BF16 weights, 16 int8 weights, or
// one whole Q4_S block), several steps' loads in flight, up to 8 vectors of
// the batch per pass over the weights (a larger batch makes more passes). A
// single vector against a tall quantised matrix takes 2 to 8 rows per warp at
// a time instead: the rows' quants of a step are in flight together and the
// step's activations are read once for them.
// fp32 accumulation; the sum order differs from the reference's 8-lane FMA
// chains (tolerance: its own tests' 1e-3 x max(1, |y|)).
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>

#include "nncu.h"

#include "common.cuh"
#include "internal.h"

namespace nncu
{
namespace
{

constexpr int GW_THREADS = 256;
constexpr int GW_MAXNB = 8;

struct GemvArgs
{
	const void* w;           // BF16 weights, Q8_0 or Q4_S quants
	const uint16_t* scales;  // Q8_0, Q4_S: BF16 [rows][cols / 32]
	const uint16_t* biases;  // Q4_S: BF16 [rows][cols / 32]
	const float* X;
	size_t x_stride;
	const float* XSUM;       // Q4_S: the vectors' block sums, cols / 32 each
	size_t xsum_stride;
	float* Y;
	size_t y_stride;
	uint32_t rows, cols, n_batch;
	unsigned long long* best; // argmax: the running (value, index) key
	// attention_forward's projections: `bias` (or NULL) added to each output;
	// with split > 0, rows come in pairs of split-row halves per head (query,
	// then gate): the first halves go to Y and the second to Y2, each
	// [n_batch][rows / 2], and the bias applies to Y's only
	const float* bias;
	float* Y2;
	uint32_t split;
};

__device__ __forceinline__ float bf16f(uint32_t h) { return __uint_as_float(h << 16); }

// Small unsigned integers to floats on the integer and FMA pipes (the
// conversion instruction is a quarter-rate one): the byte permute builds the
// bit pattern of 2^23 + n (n in [0, 255] in the low mantissa bits), then one
// subtract of 2^23 leaves exactly n.
__device__ __forceinline__ float byte_as_float(uint32_t word, uint32_t sel)
{
	uint32_t r;
	asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(word), "r"(0x4B000000u), "r"(sel));
	return __uint_as_float(r) - 8388608.0f;
}
// byte i of `word` (as 0..255) into the low byte, zeros above, then 0x4B at the top
__device__ __forceinline__ uint32_t sel_byte(int i) { return 0x7440u | (uint32_t)i; }

__device__ __forceinline__ float4 ldx4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

// One row's dot products with NB vectors (the lanes' partial sums, not yet
// reduced). X rows are read as float4 where the vectors are 16-byte aligned.
template <int FMT, int NB>
__device__ __forceinline__ void row_dots(const GemvArgs& a, uint32_t r, int lane, float (&acc)[NB])
{
#pragma unroll
	for (int v = 0; v < NB; ++v) acc[v] = 0.0f;
	const uint32_t cols = a.cols;
	const bool x4 = (reinterpret_cast<uintptr_t>(a.X) & 15u) == 0 && (NB == 1 || (a.x_stride & 3u) == 0);
	if (FMT == 0)
	{
		const uint16_t* row = static_cast<const uint16_t*>(a.w) + (size_t)r * cols;
		const bool vec = x4 && (cols & 7u) == 0 && (reinterpret_cast<uintptr_t>(a.w) & 15u) == 0;
		uint32_t k0 = 0;
		if (vec)
		{
			const uint4* row4 = reinterpret_cast<const uint4*>(row);
			const uint32_t n8 = cols / 8;
#pragma unroll 4
			for (uint32_t i = lane; i < n8; i += 32)
			{
				const uint4 w4 = __ldg(row4 + i);
				const float w[8] = {__uint_as_float(w4.x << 16), __uint_as_float(w4.x & 0xFFFF0000u),
				                    __uint_as_float(w4.y << 16), __uint_as_float(w4.y & 0xFFFF0000u),
				                    __uint_as_float(w4.z << 16), __uint_as_float(w4.z & 0xFFFF0000u),
				                    __uint_as_float(w4.w << 16), __uint_as_float(w4.w & 0xFFFF0000u)};
#pragma unroll
				for (int v = 0; v < NB; ++v)
				{
					const float* x = a.X + (size_t)v * a.x_stride + (size_t)i * 8;
					const float4 xa = ldx4(x), xb = ldx4(x + 4);
					float s = acc[v];
					s = fmaf(w[0], xa.x, s);
					s = fmaf(w[1], xa.y, s);
					s = fmaf(w[2], xa.z, s);
					s = fmaf(w[3], xa.w, s);
					s = fmaf(w[4], xb.x, s);
					s = fmaf(w[5], xb.y, s);
					s = fmaf(w[6], xb.z, s);
					s = fmaf(w[7], xb.w, s);
					acc[v] = s;
				}
			}
			k0 = n8 * 8;
		}
		for (uint32_t k = k0 + lane; k < cols; k += 32)
		{
			const float w = bf16f(row[k]);
#pragma unroll
			for (int v = 0; v < NB; ++v) acc[v] = fmaf(w, __ldg(a.X + (size_t)v * a.x_stride + k), acc[v]);
		}
	}
	else if (FMT == 1)
	{
		// 16 int8 weights per lane step: half a block, one scale. A weight q
		// is taken as (q + 128) - 128: the sign bit flipped makes it an
		// unsigned byte, and the 128 comes off with the magic subtract
		const uint4* row4 = reinterpret_cast<const uint4*>(static_cast<const int8_t*>(a.w) + (size_t)r * cols);
		const uint16_t* sc = a.scales + (size_t)r * (cols / 32);
		const uint32_t n16 = cols / 16;
#pragma unroll 2
		for (uint32_t i = lane; i < n16; i += 32)
		{
			const uint4 q4 = __ldg(row4 + i);
			const float s = bf16f(__ldg(sc + i / 2));
			const uint32_t qq[4] = {q4.x ^ 0x80808080u, q4.y ^ 0x80808080u, q4.z ^ 0x80808080u, q4.w ^ 0x80808080u};
			float w[16];
#pragma unroll
			for (int j = 0; j < 4; ++j)
#pragma unroll
				for (int t = 0; t < 4; ++t) w[4 * j + t] = byte_as_float(qq[j], sel_byte(t)) - 128.0f;
#pragma unroll
			for (int v = 0; v < NB; ++v)
			{
				const float* x = a.X + (size_t)v * a.x_stride + (size_t)i * 16;
				float d = 0.0f;
				if (x4)
				{
#pragma unroll
					for (int j = 0; j < 4; ++j)
					{
						const float4 xv = ldx4(x + 4 * j);
						d = fmaf(w[4 * j], xv.x, d);
						d = fmaf(w[4 * j + 1], xv.y, d);
						d = fmaf(w[4 * j + 2], xv.z, d);
						d = fmaf(w[4 * j + 3], xv.w, d);
					}
				}
				else
#pragma unroll
					for (int k = 0; k < 16; ++k) d = fmaf(w[k], __ldg(x + k), d);
				acc[v] = fmaf(s, d, acc[v]);
			}
		}
	}
	else
	{
		// one whole block (16 bytes, 32 nibbles) per lane step: byte k holds
		// element k (low nibble) and element k + 16 (high)
		const uint4* row4 = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.w) + (size_t)r * (cols / 2));
		const uint32_t nb = cols / 32;
		const uint16_t* sc = a.scales + (size_t)r * nb;
		const uint16_t* bi = a.biases + (size_t)r * nb;
#pragma unroll 2
		for (uint32_t b = lane; b < nb; b += 32)
		{
			const uint4 q4 = __ldg(row4 + b);
			const float s = bf16f(__ldg(sc + b)), bias = bf16f(__ldg(bi + b));
			const uint32_t qq[4] = {q4.x, q4.y, q4.z, q4.w};
			float w[32];
#pragma unroll
			for (int j = 0; j < 4; ++j)
			{
				const uint32_t lo = qq[j] & 0x0F0F0F0Fu, hi = (qq[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
				for (int t = 0; t < 4; ++t)
				{
					w[4 * j + t] = byte_as_float(lo, sel_byte(t));
					w[16 + 4 * j + t] = byte_as_float(hi, sel_byte(t));
				}
			}
#pragma unroll
			for (int v = 0; v < NB; ++v)
			{
				const float* x = a.X + (size_t)v * a.x_stride + (size_t)b * 32;
				float d = 0.0f;
				if (x4)
				{
#pragma unroll
					for (int j = 0; j < 8; ++j)
					{
						const float4 xv = ldx4(x + 4 * j);
						d = fmaf(w[4 * j], xv.x, d);
						d = fmaf(w[4 * j + 1], xv.y, d);
						d = fmaf(w[4 * j + 2], xv.z, d);
						d = fmaf(w[4 * j + 3], xv.w, d);
					}
				}
				else
#pragma unroll
					for (int k = 0; k < 32; ++k) d = fmaf(w[k], __ldg(x + k), d);
				acc[v] = fmaf(s, d, fmaf(bias, __ldg(a.XSUM + (size_t)v * a.xsum_stride + b), acc[v]));
			}
		}
	}
}

// RR consecutive rows of one warp against one vector, quantised formats: at
// each 16-byte step of a lane the RR rows' quants are loaded together (RR
// loads in flight per lane), the step's activations once for all of them,
// and each row's sum formed exactly as row_dots forms it. Rows past the end
// read the last row again; the caller drops them.
template <int FMT, int RR>
__device__ __forceinline__ void rows_dot1(const GemvArgs& a, uint32_t r0, int lane, float (&acc)[RR])
{
#pragma unroll
	for (int i = 0; i < RR; ++i) acc[i] = 0.0f;
	const uint32_t cols = a.cols, nb = cols / 32;
	const bool x4 = (reinterpret_cast<uintptr_t>(a.X) & 15u) == 0;
	uint32_t rr_[RR];
#pragma unroll
	for (int i = 0; i < RR; ++i) rr_[i] = min(r0 + i, a.rows - 1);
	if (FMT == 1)
	{
		const uint32_t n16 = cols / 16;
		for (uint32_t i = lane; i < n16; i += 32)
		{
			uint4 q[RR];
			float sc[RR];
#pragma unroll
			for (int k = 0; k < RR; ++k)
			{
				q[k] = __ldg(reinterpret_cast<const uint4*>(static_cast<const int8_t*>(a.w) + (size_t)rr_[k] * cols) + i);
				sc[k] = bf16f(__ldg(a.scales + (size_t)rr_[k] * nb + i / 2));
			}
			float x[16];
			const float* xp = a.X + (size_t)i * 16;
			if (x4)
			{
#pragma unroll
				for (int j = 0; j < 4; ++j)
				{
					const float4 xv = ldx4(xp + 4 * j);
					x[4 * j] = xv.x;
					x[4 * j + 1] = xv.y;
					x[4 * j + 2] = xv.z;
					x[4 * j + 3] = xv.w;
				}
			}
			else
#pragma unroll
				for (int k = 0; k < 16; ++k) x[k] = __ldg(xp + k);
#pragma unroll
			for (int k = 0; k < RR; ++k)
			{
				const uint32_t qq[4] = {q[k].x ^ 0x80808080u, q[k].y ^ 0x80808080u, q[k].z ^ 0x80808080u,
				                        q[k].w ^ 0x80808080u};
				float d = 0.0f;
#pragma unroll
				for (int j = 0; j < 4; ++j)
#pragma unroll
					for (int t = 0; t < 4; ++t) d = fmaf(byte_as_float(qq[j], sel_byte(t)) - 128.0f, x[4 * j + t], d);
				acc[k] = fmaf(sc[k], d, acc[k]);
			}
		}
	}
	else
	{
		for (uint32_t b = lane; b < nb; b += 32)
		{
			uint4 q[RR];
			float sc[RR], bi[RR];
#pragma unroll
			for (int k = 0; k < RR; ++k)
			{
				q[k] = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.w) + (size_t)rr_[k] * (cols / 2)) + b);
				sc[k] = bf16f(__ldg(a.scales + (size_t)rr_[k] * nb + b));
				bi[k] = bf16f(__ldg(a.biases + (size_t)rr_[k] * nb + b));
			}
			// the block's activation sum: the caller's (nnc_block_sums_f32), or,
			// without one, formed below from the 32 values once in registers
			float xs = a.XSUM ? __ldg(a.XSUM + b) : 0.0f;
			float x[32];
			const float* xp = a.X + (size_t)b * 32;
			if (x4)
			{
#pragma unroll
				for (int j = 0; j < 8; ++j)
				{
					const float4 xv = ldx4(xp + 4 * j);
					x[4 * j] = xv.x;
					x[4 * j + 1] = xv.y;
					x[4 * j + 2] = xv.z;
					x[4 * j + 3] = xv.w;
				}
			}
			else
#pragma unroll
				for (int k = 0; k < 32; ++k) x[k] = __ldg(xp + k);
			if (!a.XSUM)
			{
				float t[16];
#pragma unroll
				for (int k = 0; k < 16; ++k) t[k] = x[k] + x[k + 16];
#pragma unroll
				for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
					for (int k = 0; k < w; ++k) t[k] += t[k + w];
				xs = t[0];
			}
#pragma unroll
			for (int k = 0; k < RR; ++k)
			{
				const uint32_t qq[4] = {q[k].x, q[k].y, q[k].z, q[k].w};
				float d = 0.0f;
				// the order of row_dots: elements 0-15 (low nibbles) of j = 0..3, then 16-31 (high)
#pragma unroll
				for (int j = 0; j < 4; ++j)
#pragma unroll
					for (int t = 0; t < 4; ++t) d = fmaf(byte_as_float(qq[j] & 0x0F0F0F0Fu, sel_byte(t)), x[4 * j + t], d);
#pragma unroll
				for (int j = 0; j < 4; ++j)
#pragma unroll
					for (int t = 0; t < 4; ++t)
						d = fmaf(byte_as_float((qq[j] >> 4) & 0x0F0F0F0Fu, sel_byte(t)), x[16 + 4 * j + t], d);
				acc[k] = fmaf(sc[k], d, fmaf(bi[k], xs, acc[k]));
			}
		}
	}
}

// Where output row r goes: Y or Y2 (the query / gate split) and its index,
// with its bias (or 0).
struct OutSlot
{
	float* Y;
	uint32_t o;
	float bias;
};

__device__ __forceinline__ OutSlot out_slot(const GemvArgs& a, uint32_t r)
{
	OutSlot s{a.Y, r, 0.0f};
	if (a.split)
	{
		const uint32_t h = r / (2 * a.split), i = r - h * 2 * a.split;
		s.Y = i < a.split ? a.Y : a.Y2;
		s.o = h * a.split + (i < a.split ? i : i - a.split);
	}
	if (a.bias && s.Y == a.Y) s.bias = __ldg(a.bias + s.o);
	return s;
}

// Up to three matrices against the same vectors in one launch (a projection's
// q, k and v): grid row y takes matrix y.
constexpr int GW_MAXMAT = 3;
struct GemvSet
{
	GemvArgs m[GW_MAXMAT];
};

template <int FMT, int NB>
__global__ void __launch_bounds__(GW_THREADS) gemv_kernel(const __grid_constant__ GemvSet set, uint32_t v0)
{
	const GemvArgs& a = set.m[blockIdx.y];
	const int lane = threadIdx.x & 31;
	const uint32_t warps = gridDim.x * (GW_THREADS / 32);
	GemvArgs b = a;
	b.X = a.X + (size_t)v0 * a.x_stride;
	if (FMT == 2) b.XSUM = a.XSUM + (size_t)v0 * a.xsum_stride;
	for (uint32_t r = blockIdx.x * (GW_THREADS / 32) + (threadIdx.x >> 5); r < a.rows; r += warps)
	{
		float acc[NB];
		row_dots<FMT, NB>(b, r, lane, acc);
		const OutSlot os = out_slot(a, r);
#pragma unroll
		for (int v = 0; v < NB; ++v)
		{
			float y = warp_sum(acc[v]);
			if (a.bias) y += os.bias; // the reference adds the bias to the stored float
			if (lane == 0) os.Y[(size_t)(v0 + v) * a.y_stride + os.o] = y;
		}
	}
}

// One vector against quantised weights: RR rows per warp at a time.
template <int FMT, int RR>
__global__ void __launch_bounds__(GW_THREADS) gemv_rows_kernel(const __grid_constant__ GemvSet set)
{
	const GemvArgs& a = set.m[blockIdx.y];
	const int lane = threadIdx.x & 31;
	const uint32_t warps = gridDim.x * (GW_THREADS / 32);
	for (uint32_t r0 = (blockIdx.x * (GW_THREADS / 32) + (threadIdx.x >> 5)) * RR; r0 < a.rows; r0 += warps * RR)
	{
		float acc[RR];
		rows_dot1<FMT, RR>(a, r0, lane, acc);
#pragma unroll
		for (int k = 0; k < RR; ++k)
		{
			const float y0 = warp_sum(acc[k]);
			if (r0 + k < a.rows)
			{
				const OutSlot os = out_slot(a, r0 + k);
				const float y = a.bias ? y0 + os.bias : y0;
				if (lane == 0) os.Y[os.o] = y;
			}
		}
	}
}

// A float's order as an unsigned key: larger floats, larger keys.
__device__ __forceinline__ uint32_t order_key(float f)
{
	const uint32_t u = __float_as_uint(f);
	return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Greedy lm_head: every warp keeps its best (value, first index) and the
// CTA's best goes into one 64-bit atomic max: value key high, ~index low,
// so the larger value wins and, on a tie, the smaller index.
__global__ void __launch_bounds__(GW_THREADS) gemv_argmax_kernel(const GemvArgs a)
{
	__shared__ unsigned long long s_best[GW_THREADS / 32];
	const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
	const uint32_t warps = gridDim.x * (GW_THREADS / 32);
	unsigned long long best = 0;
	for (uint32_t r = blockIdx.x * (GW_THREADS / 32) + warp; r < a.rows; r += warps)
	{
		float acc[1];
		row_dots<0, 1>(a, r, lane, acc);
		const float y = warp_sum(acc[0]);
		if (y == y) // NaN never wins
		{
			const unsigned long long key = ((unsigned long long)order_key(y) << 32) | (0xFFFFFFFFu - r);
			best = key > best ? key : best;
		}
	}
	if (lane == 0) s_best[warp] = best;
	__syncthreads();
	if (threadIdx.x == 0)
	{
		for (int w = 1; w < GW_THREADS / 32; ++w) best = s_best[w] > best ? s_best[w] : best;
		if (best) atomicMax(a.best, best);
	}
}

// Greedy verify's argmax of each logits row (session.cpp:128-134: the first
// index of the largest value, compared with >): one CTA per row, a 64-bit
// max of (value key, ~index) as above. -0 counts as +0 (equal under >); a NaN
// never wins, and a NaN in the first place is the answer (nothing compares
// greater than it).
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* X, size_t x_stride, uint32_t n, int32_t* out)
{
	__shared__ unsigned long long s_best[32];
	const float* x = X + (size_t)blockIdx.x * x_stride;
	unsigned long long best = 0;
	for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
	{
		float v = __ldg(x + i);
		if (v == v)
		{
			if (v == 0.0f) v = 0.0f;
			const unsigned long long key = ((unsigned long long)order_key(v) << 32) | (0xFFFFFFFFu - i);
			best = key > best ? key : best;
		}
	}
#pragma unroll
	for (int o = 16; o > 0; o >>= 1)
	{
		const unsigned long long b = __shfl_xor_sync(0xffffffffu, best, o);
		best = b > best ? b : best;
	}
	if ((threadIdx.x & 31) == 0) s_best[threadIdx.x >> 5] = best;
	__syncthreads();
	if (threadIdx.x == 0)
	{
		for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = s_best[w] > best ? s_best[w] : best;
		const float x0 = __ldg(x);
		out[blockIdx.x] = (x0 != x0 || !best) ? 0 : (int32_t)(0xFFFFFFFFu - (uint32_t)(best & 0xFFFFFFFFu));
	}
}

__global__ void argmax_finish_kernel(const unsigned long long* best, int32_t* out)
{
	const unsigned long long b = *best;
	*out = b ? (int32_t)(0xFFFFFFFFu - (uint32_t)(b & 0xFFFFFFFFu)) : -1;
}

// out[b] = sum of x[32 b .. 32 b + 31]: a warp per block.
__global__ void block_sums_kernel(const float* x, float* out, size_t nb)
{
	const size_t b = (size_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
	if (b >= nb) return;
	const float s = warp_sum(x[b * 32 + (threadIdx.x & 31)]);
	if ((threadIdx.x & 31) == 0) out[b] = s;
}

int grid_for(uint32_t rows)
{
	static int sm_count[64] = {}; // per device, looked up once
	int dev = 0;
	cudaGetDevice(&dev);
	int sms = dev >= 0 && dev < 64 ? sm_count[dev] : 0;
	if (sms <= 0)
	{
		sms = 148;
		cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
		if (dev >= 0 && dev < 64) sm_count[dev] = sms;
	}
	const uint32_t want = (rows + GW_THREADS / 32 - 1) / (GW_THREADS / 32);
	return (int)(want < (uint32_t)(sms * 8) ? want : (uint32_t)(sms * 8));
}

// n (1 to GW_MAXMAT) matrices of format FMT, the same vectors and n_batch;
// grid rows beyond a shorter matrix's need return at once.
template <int FMT>
int launch_gemv_fmt(const GemvArgs* mats, int n, cudaStream_t st)
{
	GemvSet set{};
	uint32_t rows = 0;
	for (int i = 0; i < n; ++i)
	{
		set.m[i] = mats[i];
		rows = mats[i].rows > rows ? mats[i].rows : rows;
	}
	const uint32_t n_batch = mats[0].n_batch;
	if constexpr (FMT != 0)
	{
		// one vector: RR rows per warp (their quants in flight together) on
		// matrices tall enough to keep every SM busy with RR rows per warp.
		// Measured on a B200 (L2 flushed, one vector, cols 2560 and 4096):
		// Q4_S best at 8 rows per warp from 12288 rows (65536 x 4096: 256 us at
		// 1, 86 at 4, 64 at 8), at 4 from 2048; Q8_0 best at 4 from 12288
		// (65536 x 4096: 174 us at 1, 91 at 4), at 2 from 8192 (10240 x 2560:
		// 26.6 us at 1, 19.4 at 2), and at 1 row per warp below.
		// Q4_S batches too, one vector per launch (this kernel alone forms
		// the block sums itself when the caller passes none): the batched kernel's
		// per-vector arithmetic (activation loads and FMAs for every row) costs
		// more than re-reading the weights, which stay in L2 from the first
		// vector (10240 x 2560: 4 vectors 103 us batched, 70.6 one by one; 16
		// vectors 447 us against 284.7). Each row's sum is formed in the same
		// order either way.
		const int rr = FMT == 2 ? (rows >= 12288 ? 8 : rows >= 2048 ? 4 : 1) : (rows >= 12288 ? 4 : rows >= 8192 ? 2 : 0);
		if ((n_batch == 1 || FMT == 2) && rr > 0)
		{
			const dim3 grid((unsigned)grid_for((rows + rr - 1) / rr), (unsigned)n);
			for (uint32_t v = 0; v < n_batch; ++v)
			{
				GemvSet one = set;
				for (int i = 0; i < n; ++i)
				{
					GemvArgs& m = one.m[i];
					m.X = mats[i].X + (size_t)v * mats[i].x_stride;
					if (FMT == 2 && m.XSUM) m.XSUM = mats[i].XSUM + (size_t)v * mats[i].xsum_stride;
					m.Y = mats[i].Y + (size_t)v * mats[i].y_stride;
					if (m.Y2) m.Y2 = mats[i].Y2 + (size_t)v * mats[i].y_stride;
					m.n_batch = 1;
				}
				if (rr == 8)
					gemv_rows_kernel<FMT, 8><<<grid, GW_THREADS, 0, st>>>(one);
				else if (rr == 4)
					gemv_rows_kernel<FMT, 4><<<grid, GW_THREADS, 0, st>>>(one);
				else if (rr == 2)
					gemv_rows_kernel<FMT, 2><<<grid, GW_THREADS, 0, st>>>(one);
				else
					gemv_rows_kernel<FMT, 1><<<grid, GW_THREADS, 0, st>>>(one);
				note_launches(1);
			}
			return (int)cudaGetLastError();
		}
	}
	// the batched kernel reads the caller's block sums (only the rows kernel
	// forms them itself)
	if (FMT == 2)
		for (int i = 0; i < n; ++i)
			if (!mats[i].XSUM) return (int)cudaErrorInvalidValue;
	const dim3 grid((unsigned)grid_for(rows), (unsigned)n);
	for (uint32_t v0 = 0; v0 < n_batch;)
	{
		const uint32_t left = n_batch - v0;
		if (left >= 8)
			gemv_kernel<FMT, 8><<<grid, GW_THREADS, 0, st>>>(set, v0), v0 += 8;
		else if (left >= 4)
			gemv_kernel<FMT, 4><<<grid, GW_THREADS, 0, st>>>(set, v0), v0 += 4;
		else if (left >= 2)
			gemv_kernel<FMT, 2><<<grid, GW_THREADS, 0, st>>>(set, v0), v0 += 2;
		else
			gemv_kernel<FMT, 1><<<grid, GW_THREADS, 0, st>>>(set, v0), v0 += 1;
		note_launches(1);
	}
	return (int)cudaGetLastError();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

} // namespace

int check_weight(const nncu_weight& w, uint32_t rows, uint32_t cols, const char* name)
{
	char msg[160];
	msg[0] = 0;
	if (w.type < NNCU_W_BF16 || w.type > NNCU_W_Q4_S)
		snprintf(msg, sizeof msg, "%s: unknown weight type %d", name, (int)w.type);
	else if (w.rows != rows || w.cols != cols)
		snprintf(msg, sizeof msg, "%s: %u x %u weights where %u x %u are needed", name, w.rows, w.cols, rows, cols);
	else if (!w.data)
		snprintf(msg, sizeof msg, "%s: NULL weights", name);
	else if (w.type != NNCU_W_BF16 && (!w.scales || (w.type == NNCU_W_Q4_S && !w.biases)))
		snprintf(msg, sizeof msg, "%s: NULL scales or biases", name);
	else if (w.type != NNCU_W_BF16 && cols % 32)
		snprintf(msg, sizeof msg, "%s: cols must be a multiple of 32", name);
	else if (w.type != NNCU_W_BF16 && !aligned16(w.data))
		snprintf(msg, sizeof msg, "%s: quants must be 16-byte aligned", name);
	return msg[0] ? set_error(NNCU_ERR_INVALID_ARGUMENT, msg) : NNCU_OK;
}

int launch_projections(const Projection* p, int n, const float* X, size_t x_stride, const float* XSUM,
                       size_t xsum_stride, uint32_t n_batch, void* stream)
{
	const auto st = static_cast<cudaStream_t>(stream);
	// one launch per weight format present
	for (int type = NNCU_W_BF16; type <= NNCU_W_Q4_S; ++type)
	{
		GemvArgs mats[GW_MAXMAT];
		int k = 0;
		for (int i = 0; i < n; ++i)
		{
			if (p[i].w->type != type) continue;
			if (k == GW_MAXMAT) return (int)cudaErrorInvalidValue;
			const nncu_weight& w = *p[i].w;
			mats[k++] = GemvArgs{w.data, w.scales, w.biases, X, x_stride, XSUM, xsum_stride, p[i].Y, p[i].y_stride,
			                     w.rows, w.cols, n_batch, nullptr, p[i].bias, p[i].Y2, p[i].split};
		}
		if (k == 0) continue;
		const int e = type == NNCU_W_Q8_0 ? launch_gemv_fmt<1>(mats, k, st)
		              : type == NNCU_W_Q4_S ? launch_gemv_fmt<2>(mats, k, st)
		                                    : launch_gemv_fmt<0>(mats, k, st);
		if (e) return e;
	}
	return 0;
}

int launch_block_sums(const float* x, float* out, size_t n, void* stream)
{
	const size_t nb = n / 32;
	block_sums_kernel<<<(unsigned)((nb + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, out, nb);
	note_launches(1);
	return (int)cudaGetLastError();
}

} // namespace nncu

using namespace nncu;

extern "C" int nncu_gemv_bf16w_f32x_batch_dev(const void* W, const float* X, size_t x_stride, float* Y,
                                              size_t y_stride, uint32_t rows, uint32_t cols, uint32_t n_batch,
                                              void* stream)
{
	if (rows == 0 || cols == 0 || n_batch == 0) return NNCU_OK;
	if (!W || !X || !Y) return set_error(NNCU_ERR_INVALID_ARGUMENT, "gemv: NULL weights, input or output");
	if (n_batch > 1 && (x_stride < cols || y_stride < rows))
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "gemv: strides shorter than a vector");
	GemvArgs a{W, nullptr, nullptr, X, x_stride, nullptr, 0, Y, y_stride, rows, cols, n_batch, nullptr};
	const int e = launch_gemv_fmt<0>(&a, 1, static_cast<cudaStream_t>(stream));
	return e ? set_cuda_error(e, "gemv launch") : NNCU_OK;
}

extern "C" int nncu_gemv_q8_0_f32x_batch_dev(const int8_t* qs, const uint16_t* scales, const float* X,
                                             size_t x_stride, float* Y, size_t y_stride, uint32_t rows,
                                             uint32_t cols, uint32_t n_batch, void* stream)
{
	if (rows == 0 || cols == 0 || n_batch == 0) return NNCU_OK;
	if (!qs || !scales || !X || !Y) return set_error(NNCU_ERR_INVALID_ARGUMENT, "gemv: NULL weights, input or output");
	if (cols % 32) return set_error(NNCU_ERR_INVALID_ARGUMENT, "Q8_0 gemv: cols must be a multiple of 32");
	if (!aligned16(qs)) return set_error(NNCU_ERR_INVALID_ARGUMENT, "Q8_0 gemv: quants must be 16-byte aligned");
	if (n_batch > 1 && (x_stride < cols || y_stride < rows))
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "gemv: strides shorter than a vector");
	GemvArgs a{qs, scales, nullptr, X, x_stride, nullptr, 0, Y, y_stride, rows, cols, n_batch, nullptr};
	const int e = launch_gemv_fmt<1>(&a, 1, static_cast<cudaStream_t>(stream));
	return e ? set_cuda_error(e, "gemv launch") : NNCU_OK;
}

extern "C" int nncu_gemv_q4_s_f32x_batch_dev(const uint8_t* qs, const uint16_t* scales, const uint16_t* biases,
                                             const float* X, size_t x_stride, const float* XSUM, size_t xsum_stride,
                                             float* Y, size_t y_stride, uint32_t rows, uint32_t cols,
                                             uint32_t n_batch, void* stream)
{
	if (rows == 0 || cols == 0 || n_batch == 0) return NNCU_OK;
	if (!qs || !scales || !biases || !X || !XSUM || !Y)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "gemv: NULL weights, input, block sums or output");
	if (cols % 32) return set_error(NNCU_ERR_INVALID_ARGUMENT, "Q4_S gemv: cols must be a multiple of 32");
	if (!aligned16(qs)) return set_error(NNCU_ERR_INVALID_ARGUMENT, "Q4_S gemv: quants must be 16-byte aligned");
	if (n_batch > 1 && (x_stride < cols || y_stride < rows || xsum_stride < cols / 32))
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "gemv: strides shorter than a vector");
	GemvArgs a{qs, scales, biases, X, x_stride, XSUM, xsum_stride, Y, y_stride, rows, cols, n_batch, nullptr};
	const int e = launch_gemv_fmt<2>(&a, 1, static_cast<cudaStream_t>(stream));
	return e ? set_cuda_error(e, "gemv launch") : NNCU_OK;
}

extern "C" int nncu_block_sums_dev(const float* x, float* out, size_t n, void* stream)
{
	if (n == 0 || n % 32) return set_error(NNCU_ERR_INVALID_ARGUMENT, "block sums: n must be a positive multiple of 32");
	if (!x || !out) return set_error(NNCU_ERR_INVALID_ARGUMENT, "block sums: NULL input or output");
	const int e = launch_block_sums(x, out, n, stream);
	return e ? set_cuda_error(e, "block sums launch") : NNCU_OK;
}

extern "C" int nncu_gemv_bf16w_argmax_dev(const void* W, const float* x, uint32_t rows, uint32_t cols,
                                          unsigned long long* scratch, int32_t* out_index, void* stream)
{
	if (rows == 0 || cols == 0) return set_error(NNCU_ERR_INVALID_ARGUMENT, "argmax gemv: no rows or columns");
	if (!W || !x || !scratch || !out_index)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "argmax gemv: NULL weights, input, scratch or output");
	auto st = static_cast<cudaStream_t>(stream);
	cudaError_t ce = cudaMemsetAsync(scratch, 0, sizeof(unsigned long long), st);
	if (ce != cudaSuccess) return set_cuda_error((int)ce, "argmax scratch clear");
	GemvArgs a{W, nullptr, nullptr, x, cols, nullptr, 0, nullptr, 0, rows, cols, 1, scratch};
	gemv_argmax_kernel<<<grid_for(rows), GW_THREADS, 0, st>>>(a);
	argmax_finish_kernel<<<1, 1, 0, st>>>(scratch, out_index);
	note_launches(2);
	const int e = (int)cudaGetLastError();
	return e ? set_cuda_error(e, "argmax gemv launch") : NNCU_OK;
}

extern "C" int nncu_logits_batch_dev(const nncu_weight* lm_head, const float* hidden, int32_t n, float* logits,
                                     float final_softcap, float* xsum, void* stream)
{
	if (!lm_head || !hidden || !logits || n <= 0)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "logits: NULL argument or no rows");
	const int rc = check_weight(*lm_head, lm_head->rows, lm_head->cols, "lm_head");
	if (rc != NNCU_OK) return rc;
	if (final_softcap < 0.0f || final_softcap != final_softcap)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "logits: bad soft-cap");
	const uint32_t cols = lm_head->cols, rows = lm_head->rows;
	// a Q4_S lm_head's block sums: the caller's scratch filled first, or
	// (xsum NULL) formed inside the gemv
	int e = 0;
	if (lm_head->type == NNCU_W_Q4_S && xsum) e = launch_block_sums(hidden, xsum, (size_t)n * cols, stream);
	const Projection pr{lm_head, logits, rows, nullptr, 0, nullptr};
	if (!e)
		e = launch_projections(&pr, 1, hidden, cols, lm_head->type == NNCU_W_Q4_S ? xsum : nullptr, cols / 32,
		                       (uint32_t)n, stream);
	if (!e && final_softcap > 0.0f) e = launch_softcap(logits, logits, (size_t)n * rows, final_softcap, stream);
	return e ? set_cuda_error(e, "logits launch") : NNCU_OK;
}

extern "C" int nncu_argmax_rows_dev(const float* x, size_t x_stride, int32_t n_rows, uint32_t n, int32_t* out,
                                    void* stream)
{
	if (!x || !out || n_rows <= 0 || n == 0) return set_error(NNCU_ERR_INVALID_ARGUMENT, "argmax: NULL argument or empty");
	if (n_rows > 1 && x_stride < n) return set_error(NNCU_ERR_INVALID_ARGUMENT, "argmax: stride shorter than a row");
	argmax_rows_kernel<<<(unsigned)n_rows, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, x_stride, n, out);
	note_launches(1);
	const int e = (int)cudaGetLastError();
	return e ? set_cuda_error(e, "argmax launch") : NNCU_OK;
}
