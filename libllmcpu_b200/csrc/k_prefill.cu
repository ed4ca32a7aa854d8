// k_prefill.cu -- causal prefill attention on the tensor cores (tcgen05).
//
// The same attention as the reference's batched path (attend_chunks over
// nnc_attn_block / nnc_attn_merge / nnc_attn_finish, model.cpp:1251-1319,
// nn_ops.cpp:351-499): every query row of a long batch attends over its
// causal span. Here, for bf16 caches and head_dim 128, the two products run
// on the 5th-generation tensor cores. One CTA takes 256 query rows of one
// query head as two Q tiles, A and B, of 128 rows, and walks the key tiles of
// their spans, 64 keys at a time; each key tile is loaded once for both:
//
//   S = Q K^T      tcgen05.mma, M 128 x N 64 x K 128, bf16 in, fp32 in TMEM
//   P = softmax    one warpgroup per Q tile, one query row per thread (TMEM lane)
//   O += P V       tcgen05.mma, M 128 x N 128 x K 64, P (bf16) from TMEM over
//                  its own S, V from shared memory, O in TMEM
//
// Roles: warp 0 issues the TMA loads of the two Q tiles and of the K tiles,
// warp 2 those of the V tiles, each into its own 4-stage ring; warp 1 owns
// the TMEM allocation (per Q tile two S buffers of 64 columns and O of 128:
// 512 columns) and, from one lane, issues the MMAs from descriptors formed
// once. Each Q tile's S of key tile t + 2 goes into the buffer of tile t
// right after P_t V_t (tcgen05 MMAs of one thread execute in order), so the
// softmax of tile t + 1 runs while P_t V_t and S_{t+2} are computed. Warps
// 4-7 and 8-11 do the softmax of A and of B: a thread reads its row of S
// from TMEM, masks it by the row's span, writes its probabilities back as
// 16-bit pairs over the first 32 columns of the same S buffer (the A operand
// of P V), keeps O in scale and writes the output row. Online softmax in
// base 2 with a lazily moved maximum: a row's reference maximum moves (and O
// and l are rescaled) only when a new score exceeds it by more than 2^8, so O
// is rarely touched; the result is the same softmax, divided by the same l.
// After a row's first keys, a tile's exponentials are taken against the
// row's held maximum while the tile's own maximum is found on the way (no
// separate pass over the scores); a row whose scores passed the held maximum
// by more than 2^8 moves it and writes its P again. The first warpgroup
// hands registers to the two softmax warpgroups (setmaxnreg).
//
// Operands in shared memory use the 128-byte swizzled K-major layout TMA
// writes (8-row atoms of 1 KB), described to tcgen05.mma by shared memory
// descriptors; V is used as an MN-major operand straight from its tile.
// Every wait is bounded; on a timeout the CTA records an error and steps
// through without waiting further.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <math_constants.h>

#include "common.cuh"
#include "tc.cuh"

namespace nncu
{
namespace
{

constexpr int PF_BM = 128;          // query rows per Q tile; a CTA takes two (A, B)
constexpr int PF_BN = 64;           // keys per tile
constexpr int PF_D = 128;           // head_dim
constexpr int PF_STAGES = 4;        // K and V ring depth
constexpr int PF_THREADS = 384;     // warps 0-3: loads, MMA; 4-7: softmax of A; 8-11: softmax of B
constexpr float LAZY = 8.0f;        // log2 headroom before a row's reference maximum moves

// Shared memory and TMEM of the prefill (head_dim 128).
struct PfLayout
{
	static constexpr int Q_PANEL = 128 * 128;       // 128 rows x 64 bf16, 128-byte swizzled
	static constexpr int Q_TILE = 2 * Q_PANEL;      // 128 rows x 128
	static constexpr int KV_PANEL = PF_BN * 128;    // 64 rows x 64 bf16
	static constexpr int KV_TILE = 2 * KV_PANEL;    // 64 keys x 128
	static constexpr int SM_Q = 0;                  // [2] Q tiles
	static constexpr int SM_K = SM_Q + 2 * Q_TILE;  // [PF_STAGES] K stages
	static constexpr int SM_V = SM_K + PF_STAGES * KV_TILE; // [PF_STAGES] V stages
	static constexpr int SM_BAR = SM_V + PF_STAGES * KV_TILE;
	static constexpr int SMEM = SM_BAR + 256 + 1024; // + alignment slack
	// TMEM columns: S of Q tile X, buffer b at 128 X + 64 b (its P, bf16
	// pairs, in its first 32 columns); O of Q tile X at 256 + 128 X
	static constexpr uint32_t T_S = 0, T_O = 256, COLS = 512;
};

// S = Q K^T for one Q tile and one 64-key tile, eight K steps of 16 over
// head_dim 128 in one asm block: A (Q) and B (K) K-major, 128-byte swizzled;
// K step k advances each descriptor by (k >> 2) of its panels + (k & 3) x 32
// bytes (16-byte units), from descriptors formed once.
template <uint32_t AP, uint32_t BP>
__device__ __forceinline__ void mma8_s(uint32_t d, uint64_t a, uint64_t b, uint32_t id)
{
	asm volatile(
		"{\n\t.reg .pred p0, p1;\n\t.reg .b64 a, b;\n\t"
		"setp.ne.b32 p0, 0, 0;\n\tsetp.eq.b32 p1, 0, 0;\n\t"
		"tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p0;\n\t"
		"add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p1;\n\t"
		"add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p1;\n\t"
		"add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p1;\n\t"
		"add.s64 a, %1, %4;\n\tadd.s64 b, %2, %8;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p1;\n\t"
		"add.s64 a, %1, %5;\n\tadd.s64 b, %2, %9;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p1;\n\t"
		"add.s64 a, %1, %6;\n\tadd.s64 b, %2, %10;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p1;\n\t"
		"add.s64 a, %1, %7;\n\tadd.s64 b, %2, %11;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p1;\n\t}"
		::"r"(d), "l"(a), "l"(b), "r"(id), "n"(AP), "n"(AP + 2), "n"(AP + 4), "n"(AP + 6), "n"(BP), "n"(BP + 2),
		"n"(BP + 4), "n"(BP + 6)
		: "memory");
}

// O (+)= P V over a 64-key tile: A = P from TMEM (8 columns per K step of 16
// keys), B = V MN-major (2048 bytes per K step); `acc` = 0 starts O afresh.
__device__ __forceinline__ void mma4_pv(uint32_t d, uint32_t a, uint64_t b, uint32_t id, uint32_t acc)
{
	asm volatile(
		"{\n\t.reg .pred p0, p1;\n\t.reg .b64 b;\n\t.reg .b32 a;\n\t"
		"setp.ne.b32 p0, %4, 0;\n\tsetp.eq.b32 p1, 0, 0;\n\t"
		"tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p0;\n\t"
		"add.s32 a, %1, 8;\n\tadd.s64 b, %2, 128;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, p1;\n\t"
		"add.s32 a, %1, 16;\n\tadd.s64 b, %2, 256;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, p1;\n\t"
		"add.s32 a, %1, 24;\n\tadd.s64 b, %2, 384;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, p1;\n\t}"
		::"r"(d), "r"(a), "l"(b), "r"(id), "r"(acc)
		: "memory");
}

// 16 consecutive 32-bit columns into this thread's TMEM lane.
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t* v)
{
	asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
	             "%12, %13, %14, %15, %16};" ::"r"(taddr),
	             "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
	             "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
	             : "memory");
}

// Two non-negative floats to bf16, packed (lo in the low half), rounded to
// nearest with ties away from zero (an exact tie needs the low 16 bits to be
// 0x8000: a bias below 2^-16 of an ulp), on the integer pipe: bf16 keeps the
// exponent, so this is the float's top half after the carry.
__device__ __forceinline__ uint32_t pack_p_bf16(float lo, float hi)
{
	const uint32_t a = __float_as_uint(lo) + 0x8000u, b = __float_as_uint(hi) + 0x8000u;
	uint32_t r;
	asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(r) : "r"(a), "r"(b));
	return r;
}
__device__ __forceinline__ uint32_t pack_p_f16(float lo, float hi)
{
	__half2 h = __floats2half2_rn(lo, hi);
	return *reinterpret_cast<uint32_t*>(&h);
}

template <bool BF16>
__global__ void __launch_bounds__(PF_THREADS, 1)
	prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const PrefillPlan P)
{
	using L = PfLayout;
	constexpr int D = PF_D;
	extern __shared__ unsigned char smem_raw[];
	unsigned char* smem =
		reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::SM_BAR);
	uint64_t* q_full = bars + 0;
	uint64_t* k_full = bars + 1;    // [PF_STAGES]
	uint64_t* k_empty = bars + 5;   // [PF_STAGES]: a K stage is free once the S of both Q tiles are done
	uint64_t* v_full = bars + 9;    // [PF_STAGES]
	uint64_t* v_empty = bars + 13;  // [PF_STAGES]: a V stage is free once both P V are done
	uint64_t* s_full = bars + 17;   // [2 Q tiles][2 buffers]
	uint64_t* p_full = bars + 21;   // [2 Q tiles][2 buffers]: P in TMEM (and O rescaled)
	uint64_t* pv_done = bars + 25;  // [2 Q tiles]: one phase per P V of the tile (for a rescale of O)
	uint64_t* mma_done = bars + 27; // every MMA issued has completed
	uint64_t* o_done = bars + 28;   // [2 Q tiles]: the tile's last P V has completed (one phase)
	uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 30);
	volatile int* flags = reinterpret_cast<volatile int*>(bars + 31); // [0] abort

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	// the heaviest pairs of query tiles (the longest causal spans) go first;
	// neighbouring CTAs are the query heads of one KV head (its K, V in L2)
	const int h = blockIdx.x % P.n_head;
	const int q0 = (P.q_pairs - 1 - (int)blockIdx.x / P.n_head) * (2 * PF_BM);
	const int hk = h / (P.n_head / P.n_kv);
	// each Q tile's 64-key tiles [lo, hi] (the union of its rows' spans); a
	// tile past the batch is absent (lo > hi)
	int lo[2], hi[2];
#pragma unroll
	for (int X = 0; X < 2; ++X)
	{
		const int r0 = q0 + X * PF_BM;
		lo[X] = 1;
		hi[X] = 0;
		if (r0 < P.n_tok)
		{
			const int qlo = P.pos0 + r0, qhi = P.pos0 + min(P.n_tok, r0 + PF_BM) - 1;
			const int klo = (P.window > 0 && qlo + 1 > P.window) ? qlo + 1 - P.window : 0;
			lo[X] = klo / PF_BN;
			hi[X] = min(qhi, P.n_seq - 1) / PF_BN;
		}
	}
	// the tiles streamed: from A's first to the last of either (contiguous:
	// B's first row directly follows A's last)
	const int u_lo = lo[0], n_u = max(hi[0], hi[1]) - u_lo + 1;

	if (threadIdx.x == 0)
	{
		mbar_init(q_full, 1);
		for (int s = 0; s < PF_STAGES; ++s)
		{
			mbar_init(&k_full[s], 1);
			mbar_init(&k_empty[s], 1);
			mbar_init(&v_full[s], 1);
			mbar_init(&v_empty[s], 1);
		}
		for (int i = 0; i < 4; ++i)
		{
			mbar_init(&s_full[i], 1);
			mbar_init(&p_full[i], 128);
		}
		mbar_init(&pv_done[0], 1);
		mbar_init(&pv_done[1], 1);
		mbar_init(&o_done[0], 1);
		mbar_init(&o_done[1], 1);
		mbar_init(mma_done, 1);
		flags[0] = 0;
		fence_barrier_init();
	}
	if (warp == 1) tmem_alloc(tmem_slot, L::COLS);
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tmem_slot;

	// registers from the load and MMA warps to the softmax warpgroups (the
	// launch gives every thread 168; 128 x 96 + 256 x 200 = 63,488 of 64,512)
	if (warp < 4)
	{
		asm volatile("setmaxnreg.dec.sync.aligned.u32 96;" ::: "memory");
		if (warp == 0 || warp == 2)
		{
			// ---- TMA: warp 0 the Q tiles once, then the K tiles; warp 2 the V
			// tiles; each through its own PF_STAGES-deep ring ----
			if (lane == 0)
			{
				const bool is_k = warp == 0;
				const CUtensorMap* map = is_k ? &kmap : &vmap;
				uint64_t* full = is_k ? k_full : v_full;
				uint64_t* empty = is_k ? k_empty : v_empty;
				unsigned char* ring = smem + (is_k ? L::SM_K : L::SM_V);
				if (is_k)
				{
					const int nq = lo[1] <= hi[1] ? 2 : 1;
					mbar_arrive_expect_tx(q_full, nq * L::Q_TILE);
					for (int X = 0; X < nq; ++X)
						for (int p = 0; p < 2; ++p)
							tma3(smem + L::SM_Q + X * L::Q_TILE + p * L::Q_PANEL, &qmap, 64 * p, q0 + X * PF_BM, h,
							     q_full);
				}
				int issued = 0;
				for (int u = 0; u < n_u; ++u)
				{
					const int s = u % PF_STAGES;
					if (u >= PF_STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(((u / PF_STAGES) - 1) & 1), P.err,
					                                         DEVERR_WAIT_EMPTY))
					{
						flags[0] = 1;
						break;
					}
					if (flags[0]) break;
					unsigned char* t = ring + s * L::KV_TILE;
					const int key0 = (u_lo + u) * PF_BN;
					mbar_arrive_expect_tx(&full[s], L::KV_TILE);
					for (int p = 0; p < 2; ++p) tma3(t + p * L::KV_PANEL, map, 64 * p, key0, hk, &full[s]);
					issued = u + 1;
				}
				// on an abort, do not leave while a copy may still land here
				if (is_k) mbar_wait_bounded(q_full, 0, nullptr, 0);
				for (int u = max(0, issued - PF_STAGES); u < issued; ++u)
					mbar_wait_bounded(&full[u % PF_STAGES], (uint32_t)((u / PF_STAGES) & 1), nullptr, 0);
			}
			__syncwarp(); // the whole warp meets the final barrier together
		}
		else if (warp == 1)
		{
			// ---- MMA issue. Each Q tile has two S buffers: S of its tile
			// t + 2 goes into the buffer of tile t right after P_t V_t (tcgen05
			// MMAs of one thread execute in order), so the softmax of tile t + 1
			// runs while P_t V_t and S_{t+2} are computed ----
			if (lane == 0)
			{
				constexpr uint32_t ID_S = tc_idesc(128, PF_BN, BF16, false, false);
				constexpr uint32_t ID_PV = tc_idesc(128, D, BF16, false, true);
				// the operands' shared memory descriptors, formed once
				const uint64_t dq = sdesc(smem_u32(smem + L::SM_Q), 16, 1024);
				const uint64_t dk = sdesc(smem_u32(smem + L::SM_K), 16, 1024);
				const uint64_t dv = sdesc(smem_u32(smem + L::SM_V), L::KV_PANEL, 1024);
				auto has = [&](int X, int t) { return X ? (t >= lo[1] && t <= hi[1]) : (t >= lo[0] && t <= hi[0]); };
				int ns[2] = {0, 0}, np[2] = {0, 0}; // S issued, P consumed, per Q tile
				auto issue_s = [&](int X, int u) {
					const int b = ns[X] & 1;
					mma8_s<(uint32_t)(L::Q_PANEL >> 4), (uint32_t)(L::KV_PANEL >> 4)>(
						tmem + L::T_S + 128 * X + 64 * b, dq + (uint64_t)X * (L::Q_TILE >> 4),
						dk + (uint64_t)(u % PF_STAGES) * (L::KV_TILE >> 4), ID_S);
					mma_commit(&s_full[2 * X + b]);
					++ns[X];
				};
				bool ok = mbar_wait_bounded(q_full, 0, P.err, DEVERR_WAIT_FULL);
				for (int u = 0; ok && u < min(2, n_u); ++u)
				{
					ok = !flags[0] && mbar_wait_bounded(&k_full[u % PF_STAGES], (uint32_t)((u / PF_STAGES) & 1), P.err,
					                                    DEVERR_WAIT_FULL);
					if (!ok) break;
					tc_fence_after();
					for (int X = 0; X < 2; ++X)
						if (has(X, u_lo + u)) issue_s(X, u);
					mma_commit(&k_empty[u % PF_STAGES]);
				}
				for (int u = 0; ok && u < n_u; ++u)
				{
					const int t = u_lo + u, s = u % PF_STAGES;
					ok = !flags[0] && mbar_wait_bounded(&v_full[s], (uint32_t)((u / PF_STAGES) & 1), P.err,
					                                    DEVERR_WAIT_FULL);
					const bool ahead = u + 2 < n_u;
					bool k_ready = false;
					for (int X = 0; ok && X < 2; ++X)
					{
						if (has(X, t))
						{
							const int b = np[X] & 1;
							ok = !flags[0] && mbar_wait_bounded(&p_full[2 * X + b], (uint32_t)((np[X] >> 1) & 1), P.err,
							                                    DEVERR_WAIT_FULL);
							if (!ok) break;
							tc_fence_after();
							mma4_pv(tmem + L::T_O + 128 * X, tmem + L::T_S + 128 * X + 64 * b,
							        dv + (uint64_t)s * (L::KV_TILE >> 4), ID_PV, np[X] > 0 ? 1u : 0u);
							mma_commit(&pv_done[X]);
							if (t == (X ? hi[1] : hi[0])) mma_commit(&o_done[X]);
							++np[X];
						}
						if (ahead && has(X, t + 2))
						{
							if (!k_ready)
							{
								const int u2 = u + 2;
								ok = !flags[0] && mbar_wait_bounded(&k_full[u2 % PF_STAGES],
								                                    (uint32_t)((u2 / PF_STAGES) & 1), P.err,
								                                    DEVERR_WAIT_FULL);
								if (!ok) break;
								tc_fence_after();
								k_ready = true;
							}
							issue_s(X, u + 2);
						}
					}
					if (!ok) break;
					mma_commit(&v_empty[s]);
					if (ahead)
					{
						const int u2 = u + 2;
						if (!k_ready) // (every streamed tile belongs to a Q tile; kept for the ring's phases)
							ok = mbar_wait_bounded(&k_full[u2 % PF_STAGES], (uint32_t)((u2 / PF_STAGES) & 1), P.err,
							                       DEVERR_WAIT_FULL);
						mma_commit(&k_empty[u2 % PF_STAGES]);
					}
				}
				if (!ok) flags[0] = 1;
				// every MMA issued has completed before TMEM is freed
				mma_commit(mma_done);
				mbar_wait_bounded(mma_done, 0, nullptr, 0);
			}
			__syncwarp(); // the whole warp meets the final barrier together
		}
	}
	else
	{
		asm volatile("setmaxnreg.inc.sync.aligned.u32 200;" ::: "memory");
		// ---- softmax of Q tile X, one query row per thread (TMEM lane r),
		// O kept in scale, then the output ----
		const int X = (warp - 4) >> 2, wq = warp & 3;
		const int r = wq * 32 + lane;
		const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
		const uint32_t ts0 = tmem + L::T_S + 128 * X + lane_off, to = tmem + L::T_O + 128 * X + lane_off;
		const int row = q0 + X * PF_BM + r;
		const int qp = P.pos0 + row;
		const int kf = (P.window > 0 && qp + 1 > P.window) ? qp + 1 - P.window : 0;
		const int kl = min(qp, P.n_seq - 1);
		float m_used = -CUDART_INF_F, l = 0.0f;
		bool ok = true;
		int n = 0;
		const int t_lo = X ? lo[1] : lo[0], t_hi = X ? hi[1] : hi[0];
		for (int t = t_lo; t <= t_hi; ++t, ++n)
		{
			const int b = n & 1;
			const uint32_t ts = ts0 + 64 * b;
			ok = ok && !flags[0] &&
			     mbar_wait_bounded(&s_full[2 * X + b], (uint32_t)((n >> 1) & 1), P.err, DEVERR_WAIT_FULL);
			if (!__all_sync(0xffffffffu, ok))
			{
				ok = false;
				break;
			}
			tc_fence_after();
			float x[PF_BN];
			tmem_ld32(ts, x);
			tmem_ld32(ts + 32, x + 32);
			tmem_wait_ld();
			// scores in log2 units: sl * s, folded into the exponentials' FMA
			// (sl > 0 keeps the maximum's place); with a soft-cap, capped first
			float sl = P.scale * P.log2e;
			if (P.softcap > 0.0f)
			{
				const float cs = P.scale / P.softcap, cl = P.softcap * P.log2e;
#pragma unroll
				for (int c = 0; c < PF_BN; ++c) x[c] = tanhf(x[c] * cs) * cl;
				sl = 1.0f;
			}
			const int key0 = t * PF_BN;
			if (key0 < kf || key0 + PF_BN - 1 > kl)
			{
#pragma unroll
				for (int c = 0; c < PF_BN; ++c)
					if (key0 + c < kf || key0 + c > kl) x[c] = -CUDART_INF_F;
			}
			// P into the first 32 columns of this S buffer as 16-bit pairs (S is
			// in registers), p = 2^(x sl + nm); with `track`, the largest
			// exponent x sl + nm is returned
			float ls[4];
			auto write_p = [&](float nm, bool track) -> float {
				float mq[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
				for (int i = 0; i < 4; ++i) ls[i] = 0.0f;
#pragma unroll
				for (int c0 = 0; c0 < PF_BN; c0 += 32)
				{
					uint32_t pk[16];
#pragma unroll
					for (int c = 0; c < 32; c += 2)
					{
						const float e0 = fmaf(x[c0 + c], sl, nm), e1 = fmaf(x[c0 + c + 1], sl, nm);
						if (track)
						{
							mq[(c >> 1) & 3] = fmaxf(mq[(c >> 1) & 3], e0);
							mq[(c >> 1) & 3] = fmaxf(mq[(c >> 1) & 3], e1);
						}
						const float p0 = ex2(e0), p1 = ex2(e1); // masked (-inf): 0
						ls[(c >> 1) & 3] += p0 + p1;
						pk[c >> 1] = BF16 ? pack_p_bf16(p0, p1) : pack_p_f16(p0, p1);
					}
					tmem_st16u(ts + c0 / 2, pk);
				}
				return fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
			};
			// the row's reference maximum moves only when a score exceeds it by
			// more than 2^LAZY; then O (in TMEM) and l are rescaled
			float m_new = m_used;
			bool rescale = false;
			if (__any_sync(0xffffffffu, m_used == -CUDART_INF_F))
			{
				// a row without a reference maximum yet (its first keys): the
				// tile's maximum first, then the exponentials
				float mq[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F};
#pragma unroll
				for (int c = 0; c < PF_BN; ++c) mq[c & 3] = fmaxf(mq[c & 3], x[c]);
				const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl;
				const bool move = mx > m_used + LAZY;
				rescale = move && m_used != -CUDART_INF_F;
				m_new = move ? mx : m_used;
				write_p(m_new == -CUDART_INF_F ? 0.0f : -m_new, false); // no key yet: every p is 0
			}
			else
			{
				// the usual tile: the exponentials against the held maximum, the
				// tile's own maximum found on the way; a row whose scores passed
				// the held maximum by more than 2^LAZY moves it and writes its P
				// again (rare after a row's first tiles)
				const float top = write_p(-m_used, true);
				const bool move = top > LAZY;
				if (__any_sync(0xffffffffu, move))
				{
					rescale = move;
					m_new = move ? m_used + top : m_used;
					write_p(-m_new, false);
				}
			}
			const float alpha = rescale ? ex2(m_used - m_new) : 1.0f;
			if (__any_sync(0xffffffffu, rescale))
			{
				// O must hold every P V before this tile's: wait for the last
				// one (a row rescales only after its first tile, so n >= 1; S of
				// this tile completed after P V of tile n - 2, so pv_done is at
				// most one phase behind and its parity wait cannot alias)
				bool done = !flags[0] && mbar_wait_bounded(&pv_done[X], (uint32_t)((n - 1) & 1), P.err,
				                                          DEVERR_WAIT_FULL);
				if (!__all_sync(0xffffffffu, done))
				{
					ok = false;
					break;
				}
				tc_fence_after();
#pragma unroll
				for (int c = 0; c < D; c += 32)
				{
					float o[32];
					tmem_ld32(to + c, o);
					tmem_wait_ld();
#pragma unroll
					for (int i = 0; i < 32; ++i) o[i] *= alpha;
					tmem_st32(to + c, o);
				}
			}
			tmem_wait_st();
			l = fmaf(l, alpha, (ls[0] + ls[1]) + (ls[2] + ls[3]));
			m_used = m_new;
			tc_fence_before();
			mbar_arrive(&p_full[2 * X + b]);
		}
		// the output: O / l once the tile's last P V is done (its own barrier:
		// the softmax may finish its last tile while the P V before it still
		// runs, two phases of pv_done behind, where a parity wait would alias)
		if (ok && n > 0) ok = !flags[0] && mbar_wait_bounded(&o_done[X], 0, P.err, DEVERR_WAIT_FULL);
		if (__all_sync(0xffffffffu, ok) && n > 0)
		{
			tc_fence_after();
			const float inv = l > 0.0f ? 1.0f / l : 0.0f;
			const size_t orow0 = ((size_t)row * P.n_head + h) * D;
#pragma unroll
			for (int c = 0; c < D; c += 32)
			{
				float o[32];
				tmem_ld32(to + c, o);
				tmem_wait_ld();
				if (row < P.n_tok)
				{
					float* orow = P.out + orow0 + c;
#pragma unroll
					for (int i = 0; i < 32; i += 4)
						*reinterpret_cast<float4*>(orow + i) = gated4(
							make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv), P.gate, orow0 + c + i);
				}
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 1)
	{
		tc_fence_after();
		tmem_dealloc(tmem, L::COLS);
	}
}

// The per-head work of a prefill's tokens before the attention (model.cpp:
// 1616-1694), one CTA per token, a warp per head vector: the q rows get
// RMSNorm with the gains and RoPE and go out in the tensor-core kernel's
// operand form (bf16, head-major [n_head][n_tok][128]); the k rows get
// RMSNorm and RoPE, the v rows the plain norm where asked, and both are
// appended to the cache at row pos % rows in its type. The rotation's
// cosines and sines depend only on the token, so each CTA forms them once
// (64 angles) for all its heads.
template <typename KV>
__global__ void __launch_bounds__(256) prefill_prep_kernel(const __grid_constant__ DevJob j, __nv_bfloat16* qb)
{
	using T = typename KV::T;
	static_assert(sizeof(T) == 2, "the prefill's cache and q rows are bf16");
	__shared__ __align__(16) float s_qg[PF_D], s_kg[PF_D], s_cs[PF_D / 2], s_sn[PF_D / 2];
	const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int half = j.n_rot / 2;
	const int pos = j.pos0 + t;
	const bool append = !j.reuse_kv && pos >= j.key_lo && pos < j.key_hi;
	const int n_head = j.n_head, n_kv = j.n_kv;
	const int n_tasks = n_head + (append ? 2 * n_kv : 0); // q heads, then k heads, then v heads
	auto src_of = [&](int task) -> const float* {
		if (task < n_head) return j.q + ((size_t)t * n_head + task) * PF_D;
		const int u = task - n_head;
		return u < n_kv ? j.k + ((size_t)t * n_kv + u) * PF_D : j.v + ((size_t)t * n_kv + (u - n_kv)) * PF_D;
	};
	// head vectors in registers, elements 4 lane .. 4 lane + 3 in v[0..3]
	// (one 16-byte load per lane); a warp issues the loads of all its vectors
	// of a round (up to PREP_PER_WARP) before working on the first, so their
	// latencies overlap
	auto load = [&](float* dst, int task) {
		const float4 x = reinterpret_cast<const float4*>(src_of(task))[lane];
		dst[0] = x.x;
		dst[1] = x.y;
		dst[2] = x.z;
		dst[3] = x.w;
	};
	constexpr int PREP_PER_WARP = 8;
	float vv[PREP_PER_WARP][4];
#pragma unroll
	for (int r = 0; r < PREP_PER_WARP; ++r)
		if (warp + 8 * r < n_tasks) load(vv[r], warp + 8 * r);
	const float rpos = (float)pos * j.rope_scale;
	for (int i = threadIdx.x; i < PF_D; i += blockDim.x)
	{
		s_qg[i] = j.q_gamma ? j.q_gamma[i] : 0.0f;
		s_kg[i] = j.k_gamma ? j.k_gamma[i] : 0.0f;
		if (i < half)
		{
			float theta = rpos * j.rope_inv[i];
			if (j.freq_factors) theta = __fdiv_rn(theta, j.freq_factors[i]);
			sincosf(theta, &s_sn[i], &s_cs[i]);
		}
	}
	__syncthreads();
	// NEOX pairs elements e and e + n_rot/2 (n_rot/2 is 32 or 64, checked on
	// the host): the partner sits in lane ^ 8 or lane ^ 16 at the same place
	// of its four; NORM pairs e and e ^ 1: within a lane's four
	const bool neox = j.rope_mode == 0;
	const int row = pos % j.rows;
	const int partner = half == 64 ? 16 : 8;
	auto process = [&](float* v, int task) {
		const bool is_q = task < n_head, is_k = !is_q && task - n_head < n_kv;
		const float* gamma = is_q ? (j.q_gamma ? s_qg : nullptr) : (is_k && j.k_gamma ? s_kg : nullptr);
		const bool plain = !is_q && !is_k && j.v_rmsnorm;
		if (gamma || plain)
		{
			// RMSNorm as rms_scale does: squares in fp32, the scale in double
			float ss = v[0] * v[0];
			ss = fmaf(v[1], v[1], ss);
			ss = fmaf(v[2], v[2], ss);
			ss = fmaf(v[3], v[3], ss);
			ss = warp_sum(ss);
			const double mean = gamma ? (double)ss * (double)(1.0f / (float)PF_D) : (double)ss / (double)PF_D;
			const float sc = (float)(1.0 / sqrt(mean + (double)j.eps));
			if (gamma)
			{
				const float4 g = reinterpret_cast<const float4*>(gamma)[lane];
				v[0] = v[0] * sc * g.x;
				v[1] = v[1] * sc * g.y;
				v[2] = v[2] * sc * g.z;
				v[3] = v[3] * sc * g.w;
			}
			else
#pragma unroll
				for (int i = 0; i < 4; ++i) v[i] *= sc;
		}
		if ((is_q || is_k) && half > 0)
		{
			if (neox)
			{
				float o[4];
#pragma unroll
				for (int i = 0; i < 4; ++i) o[i] = __shfl_xor_sync(0xffffffffu, v[i], partner);
				const int e = 4 * lane; // this lane's first element
				if (e < 2 * half)
				{
					const bool first = (lane & partner) == 0; // holds e of the pair (e, e + half)
					const float4 cs = reinterpret_cast<const float4*>(s_cs)[lane & (partner - 1)];
					const float4 sn = reinterpret_cast<const float4*>(s_sn)[lane & (partner - 1)];
					const float c[4] = {cs.x, cs.y, cs.z, cs.w}, n[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
					for (int i = 0; i < 4; ++i) v[i] = first ? c[i] * v[i] - n[i] * o[i] : n[i] * o[i] + c[i] * v[i];
				}
			}
			else if (4 * lane < j.n_rot)
			{
				const float2 cs = reinterpret_cast<const float2*>(s_cs)[lane], sn = reinterpret_cast<const float2*>(s_sn)[lane];
				const float a0 = v[0], b0 = v[1], a1 = v[2], b1 = v[3];
				v[0] = cs.x * a0 - sn.x * b0;
				v[1] = sn.x * a0 + cs.x * b0;
				if (4 * lane + 2 < j.n_rot)
				{
					v[2] = cs.y * a1 - sn.y * b1;
					v[3] = sn.y * a1 + cs.y * b1;
				}
			}
		}
		T* dst;
		if (is_q)
			dst = reinterpret_cast<T*>(qb) + ((size_t)task * j.n_tok + t) * PF_D;
		else
		{
			const int h = is_k ? task - n_head : task - n_head - n_kv;
			dst = reinterpret_cast<T*>((is_k ? j.K : j.V) + (size_t)h * j.head_bytes) + (size_t)row * PF_D;
		}
		// four bf16 (round to nearest even) in one 8-byte store
		const __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
		reinterpret_cast<uint2*>(dst)[lane] =
			make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
	};
	for (int base = 0; base < n_tasks; base += 8 * PREP_PER_WARP)
	{
		if (base > 0)
#pragma unroll
			for (int r = 0; r < PREP_PER_WARP; ++r)
				if (base + warp + 8 * r < n_tasks) load(vv[r], base + warp + 8 * r);
#pragma unroll
		for (int r = 0; r < PREP_PER_WARP; ++r)
			if (base + warp + 8 * r < n_tasks) process(vv[r], base + warp + 8 * r);
	}
}

// A 3-D tensor map over a head-major bf16 array [z][y][128] with a
// 64 x 128 x 1 box, 128-byte swizzled (the kernels' operand layout).
int make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t heads)
{
	return make_tensor_map(map, base, true, PF_D, rows, heads, 128);
}

} // namespace

int make_tensor_map(CUtensorMap* map, const void* base, bool bf16, uint64_t D, uint64_t rows, uint64_t planes,
                    uint32_t box_rows)
{
	const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)planes};
	const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)rows * D * 2};
	const cuuint32_t box[3] = {64, box_rows, 1};
	const cuuint32_t estr[3] = {1, 1, 1};
	// the driver's encoder, looked up through the runtime (the library loads
	// without the driver library present, e.g. for its CPU-side checks)
	using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
	                            const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
	                            CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
	static Encode encode = nullptr;
	if (!encode)
	{
		void* fn = nullptr;
		cudaDriverEntryPointQueryResult q;
		if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
		    q != cudaDriverEntryPointSuccess || !fn)
			return (int)cudaErrorNotSupported;
		encode = reinterpret_cast<Encode>(fn);
	}
	const CUresult r = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
	                          const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
	                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
	                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
	return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

bool prefill_supported(int D, int kv_type) { return D == PF_D && kv_type == KV_BF16; }

size_t prefill_qbuf_bytes(int n_tok, int n_head) { return (size_t)n_head * n_tok * PF_D * 2; }

int launch_prefill_prep(const DevJob& j, void* qbuf, void* stream)
{
	if (j.D != PF_D || j.n_tok <= 0) return (int)cudaErrorInvalidValue;
	prefill_prep_kernel<kv_bf16><<<(unsigned)j.n_tok, 256, 0, static_cast<cudaStream_t>(stream)>>>(
		j, static_cast<__nv_bfloat16*>(qbuf));
	return (int)cudaGetLastError();
}

int launch_prefill(const DevJob& j, void* qbuf, int* err, void* stream)
{
	if (j.D != PF_D || j.n_tok <= 0 || j.n_head % j.n_kv) return (int)cudaErrorInvalidValue;
	auto st = static_cast<cudaStream_t>(stream);
	CUtensorMap qmap, kmap, vmap;
	int e = make_map(&qmap, qbuf, (uint64_t)j.n_tok, (uint64_t)j.n_head);
	if (!e) e = make_tensor_map(&kmap, j.K, true, PF_D, (uint64_t)j.rows, (uint64_t)j.n_kv, PF_BN);
	if (!e) e = make_tensor_map(&vmap, j.V, true, PF_D, (uint64_t)j.rows, (uint64_t)j.n_kv, PF_BN);
	if (e) return e;
	cudaError_t ce;
	static bool configured[64] = {};
	int dev = 0;
	cudaGetDevice(&dev);
	if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
	auto kernel = prefill_kernel<true>;
	constexpr int smem = PfLayout::SMEM;
	if (!configured[dev])
	{
		ce = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
		if (ce != cudaSuccess) return (int)ce;
		configured[dev] = true;
	}
	PrefillPlan P{};
	P.n_tok = j.n_tok;
	P.pos0 = j.pos0;
	P.n_seq = j.n_seq;
	P.n_head = j.n_head;
	P.n_kv = j.n_kv;
	P.window = j.window;
	P.q_pairs = (j.n_tok + 2 * PF_BM - 1) / (2 * PF_BM);
	P.scale = j.scale;
	P.log2e = 1.4426950408889634f;
	P.softcap = j.softcap;
	P.out = j.out;
	P.gate = j.gate;
	P.err = err;
	kernel<<<(unsigned)(P.q_pairs * j.n_head), PF_THREADS, smem, st>>>(qmap, kmap, vmap, P);
	return (int)cudaGetLastError();
}

} // namespace nncu
