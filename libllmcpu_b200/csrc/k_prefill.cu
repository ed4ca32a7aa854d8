// k_prefill.cu -- causal prefill attention on the tensor cores (tcgen05).
//
// The same attention as the reference's batched path (attend_chunks over
// nnc_attn_block / nnc_attn_merge / nnc_attn_finish, model.cpp:1251-1319,
// nn_ops.cpp:351-499): every query row of a long batch attends over its
// causal span. Here, for bf16 caches and head_dim 128, the two products run
// on the 5th-generation tensor cores: one CTA takes 128 query rows of one
// query head and walks the key tiles of its span, 128 keys at a time:
//
//   S = Q K^T      tcgen05.mma, M 128 x N 128 x K 128, bf16 in, fp32 in TMEM
//   P = softmax    4 warps, one query row per thread, read from TMEM
//   O += P V       tcgen05.mma, P (bf16) from shared memory, O in TMEM
//
// Roles: warps 0 and 2 issue the TMA loads (Q once and the K tiles; the V
// tiles), each into its own 2-stage ring, K free again as soon as its S is
// done; warp 1 owns the TMEM allocation and, from one lane, issues the MMAs
// (S into two TMEM buffers in turn, so the next tile's S is computed while
// this tile's softmax runs); warps 4 on do the softmax, PF_NH threads per
// query row (the row maximum exchanged through shared memory),
// keep O in scale and write the output. Online softmax in base 2 with a
// lazily moved maximum: a row's reference maximum moves (and O and l are
// rescaled) only when a new score exceeds it by more than 2^8, so O is rarely
// touched; the result is the same softmax, divided by the same l.
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

constexpr int PF_BM = 128;                      // query rows per CTA
constexpr int PF_BN = 128;                      // keys per tile
constexpr int PF_D = 128;                       // head_dim
constexpr int PF_NH = 4;                        // softmax threads per query row (32 columns each)
constexpr int PF_CW = PF_BN / PF_NH;            // columns per softmax thread
constexpr int PF_THREADS = 128 + 128 * PF_NH;   // warps 0-3: TMA, MMA; then the softmax warps
constexpr int PANEL = 128 * 128;                // 128 rows x 64 bf16: one 128-byte-swizzled panel
constexpr int TILE = 2 * PANEL;                 // 128 rows x 128 bf16
constexpr int SM_Q = 0;                         // Q tile
constexpr int SM_K = SM_Q + TILE;               // [2] K tiles
constexpr int SM_V = SM_K + 2 * TILE;           // [2] V tiles
constexpr int SM_P = SM_V + 2 * TILE;           // P tile
constexpr int SM_RED = SM_P + TILE;             // [2 tiles][PF_NH parts][128 rows] row maxima, then [PF_NH][128] row sums
constexpr int SM_BAR = SM_RED + 3 * PF_NH * 128 * 4; // barriers, TMEM address
constexpr int PF_SMEM = SM_BAR + 256 + 1024;    // + alignment slack
constexpr int TMEM_COLS = 512;                  // S0, S1, O (128 columns each)
constexpr float LAZY = 8.0f;                    // log2 headroom before the row maximum moves

// tcgen05 instruction descriptors for the prefill: bf16 A and B, fp32
// accumulate, M = 128, N = 128; A K-major; B K-major (Q K^T) or MN-major (P V).
constexpr uint32_t idesc(bool b_mn_major) { return tc_idesc(128, 128, true, false, b_mn_major); }

} // namespace

namespace
{

__global__ void __launch_bounds__(PF_THREADS, 1)
	prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const PrefillPlan P)
{
	extern __shared__ unsigned char smem_raw[];
	unsigned char* smem =
		reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);
	uint64_t* q_full = bars + 0;
	uint64_t* k_full = bars + 1;   // [2]
	uint64_t* k_empty = bars + 3;  // [2]: K_j no longer needed once S_j is done
	uint64_t* v_full = bars + 5;   // [2]
	uint64_t* v_empty = bars + 7;  // [2]: V_j no longer needed once P_j V_j is done
	uint64_t* s_full = bars + 9;   // [2]
	uint64_t* s_empty = bars + 11; // [2]
	uint64_t* p_full = bars + 13;
	uint64_t* pv_done = bars + 14;
	uint64_t* mma_done = bars + 16;
	uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
	volatile int* flags = reinterpret_cast<volatile int*>(bars + 18); // [0] abort

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	// the heaviest query tiles (the longest causal spans) go first
	const int h = blockIdx.x % P.n_head;
	const int qt = P.q_tiles - 1 - blockIdx.x / P.n_head;
	const int q0 = qt * PF_BM;
	const int qlo = P.pos0 + q0, qhi = P.pos0 + min(P.n_tok, q0 + PF_BM) - 1;
	const int klo = (P.window > 0 && qlo + 1 > P.window) ? qlo + 1 - P.window : 0;
	const int khi = min(qhi, P.n_seq - 1);
	const int j_lo = klo / PF_BN, n_tiles = khi / PF_BN - j_lo + 1;
	const int hk = h / (P.n_head / P.n_kv);

	if (threadIdx.x == 0)
	{
		mbar_init(q_full, 1);
		for (int s = 0; s < 2; ++s)
		{
			mbar_init(&k_full[s], 1);
			mbar_init(&k_empty[s], 1);
			mbar_init(&v_full[s], 1);
			mbar_init(&v_empty[s], 1);
			mbar_init(&s_full[s], 1);
			mbar_init(&s_empty[s], 128 * PF_NH);
		}
		mbar_init(p_full, 128 * PF_NH);
		mbar_init(pv_done, 1);
		mbar_init(mma_done, 1);
		flags[0] = 0;
		fence_barrier_init();
	}
	if (warp == 1)
	{
		asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
		             "r"(TMEM_COLS)
		             : "memory");
		asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tmem_slot;
	const uint32_t TS[2] = {tmem, tmem + 128};
	const uint32_t TO = tmem + 256;

	if (warp == 0 || warp == 2)
	{
		// ---- TMA: warp 0 Q once, then the K tiles; warp 2 the V tiles; each
		// through its own 2-stage ring (K is free again as soon as S is done) ----
		if (lane == 0)
		{
			const bool is_k = warp == 0;
			const CUtensorMap* map = is_k ? &kmap : &vmap;
			uint64_t* full = is_k ? k_full : v_full;
			uint64_t* empty = is_k ? k_empty : v_empty;
			unsigned char* ring = smem + (is_k ? SM_K : SM_V);
			if (is_k)
			{
				mbar_arrive_expect_tx(q_full, TILE);
				tma3(smem + SM_Q, &qmap, 0, q0, h, q_full);
				tma3(smem + SM_Q + PANEL, &qmap, 64, q0, h, q_full);
			}
			int issued = 0;
			for (int jj = 0; jj < n_tiles; ++jj)
			{
				const int s = jj & 1;
				if (jj >= 2 &&
				    !mbar_wait_bounded(&empty[s], (uint32_t)(((jj >> 1) - 1) & 1), P.err, DEVERR_WAIT_EMPTY))
				{
					flags[0] = 1;
					break;
				}
				if (flags[0]) break;
				unsigned char* t = ring + s * TILE;
				const int key0 = (j_lo + jj) * PF_BN;
				mbar_arrive_expect_tx(&full[s], TILE);
				tma3(t, map, 0, key0, hk, &full[s]);
				tma3(t + PANEL, map, 64, key0, hk, &full[s]);
				issued = jj + 1;
			}
			// on an abort, do not leave while a copy may still land here
			if (is_k) mbar_wait_bounded(q_full, 0, nullptr, 0);
			for (int jj = max(0, issued - 2); jj < issued; ++jj)
				mbar_wait_bounded(&full[jj & 1], (uint32_t)((jj >> 1) & 1), nullptr, 0);
		}
		__syncwarp(); // the whole warp meets the final barrier together
	}
	else if (warp == 1)
	{
		// ---- MMA issue: S_j = Q K_j^T into S[j % 2], then O += P_{j-1} V_{j-1} ----
		if (lane == 0)
		{
			constexpr uint32_t ID_QK = idesc(false), ID_PV = idesc(true);
			const uint32_t qa = smem_u32(smem + SM_Q), pa0 = smem_u32(smem + SM_P);
			bool ok = mbar_wait_bounded(q_full, 0, P.err, DEVERR_WAIT_FULL);
			auto issue_pv = [&](int jj) -> bool {
				if (!mbar_wait_bounded(p_full, (uint32_t)(jj & 1), P.err, DEVERR_WAIT_FULL) ||
				    !mbar_wait_bounded(&v_full[jj & 1], (uint32_t)((jj >> 1) & 1), P.err, DEVERR_WAIT_FULL))
					return false;
				tc_fence_after();
				const uint32_t va = smem_u32(smem + SM_V + (jj & 1) * TILE);
				const uint32_t pa = pa0;
#pragma unroll
				for (int k = 0; k < PF_BN / 16; ++k)
					mma_f16(TO, sdesc(pa + (k >> 2) * PANEL + (k & 3) * 32, 16, 1024), sdesc(va + k * 2048, PANEL, 1024),
					        ID_PV, (jj > 0 || k > 0) ? 1u : 0u);
				mma_commit(pv_done);
				mma_commit(&v_empty[jj & 1]);
				return true;
			};
			int jj = 0;
			for (; ok && jj < n_tiles; ++jj)
			{
				const int s = jj & 1;
				ok = !flags[0] && mbar_wait_bounded(&k_full[s], (uint32_t)((jj >> 1) & 1), P.err, DEVERR_WAIT_FULL);
				if (ok && jj >= 2)
					ok = mbar_wait_bounded(&s_empty[s], (uint32_t)(((jj >> 1) - 1) & 1), P.err, DEVERR_WAIT_EMPTY);
				if (!ok) break;
				tc_fence_after();
				const uint32_t ka = smem_u32(smem + SM_K + s * TILE);
#pragma unroll
				for (int k = 0; k < PF_D / 16; ++k)
					mma_f16(TS[s], sdesc(qa + (k >> 2) * PANEL + (k & 3) * 32, 16, 1024),
					        sdesc(ka + (k >> 2) * PANEL + (k & 3) * 32, 16, 1024), ID_QK, k > 0 ? 1u : 0u);
				mma_commit(&s_full[s]);
				mma_commit(&k_empty[s]);
				if (jj >= 1) ok = issue_pv(jj - 1);
			}
			if (ok && n_tiles > 0) ok = issue_pv(n_tiles - 1);
			if (!ok) flags[0] = 1;
			// every MMA issued has completed before TMEM is freed
			mma_commit(mma_done);
			mbar_wait_bounded(mma_done, 0, nullptr, 0);
		}
		__syncwarp(); // the whole warp meets the final barrier together
	}
	else if (warp >= 4)
	{
		// ---- softmax, O in scale, output: PF_NH threads per query row (warp
		// 4 + 4 part + lane group takes columns [32 part, 32 part + 32); a warp
		// reaches TMEM lanes 32 (warp % 4) .. +31), the row maximum shared
		// through shared memory by the warps on the same lanes ----
		const int wq = warp & 3;
		const int hf = (warp >> 2) - 1; // column part
		const int r = wq * 32 + lane;
		const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
		const uint32_t col0 = (uint32_t)(hf * PF_CW);
		const int qp = P.pos0 + q0 + r;
		const int kf = (P.window > 0 && qp + 1 > P.window) ? qp + 1 - P.window : 0;
		const int kl = min(qp, P.n_seq - 1);
		float* red = reinterpret_cast<float*>(smem + SM_RED); // maxima [2][PF_NH][128], then sums [PF_NH][128]
		float m_used = -CUDART_INF_F, l = 0.0f;
		bool ok = true;
		// this thread's 32 columns: 4 chunks of 8 in its row of panel hf / 2
		unsigned char* prow = smem + SM_P + (hf >> 1) * PANEL + r * 128;
		for (int jj = 0; jj < n_tiles; ++jj)
		{
			const int s = jj & 1;
			if (ok) ok = !flags[0] && mbar_wait_bounded(&s_full[s], (uint32_t)((jj >> 1) & 1), P.err, DEVERR_WAIT_FULL);
			ok = __all_sync(0xffffffffu, ok); // (the warps on these lanes leave together, at the barrier below)
			tc_fence_after();
			float x[PF_CW];
			tmem_ld32(TS[s] + lane_off + col0, x);
			tmem_wait_ld();
			tc_fence_before();
			mbar_arrive(&s_empty[s]);
			const int key0 = (j_lo + jj) * PF_BN + hf * PF_CW;
			// scores in log2 units: sl * s, folded into the exponentials' FMA
			// (sl > 0 keeps the maximum's place); with a soft-cap, capped first
			// in their own loop (a select would evaluate tanh for every score)
			float sl = P.scale * P.log2e;
			if (P.softcap > 0.0f)
			{
				const float cs = P.scale / P.softcap, cl = P.softcap * P.log2e;
#pragma unroll
				for (int c = 0; c < PF_CW; ++c) x[c] = tanhf(x[c] * cs) * cl;
				sl = 1.0f;
			}
			if (key0 < kf || key0 + PF_CW - 1 > kl)
			{
#pragma unroll
				for (int c = 0; c < PF_CW; ++c)
					if (key0 + c < kf || key0 + c > kl) x[c] = -CUDART_INF_F;
			}
			float mq[4] = {-CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F, -CUDART_INF_F}; // four chains
#pragma unroll
			for (int c = 0; c < PF_CW; ++c) mq[c & 3] = fmaxf(mq[c & 3], x[c]);
			float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3])) * sl;
			float* mxs = red + s * PF_NH * 128;
			mxs[hf * 128 + r] = mx;
			// the warps on these TMEM lanes; a timed-out wait in any of them ends
			// the loop for all of them
			if (named_sync_or(2 + wq, 32 * PF_NH, !ok))
			{
				ok = false;
				break;
			}
#pragma unroll
			for (int o = 1; o < PF_NH; ++o) mx = fmaxf(mx, mxs[((hf + o) % PF_NH) * 128 + r]);
			// the row's reference maximum moves only when a score exceeds it by
			// more than 2^LAZY; then O (in TMEM) and l are rescaled
			const bool move = mx > m_used + LAZY;
			const float m_new = move ? mx : m_used;
			const float alpha = (move && m_used != -CUDART_INF_F) ? ex2(m_used - m_new) : 1.0f;
			const bool rescale = move && m_used != -CUDART_INF_F;
			const float m_ref = m_new == -CUDART_INF_F ? 0.0f : m_new; // a row with no key yet: all p are 0
			// the weights and their bf16 pairs, in registers first, then into the
			// P tile once the previous P V has read it
			uint32_t pk[PF_CW / 2];
			float ls[4] = {0.0f, 0.0f, 0.0f, 0.0f};
			const float nm = -m_ref;
#pragma unroll
			for (int c = 0; c < PF_CW; c += 2)
			{
				const float p0 = ex2(fmaf(x[c], sl, nm)), p1 = ex2(fmaf(x[c + 1], sl, nm)); // masked (-inf): 0
				ls[(c >> 1) & 3] += p0 + p1;
				__nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
				pk[c >> 1] = *reinterpret_cast<uint32_t*>(&b2);
			}
			if (jj > 0)
			{
				ok = mbar_wait_bounded(pv_done, (uint32_t)((jj - 1) & 1), P.err, DEVERR_WAIT_FULL);
				ok = __all_sync(0xffffffffu, ok); // (a failure ends the loop at the next barrier)
				tc_fence_after();
				if (ok && __any_sync(0xffffffffu, rescale))
				{
					float o[32];
					tmem_ld32(TO + lane_off + col0, o);
					tmem_wait_ld();
#pragma unroll
					for (int i = 0; i < 32; ++i) o[i] *= alpha;
					tmem_st32(TO + lane_off + col0, o);
					tmem_wait_st();
				}
			}
#pragma unroll
			for (int c4 = 0; c4 < PF_CW / 8; ++c4)
			{
				const int chunk = ((hf & 1) * (PF_CW / 8) + c4) ^ (r & 7);
				*reinterpret_cast<uint4*>(prow + chunk * 16) =
					make_uint4(pk[4 * c4], pk[4 * c4 + 1], pk[4 * c4 + 2], pk[4 * c4 + 3]);
			}
			l = fmaf(l, alpha, (ls[0] + ls[1]) + (ls[2] + ls[3]));
			m_used = m_new;
			asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
			tc_fence_before();
			mbar_arrive(p_full);
		}
		// the output: O / l, once the last P V is done (l: the parts' sums)
		if (ok && n_tiles > 0) ok = mbar_wait_bounded(pv_done, (uint32_t)((n_tiles - 1) & 1), P.err, DEVERR_WAIT_FULL);
		ok = __all_sync(0xffffffffu, ok);
		float* sums = red + 2 * PF_NH * 128;
		sums[hf * 128 + r] = l;
		named_sync(2 + wq, 32 * PF_NH);
#pragma unroll
		for (int o = 1; o < PF_NH; ++o) l += sums[((hf + o) % PF_NH) * 128 + r];
		if (ok)
		{
			tc_fence_after();
			const float inv = l > 0.0f ? 1.0f / l : 0.0f;
			float o[32];
			tmem_ld32(TO + lane_off + col0, o);
			tmem_wait_ld();
			if (q0 + r < P.n_tok)
			{
				const size_t orow0 = ((size_t)(q0 + r) * P.n_head + h) * PF_D + col0;
				float* orow = P.out + orow0;
#pragma unroll
				for (int i = 0; i < 32; i += 4)
					*reinterpret_cast<float4*>(orow + i) =
						gated4(make_float4(o[i] * inv, o[i + 1] * inv, o[i + 2] * inv, o[i + 3] * inv), P.gate, orow0 + i);
			}
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 1)
	{
		tc_fence_after();
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
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
	__shared__ float s_qg[PF_D], s_kg[PF_D], s_cs[PF_D / 2], s_sn[PF_D / 2];
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
	// a head vector in registers, element lane + 32 i in v[i]; the warp's
	// next vector is loaded while this one is worked on
	float v[PF_D / 32], vn[PF_D / 32];
	auto load = [&](float* dst, int task) {
		const float* src = src_of(task);
#pragma unroll
		for (int i = 0; i < PF_D / 32; ++i) dst[i] = src[lane + 32 * i];
	};
	if (warp < n_tasks) load(v, warp);
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
	// NEOX pairs elements e and e + n_rot/2: the same lane when n_rot/2 is a
	// multiple of 32; NORM pairs e and e ^ 1: neighbouring lanes
	const bool neox = j.rope_mode == 0;
	const int row = pos % j.rows;
	for (int task = warp; task < n_tasks; task += 8)
	{
		if (task + 8 < n_tasks) load(vn, task + 8);
		const bool is_q = task < n_head, is_k = !is_q && task - n_head < n_kv;
		const float* gamma = is_q ? (j.q_gamma ? s_qg : nullptr) : (is_k && j.k_gamma ? s_kg : nullptr);
		const bool plain = !is_q && !is_k && j.v_rmsnorm;
		if (gamma || plain)
		{
			// RMSNorm as rms_scale does: squares in fp32, the scale in double
			float ss = 0.0f;
#pragma unroll
			for (int i = 0; i < PF_D / 32; ++i) ss = fmaf(v[i], v[i], ss);
			ss = warp_sum(ss);
			const double mean = gamma ? (double)ss * (double)(1.0f / (float)PF_D) : (double)ss / (double)PF_D;
			const float sc = (float)(1.0 / sqrt(mean + (double)j.eps));
#pragma unroll
			for (int i = 0; i < PF_D / 32; ++i) v[i] = gamma ? v[i] * sc * gamma[lane + 32 * i] : v[i] * sc;
		}
		if ((is_q || is_k) && half > 0)
		{
			if (neox)
			{
				// half is 32 or 64 here (a multiple of 32, checked on the host)
				auto rot = [&](float& a_, float& b_, int e) {
					const float a = a_, b = b_;
					a_ = s_cs[e] * a - s_sn[e] * b;
					b_ = s_sn[e] * a + s_cs[e] * b;
				};
				if (half == 64)
				{
					rot(v[0], v[2], lane);
					rot(v[1], v[3], lane + 32);
				}
				else
					rot(v[0], v[1], lane);
			}
			else
			{
#pragma unroll
				for (int i = 0; i < PF_D / 32; ++i)
				{
					const int e = lane + 32 * i;
					const float other = __shfl_xor_sync(0xffffffffu, v[i], 1);
					if (e < j.n_rot)
					{
						const float cs = s_cs[e >> 1], sn = s_sn[e >> 1];
						v[i] = (lane & 1) ? sn * other + cs * v[i] : cs * v[i] - sn * other;
					}
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
		// rounded to bf16 on the integer pipe (the conversion instruction would
		// queue on the transcendental unit)
#pragma unroll
		for (int i = 0; i < PF_D / 32; ++i)
		{
			reinterpret_cast<uint16_t*>(dst)[lane + 32 * i] = (uint16_t)bf16_rne_bits(v[i]);
			v[i] = vn[i];
		}
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
	if (!e) e = make_map(&kmap, j.K, (uint64_t)j.rows, (uint64_t)j.n_kv);
	if (!e) e = make_map(&vmap, j.V, (uint64_t)j.rows, (uint64_t)j.n_kv);
	if (e) return e;
	cudaError_t ce;
	static bool configured[64] = {};
	int dev = 0;
	cudaGetDevice(&dev);
	if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
	if (!configured[dev])
	{
		ce = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_SMEM);
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
	P.q_tiles = (j.n_tok + PF_BM - 1) / PF_BM;
	P.scale = j.scale;
	P.log2e = 1.4426950408889634f;
	P.softcap = j.softcap;
	P.out = j.out;
	P.gate = j.gate;
	P.err = err;
	prefill_kernel<<<(unsigned)(P.q_tiles * j.n_head), PF_THREADS, PF_SMEM, st>>>(qmap, kmap, vmap, P);
	return (int)cudaGetLastError();
}

} // namespace nncu
