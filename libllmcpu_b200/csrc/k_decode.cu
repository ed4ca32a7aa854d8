// k_decode.cu -- K2 + K3: attention of a few query rows per KV head over the
// HBM K/V cache, for decode (1 token) and speculative verify (a few tokens).
//
// It replaces libnnc's blocked attention (nnc_attn_block / nnc_attn_merge /
// nnc_attn_finish, src/libnnc/nn_ops.cpp:351-499) and its dispatch
// (attend_token / attend_blocks, src/libnnc/model.cpp:1251-1319, 1696-1749).
// The same algorithm, laid out for the GPU:
//
//  * Work unit. A segment is one (job, KV head, group of RM query rows): the
//    query heads that share a KV head, times the job's tokens, read that KV
//    head's keys together, as the reference's group of heads does. Its keys
//    are the union of the rows' spans, cut into tiles of T keys aligned to
//    absolute positions (T divides 256, so a tile never straddles a ring's
//    end); a row ignores the keys outside its own span.
//  * Split. The tiles of all segments of the launch are concatenated and cut
//    into equal runs, one per CTA (stream-K). A segment that falls into
//    several runs is computed as several pieces, each giving a partial
//    (o, m, l) exactly like nnc_attn_block's; the CTA that finishes a
//    segment's last piece merges the pieces in key order (nnc_attn_merge)
//    and divides by l (nnc_attn_finish). No second launch.
//  * Memory. One producer warp streams each tile's K rows and V rows (one
//    contiguous run each in the head-major cache) into a 4-stage shared
//    memory ring with cp.async.bulk, completing on mbarriers; 8 consumer
//    warps compute while the next tiles are in flight.
//  * Math. fp32 throughout. A warp owns T/8 keys of each tile; its lanes
//    split head_dim (D/32 elements each). The q.k partial sums of a batch of
//    keys x rows are summed across lanes with a transposing reduction, the
//    online softmax runs in registers in base 2, and o accumulates in
//    registers. Warps merge their (o, m, l) in shared memory at piece end.
#include <cuda_runtime.h>

#include <math_constants.h>

#include "common.cuh"

namespace nncu
{
namespace
{

constexpr int NW = 8;          // consumer warps
constexpr int STAGES = 4;      // K/V tiles in flight per CTA
constexpr int TILE_BYTES = 16384;
constexpr float LOG2E = 1.4426950408889634f;

template <int D, typename KV, int RM>
struct Cfg
{
	static constexpr int E = D / 32;                       // elements per lane
	static constexpr int RS = RM * E > 32 ? RM * E / 32 : 1; // row slices: warps sharing keys, splitting rows
	static constexpr int RMW = RM / RS;                    // rows per warp
	static constexpr int NKG = NW / RS;                    // key groups
	static constexpr int T = TILE_BYTES / (D * KV::esize); // keys per tile
	static constexpr int KB = T / NKG;                     // keys per warp per tile
	static constexpr int KS = KB < 32 / RMW ? KB : 32 / RMW; // keys per reduction batch
	static constexpr int N = KS * RMW;                     // values per reduction
	static constexpr int LOG2N = N >= 32 ? 5 : N >= 16 ? 4 : N >= 8 ? 3 : N >= 4 ? 2 : N >= 2 ? 1 : 0;
	static constexpr int SHIFT = 5 - LOG2N;                // lane >> SHIFT = value index after the reduction
	static constexpr int LOG2RMW = RMW >= 32 ? 5 : RMW >= 16 ? 4 : RMW >= 8 ? 3 : RMW >= 4 ? 2 : RMW >= 2 ? 1 : 0;
	static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
	static constexpr int MERGE_FLOATS = NW * RMW * D + 2 * NW * RMW;
	static constexpr int SMEM = STAGES * STAGE_BYTES + MERGE_FLOATS * 4 + 2 * STAGES * 8 + 64;
	static_assert(D % 32 == 0, "D: a multiple of 32");
	static_assert(RM % RS == 0 && NW % RS == 0, "row slices");
	static_assert(T >= NKG && T <= ATTN_BLOCK && ATTN_BLOCK % T == 0 && T % NKG == 0, "tile keys");
	static_assert(KB % KS == 0, "batches per warp");
	static_assert(RMW * E <= 32, "accumulator registers");
};

// Where global tile g of the launch lies.
struct TileLoc
{
	int job;
	int seg_local;   // segment within the job: h * n_rowgroups + rg
	int tis;         // tile within the segment
};

struct JobCursor
{
	int j = -1;
	long long g0 = 0, g1 = 0; // global tiles of job j: [g0, g1)
	int n_tiles = 1;
};

__device__ __forceinline__ void locate(const DecodePlan& P, JobCursor& c, long long g, TileLoc& loc)
{
	if (c.j < 0 || g < c.g0 || g >= c.g1)
	{
		int lo = 0, hi = P.n_jobs - 1;
		while (lo < hi)
		{
			const int mid = (lo + hi + 1) >> 1;
			if (P.jobs[mid].gtile0 <= g) lo = mid;
			else hi = mid - 1;
		}
		// skip jobs with no tiles that share the same gtile0
		while (lo + 1 < P.n_jobs && P.jobs[lo + 1].gtile0 <= g) ++lo;
		const DevJob& J = P.jobs[lo];
		c.j = lo;
		c.g0 = J.gtile0;
		c.n_tiles = J.n_tiles;
		c.g1 = J.gtile0 + (long long)J.n_kv * J.n_rowgroups * J.n_tiles;
	}
	const long long local = g - c.g0;
	loc.job = c.j;
	loc.seg_local = (int)(local / c.n_tiles);
	loc.tis = (int)(local % c.n_tiles);
}

template <int D, typename KV, int RM>
__global__ void __launch_bounds__((NW + 1) * 32, 1) decode_kernel(const DecodePlan P)
{
	using C = Cfg<D, KV, RM>;
	using T_ = typename KV::T;
	constexpr int E = C::E, T = C::T, KB = C::KB, KS = C::KS, N = C::N, SHIFT = C::SHIFT;
	constexpr int VEC = LaneVec<E, KV::esize>::VEC; // lane <-> element mapping of K, V, q and o

	extern __shared__ __align__(1024) unsigned char smem[];
	unsigned char* stages = smem;
	float* m_s = reinterpret_cast<float*>(smem + STAGES * C::STAGE_BYTES); // [NW][RMW]
	float* l_s = m_s + NW * C::RMW;                                        // [NW][RMW]
	float* o_s = l_s + NW * C::RMW;                                        // [NW][RMW][D]
	uint64_t* full = reinterpret_cast<uint64_t*>(o_s + NW * C::RMW * D);
	uint64_t* empty = full + STAGES;
	volatile int* s_flags = reinterpret_cast<volatile int*>(empty + STAGES); // [0] abort, [1] last-piece vote

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const long long g_begin = (long long)blockIdx.x * P.tiles_per_cta;
	const long long g_end = min(g_begin + P.tiles_per_cta, P.total_tiles);

	if (threadIdx.x == 0)
	{
		for (int s = 0; s < STAGES; ++s)
		{
			mbar_init(&full[s], 1);
			mbar_init(&empty[s], NW);
		}
		s_flags[0] = 0;
		s_flags[1] = 0;
		fence_barrier_init();
	}
	__syncthreads();

	if (warp == NW)
	{
		// ---- producer: one lane streams the CTA's tiles into the stage ring ----
		if (lane == 0)
		{
			JobCursor cur;
			TileLoc loc;
			long long i = 0;
			for (long long g = g_begin; g < g_end; ++g, ++i)
			{
				locate(P, cur, g, loc);
				const DevJob& J = P.jobs[loc.job];
				const int h = loc.seg_local / J.n_rowgroups;
				const long long key0 = (long long)(J.tile_lo + loc.tis) * T;
				const size_t row0 = (size_t)(key0 % J.rows);
				const size_t off = (size_t)h * J.head_bytes + row0 * D * KV::esize;
				const int s = (int)(i % STAGES);
				if (i >= STAGES && !mbar_wait_bounded(&empty[s], (uint32_t)(((i / STAGES) - 1) & 1), P.err,
				                                      DEVERR_WAIT_EMPTY))
				{
					s_flags[0] = 1;
					break;
				}
				if (s_flags[0]) break;
				unsigned char* st = stages + s * C::STAGE_BYTES;
				mbar_arrive_expect_tx(&full[s], 2 * TILE_BYTES);
				bulk_g2s(st, J.K + off, TILE_BYTES, &full[s]);
				bulk_g2s(st + TILE_BYTES, J.V + off, TILE_BYTES, &full[s]);
			}
		}
		return;
	}

	// ---- consumers ----
	// Warp w takes rows [rs*RMW, rs*RMW + RMW) of the segment (rs = w % RS)
	// for the keys [kg*KB, kg*KB + KB) of every tile (kg = w / RS).
	constexpr int RS = C::RS, RMW = C::RMW;
	const int ctid = threadIdx.x; // 0 .. NW*32-1
	const int rs = warp % RS, kg = warp / RS;
	const int r_v = (lane >> SHIFT) % RMW;  // the row (within the warp's rows) of this lane's reduced value
	const int kk_v = (lane >> SHIFT) / RMW; // its key within the batch

	float q[RMW][E];
	float o[RMW][E];
	float m[RMW];
	float l_lane = 0.0f;
	int first_v = 0, last_v = -1; // this lane's row span
	bool softcap = false;
	float cap = 0.0f;

	JobCursor cur;
	TileLoc loc;
	int cur_job = -1, cur_seg = -1;
	long long piece_g0 = 0; // first global tile of the current segment

	auto start_piece = [&](const DevJob& J, int seg_local) {
		const int G = J.n_head / J.n_kv;
		const int h = seg_local / J.n_rowgroups, rg = seg_local % J.n_rowgroups;
		softcap = J.softcap > 0.0f;
		cap = J.softcap;
		const float qmul = softcap ? J.scale : J.scale * LOG2E;
#pragma unroll
		for (int r = 0; r < RMW; ++r)
		{
			const int gr = rg * RM + rs * RMW + r;
			const bool ok = gr < G * J.n_tok;
			const int t = ok ? gr / G : 0, g = ok ? gr % G : 0;
			const float* src = J.q_rot + ((size_t)t * J.n_head + (size_t)h * G + g) * D;
			float tmp[E];
			if (ok) load_lane_f<E, VEC>(src, lane, tmp);
#pragma unroll
			for (int e = 0; e < E; ++e)
			{
				q[r][e] = ok ? tmp[e] * qmul : 0.0f;
				o[r][e] = 0.0f;
			}
			m[r] = -CUDART_INF_F;
		}
		l_lane = 0.0f;
		const int gr_v = rg * RM + rs * RMW + r_v;
		if (gr_v < G * J.n_tok)
			span_of(J.causal, J.window, J.pos0 + gr_v / G, J.n_seq, first_v, last_v);
		else
			first_v = 0, last_v = -1; // a padding row sees nothing
	};

	// Merge the warps' states of the finished piece; write the output (whole
	// segment in this CTA) or a partial, and fold the partials if this CTA
	// completes the segment.
	auto finish_piece = [&](const DevJob& J, int seg_local, long long seg_gstart) {
		// l of row r: sum over the batch's key slots (lanes differing in the key bits)
		float lsum = l_lane;
#pragma unroll
		for (int off = 1 << (SHIFT + C::LOG2RMW); off < 32; off <<= 1)
			lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
#pragma unroll
		for (int r = 0; r < RMW; ++r)
		{
#pragma unroll
			for (int e = 0; e < E; ++e) o_s[(warp * RMW + r) * D + lane_elem<E, VEC>(lane, e)] = o[r][e];
			if (lane == (r << SHIFT))
			{
				m_s[warp * RMW + r] = m[r];
				l_s[warp * RMW + r] = lsum;
			}
		}
		named_sync(1, NW * 32);

		const int G = J.n_head / J.n_kv;
		const int h = seg_local / J.n_rowgroups, rg = seg_local % J.n_rowgroups;
		const long long W = P.tiles_per_cta;
		const long long seg_gend = seg_gstart + J.n_tiles;
		const int c_first = (int)(seg_gstart / W), c_last = (int)((seg_gend - 1) / W);
		const bool single = c_first == c_last;
		const int seg = J.seg0 + seg_local;
		float* part = P.parts + (size_t)(seg + (int)blockIdx.x) * RM * (D + 2);

		for (int idx = ctid; idx < RM * D; idx += NW * 32)
		{
			const int R = idx / D, d = idx % D;
			const int sl = R / RMW, r = R % RMW; // the row's slice and its row within the slice
			float M = -CUDART_INF_F;
#pragma unroll
			for (int k = 0; k < C::NKG; ++k) M = fmaxf(M, m_s[(k * RS + sl) * RMW + r]);
			float acc = 0.0f, L = 0.0f;
#pragma unroll
			for (int k = 0; k < C::NKG; ++k)
			{
				const int w = k * RS + sl;
				const float mw = m_s[w * RMW + r];
				const float c = mw == -CUDART_INF_F ? 0.0f : ex2(mw - M);
				acc = fmaf(o_s[(w * RMW + r) * D + d], c, acc);
				L = fmaf(l_s[w * RMW + r], c, L);
			}
			if (single)
			{
				const int gr = rg * RM + R;
				if (gr < G * J.n_tok)
				{
					const int t = gr / G, g = gr % G;
					J.out[((size_t)t * J.n_head + (size_t)h * G + g) * D + d] = L > 0.0f ? acc / L : 0.0f;
				}
			}
			else
			{
				part[R * (D + 2) + d] = acc;
				if (d == 0)
				{
					part[R * (D + 2) + D] = M;
					part[R * (D + 2) + D + 1] = L;
				}
			}
		}
		if (!single)
		{
			__threadfence();
			named_sync(1, NW * 32);
			if (ctid == 0)
			{
				const int n_pieces = c_last - c_first + 1;
				const int prev = atomicAdd(&P.counters[seg], 1);
				s_flags[1] = prev == n_pieces - 1;
			}
			named_sync(1, NW * 32);
			if (s_flags[1])
			{
				__threadfence();
				// fold the pieces in key order: merge (o, m, l), then o / l
				for (int idx = ctid; idx < RM * D; idx += NW * 32)
				{
					const int R = idx / D, d = idx % D;
					const int gr = rg * RM + R;
					if (gr >= G * J.n_tok) continue;
					float M = -CUDART_INF_F;
					for (int c = c_first; c <= c_last; ++c)
						M = fmaxf(M, __ldcg(P.parts + (size_t)(seg + c) * RM * (D + 2) + R * (D + 2) + D));
					float acc = 0.0f, L = 0.0f;
					for (int c = c_first; c <= c_last; ++c)
					{
						const float* pc = P.parts + (size_t)(seg + c) * RM * (D + 2) + R * (D + 2);
						const float mc = __ldcg(pc + D);
						const float w = mc == -CUDART_INF_F ? 0.0f : ex2(mc - M);
						acc = fmaf(__ldcg(pc + d), w, acc);
						L = fmaf(__ldcg(pc + D + 1), w, L);
					}
					const int t = gr / G, g = gr % G;
					J.out[((size_t)t * J.n_head + (size_t)h * G + g) * D + d] = L > 0.0f ? acc / L : 0.0f;
				}
				if (ctid == 0) P.counters[seg] = 0; // ready for the next launch
			}
		}
		named_sync(1, NW * 32); // the merge area is free again
	};

	long long i = 0;
	for (long long g = g_begin; g < g_end; ++g, ++i)
	{
		locate(P, cur, g, loc);
		const DevJob& J = P.jobs[loc.job];
		if (loc.job != cur_job || loc.seg_local != cur_seg)
		{
			if (cur_job >= 0) finish_piece(P.jobs[cur_job], cur_seg, piece_g0);
			cur_job = loc.job;
			cur_seg = loc.seg_local;
			piece_g0 = J.gtile0 + (long long)loc.seg_local * J.n_tiles;
			start_piece(J, loc.seg_local);
		}
		const int s = (int)(i % STAGES);
		// After a timed-out wait the CTA stops waiting (fail fast) but keeps
		// stepping through its tiles, so every consumer warp still meets the
		// same named barriers; the error word tells the host the result is void.
		if (!s_flags[0] && !mbar_wait_bounded(&full[s], (uint32_t)((i / STAGES) & 1), P.err, DEVERR_WAIT_FULL))
			s_flags[0] = 1;
		if (s_flags[0])
		{
			__syncwarp();
			continue;
		}
		const T_* Kt = reinterpret_cast<const T_*>(stages + s * C::STAGE_BYTES);
		const T_* Vt = reinterpret_cast<const T_*>(stages + s * C::STAGE_BYTES + TILE_BYTES);
		const int key_base = (J.tile_lo + loc.tis) * T; // absolute position of the tile's first key

#pragma unroll
		for (int b = 0; b < KB / KS; ++b)
		{
			const int k0 = kg * KB + b * KS; // key index within the tile
			// scores of KS keys x RMW rows: lane-partial dot products, then reduced
			float part[N];
#pragma unroll
			for (int kk = 0; kk < KS; ++kk)
			{
				float kv[E];
				load_lane<E>(Kt + (size_t)(k0 + kk) * D, lane, kv);
#pragma unroll
				for (int r = 0; r < RMW; ++r)
				{
					float acc = 0.0f;
#pragma unroll
					for (int e = 0; e < E; ++e) acc = fmaf(q[r][e], kv[e], acc);
					part[kk * RMW + r] = acc;
				}
			}
			float sv = transpose_reduce<N>(part, lane);
			const int pos = key_base + k0 + kk_v;
			if (softcap) sv = cap * tanhf(sv / cap) * LOG2E;
			if (pos < first_v || pos > last_v) sv = -CUDART_INF_F;
			// the batch's max of each row, then the new running max of every row
			float mx = sv;
#pragma unroll
			for (int off = 1 << (SHIFT + C::LOG2RMW); off < 32; off <<= 1)
				mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
			float alpha[RMW];
#pragma unroll
			for (int r = 0; r < RMW; ++r)
			{
				const float mn = fmaxf(m[r], __shfl_sync(0xffffffffu, mx, r << SHIFT));
				alpha[r] = mn == -CUDART_INF_F ? 1.0f : ex2(m[r] - mn);
				m[r] = mn;
			}
			const float pv = sv == -CUDART_INF_F ? 0.0f : ex2(sv - m[r_v]);
			l_lane = fmaf(l_lane, alpha[r_v], pv);
#pragma unroll
			for (int r = 0; r < RMW; ++r)
#pragma unroll
				for (int e = 0; e < E; ++e) o[r][e] *= alpha[r];
			// o += p v over the batch's keys
#pragma unroll
			for (int kk = 0; kk < KS; ++kk)
			{
				float vv[E];
				load_lane<E>(Vt + (size_t)(k0 + kk) * D, lane, vv);
#pragma unroll
				for (int r = 0; r < RMW; ++r)
				{
					const float p = __shfl_sync(0xffffffffu, pv, (kk * RMW + r) << SHIFT);
#pragma unroll
					for (int e = 0; e < E; ++e) o[r][e] = fmaf(p, vv[e], o[r][e]);
				}
			}
		}
		__syncwarp();
		if (lane == 0) mbar_arrive(&empty[s]);
	}
	if (cur_job >= 0) finish_piece(P.jobs[cur_job], cur_seg, piece_g0);
	if (s_flags[0] && ctid == 0)
	{
		// Do not leave while a copy issued into this CTA's shared memory may
		// still land: wait (bounded again) for every stage's last phase.
		const long long n = g_end - g_begin;
		for (long long k = n > STAGES ? n - STAGES : 0; k < n; ++k)
			mbar_wait_bounded(&full[k % STAGES], (uint32_t)((k / STAGES) & 1), nullptr, 0);
	}
}

// ---- unit seam: nnc_attn_block / merge / finish on device pointers ---------------

// One block of keys for n_heads query heads, any head_dim up to 512 and any
// kv_stride. A CTA per head; its warps take keys in turn with their own
// online softmax, merged at the end. Partial layout and meaning as
// nnc_attn_block's: o (relative to m), m (natural log units), l.
template <typename KV>
__global__ void attn_block_kernel(const float* q, size_t q_stride, const void* Kp, const void* Vp, size_t kv_stride,
                                  size_t n_keys, int hd, float scale, float cap, float* part)
{
	using T_ = typename KV::T;
	constexpr int MAXE = 16;
	__shared__ float sm_m[8], sm_l[8];
	__shared__ float sm_o[8][512];
	const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const float* qh = q + (size_t)h * q_stride;
	const T_* K = static_cast<const T_*>(Kp);
	const T_* V = static_cast<const T_*>(Vp);
	float qr[MAXE], o[MAXE];
#pragma unroll
	for (int e = 0; e < MAXE; ++e)
	{
		const int i = lane + 32 * e;
		qr[e] = i < hd ? qh[i] : 0.0f;
		o[e] = 0.0f;
	}
	float m = -CUDART_INF_F, l = 0.0f;
	for (size_t t = warp; t < n_keys; t += 8)
	{
		float s = 0.0f;
#pragma unroll
		for (int e = 0; e < MAXE; ++e)
		{
			const int i = lane + 32 * e;
			if (i < hd) s = fmaf(qr[e], load_elem(K + t * kv_stride + i), s);
		}
		s = warp_sum(s) * scale;
		if (cap > 0.0f) s = tanhf(s * (1.0f / cap)) * cap;
		const float mn = fmaxf(m, s);
		const float a = m == -CUDART_INF_F ? 0.0f : expf(m - mn);
		const float p = expf(s - mn);
		l = l * a + p;
#pragma unroll
		for (int e = 0; e < MAXE; ++e)
		{
			const int i = lane + 32 * e;
			if (i < hd) o[e] = fmaf(p, load_elem(V + t * kv_stride + i), o[e] * a);
		}
		m = mn;
	}
	if (lane == 0)
	{
		sm_m[warp] = m;
		sm_l[warp] = l;
	}
#pragma unroll
	for (int e = 0; e < MAXE; ++e)
	{
		const int i = lane + 32 * e;
		if (i < hd) sm_o[warp][i] = o[e];
	}
	__syncthreads();
	float M = -CUDART_INF_F;
	for (int w = 0; w < 8; ++w) M = fmaxf(M, sm_m[w]);
	float* ph = part + (size_t)h * (hd + 2);
	for (int i = threadIdx.x; i < hd; i += blockDim.x)
	{
		float acc = 0.0f;
		for (int w = 0; w < 8; ++w)
			if (sm_m[w] != -CUDART_INF_F) acc = fmaf(sm_o[w][i], expf(sm_m[w] - M), acc);
		ph[i] = acc;
	}
	if (threadIdx.x == 0)
	{
		float L = 0.0f;
		for (int w = 0; w < 8; ++w)
			if (sm_m[w] != -CUDART_INF_F) L = fmaf(sm_l[w], expf(sm_m[w] - M), L);
		ph[hd] = M;
		ph[hd + 1] = L;
	}
}

__global__ void attn_merge_kernel(float* acc, const float* part, int hd, int n_heads)
{
	const int h = blockIdx.x;
	float* a = acc + (size_t)h * (hd + 2);
	const float* b = part + (size_t)h * (hd + 2);
	const float ma = a[hd], mb = b[hd];
	const float mx = fmaxf(ma, mb);
	const float ca = expf(ma - mx), cb = expf(mb - mx);
	for (int i = threadIdx.x; i < hd; i += blockDim.x) a[i] = fmaf(b[i], cb, a[i] * ca);
	__syncthreads();
	if (threadIdx.x == 0)
	{
		a[hd] = mx;
		a[hd + 1] = a[hd + 1] * ca + b[hd + 1] * cb;
	}
}

__global__ void attn_finish_kernel(float* out, size_t out_stride, const float* acc, int hd)
{
	const int h = blockIdx.x;
	const float* a = acc + (size_t)h * (hd + 2);
	const float l = a[hd + 1];
	const float inv = l > 0.0f ? 1.0f / l : 0.0f;
	for (int i = threadIdx.x; i < hd; i += blockDim.x) out[(size_t)h * out_stride + i] = a[i] * inv;
}

// ---- dispatch over (D, element type, rows) -----------------------------------------

template <int D, typename KV, int RM>
int launch_one(const DecodePlan& P, cudaStream_t st)
{
	using C = Cfg<D, KV, RM>;
	static bool configured = false;
	if (!configured)
	{
		cudaError_t e = cudaFuncSetAttribute(decode_kernel<D, KV, RM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
		                                     C::SMEM);
		if (e != cudaSuccess) return (int)e;
		configured = true;
	}
	decode_kernel<D, KV, RM><<<P.n_ctas, (NW + 1) * 32, C::SMEM, st>>>(P);
	return (int)cudaGetLastError();
}

template <int D, typename KV>
int launch_rows(const DecodePlan& P, cudaStream_t st)
{
	constexpr int E = D / 32;
	switch (P.RM)
	{
	case 1: return launch_one<D, KV, 1>(P, st);
	case 2: return launch_one<D, KV, 2>(P, st);
	case 4: return launch_one<D, KV, 4>(P, st);
	case 8:
		if constexpr (8 * E <= 64) return launch_one<D, KV, 8>(P, st);
		break;
	case 16:
		if constexpr (16 * E <= 64) return launch_one<D, KV, 16>(P, st);
		break;
	case 32:
		if constexpr (32 * E <= 64) return launch_one<D, KV, 32>(P, st);
		break;
	default: break;
	}
	return (int)cudaErrorInvalidValue;
}

template <typename KV>
int launch_dims(const DecodePlan& P, cudaStream_t st)
{
	switch (P.D)
	{
	case 64: return launch_rows<64, KV>(P, st);
	case 128: return launch_rows<128, KV>(P, st);
	case 256: return launch_rows<256, KV>(P, st);
	case 512: return launch_rows<512, KV>(P, st);
	default: return (int)cudaErrorInvalidValue;
	}
}

} // namespace

bool decode_supported(int D, int kv_type)
{
	(void)kv_type;
	return D == 64 || D == 128 || D == 256 || D == 512;
}

int decode_tile_keys(int D, int kv_type) { return TILE_BYTES / (D * kv_esize(kv_type)); }

int decode_rows_max(int D) { return 64 / (D / 32) < 32 ? 64 / (D / 32) : 32; }

int decode_smem_bytes(int D, int kv_type, int RM)
{
	(void)kv_type;
	const int E = D / 32, RS = RM * E > 32 ? RM * E / 32 : 1, RMW = RM / RS;
	return STAGES * 2 * TILE_BYTES + (NW * RMW * D + 2 * NW * RMW) * 4 + 2 * STAGES * 8 + 64;
}

int launch_decode(const DecodePlan& P, void* stream)
{
	if (P.total_tiles == 0) return 0;
	auto st = static_cast<cudaStream_t>(stream);
	switch (P.kv_type)
	{
	case KV_F32: return launch_dims<kv_f32>(P, st);
	case KV_BF16: return launch_dims<kv_bf16>(P, st);
	default: return launch_dims<kv_f16>(P, st);
	}
}

int launch_attn_block(const float* q, size_t q_stride, const void* K, const void* V, int kv_type, size_t kv_stride,
                      size_t n_keys, size_t head_dim, size_t n_heads, float scale, float softcap, float* part,
                      void* stream)
{
	if (head_dim == 0 || head_dim > 512) return (int)cudaErrorInvalidValue;
	if (n_heads == 0) return 0;
	auto st = static_cast<cudaStream_t>(stream);
	const int hd = (int)head_dim;
	switch (kv_type)
	{
	case KV_F32:
		attn_block_kernel<kv_f32><<<(unsigned)n_heads, 256, 0, st>>>(q, q_stride, K, V, kv_stride, n_keys, hd, scale,
		                                                               softcap, part);
		break;
	case KV_BF16:
		attn_block_kernel<kv_bf16><<<(unsigned)n_heads, 256, 0, st>>>(q, q_stride, K, V, kv_stride, n_keys, hd,
		                                                                scale, softcap, part);
		break;
	default:
		attn_block_kernel<kv_f16><<<(unsigned)n_heads, 256, 0, st>>>(q, q_stride, K, V, kv_stride, n_keys, hd, scale,
		                                                               softcap, part);
		break;
	}
	return (int)cudaGetLastError();
}

int launch_attn_merge(float* acc, const float* part, size_t head_dim, size_t n_heads, void* stream)
{
	if (n_heads == 0) return 0;
	attn_merge_kernel<<<(unsigned)n_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(acc, part, (int)head_dim,
	                                                                                   (int)n_heads);
	return (int)cudaGetLastError();
}

int launch_attn_finish(float* out, size_t out_stride, const float* acc, size_t head_dim, size_t n_heads,
                       void* stream)
{
	if (n_heads == 0) return 0;
	attn_finish_kernel<<<(unsigned)n_heads, 128, 0, static_cast<cudaStream_t>(stream)>>>(out, out_stride, acc,
	                                                                                    (int)head_dim);
	return (int)cudaGetLastError();
}

} // namespace nncu
