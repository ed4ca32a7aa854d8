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
//    contiguous 32 KB run each in the head-major cache) into a 3-stage shared
//    memory ring with cp.async.bulk, completing on mbarriers; 8 consumer
//    warps compute while the next tiles are in flight. Each piece's q rows
//    come the same way, into one of two q slots, ahead of the piece's tiles,
//    so no consumer ever waits on a plain global load behind the tile stream.
//  * Order. The kernel is a programmatic dependent of K1 (k_prep.cu): its
//    CTAs become resident while K1 runs, and the producer starts streaming as
//    soon as K1's q rows and appended K/V rows are complete.
//  * Math. fp32 throughout. A warp owns T/8 keys of each tile; its lanes
//    split head_dim (D/32 elements each). The q.k partial sums of a batch of
//    keys x rows are summed across lanes with a transposing reduction, the
//    online softmax runs in registers in base 2, and o accumulates in
//    registers. Warps merge their (o, m, l) in shared memory at piece end.
#include <cuda_runtime.h>

#include <math_constants.h>

#include <algorithm>

#include "common.cuh"

namespace nncu
{
namespace
{

constexpr int NW = 8;              // consumer warps
constexpr int MAX_STAGES = 4;      // K/V tiles in flight per CTA, as shared memory allows
constexpr int SMEM_LIMIT = 232448; // 227 KB of shared memory per CTA
constexpr int TILE_BYTES = 32768;  // one tile's K (or V) rows
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
	// the warps' (o, m, l) at a piece's end pass through two warps' worth of
	// area in a pairwise tree; the fold's weights reuse the same area
	static constexpr int AREA_FLOATS = 2 * RMW * D;
	// one piece's slot: its job descriptor, its tile count / first tile /
	// segment, its raw q rows, the q gains and the RoPE tables
	static constexpr int QHEAD_FLOATS = (int)(sizeof(DevJob) / 4) + 4;
	static constexpr int QROWS = QHEAD_FLOATS;             // RM * D
	static constexpr int QGAIN = QROWS + RM * D;           // D
	static constexpr int QINV = QGAIN + D;                 // D / 2
	static constexpr int QFF = QINV + D / 2;               // D / 2
	static constexpr int QSLOT_FLOATS = QFF + D / 2;
	static constexpr int FIXED_BYTES = (AREA_FLOATS + 2 * NW * RMW + 2 * QSLOT_FLOATS) * 4 + 256;
	static constexpr int FIT = (SMEM_LIMIT - FIXED_BYTES) / STAGE_BYTES;
	static constexpr int STAGES = FIT < MAX_STAGES ? FIT : MAX_STAGES;
	static constexpr int SMEM = STAGES * STAGE_BYTES + FIXED_BYTES;
	static_assert(STAGES >= 3, "shared memory for at least three stages");
	static_assert(D % 32 == 0, "D: a multiple of 32");
	static_assert(RM % RS == 0 && NW == 8 && RS <= 2, "row slices");
	static_assert(T >= NKG && T <= ATTN_BLOCK && ATTN_BLOCK % T == 0 && T % NKG == 0, "tile keys");
	static_assert(KB % KS == 0, "batches per warp");
	static_assert(RMW * E <= 32, "accumulator registers");
};

// The CTA's walk over its run of the launch's tiles: (job, segment within
// the job, tile within the segment), advanced one tile at a time.
struct Cursor
{
	int job = 0, seg = 0, tis = 0;
	int n_tiles = 1, n_segs = 1;
};

__device__ __forceinline__ void cursor_load(const DecodePlan& P, Cursor& c)
{
	const DevJob& J = P.jobs[c.job];
	c.n_tiles = J.n_tiles;
	c.n_segs = J.n_kv * J.n_rowgroups;
	if (c.job + 1 < P.n_jobs)
	{
		// the next job's descriptor into L1 ahead of the job change
		const char* nx = reinterpret_cast<const char*>(P.jobs + c.job + 1);
		for (int b = 0; b < (int)sizeof(DevJob); b += 128) asm volatile("prefetch.global.L1 [%0];" ::"l"(nx + b));
	}
}

__device__ __forceinline__ void cursor_start(const DecodePlan& P, Cursor& c)
{
	const int4 st = P.cta_start[blockIdx.x]; // placed by the host: (job, segment, tile)
	c.job = st.x;
	c.seg = st.y;
	c.tis = st.z;
	cursor_load(P, c);
}

__device__ __forceinline__ void cursor_next(const DecodePlan& P, Cursor& c)
{
	if (++c.tis < c.n_tiles) return;
	c.tis = 0;
	if (++c.seg < c.n_segs) return;
	c.seg = 0;
	do
		++c.job;
	while (c.job < P.n_jobs && P.jobs[c.job].n_tiles == 0);
	if (c.job < P.n_jobs) cursor_load(P, c);
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

// The rows of a segment that exist (the last row group may be short).
__device__ __forceinline__ int seg_rows(const DevJob& J, int rg, int RM)
{
	return min(RM, (J.n_head / J.n_kv) * J.n_tok - rg * RM);
}

template <int D, typename KV, int RM>
__global__ void __launch_bounds__((NW + 1) * 32, 1) decode_kernel(const DecodePlan P)
{
	using C = Cfg<D, KV, RM>;
	using T_ = typename KV::T;
	constexpr int E = C::E, T = C::T, KB = C::KB, KS = C::KS, N = C::N, SHIFT = C::SHIFT;
	constexpr int VEC = LaneVec<E, KV::esize>::VEC; // lane <-> element mapping of K, V, q and o
	constexpr int RS = C::RS, RMW = C::RMW;
	constexpr int PW = D + 4; // a partial row: o[D], m, l, two pad floats (16-byte rows)
	constexpr int STAGES = C::STAGES;

	extern __shared__ __align__(1024) unsigned char smem[];
	unsigned char* stages = smem;
	float* area = reinterpret_cast<float*>(smem + STAGES * C::STAGE_BYTES); // [NW/2][RMW][D]
	float* m_s = area + C::AREA_FLOATS;                                      // [NW][RMW]
	float* l_s = m_s + NW * RMW;                                             // [NW][RMW]
	float* qslot = l_s + NW * RMW;                                           // [2][RM][D]
	uint64_t* full = reinterpret_cast<uint64_t*>(qslot + 2 * C::QSLOT_FLOATS);
	uint64_t* empty = full + STAGES;
	uint64_t* qfull = empty + STAGES;  // [2]
	uint64_t* qempty = qfull + 2;      // [2]
	volatile int* s_flags = reinterpret_cast<volatile int*>(qempty + 2); // [0] abort, [1] last-piece vote

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const long long g_begin = (long long)blockIdx.x * P.tiles_per_cta;
	const long long g_end = min(g_begin + P.tiles_per_cta, P.total_tiles);
	const int n_mine = (int)(g_end - g_begin);

	if (threadIdx.x == 0)
	{
		for (int s = 0; s < STAGES; ++s)
		{
			mbar_init(&full[s], 1);
			mbar_init(&empty[s], NW);
		}
		for (int s = 0; s < 2; ++s)
		{
			mbar_init(&qfull[s], 1);
			mbar_init(&qempty[s], NW);
		}
		s_flags[0] = 0;
		s_flags[1] = 0;
		fence_barrier_init();
	}
	__syncthreads();

	if (warp == NW)
	{
		// ---- producer: one lane streams each piece's q rows and the CTA's tiles ----
		if (lane == 0 && n_mine > 0)
		{
			Cursor cur;
			cursor_start(P, cur);
			int pj = -1, ps = -1, piece = 0;
			bool waited = false;
			for (int i = 0; i < n_mine; ++i)
			{
				const DevJob& J = P.jobs[cur.job];
				const int h = cur.seg / J.n_rowgroups, rg = cur.seg % J.n_rowgroups;
				if (cur.job != pj || cur.seg != ps)
				{
					// a new piece: its descriptor, tile count and q rows into slot piece % 2,
					// once the consumers are done with what that slot held
					const int sl = piece & 1;
					if (piece >= 2 &&
					    !mbar_wait_bounded(&qempty[sl], (uint32_t)(((piece >> 1) - 1) & 1), P.err, DEVERR_WAIT_EMPTY))
					{
						s_flags[0] = 1;
						break;
					}
					const int G = J.n_head / J.n_kv;
					const int rows = seg_rows(J, rg, RM);
					float* slot = qslot + sl * C::QSLOT_FLOATS;
					int* info = reinterpret_cast<int*>(slot + C::QHEAD_FLOATS - 4);
					info[0] = min(cur.n_tiles - cur.tis, n_mine - i); // tiles of this piece in this CTA
					info[1] = cur.tis;
					info[2] = cur.seg;
					const int half = J.n_rot / 2;
					const uint32_t inv_bytes = (uint32_t)((half * 4 + 15) & ~15); // the table is padded
					const uint32_t bytes = (uint32_t)(sizeof(DevJob) + rows * D * 4 + (J.q_gamma ? D * 4 : 0) +
					                                  inv_bytes + (J.freq_factors ? half * 4 : 0));
					mbar_arrive_expect_tx(&qfull[sl], bytes);
					bulk_g2s(slot, P.jobs + cur.job, (uint32_t)sizeof(DevJob), &qfull[sl]);
					if (J.q_gamma) bulk_g2s(slot + C::QGAIN, J.q_gamma, (uint32_t)(D * 4), &qfull[sl]);
					if (inv_bytes) bulk_g2s(slot + C::QINV, J.rope_inv, inv_bytes, &qfull[sl]);
					if (J.freq_factors) bulk_g2s(slot + C::QFF, J.freq_factors, (uint32_t)(half * 4), &qfull[sl]);
					// rows (t, g) of the segment: per token, its G heads are contiguous
					for (int r = 0; r < rows;)
					{
						const int gr = rg * RM + r, t = gr / G, g = gr % G;
						const int run = min(G - g, rows - r);
						bulk_g2s(slot + C::QROWS + r * D, J.q + ((size_t)t * J.n_head + (size_t)h * G + g) * D,
						         (uint32_t)(run * D * 4), &qfull[sl]);
						r += run;
					}
					pj = cur.job;
					ps = cur.seg;
					++piece;
				}
				const int key0 = (J.tile_lo + cur.tis) * T;
				// the rows K1 appends come from the preceding grid: wait for it
				// before streaming a tile that holds them (earlier tiles need not)
				if (!waited && !J.reuse_kv && key0 <= J.pos0 + J.n_tok - 1 && key0 + T - 1 >= J.pos0)
				{
					griddep_wait();
					waited = true;
				}
				const size_t off = (size_t)h * J.head_bytes + (size_t)(key0 % J.rows) * D * KV::esize;
				const int s = i % STAGES;
				if (i >= STAGES &&
				    !mbar_wait_bounded(&empty[s], (uint32_t)(((i / STAGES) - 1) & 1), P.err, DEVERR_WAIT_EMPTY))
				{
					s_flags[0] = 1;
					break;
				}
				if (s_flags[0]) break;
				unsigned char* st = stages + s * C::STAGE_BYTES;
				mbar_arrive_expect_tx(&full[s], 2 * TILE_BYTES);
				bulk_g2s(st, J.K + off, TILE_BYTES, &full[s]);
				bulk_g2s(st + TILE_BYTES, J.V + off, TILE_BYTES, &full[s]);
				cursor_next(P, cur);
			}
		}
		return;
	}

	// ---- consumers ----
	// Warp w takes rows [rs*RMW, rs*RMW + RMW) of the segment (rs = w % RS)
	// for the keys [kg*KB, kg*KB + KB) of every tile (kg = w / RS).
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

	// What the end of a piece needs from its job, kept in registers (the slot
	// it came in may be refilled before the piece ends).
	struct PieceEnd
	{
		float* out;
		int n_head, G, h, rg, n_tok, seg, c_first, c_last;
	} pe;

	// Piece start: the piece's q rows from its slot into registers, and what
	// its end will need; then the slot goes back to the producer.
	auto start_piece = [&](const DevJob& J, int seg_local, int sl) {
		const int G = J.n_head / J.n_kv;
		const int h = seg_local / J.n_rowgroups, rg = seg_local % J.n_rowgroups;
		const int rows = seg_rows(J, rg, RM);
		softcap = J.softcap > 0.0f;
		cap = J.softcap;
		const float qmul = softcap ? J.scale : J.scale * LOG2E;
		float* slot = qslot + sl * C::QSLOT_FLOATS;
		float* qs = slot + C::QROWS;
		// attention_forward's q work (model.cpp:1616-1660), a warp per row:
		// RMSNorm with the gains, then RoPE at the row's token position
		for (int r = warp; r < rows; r += NW)
		{
			float* buf = qs + r * D;
			if (J.q_gamma)
			{
				const float sc = rms_scale(buf, D, J.eps, true);
				for (int i2 = lane; i2 < D; i2 += 32) buf[i2] = buf[i2] * sc * slot[C::QGAIN + i2];
				__syncwarp();
			}
			rope_vec(buf, J.n_rot, J.rope_mode, (float)(J.pos0 + (rg * RM + r) / G) * J.rope_scale, slot + C::QINV,
			         J.freq_factors ? slot + C::QFF : nullptr);
			__syncwarp();
		}
		named_sync(1, NW * 32);
#pragma unroll
		for (int r = 0; r < RMW; ++r)
		{
			const int R = rs * RMW + r;
			const bool ok = R < rows; // warp-uniform
			float tmp[E];
			if (ok) load_lane_f<E, VEC>(qs + R * D, lane, tmp);
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
		const long long W = P.tiles_per_cta;
		const long long seg_gstart = J.gtile0 + (long long)seg_local * J.n_tiles;
		pe.out = J.out;
		pe.n_head = J.n_head;
		pe.G = G;
		pe.h = h;
		pe.rg = rg;
		pe.n_tok = J.n_tok;
		pe.seg = J.seg0 + seg_local;
		pe.c_first = (int)(seg_gstart / W);
		pe.c_last = (int)((seg_gstart + J.n_tiles - 1) / W);
		// the slot is refilled by bulk copies (the async proxy): order this warp's
		// writes to it first, then hand it back
		asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
		__syncwarp();
		if (lane == 0) mbar_arrive(&qempty[sl]);
	};

	// Merge the warps' states of the finished piece (two rounds: the upper half
	// of the warps hands its state to the lower half, which folds it in
	// registers and leaves the result for the CTA); write the output (whole
	// segment in this CTA) or a partial, and fold the partials if this CTA
	// completes the segment.
	auto finish_piece = [&]() {
		// l of each row: sum over the batch's key slots (lanes differing in the
		// key bits), then every row's l in every lane
		float lsum = l_lane;
#pragma unroll
		for (int off = 1 << (SHIFT + C::LOG2RMW); off < 32; off <<= 1)
			lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
		float lrow[RMW];
#pragma unroll
		for (int r = 0; r < RMW; ++r) lrow[r] = __shfl_sync(0xffffffffu, lsum, r << SHIFT);
		// Pairwise tree over the warps through two warps' worth of area: 6,7 into
		// 2,3; 4,5 into 0,1; 2,3 into 0,1. Partners have the same row slice.
		auto put = [&](int slot_i) {
#pragma unroll
			for (int r = 0; r < RMW; ++r)
			{
#pragma unroll
				for (int e = 0; e < E; ++e) area[(slot_i * RMW + r) * D + lane_elem<E, VEC>(lane, e)] = o[r][e];
				if (lane == 0)
				{
					m_s[slot_i * RMW + r] = m[r];
					l_s[slot_i * RMW + r] = lrow[r];
				}
			}
		};
		auto take = [&](int slot_i) {
#pragma unroll
			for (int r = 0; r < RMW; ++r)
			{
				const float mo = m_s[slot_i * RMW + r], lo = l_s[slot_i * RMW + r];
				const float M = fmaxf(m[r], mo);
				const float ca = m[r] == -CUDART_INF_F ? 0.0f : ex2(m[r] - M);
				const float cb = mo == -CUDART_INF_F ? 0.0f : ex2(mo - M);
#pragma unroll
				for (int e = 0; e < E; ++e)
					o[r][e] = fmaf(o[r][e], ca, area[(slot_i * RMW + r) * D + lane_elem<E, VEC>(lane, e)] * cb);
				m[r] = M;
				lrow[r] = fmaf(lrow[r], ca, lo * cb);
			}
		};
		if (warp >= 6) put(warp - 6);
		named_sync(1, NW * 32);
		if (warp == 2 || warp == 3) take(warp - 2);
		named_sync(1, NW * 32);
		if (warp == 4 || warp == 5) put(warp - 4);
		named_sync(1, NW * 32);
		if (warp < 2) take(warp);
		named_sync(1, NW * 32);
		if (warp == 2 || warp == 3) put(warp - 2);
		named_sync(1, NW * 32);
		if (warp < 2) take(warp);
		named_sync(1, NW * 32);
		if (warp < 2) put(warp);
		named_sync(1, NW * 32);
		// area slot 0 holds warp 0's merged state, slot 1 warp 1's: the same rows
		// (one row slice) or the two slices

		const int G = pe.G, h = pe.h, rg = pe.rg, n_tok = pe.n_tok, n_head = pe.n_head;
		const int c_first = pe.c_first, c_last = pe.c_last, seg = pe.seg;
		const bool single = c_first == c_last;
		float* part = P.parts + (size_t)(seg + (int)blockIdx.x) * RM * PW;

		for (int idx = ctid; idx < RM * D; idx += NW * 32)
		{
			const int R = idx / D, d = idx % D;
			const int sl = R / RMW, r = R % RMW; // the row's slice and its row within the slice
			float M = -CUDART_INF_F;
#pragma unroll
			for (int k = 0; k < 2 / RS; ++k) M = fmaxf(M, m_s[(k * RS + sl) * RMW + r]);
			float acc = 0.0f, L = 0.0f;
#pragma unroll
			for (int k = 0; k < 2 / RS; ++k)
			{
				const int w = k * RS + sl;
				const float mw = m_s[w * RMW + r];
				const float c = mw == -CUDART_INF_F ? 0.0f : ex2(mw - M);
				acc = fmaf(area[(w * RMW + r) * D + d], c, acc);
				L = fmaf(l_s[w * RMW + r], c, L);
			}
			if (single)
			{
				const int gr = rg * RM + R;
				if (gr < G * n_tok)
				{
					const int t = gr / G, g = gr % G;
					pe.out[((size_t)t * n_head + (size_t)h * G + g) * D + d] = L > 0.0f ? acc / L : 0.0f;
				}
			}
			else
			{
				part[R * PW + d] = acc;
				if (d == 0)
				{
					part[R * PW + D] = M;
					part[R * PW + D + 1] = L;
				}
			}
		}
		if (!single)
		{
			named_sync(1, NW * 32);
			if (ctid == 0)
			{
				const int n_pieces = c_last - c_first + 1;
				const int prev = atomic_add_acq_rel(&P.counters[seg], 1);
				s_flags[1] = prev == n_pieces - 1;
			}
			named_sync(1, NW * 32);
			if (s_flags[1])
			{
				// Fold the pieces (nnc_attn_merge in key order, then
				// nnc_attn_finish) in two rounds of independent loads: a warp
				// per row takes every piece's (m, l) at once and leaves the
				// weights exp2(m_c - M) / L in the area; then each thread sums
				// its 4 output columns over the pieces with 16-byte loads.
				const int np = c_last - c_first + 1; // the planner keeps np * RM within the area
				const float* base = P.parts + (size_t)(seg + c_first) * RM * PW;
				float* wgt = area; // [np][RM]
				for (int R = warp; R < RM; R += NW)
				{
					float2 ml[4];
#pragma unroll
					for (int k = 0; k < 4; ++k)
					{
						const int c = lane + 32 * k;
						ml[k] = c < np ? __ldcg(reinterpret_cast<const float2*>(base + (size_t)c * RM * PW + R * PW + D))
						               : make_float2(-CUDART_INF_F, 0.0f);
					}
					float mx = fmaxf(fmaxf(ml[0].x, ml[1].x), fmaxf(ml[2].x, ml[3].x));
					for (int c = lane + 128; c < np; c += 32)
						mx = fmaxf(mx, __ldcg(base + (size_t)c * RM * PW + R * PW + D));
					mx = warp_max(mx);
					float L = 0.0f;
#pragma unroll
					for (int k = 0; k < 4; ++k)
					{
						const int c = lane + 32 * k;
						const float w = ml[k].x == -CUDART_INF_F ? 0.0f : ex2(ml[k].x - mx);
						if (c < np) wgt[c * RM + R] = w;
						L = fmaf(ml[k].y, w, L);
					}
					for (int c = lane + 128; c < np; c += 32)
					{
						const float2 v = __ldcg(reinterpret_cast<const float2*>(base + (size_t)c * RM * PW + R * PW + D));
						const float w = v.x == -CUDART_INF_F ? 0.0f : ex2(v.x - mx);
						wgt[c * RM + R] = w;
						L = fmaf(v.y, w, L);
					}
					L = warp_sum(L);
					const float inv = L > 0.0f ? 1.0f / L : 0.0f;
					for (int c = lane; c < np; c += 32) wgt[c * RM + R] *= inv;
				}
				named_sync(1, NW * 32);
				for (int idx = ctid; idx < RM * (D / 4); idx += NW * 32)
				{
					const int R = idx / (D / 4), d = 4 * (idx % (D / 4));
					const int gr = rg * RM + R;
					if (gr >= G * n_tok) continue;
					const float* col = base + R * PW + d;
					float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
					int c = 0;
					for (; c + 4 <= np; c += 4)
					{
						float4 v[4];
#pragma unroll
						for (int u = 0; u < 4; ++u) v[u] = __ldcg(reinterpret_cast<const float4*>(col + (size_t)(c + u) * RM * PW));
#pragma unroll
						for (int u = 0; u < 4; ++u)
						{
							const float w = wgt[(c + u) * RM + R];
							acc.x = fmaf(v[u].x, w, acc.x);
							acc.y = fmaf(v[u].y, w, acc.y);
							acc.z = fmaf(v[u].z, w, acc.z);
							acc.w = fmaf(v[u].w, w, acc.w);
						}
					}
					for (; c < np; ++c)
					{
						const float4 v = __ldcg(reinterpret_cast<const float4*>(col + (size_t)c * RM * PW));
						const float w = wgt[c * RM + R];
						acc.x = fmaf(v.x, w, acc.x);
						acc.y = fmaf(v.y, w, acc.y);
						acc.z = fmaf(v.z, w, acc.z);
						acc.w = fmaf(v.w, w, acc.w);
					}
					const int t = gr / G, g = gr % G;
					*reinterpret_cast<float4*>(pe.out + ((size_t)t * n_head + (size_t)h * G + g) * D + d) = acc;
				}
				if (ctid == 0) P.counters[seg] = 0; // ready for the next launch
			}
		}
		named_sync(1, NW * 32); // the merge area is free again
	};

	// Pieces as the producer announces them in the q slots: start, tiles, end.
	int i = 0;
	for (int piece = 0; i < n_mine; ++piece)
	{
		const int sl = piece & 1;
		if (!s_flags[0] && !mbar_wait_bounded(&qfull[sl], (uint32_t)((piece >> 1) & 1), P.err, DEVERR_WAIT_FULL))
			s_flags[0] = 1;
		named_sync(1, NW * 32); // every warp has its answer: the decision below is uniform
		if (s_flags[0]) break;
		const float* slot = qslot + sl * C::QSLOT_FLOATS;
		const DevJob& J = *reinterpret_cast<const DevJob*>(slot);
		const int* info = reinterpret_cast<const int*>(slot + C::QHEAD_FLOATS - 4);
		const int n_piece = info[0], tis0 = info[1], seg_local = info[2];
		int key_base = (J.tile_lo + tis0) * T;
		start_piece(J, seg_local, sl);
		for (int k = 0; k < n_piece; ++k, ++i)
		{
			const int s = i % STAGES;
			// After a timed-out wait the CTA stops waiting (fail fast) but keeps
			// stepping through the piece, so every consumer warp still meets the
			// same named barriers; the error word tells the host the result is void.
			if (!s_flags[0] && !mbar_wait_bounded(&full[s], (uint32_t)((i / STAGES) & 1), P.err, DEVERR_WAIT_FULL))
				s_flags[0] = 1;
			const T_* Kt = reinterpret_cast<const T_*>(stages + s * C::STAGE_BYTES);
			const T_* Vt = reinterpret_cast<const T_*>(stages + s * C::STAGE_BYTES + TILE_BYTES);
			if (!s_flags[0])
			{
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
					bool moved = false;
					float m_v = 0.0f, alpha_v = 1.0f; // this lane's row's, picked without dynamic indexing
#pragma unroll
					for (int r = 0; r < RMW; ++r)
					{
						const float mn = fmaxf(m[r], __shfl_sync(0xffffffffu, mx, r << SHIFT));
						moved |= mn != m[r];
						alpha[r] = mn == -CUDART_INF_F ? 1.0f : ex2(m[r] - mn);
						m[r] = mn;
						if (r == r_v)
						{
							m_v = mn;
							alpha_v = alpha[r];
						}
					}
					const float pv = sv == -CUDART_INF_F ? 0.0f : ex2(sv - m_v);
					l_lane = fmaf(l_lane, alpha_v, pv);
					if (moved) // warp-uniform: m is the same in every lane
					{
#pragma unroll
						for (int r = 0; r < RMW; ++r)
#pragma unroll
							for (int e = 0; e < E; ++e) o[r][e] *= alpha[r];
					}
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
			}
			__syncwarp();
			if (lane == 0) mbar_arrive(&empty[s]);
			key_base += T;
		}
		finish_piece();
	}
	const int n_done = i;
	if (s_flags[0] && ctid == 0)
	{
		// Do not leave while a copy issued into this CTA's shared memory may
		// still land: wait (bounded again) for the stages the producer may
		// have filled beyond the last consumed tile.
		for (int k = n_done; k < n_mine && k < n_done + STAGES; ++k)
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
	static bool configured[64] = {};
	int dev = 0;
	cudaGetDevice(&dev);
	if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
	if (!configured[dev])
	{
		cudaError_t e = cudaFuncSetAttribute(decode_kernel<D, KV, RM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
		                                     C::SMEM);
		if (e != cudaSuccess) return (int)e;
		configured[dev] = true;
	}
	// launched as a programmatic dependent of the K1 grid before it (when there
	// is one): it starts while K1 runs and waits for it where it must
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3((unsigned)P.n_ctas);
	cfg.blockDim = dim3((NW + 1) * 32);
	cfg.dynamicSmemBytes = C::SMEM;
	cfg.stream = st;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = attr;
	cfg.numAttrs = 1;
	return (int)cudaLaunchKernelEx(&cfg, decode_kernel<D, KV, RM>, P);
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

namespace
{
constexpr int slices(int D, int RM) { return RM * (D / 32) > 32 ? RM * (D / 32) / 32 : 1; }
} // namespace

int decode_smem_bytes(int D, int kv_type, int RM)
{
	(void)kv_type;
	const int RMW = RM / slices(D, RM);
	const int qslot = (int)(sizeof(DevJob) / 4) + 4 + RM * D + 2 * D;
	const int fixed = (2 * RMW * D + 2 * NW * RMW + 2 * qslot) * 4 + 256;
	const int stages = std::min(MAX_STAGES, (SMEM_LIMIT - fixed) / (2 * TILE_BYTES));
	return stages * 2 * TILE_BYTES + fixed;
}

int decode_fold_pieces(int D, int RM) { return 2 * (RM / slices(D, RM)) * D / RM; }

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
