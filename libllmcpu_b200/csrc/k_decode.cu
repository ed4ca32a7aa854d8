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
//  * Split. Each segment is cut into a few equal chunks of whole tiles and
//    each CTA streams a run of consecutive chunks (plan.cpp), most CTAs a
//    single one. A chunk is computed as one piece giving a partial (o, m, l)
//    like nnc_attn_block's; the CTA that finishes a segment's last piece
//    merges the pieces (nnc_attn_merge) and divides by l (nnc_attn_finish).
//    A segment of one chunk writes the output directly. No second launch.
//  * Memory. One producer warp streams each tile's K rows and V rows (one
//    contiguous 32 KB run each in the head-major cache) into a 3-stage shared
//    memory ring with cp.async.bulk, completing on mbarriers; 8 consumer
//    warps compute while the next tiles are in flight. The first tile goes
//    out before the job is even read (its address is in the CTA's start).
//    Each piece's job descriptor, raw q rows, gains and RoPE tables come the
//    same way, into one of two q slots, ahead of the piece's tiles, so no
//    consumer ever waits on a plain global load behind the tile stream.
//  * Per-head work. The consumers give the q rows their RMSNorm and RoPE in
//    the slot. For decode and short verify the kernel also appends the new
//    tokens' K/V rows itself: the piece holding them normalises, rotates and
//    narrows the raw k, v rows from its slot, reads them from there in place
//    of the cache rows, and (first row group only) stores them to the cache.
//    Longer batches have K1 (k_prep.cu) append first; the kernel is then its
//    programmatic dependent, starts while K1 runs, and waits for K1 only
//    before the tiles that hold the new rows, which it streams last.
//  * Math. fp32 throughout. A warp owns T/8 keys of each tile. For head_dim
//    256 and up its lanes split head_dim (D/32 elements each); below that a
//    key takes LK = D/8 lanes (8 elements each) and the warp works on 32/LK
//    keys side by side, each lane group with its own softmax state. The
//    q.k partial sums of a batch of keys x rows are summed across a key's
//    lanes with a transposing reduction, the online softmax runs in
//    registers in base 2, and o accumulates in registers. The lane groups,
//    then the warps, merge their (o, m, l) at piece end.
#include <cuda_runtime.h>

#include <math_constants.h>

#include <algorithm>

#include "common.cuh"
#include "decode.cuh"

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
	// lanes per key: a key row spans the warp for head_dim 256 and up (and
	// for many rows); below that each lane takes 8 elements and the warp
	// works on 32 / LK keys side by side, so a score is summed over LK lanes
	// instead of 32
	static constexpr int LK = (D < 256 && RM <= 8) ? D / 8 : 32;
	static constexpr int LG = 32 / LK;                     // lane groups (keys side by side) per warp
	static constexpr int LOG2LK = LK >= 32 ? 5 : LK >= 16 ? 4 : LK >= 8 ? 3 : LK >= 4 ? 2 : 1;
	static constexpr int E = D / LK;                       // elements per lane
	static constexpr int RS = RM * E > 32 ? RM * E / 32 : 1; // row slices: warps sharing keys, splitting rows
	static constexpr int RMW = RM / RS;                    // rows per warp
	static constexpr int NKG = NW / RS;                    // key groups
	static constexpr int T = TILE_BYTES / (D * KV::esize); // keys per tile
	static constexpr int KB = T / NKG;                     // keys per warp per tile
	static constexpr int KS = KB / LG < LK / RMW ? KB / LG : LK / RMW; // keys per lane group per reduction batch
	static constexpr int N = KS * RMW;                     // values per reduction
	static constexpr int LOG2N = N >= 32 ? 5 : N >= 16 ? 4 : N >= 8 ? 3 : N >= 4 ? 2 : N >= 2 ? 1 : 0;
	static constexpr int SHIFT = LOG2LK - LOG2N;           // (lane % LK) >> SHIFT = value index after the reduction
	static constexpr int LOG2RMW = RMW >= 32 ? 5 : RMW >= 16 ? 4 : RMW >= 8 ? 3 : RMW >= 4 ? 2 : RMW >= 2 ? 1 : 0;
	static constexpr int NB = KB / (KS * LG);              // reduction batches per warp per tile
	// batches sharing one softmax update: with lane groups, all of a tile's
	// (their weights fit 128 floats of warp scratch); otherwise one, as a
	// batch then already spans 32 / RMW keys
	static constexpr int NBS = LG == 1 ? 1 : NB * LG * N <= 128 ? NB : (128 / (LG * N) >= 1 ? 128 / (LG * N) : 1);
	static constexpr int PBW = NBS * LG * N > 32 ? NBS * LG * N : 32; // warp scratch floats
	static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
	// the warps' (o, m, l) at a piece's end pass through two warps' worth of
	// area in a pairwise tree; the fold's weights reuse the same area
	static constexpr int AREA_FLOATS = 2 * RMW * D;
	// one piece's slot: its job descriptor, its tile count / first tile /
	// segment / whether it appends, its raw q rows, the q and k gains, the RoPE
	// tables, and (when this kernel appends the new rows itself) the new
	// tokens' k rows and v rows of its KV head
	static constexpr int QHEAD_FLOATS = (int)(sizeof(DevJob) / 4) + 4;
	static constexpr int QROWS = QHEAD_FLOATS;             // RM * D
	static constexpr int QGAIN = QROWS + RM * D;           // D
	static constexpr int QINV = QGAIN + D;                 // D / 2
	static constexpr int QFF = QINV + D / 2;               // D / 2
	static constexpr int QKG = QFF + D / 2;                // D (only with NT > 0)
	static constexpr int QNEW = QKG + D;                   // NT * D k rows, then NT * D v rows
	static constexpr int FIXED0 = (AREA_FLOATS + 2 * NW * RMW + NW * PBW + 2 * QKG) * 4 + 256;
	static constexpr int FIT = (SMEM_LIMIT - FIXED0) / STAGE_BYTES;
	static constexpr int STAGES = FIT < MAX_STAGES ? FIT : MAX_STAGES;
	// new tokens per launch this kernel can append itself, in what the stages leave
	static constexpr int NT_FIT = (SMEM_LIMIT - FIXED0 - STAGES * STAGE_BYTES - 2 * D * 4) / (2 * 2 * D * 4);
	static constexpr int NT = NT_FIT < 0 ? 0 : NT_FIT < 16 ? NT_FIT : 16;
	static constexpr int QSLOT_FLOATS = NT > 0 ? QNEW + 2 * NT * D : QKG;
	static constexpr int FIXED_BYTES = (AREA_FLOATS + 2 * NW * RMW + NW * PBW + 2 * QSLOT_FLOATS) * 4 + 256;
	static constexpr int SMEM = STAGES * STAGE_BYTES + FIXED_BYTES;
	static_assert(SMEM <= SMEM_LIMIT, "shared memory");
	static_assert(STAGES >= 3, "shared memory for at least three stages");
	static_assert(D % 32 == 0, "D: a multiple of 32");
	static_assert(RM % RS == 0 && NW == 8 && RS <= 2, "row slices");
	static_assert(T >= NKG && T <= ATTN_BLOCK && ATTN_BLOCK % T == 0 && T % NKG == 0, "tile keys");
	static_assert(KS >= 1 && KB % (KS * LG) == 0 && NB % NBS == 0, "batches per warp");
	static_assert(N <= LK && LK * LG == 32, "lane groups");
	static_assert(RMW * E <= 32, "accumulator registers");
};

// The kernel's body. INL: the job table and the CTA starts are the bytes
// `tab` of the kernel's parameters (a small launch, no upload) instead of
// P.jobs and P.cta_start in global memory.
template <int D, typename KV, int RM, bool INL>
__device__ __forceinline__ void decode_body(const DecodePlan& P, const unsigned char* tab)
{
	using C = Cfg<D, KV, RM>;
	using T_ = typename KV::T;
	constexpr int E = C::E, T = C::T, KB = C::KB, KS = C::KS, N = C::N, SHIFT = C::SHIFT, NBS = C::NBS;
	constexpr int VEC = LaneVec<E, KV::esize>::VEC; // lane <-> element mapping of K, V, q and o
	constexpr int RS = C::RS, RMW = C::RMW;
	constexpr int PW = D + 4; // a partial row: o[D], m, l, two pad floats (16-byte rows)
	constexpr int STAGES = C::STAGES;

	extern __shared__ __align__(1024) unsigned char smem[];
	unsigned char* stages = smem;
	float* area = reinterpret_cast<float*>(smem + STAGES * C::STAGE_BYTES); // [NW/2][RMW][D]
	float* m_s = area + C::AREA_FLOATS;                                      // [NW][RMW]
	float* l_s = m_s + NW * RMW;                                             // [NW][RMW]
	float* pbuf = l_s + NW * RMW;                                            // [NW][PBW] batches' weights
	float* qslot = pbuf + NW * C::PBW;                                       // [2][RM][D]
	uint64_t* full = reinterpret_cast<uint64_t*>(qslot + 2 * C::QSLOT_FLOATS);
	uint64_t* empty = full + STAGES;
	uint64_t* qfull = empty + STAGES;  // [2]
	uint64_t* qempty = qfull + 2;      // [2]
	// [0] abort, [1] last-piece vote, [2] the GPUs whose split merge this CTA does
	volatile int* s_flags = reinterpret_cast<volatile int*>(qempty + 2);
	CtaStart* s_start = reinterpret_cast<CtaStart*>(qempty + 4);          // this CTA's start (16-byte aligned)

	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const DevJob* jobs = INL ? reinterpret_cast<const DevJob*>(tab) : P.jobs;
	const CtaStart* starts =
		INL ? reinterpret_cast<const CtaStart*>(tab + ((P.n_jobs * sizeof(DevJob) + 15) & ~size_t(15))) : P.cta_start;

	if (threadIdx.x == 0)
	{
		*s_start = starts[blockIdx.x];
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
	const int n_mine = s_start->n_tiles;

	if (warp == NW)
	{
		// ---- producer: one lane streams each piece's q rows and the CTA's tiles ----
		// A piece is one chunk of a segment (or the part of it in this CTA). The
		// first tiles go out before anything else, from addresses the plan
		// gives. While K1 appends, the pieces go in two passes: first those
		// without any key K1 appends, then those with them, so that the wait for
		// K1 comes as late in the CTA's stream as it can (a piece's own tiles
		// stay in key order; so do its new keys, last).
		if (lane == 0 && n_mine > 0)
		{
			const CtaStart S = *s_start;
			for (int t = 0; t < S.pre; ++t)
			{
				unsigned char* st = stages + t * C::STAGE_BYTES;
				mbar_arrive_expect_tx(&full[t], 2 * TILE_BYTES);
				bulk_g2s(st, S.k0 + (size_t)t * TILE_BYTES, TILE_BYTES, &full[t]);
				bulk_g2s(st + TILE_BYTES, S.v0 + (size_t)t * TILE_BYTES, TILE_BYTES, &full[t]);
			}
			Cursor c0;
			c0.job = S.job;
			c0.seg = S.seg;
			c0.tis = S.tis;
			cursor_load<INL>(jobs, P.n_jobs, c0);
			int piece = 0, i = 0;
			bool waited = false;
			for (int pass = 0; pass < (P.fused ? 1 : 2) && !s_flags[0]; ++pass)
			{
				Cursor cur = c0;
				for (int left = n_mine; left > 0 && !s_flags[0];)
				{
					const DevJob& J = jobs[cur.job];
					const int n = min(min(cur.n_tiles - cur.tis, J.chunk - cur.tis % J.chunk), left);
					const bool fresh = holds_new_rows(J, cur.tis, n, T);
					if (P.fused || (int)fresh == pass)
					{
						// a piece holding new keys appends them itself when K1 does not run
						const bool append = P.fused && fresh;
						const int h = cur.seg / J.n_rowgroups, rg = cur.seg % J.n_rowgroups;
						// the piece's descriptor, tile count and q rows into slot piece % 2,
						// once the consumers are done with what that slot held
						const int sl = piece & 1;
						if (piece >= 2 && !mbar_wait_bounded(&qempty[sl], (uint32_t)(((piece >> 1) - 1) & 1), P.err,
						                                     DEVERR_WAIT_EMPTY))
						{
							s_flags[0] = 1;
							break;
						}
						const int G = J.n_head / J.n_kv;
						const int rows = seg_rows(J, rg, RM);
						float* slot = qslot + sl * C::QSLOT_FLOATS;
						int* info = reinterpret_cast<int*>(slot + C::QHEAD_FLOATS - 4);
						info[0] = n;       // tiles of this piece in this CTA
						info[1] = cur.tis; // its first tile within the segment
						info[2] = cur.seg;
						info[3] = append;
						const int half = J.n_rot / 2;
						const uint32_t inv_bytes = (uint32_t)((half * 4 + 15) & ~15); // the table is padded
						const uint32_t bytes =
							(uint32_t)(sizeof(DevJob) + rows * D * 4 + (J.q_gamma ? D * 4 : 0) + inv_bytes +
						               (J.freq_factors ? half * 4 : 0) +
						               (append ? (J.k_gamma ? D * 4 : 0) + 2 * J.n_tok * D * 4 : 0));
						if constexpr (INL)
						{
							// from the parameters: plain copies (the bulk copy reads global memory only)
#pragma unroll
							for (int w = 0; w < (int)(sizeof(DevJob) / 16); ++w)
								reinterpret_cast<uint4*>(slot)[w] = reinterpret_cast<const uint4*>(&J)[w];
						}
						mbar_arrive_expect_tx(&qfull[sl], bytes - (INL ? (uint32_t)sizeof(DevJob) : 0u)); // also releases the stores above
						if constexpr (!INL) bulk_g2s(slot, &J, (uint32_t)sizeof(DevJob), &qfull[sl]);
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
						if (append)
						{
							// the new tokens' raw k and v rows of this KV head, and the k gains
							if (J.k_gamma) bulk_g2s(slot + C::QKG, J.k_gamma, (uint32_t)(D * 4), &qfull[sl]);
							for (int t = 0; t < J.n_tok; ++t)
							{
								const size_t src = ((size_t)t * J.n_kv + h) * D;
								bulk_g2s(slot + C::QNEW + t * D, J.k + src, (uint32_t)(D * 4), &qfull[sl]);
								bulk_g2s(slot + C::QNEW + (C::NT + t) * D, J.v + src, (uint32_t)(D * 4), &qfull[sl]);
							}
						}
						++piece;
						for (int k = 0; k < n; ++k, ++i)
						{
							const int key0 = (J.tile_lo + cur.tis + k) * T;
							// the rows K1 appends come from the preceding grid: wait for it
							// before streaming a tile that holds them
							if (!P.fused && !waited && fresh && holds_new_rows(J, cur.tis + k, 1, T))
							{
								griddep_wait();
								waited = true;
							}
							if (i < S.pre) continue; // issued at the start
							const size_t off = (size_t)h * J.head_bytes + (size_t)(key0 % J.rows) * D * KV::esize;
							const int s = i % STAGES;
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
					left -= n;
					cur.tis += n;
					if (cur.tis >= cur.n_tiles) cursor_next_segment<INL>(jobs, P.n_jobs, cur);
				}
			}
		}
		return;
	}

	// ---- consumers ----
	// Warp w takes rows [rs*RMW, rs*RMW + RMW) of the segment (rs = w % RS)
	// for the keys [kg*KB, kg*KB + KB) of every tile (kg = w / RS). Within
	// the warp, lane group lg (LK lanes) takes KS keys of each batch and
	// keeps its own softmax state; the groups merge at the piece's end.
	constexpr int LK = C::LK, LG = C::LG;
	const int ctid = threadIdx.x; // 0 .. NW*32-1
	const int rs = warp % RS, kg = warp / RS;
	const int lj = lane & (LK - 1);        // this lane within its group
	const int lg = lane / LK;              // its group
	const int gbase = lane & ~(LK - 1);    // the group's first lane
	const int r_v = (lj >> SHIFT) % RMW;   // the row (within the warp's rows) of this lane's reduced value
	const int kk_v = (lj >> SHIFT) / RMW;  // its key within the group's batch

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
		const float* gate;
		int n_head, G, h, rg, n_tok, seg, n_pieces, part, chunk, out_row0;
	} pe;

	// The new keys a piece appends itself, in its slot in the cache's element
	// type (row t of the k rows at new_k + t * NSTRIDE), used in place of the
	// cache rows of positions [new_lo, new_lo + n_new) of its tiles.
	constexpr int NSTRIDE = D * 4 / KV::esize;
	int new_lo = 0, n_new = 0;
	const T_* new_k = nullptr;
	const T_* new_v = nullptr;

	// Piece start: the piece's q rows from its slot into registers, and what
	// its end will need; then the slot goes back to the producer (at the
	// piece's end instead when the slot holds the new keys it appends).
	auto start_piece = [&](const DevJob& J, int seg_local, int sl, bool append, int tis0, int n_piece) {
		const int G = J.n_head / J.n_kv;
		const int h = seg_local / J.n_rowgroups, rg = seg_local % J.n_rowgroups;
		const int rows = seg_rows(J, rg, RM);
		softcap = J.softcap > 0.0f;
		cap = J.softcap;
		const float qmul = softcap ? J.scale : J.scale * LOG2E;
		float* slot = qslot + sl * C::QSLOT_FLOATS;
		float* qs = slot + C::QROWS;
		const float* ff = J.freq_factors ? slot + C::QFF : nullptr;
		// attention_forward's per-head work (model.cpp:1616-1694), a warp per
		// vector: each q row gets RMSNorm with the gains and RoPE at its token's
		// position; when the piece appends, each new k row gets RMSNorm with the
		// k gains and RoPE, each new v row the plain norm if asked, both are
		// narrowed to the cache's type and, by the first row group's piece,
		// stored at row pos % rows of the cache (the append loop, :1662-1694)
		const int n_app = append ? 2 * J.n_tok : 0;
		for (int task = warp; task < rows + n_app; task += NW)
		{
			if (task < rows)
			{
				prep_buf(qs + task * D, D, J.q_gamma ? slot + C::QGAIN : nullptr, false, J.eps, true, J.n_rot,
				         J.rope_mode, (float)(J.pos0 + (rg * RM + task) / G) * J.rope_scale, slot + C::QINV, ff);
				continue;
			}
			const int u = task - rows;
			const bool is_k = u < J.n_tok;
			const int t = is_k ? u : u - J.n_tok;
			float* buf = slot + C::QNEW + (is_k ? t : C::NT + t) * D;
			prep_buf(buf, D, is_k && J.k_gamma ? slot + C::QKG : nullptr, !is_k && J.v_rmsnorm, J.eps, is_k, J.n_rot,
			         J.rope_mode, (float)(J.pos0 + t) * J.rope_scale, slot + C::QINV, ff);
			narrow_buf<KV>(buf, D);
			const int pos = J.pos0 + t;
			const int lo = (J.tile_lo + tis0) * T;
			if (rg == 0 && pos >= lo && pos < lo + n_piece * T && pos >= J.key_lo && pos < J.key_hi)
			{
				const T_* src = reinterpret_cast<const T_*>(buf);
				T_* dst = reinterpret_cast<T_*>((is_k ? J.K : J.V) + (size_t)h * J.head_bytes) + (size_t)(pos % J.rows) * D;
				for (int i2 = lane; i2 < D; i2 += 32) dst[i2] = src[i2];
			}
		}
		new_lo = J.pos0;
		n_new = append ? J.n_tok : 0;
		new_k = reinterpret_cast<const T_*>(slot + C::QNEW);
		new_v = reinterpret_cast<const T_*>(slot + C::QNEW + C::NT * D);
		named_sync(1, NW * 32);
#pragma unroll
		for (int r = 0; r < RMW; ++r)
		{
			const int R = rs * RMW + r;
			const bool ok = R < rows; // warp-uniform
			float tmp[E];
			if (ok) load_lane_f<E, VEC, LK>(qs + R * D, lj, tmp);
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
		{
			span_of(J.causal, J.window, J.pos0 + gr_v / G, J.n_seq, first_v, last_v);
			first_v = max(first_v, J.key_lo);
			last_v = min(last_v, J.key_hi - 1);
		}
		else
			first_v = 0, last_v = -1; // a padding row sees nothing
		pe.out = J.out;
		pe.gate = J.gate;
		pe.n_head = J.n_head;
		pe.G = G;
		pe.h = h;
		pe.rg = rg;
		pe.n_tok = J.n_tok;
		pe.seg = J.seg0 + seg_local;
		pe.n_pieces = J.n_chunks;
		pe.part = J.part0 + seg_local * J.n_chunks; // the segment's first partial slot
		pe.chunk = tis0 / J.chunk;
		pe.out_row0 = J.out_row0;
		// the slot is refilled by bulk copies (the async proxy): order this warp's
		// writes to it first, then hand it back
		asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
		__syncwarp();
		if (lane == 0 && !append) mbar_arrive(&qempty[sl]);
	};

	// Merge the warps' states of the finished piece; write the output (whole
	// segment in this CTA) or a partial, and fold the partials if this CTA
	// completes the segment. After the CTA's last tile (`flat`) the stage
	// buffers are free: every warp leaves its state there and the CTA merges
	// all of them in one round. Otherwise the states go through two warps'
	// worth of area in a pairwise tree.
	auto finish_piece = [&](bool flat) {
		// l of each row: sum over the batch's key slots (lanes differing in the
		// key bits), then every row's l in every lane
		float lsum = l_lane;
#pragma unroll
		for (int off = 1 << (SHIFT + C::LOG2RMW); off < LK; off <<= 1)
			lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
		float lrow[RMW];
#pragma unroll
		for (int r = 0; r < RMW; ++r) lrow[r] = __shfl_sync(0xffffffffu, lsum, gbase + (r << SHIFT));
		// the lane groups' states merged across the warp: every group then
		// holds the warp's (o, m, l)
		if constexpr (LG > 1)
		{
#pragma unroll
			for (int r = 0; r < RMW; ++r)
			{
				float M = m[r];
#pragma unroll
				for (int off = LK; off < 32; off <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
				const float c = m[r] == -CUDART_INF_F ? 0.0f : ex2(m[r] - M);
				float lr = lrow[r] * c;
#pragma unroll
				for (int off = LK; off < 32; off <<= 1) lr += __shfl_xor_sync(0xffffffffu, lr, off);
				lrow[r] = lr;
#pragma unroll
				for (int e = 0; e < E; ++e)
				{
					float x = o[r][e] * c;
#pragma unroll
					for (int off = LK; off < 32; off <<= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
					o[r][e] = x;
				}
				m[r] = M;
			}
		}
		// one round: fo[w][r][:] = warp w's o of its row r, fm / fl its m and l;
		// fc[w][r] the weight of warp w's state in its row's merge, and fM / fL
		// each segment row's merged m and l
		float* fo = reinterpret_cast<float*>(stages); // [NW][RMW][D]
		float* fm = fo + NW * RMW * D;                // [NW][RMW]
		float* fl = fm + NW * RMW;                    // [NW][RMW]
		float* fc = fl + NW * RMW;                    // [NW][RMW]
		float* fM = fc + NW * RMW;                    // [RM]
		float* fL = fM + RM;                          // [RM]
		if (flat)
		{
			named_sync(1, NW * 32); // every warp is done reading the last tile's stage
#pragma unroll
			for (int r = 0; r < RMW; ++r)
			{
#pragma unroll
				for (int e = 0; e < E; ++e) fo[(warp * RMW + r) * D + lane_elem<E, VEC, LK>(lj, e)] = o[r][e];
			}
			if (lane < RMW)
			{
#pragma unroll
				for (int r = 0; r < RMW; ++r)
					if (r == lane)
					{
						fm[warp * RMW + r] = m[r];
						fl[warp * RMW + r] = lrow[r];
					}
			}
			named_sync(1, NW * 32);
			if (ctid < NW * RMW)
			{
				const int w = ctid / RMW, r = ctid % RMW, sl = w % RS;
				float M = -CUDART_INF_F;
#pragma unroll
				for (int k = 0; k < NW / RS; ++k) M = fmaxf(M, fm[(k * RS + sl) * RMW + r]);
				const float mw = fm[ctid];
				fc[ctid] = mw == -CUDART_INF_F ? 0.0f : ex2(mw - M);
				if (w == sl) // the slice's first warp: the row's m and l
				{
					float L = 0.0f;
#pragma unroll
					for (int k = 0; k < NW / RS; ++k)
					{
						const float mk = fm[(k * RS + sl) * RMW + r];
						L = fmaf(fl[(k * RS + sl) * RMW + r], mk == -CUDART_INF_F ? 0.0f : ex2(mk - M), L);
					}
					fM[sl * RMW + r] = M;
					fL[sl * RMW + r] = L;
				}
			}
			named_sync(1, NW * 32);
		}
		else
		{
			// Pairwise tree over the warps through two warps' worth of area: 6,7 into
			// 2,3; 4,5 into 0,1; 2,3 into 0,1. Partners have the same row slice.
			auto put = [&](int slot_i) {
#pragma unroll
				for (int r = 0; r < RMW; ++r)
				{
#pragma unroll
					for (int e = 0; e < E; ++e) area[(slot_i * RMW + r) * D + lane_elem<E, VEC, LK>(lj, e)] = o[r][e];
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
						o[r][e] = fmaf(o[r][e], ca, area[(slot_i * RMW + r) * D + lane_elem<E, VEC, LK>(lj, e)] * cb);
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
		}

		const int G = pe.G, h = pe.h, rg = pe.rg, n_tok = pe.n_tok, n_head = pe.n_head;
		const int seg = pe.seg, n_pieces = pe.n_pieces;
		const bool single = n_pieces == 1;
		const bool split = P.world > 1;
		float* part = P.parts + (size_t)(pe.part + pe.chunk) * RM * PW;
		const int rows_valid = G * n_tok - rg * RM;
		// where row R of this segment goes: the output (t, head) row, and, split,
		// the segment's partial slot in GPU g's receive block of this rank
		// the offset of row R of this segment in the job's output (and gate)
		auto row_off = [&](int R) -> size_t {
			const int gr = rg * RM + R;
			return ((size_t)(gr / G) * n_head + (size_t)h * G + gr % G) * D;
		};
		auto out_row = [&](float* base_out, int R) -> float* { return base_out + row_off(R); };
		auto recv_row = [&](int g, int rank, int R) {
			return P.recv[g] + (size_t)rank * P.recv_stride + ((size_t)seg * RM + R) * PW;
		};

		for (int idx = ctid; idx < RM * D; idx += NW * 32)
		{
			const int R = idx / D, d = idx % D;
			const int sl = R / RMW, r = R % RMW; // the row's slice and its row within the slice
			float M = -CUDART_INF_F, acc = 0.0f, L = 0.0f;
			if (flat)
			{
				M = fM[R];
				L = fL[R];
#pragma unroll
				for (int k = 0; k < NW / RS; ++k)
				{
					const int w = k * RS + sl;
					acc = fmaf(fo[(w * RMW + r) * D + d], fc[w * RMW + r], acc);
				}
			}
			else
			{
#pragma unroll
				for (int k = 0; k < 2 / RS; ++k) M = fmaxf(M, m_s[(k * RS + sl) * RMW + r]);
#pragma unroll
				for (int k = 0; k < 2 / RS; ++k)
				{
					const int w = k * RS + sl;
					const float mw = m_s[w * RMW + r];
					const float c = mw == -CUDART_INF_F ? 0.0f : ex2(mw - M);
					acc = fmaf(area[(w * RMW + r) * D + d], c, acc);
					L = fmaf(l_s[w * RMW + r], c, L);
				}
			}
			if (single && !split)
			{
				if (R < rows_valid) out_row(pe.out, R)[d] = gated(L > 0.0f ? acc / L : 0.0f, pe.gate, row_off(R) + d);
			}
			else if (single)
			{
				// the segment's result over this GPU's keys, to every GPU of the split
				for (int g = 0; g < P.world; ++g)
				{
					float* dst = recv_row(g, P.rank, R);
					dst[d] = acc;
					if (d == 0)
					{
						dst[D] = M;
						dst[D + 1] = L;
					}
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
		bool have = single; // this CTA holds the segment's result over this GPU's keys
		if (!single)
		{
			named_sync(1, NW * 32);
			if (ctid == 0)
			{
				const int prev = atomic_add_acq_rel(&P.counters[seg], 1);
				s_flags[1] = prev == n_pieces - 1;
			}
			named_sync(1, NW * 32);
			if (s_flags[1])
			{
				// Fold the pieces (nnc_attn_merge over the chunks, then
				// nnc_attn_finish), or, split, merge them into the partial this
				// GPU sends
				const float* base = P.parts + (size_t)pe.part * RM * PW;
				if (!split)
					merge_pieces<D, RM>(base, (size_t)RM * PW, n_pieces, rows_valid, ctid, NW * 32,
					                    [&](int R, int d, float4 acc, float M, float L) {
						                    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
						                    acc.x *= inv;
						                    acc.y *= inv;
						                    acc.z *= inv;
						                    acc.w *= inv;
						                    *reinterpret_cast<float4*>(out_row(pe.out, R) + d) =
							                    gated4(acc, pe.gate, row_off(R) + d);
					                    });
				else
					merge_pieces<D, RM>(base, (size_t)RM * PW, n_pieces, rows_valid, ctid, NW * 32,
					                    [&](int R, int d, float4 acc, float M, float L) {
						                    for (int g = 0; g < P.world; ++g)
						                    {
							                    float* dst = recv_row(g, P.rank, R);
							                    *reinterpret_cast<float4*>(dst + d) = acc;
							                    if (d == 0) *reinterpret_cast<float2*>(dst + D) = make_float2(M, L);
						                    }
					                    });
				if (ctid == 0) P.counters[seg] = 0; // ready for the next launch
				have = true;
			}
		}
		if (split && have)
		{
			// This GPU's result for the segment is in every GPU's receive buffer:
			// one system-scope fence orders those stores (every thread's, through
			// the CTA barrier) before the arrivals, which then go out together.
			// Each GPU merges the world's partials at the end of its own call
			// (split_merge_kernel), with loads and stores of its own memory.
			named_sync(1, NW * 32);
			if (ctid == 0 && !P.drop_arrivals) // (a test drops them to make the merges' waits run out)
			{
				fence_acq_rel_sys();
#pragma unroll
				for (int g = 0; g < MAX_WORLD; ++g)
					if (g < P.world) atomic_add_relaxed_sys(P.arrive[g] + seg, 1);
			}
		}
		named_sync(1, NW * 32); // the merge area is free again
	};

	// Pieces as the producer announces them in the q slots: start, tiles, end.
	int i = 0;
	for (int piece = 0; i < n_mine; ++piece)
	{
		const int sl = piece & 1;
		const bool ok = !s_flags[0] && mbar_wait_bounded(&qfull[sl], (uint32_t)((piece >> 1) & 1), P.err, DEVERR_WAIT_FULL);
		if (named_sync_or(1, NW * 32, !ok)) // every consumer takes the same decision
		{
			s_flags[0] = 1;
			break;
		}
		const float* slot = qslot + sl * C::QSLOT_FLOATS;
		const DevJob& J = *reinterpret_cast<const DevJob*>(slot);
		const int* info = reinterpret_cast<const int*>(slot + C::QHEAD_FLOATS - 4);
		const int n_piece = info[0], tis0 = info[1], seg_local = info[2];
		const bool append = info[3] != 0;
		int key_base = (J.tile_lo + tis0) * T;
		start_piece(J, seg_local, sl, append, tis0, n_piece);
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
				for (int sb = 0; sb < C::NB / NBS; ++sb)
				{
					// The scores of NBS batches (each KS keys x RMW rows per lane
					// group): lane-partial dot products, reduced across the key's
					// lanes; then one softmax update for all of them
					float sv[NBS];
#pragma unroll
					for (int bb = 0; bb < NBS; ++bb)
					{
						const int k0 = kg * KB + ((sb * NBS + bb) * LG + lg) * KS; // the lane group's first key, in the tile
						float part[N];
#pragma unroll
						for (int kk = 0; kk < KS; ++kk)
						{
							float kv[E];
							const int np = key_base + k0 + kk - new_lo; // a new key: its row from the slot
							load_lane<E, LK>((unsigned)np < (unsigned)n_new ? new_k + np * NSTRIDE
							                                                : Kt + (size_t)(k0 + kk) * D,
							                 lj, kv);
#pragma unroll
							for (int r = 0; r < RMW; ++r)
							{
								float acc = 0.0f;
#pragma unroll
								for (int e = 0; e < E; ++e) acc = fmaf(q[r][e], kv[e], acc);
								part[kk * RMW + r] = acc;
							}
						}
						float x = transpose_reduce<N, LK>(part, lane);
						const int pos = key_base + k0 + kk_v;
						if (softcap) x = cap * tanhf(x / cap) * LOG2E;
						if (pos < first_v || pos > last_v) x = -CUDART_INF_F;
						sv[bb] = x;
					}
					// the batches' max of each row, then the new running max of every row
					float mx = sv[0];
#pragma unroll
					for (int bb = 1; bb < NBS; ++bb) mx = fmaxf(mx, sv[bb]);
#pragma unroll
					for (int off = 1 << (SHIFT + C::LOG2RMW); off < LK; off <<= 1)
						mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
					float alpha[RMW];
					bool moved = false;
					float m_v = 0.0f, alpha_v = 1.0f; // this lane's row's, picked without dynamic indexing
#pragma unroll
					for (int r = 0; r < RMW; ++r)
					{
						const float mn = fmaxf(m[r], __shfl_sync(0xffffffffu, mx, gbase + (r << SHIFT)));
						moved |= mn != m[r];
						alpha[r] = mn == -CUDART_INF_F ? 1.0f : ex2(m[r] - mn);
						m[r] = mn;
						if (r == r_v)
						{
							m_v = mn;
							alpha_v = alpha[r];
						}
					}
					// the weights; with four or more rows per warp they go through this
					// warp's scratch and come back four at a time as broadcast loads,
					// instead of a shuffle each
					float* pb = pbuf + warp * C::PBW;
					float pv[NBS];
					float psum = 0.0f;
#pragma unroll
					for (int bb = 0; bb < NBS; ++bb)
					{
						pv[bb] = sv[bb] == -CUDART_INF_F ? 0.0f : ex2(sv[bb] - m_v);
						psum += pv[bb];
						if constexpr (RMW >= 4)
							if ((lj & ((1 << SHIFT) - 1)) == 0) pb[(bb * LG + lg) * N + (lj >> SHIFT)] = pv[bb];
					}
					l_lane = fmaf(l_lane, alpha_v, psum);
					if (moved) // uniform in the lane group: its lanes share m
					{
#pragma unroll
						for (int r = 0; r < RMW; ++r)
#pragma unroll
							for (int e = 0; e < E; ++e) o[r][e] *= alpha[r];
					}
					if constexpr (RMW >= 4) __syncwarp();
					// o += p v over the batches' keys
#pragma unroll
					for (int bb = 0; bb < NBS; ++bb)
					{
						const int k0 = kg * KB + ((sb * NBS + bb) * LG + lg) * KS;
#pragma unroll
						for (int kk = 0; kk < KS; ++kk)
						{
							float vv[E];
							const int np = key_base + k0 + kk - new_lo;
							load_lane<E, LK>((unsigned)np < (unsigned)n_new ? new_v + np * NSTRIDE
							                                                : Vt + (size_t)(k0 + kk) * D,
							                 lj, vv);
#pragma unroll
							for (int r = 0; r < RMW; ++r)
							{
								float p;
								if constexpr (RMW >= 4)
								{
									const float4 p4 = *reinterpret_cast<const float4*>(pb + (bb * LG + lg) * N + kk * RMW +
									                                                    (r & ~3));
									p = (r & 3) == 0 ? p4.x : (r & 3) == 1 ? p4.y : (r & 3) == 2 ? p4.z : p4.w;
								}
								else
									p = __shfl_sync(0xffffffffu, pv[bb], gbase + ((kk * RMW + r) << SHIFT));
#pragma unroll
								for (int e = 0; e < E; ++e) o[r][e] = fmaf(p, vv[e], o[r][e]);
							}
						}
					}
					if constexpr (RMW >= 4) __syncwarp(); // the scratch is read before the next batches write it
				}
			}
			__syncwarp();
			if (lane == 0) mbar_arrive(&empty[s]);
			key_base += T;
		}
		if (append && lane == 0) mbar_arrive(&qempty[sl]); // the new keys are no longer needed
		n_new = 0;
		finish_piece(i == n_mine && !s_flags[0]);
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

template <int D, typename KV, int RM>
__global__ void __launch_bounds__((NW + 1) * 32, 1) decode_kernel(const DecodePlan P)
{
	decode_body<D, KV, RM, false>(P, nullptr);
}

// A small launch: its job table and CTA starts come with the parameters.
template <int D, typename KV, int RM>
__global__ void __launch_bounds__((NW + 1) * 32, 1)
	decode_kernel_inline(const DecodePlan P, const __grid_constant__ InlineTable tab)
{
	decode_body<D, KV, RM, true>(P, tab.b);
}

// The end of a split call on this GPU: a CTA per segment waits (bounded)
// until every GPU's partial of the segment has landed in this GPU's receive
// buffer, merges them in rank order (nnc_attn_merge, then nnc_attn_finish)
// into this GPU's output rows, and clears the segment's count for this
// parity's next call. A rank that never arrives makes the wait time out with
// DEVERR_SPLIT instead of hanging; the host reports it as NNCU_ERR_TIMEOUT.
// The timeout also poisons this GPU's group: a late arrival may still count
// into this call's counters, so no later merge trusts them (each fails at
// once with DEVERR_SPLIT) until the host resets the group.
__global__ void split_merge_kernel(const DecodePlan P)
{
	const int seg = blockIdx.x;
	__shared__ int s_ok, s_job;
	if (threadIdx.x == 0)
	{
		const int* cnt = P.arrive[P.rank] + seg;
		int ok = 1;
		if (ld_acquire_sys(P.poison) != 0)
		{
			atomicExch(P.err, DEVERR_SPLIT);
			ok = 0;
		}
		const uint64_t t0 = globaltimer_ns();
		while (ok && ld_acquire_sys(cnt) < P.world)
		{
			if (globaltimer_ns() - t0 > P.wait_ns)
			{
				atomicExch(P.err, DEVERR_SPLIT);
				atomicExch(P.poison, 1);
				ok = 0;
				break;
			}
			__nanosleep(100);
		}
		int j = 0; // the segment's job (jobs hold consecutive segment ranges)
		while (j + 1 < P.n_jobs && P.jobs[j + 1].seg0 <= seg) ++j;
		s_ok = ok;
		s_job = j;
	}
	__syncthreads();
	if (!s_ok) return;
	const DevJob& J = P.jobs[s_job];
	const int seg_local = seg - J.seg0;
	const int h = seg_local / J.n_rowgroups, rg = seg_local % J.n_rowgroups;
	const int G = J.n_head / J.n_kv, RM = P.RM, D = P.D, PW = D + 4;
	const int rows_valid = min(RM, G * J.n_tok - rg * RM);
	float* out = P.out[P.rank] + (size_t)J.out_row0 * D;
	const float* base = P.recv[P.rank] + (size_t)seg * RM * PW; // rank r's partial at + r * recv_stride
	for (int idx = threadIdx.x; idx < rows_valid * D; idx += blockDim.x)
	{
		const int R = idx / D, d = idx % D;
		float M = -CUDART_INF_F;
		for (int r = 0; r < P.world; ++r) M = fmaxf(M, __ldcg(base + (size_t)r * P.recv_stride + R * PW + D));
		float acc = 0.0f, L = 0.0f;
		for (int r = 0; r < P.world; ++r)
		{
			const float* pr = base + (size_t)r * P.recv_stride + R * PW;
			const float m = __ldcg(pr + D);
			const float c = m == -CUDART_INF_F ? 0.0f : ex2(m - M);
			acc = fmaf(__ldcg(pr + d), c, acc);
			L = fmaf(__ldcg(pr + D + 1), c, L);
		}
		const int gr = rg * RM + R;
		const size_t oi = ((size_t)(gr / G) * J.n_head + (size_t)h * G + gr % G) * D + d;
		out[oi] = gated(acc * (L > 0.0f ? 1.0f / L : 0.0f), J.gate, oi);
	}
	__syncthreads();
	if (threadIdx.x == 0) atomicExch(P.arrive[P.rank] + seg, 0); // ready for this parity's next call
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
int launch_one(const DecodePlan& P, const InlineTable* tab, cudaStream_t st)
{
	using C = Cfg<D, KV, RM>;
	static bool configured[2][64] = {};
	int dev = 0;
	cudaGetDevice(&dev);
	if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
	if (!configured[tab != nullptr][dev])
	{
		cudaError_t e = tab ? cudaFuncSetAttribute(decode_kernel_inline<D, KV, RM>,
		                                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM)
		                    : cudaFuncSetAttribute(decode_kernel<D, KV, RM>,
		                                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
		if (e != cudaSuccess) return (int)e;
		configured[tab != nullptr][dev] = true;
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
	cfg.numAttrs = P.fused ? 0 : 1; // appending itself, it follows the stream's previous work in full
	if (tab) return (int)cudaLaunchKernelEx(&cfg, decode_kernel_inline<D, KV, RM>, P, *tab);
	return (int)cudaLaunchKernelEx(&cfg, decode_kernel<D, KV, RM>, P);
}

template <int D, typename KV>
int launch_rows(const DecodePlan& P, const InlineTable* tab, cudaStream_t st)
{
	constexpr int E = D / 32;
	switch (P.RM)
	{
	case 1: return launch_one<D, KV, 1>(P, tab, st);
	case 2: return launch_one<D, KV, 2>(P, tab, st);
	case 4: return launch_one<D, KV, 4>(P, tab, st);
	case 8:
		if constexpr (8 * E <= 64) return launch_one<D, KV, 8>(P, tab, st);
		break;
	case 16:
		if constexpr (16 * E <= 64) return launch_one<D, KV, 16>(P, tab, st);
		break;
	case 32:
		if constexpr (32 * E <= 64) return launch_one<D, KV, 32>(P, tab, st);
		break;
	default: break;
	}
	return (int)cudaErrorInvalidValue;
}

template <typename KV>
int launch_dims(const DecodePlan& P, const InlineTable* tab, cudaStream_t st)
{
	switch (P.D)
	{
	case 64: return launch_rows<64, KV>(P, tab, st);
	case 128: return launch_rows<128, KV>(P, tab, st);
	case 256: return launch_rows<256, KV>(P, tab, st);
	case 512: return launch_rows<512, KV>(P, tab, st);
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
template <int D, typename KV>
int fuse_tokens_rows(int RM)
{
	constexpr int E = D / 32;
	switch (RM)
	{
	case 1: return Cfg<D, KV, 1>::NT;
	case 2: return Cfg<D, KV, 2>::NT;
	case 4: return Cfg<D, KV, 4>::NT;
	case 8:
		if constexpr (8 * E <= 64) return Cfg<D, KV, 8>::NT;
		break;
	case 16:
		if constexpr (16 * E <= 64) return Cfg<D, KV, 16>::NT;
		break;
	case 32:
		if constexpr (32 * E <= 64) return Cfg<D, KV, 32>::NT;
		break;
	default: break;
	}
	return 0;
}

template <typename KV>
int fuse_tokens_dims(int D, int RM)
{
	switch (D)
	{
	case 64: return fuse_tokens_rows<64, KV>(RM);
	case 128: return fuse_tokens_rows<128, KV>(RM);
	case 256: return fuse_tokens_rows<256, KV>(RM);
	case 512: return fuse_tokens_rows<512, KV>(RM);
	default: return 0;
	}
}
} // namespace

int decode_fuse_tokens(int D, int kv_type, int RM)
{
	switch (kv_type)
	{
	case KV_F32: return fuse_tokens_dims<kv_f32>(D, RM);
	case KV_BF16: return fuse_tokens_dims<kv_bf16>(D, RM);
	default: return fuse_tokens_dims<kv_f16>(D, RM);
	}
}


int launch_decode(const DecodePlan& P, void* stream, const InlineTable* tab)
{
	if (P.n_ctas == 0) return 0;
	auto st = static_cast<cudaStream_t>(stream);
	switch (P.kv_type)
	{
	case KV_F32: return launch_dims<kv_f32>(P, tab, st);
	case KV_BF16: return launch_dims<kv_bf16>(P, tab, st);
	default: return launch_dims<kv_f16>(P, tab, st);
	}
}

int launch_split_wait(const DecodePlan& P, void* stream)
{
	split_merge_kernel<<<(unsigned)P.n_segments, 256, 0, static_cast<cudaStream_t>(stream)>>>(P);
	return (int)cudaGetLastError();
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
