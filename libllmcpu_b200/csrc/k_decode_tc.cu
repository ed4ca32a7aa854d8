// k_decode_tc.cu -- decode and verify attention on the tensor cores, for
// 16-bit (f16 or bf16) caches with several query rows per KV head.
//
// The same attention as k_decode.cu (libnnc's nnc_attn_block / merge /
// finish, src/libnnc/nn_ops.cpp:351-499, dispatched by attend_token /
// attend_blocks, src/libnnc/model.cpp:1251-1319) and the same work plan
// (segments of RM query rows, cut into chunks of whole tiles of T keys at
// absolute positions, plan.cpp), but the two products run on tcgen05:
//
//   S^T = K Q^T    M = the tile's keys, N = the segment's rows, K = head_dim
//   O^T = V^T P^T  M = head_dim,        N = the segment's rows, K = the keys
//
// The keys are the M dimension because a segment has only a few rows (8 for
// a Gemma-3-4B verify block, 4 for a Llama decode token): the rows are N.
// fp32 accuracy is kept by splitting each 16-bit operand the cache type
// cannot hold exactly into a high and a low half: Q = Q_hi + Q_lo and
// P = P_hi + P_lo, the halves side by side along N (N = 2 RM), so one MMA
// gives both products and the two columns are summed in fp32 (the cache's K
// and V are exact in their own type). The weights are formed as
// 2^8 exp2(s - m) so that their low halves stay in the normal range.
//
// Roles (12 warps):
//  * warp 0 streams the K tiles with TMA (128-byte-swizzled 64-column
//    panels, a tensor map over the cache buffer [planes][rows][head_dim])
//    and fills the q slot (job descriptor, raw q rows, gains, RoPE tables)
//    of each piece; warp 2 streams the V tiles; each into its own ring;
//  * warp 1 owns the TMEM allocation and, from one lane, issues the MMAs,
//    polling for whichever is ready first: the next S (into one of four TMEM
//    buffers, up to three tiles ahead of the softmax) or the next O (into
//    one of two);
//  * warp 3 appends the new tokens' K/V rows when their raw rows fit the q
//    slot (decode and short verify): the piece holding them normalises,
//    rotates and narrows them, stores them to the cache (first row group),
//    and writes them into the K and V stages of the tiles that hold them once
//    those have landed, before the MMAs read the stages. Longer batches have
//    K1 (k_prep.cu) append first; this kernel is then its programmatic
//    dependent and waits for it only before the tiles that hold the new rows;
//  * warps 4-7 and 8-11 are two softmax groups (each reaching TMEM lanes
//    0-127): together they normalise and rotate the q rows and write the Q
//    operand; then group g takes the tiles i with i % 2 == g, keeping its own
//    online softmax state: read S, scale, soft-cap, mask by each row's span,
//    take the row maxima across the tile (warp shuffles, then the group's
//    warps through shared memory), fold the group's previous O into
//    registers with the running maximum's correction (base 2), write P. At a
//    piece's end group 1 hands its (m, l, o) to group 0 through TMEM and
//    shared memory; group 0 merges them and writes the output, or a partial
//    (o, m, l) merged in order by the segment's last piece (decode.cuh), as
//    in k_decode.cu.
// Every wait is bounded; a timed-out wait records an error and the CTA steps
// through without waiting further.
#include <cuda.h>
#include <cuda_runtime.h>

#include <math_constants.h>

#include "common.cuh"
#include "decode.cuh"
#include "tc.cuh"

namespace nncu
{
namespace
{

constexpr int TC_THREADS = 384;   // 12 warps (roles above)
constexpr int CW0 = 4;            // the first softmax warp; warps 4-7 and 8-11 each reach TMEM lanes 0-127
constexpr int NCW = 4;            // warps per softmax group
constexpr int NSG = 2;            // softmax groups: group g takes the tiles i with i % 2 == g
constexpr int TC_SMEM_LIMIT = 232448;
constexpr int TC_TILE = 32768;    // one tile's K (or V) rows in bytes
constexpr float TC_LOG2E = 1.4426950408889634f;
constexpr float P_SHIFT = 8.0f;   // weights are 2^P_SHIFT exp2(s - m)

template <int D, int NR>
struct TcCfg
{
	static constexpr int T = TC_TILE / (D * 2);     // keys per tile: 256, 128, 64
	static constexpr int MQ = T >= 128 ? 128 : 64;  // M of a Q K^T MMA (keys)
	static constexpr int NQB = T / MQ;              // Q K^T MMA blocks per tile
	static constexpr int MP = D >= 128 ? 128 : 64;  // M of a P V MMA (head_dim)
	static constexpr int NPB = D / MP;              // P V MMA blocks
	static constexpr int N = 2 * NR;                // MMA N: the rows' high halves, then their low halves
	static constexpr int KP = D / 64;               // 64-column panels of a row
	static constexpr int PANEL = T * 128;           // one panel of a tile: T rows of 128 bytes
	static constexpr int QPANEL = N * 128;          // one panel of the Q operand
	static constexpr int QBYTES = KP * QPANEL;
	static constexpr int PPANEL = N * 128;          // one 64-key panel of the P operand
	static constexpr int PBYTES = (T / 64) * PPANEL;
	// the q slot (floats): descriptor and 4 info words, raw q rows, q gains,
	// inverse frequencies, frequency factors; when this kernel appends the new
	// tokens itself, the k gains and the new tokens' raw k rows, then v rows
	static constexpr int QHEAD = (int)(sizeof(DevJob) / 4) + 4;
	static constexpr int QROWS = QHEAD;
	static constexpr int QGAIN = QROWS + NR * D;
	static constexpr int QINV = QGAIN + D;
	static constexpr int QFF = QINV + D / 2;
	static constexpr int QKG = QFF + D / 2;
	static constexpr int QNEW = QKG + D;
	static constexpr int RED = NSG * 2 * NCW * NR + 2 * NR; // per group two buffers of per-warp row values; m, l of group 1
	static constexpr int FIXED0 = QBYTES + 2 * PBYTES + QNEW * 4 + RED * 4 + 512;
	// three stages of K and V tiles where they fit, else two; then as many new
	// tokens (up to 8) as what is left holds
	static constexpr int LEFT3 = TC_SMEM_LIMIT - 1024 - 3 * 2 * TC_TILE - FIXED0;
	static constexpr int STAGES = LEFT3 >= 0 ? 3 : 2;
	static constexpr int LEFT = TC_SMEM_LIMIT - 1024 - STAGES * 2 * TC_TILE - FIXED0;
	static constexpr int NT_FIT = LEFT / (2 * D * 4);
	static constexpr int NT = NT_FIT > 8 ? 8 : NT_FIT; // (their narrowed rows stay in the append warp's registers)
	static constexpr int SLOT = QNEW + 2 * NT * D;
	static constexpr int OFF_K = 0;
	static constexpr int OFF_V = STAGES * TC_TILE;
	static constexpr int OFF_Q = 2 * STAGES * TC_TILE;
	static constexpr int OFF_P = OFF_Q + QBYTES;
	static constexpr int OFF_SLOT = OFF_P + 2 * PBYTES;
	static constexpr int OFF_RED = OFF_SLOT + SLOT * 4;
	static constexpr int OFF_BAR = OFF_RED + RED * 4;
	static constexpr int SMEM = OFF_BAR + 512 + 1024; // + alignment slack
	static constexpr int S_COLS = NQB * N;            // TMEM columns of one S buffer
	static constexpr int O_COLS = NPB * N;            // of one O buffer
	static constexpr int X_COLS = NPB * NR;           // group 1's o, handed to group 0 at a piece's end
	// S buffers: four where TMEM holds them (S runs three tiles ahead of P V), else two
	static constexpr int NSB = 4 * S_COLS + 2 * O_COLS + X_COLS <= 256 ? 4 : 2;
	static constexpr int SA = NSB - 1;                // tiles S runs ahead
	static constexpr int O_BASE = NSB * S_COLS;       // first column of the O buffers
	static constexpr int X_BASE = O_BASE + 2 * O_COLS;
	static constexpr int TMEM_COLS = X_BASE + X_COLS <= 128 ? 128 : 256;
	static_assert(X_BASE + X_COLS <= 256, "TMEM columns");
	static_assert(LEFT >= 0, "shared memory for two stages");
	static_assert(SMEM <= TC_SMEM_LIMIT, "shared memory");
	static_assert(NR == 8 || NR == 16, "rows per segment");
	static_assert(QBYTES % 1024 == 0 && PBYTES % 1024 == 0 && (SLOT * 4) % 16 == 0, "operand alignment");
};

// The tensor maps of a launch whose jobs carry none (the no-allocation call).
struct alignas(64) TcMaps
{
	CUtensorMap k, v;
};

// Byte offset of element (row n, column c) in a 128-byte-swizzled K-major
// operand panel of 64 columns (the layout TMA writes with SWIZZLE_128B and
// tcgen05 reads through sdesc): 16-byte chunk c / 8 of row n sits at chunk
// (c / 8) ^ (n % 8).
__device__ __forceinline__ int swz(int n, int c) { return n * 128 + ((((c >> 3) ^ n) & 7) << 4) + ((c & 7) << 1); }

template <typename KV>
struct Half16;
template <>
struct Half16<kv_f16>
{
	static __device__ __forceinline__ uint16_t bits(float x, float& back)
	{
		const __half h = __float2half_rn(x);
		back = __half2float(h);
		return __half_as_ushort(h);
	}
};
template <>
struct Half16<kv_bf16>
{
	static __device__ __forceinline__ uint16_t bits(float x, float& back)
	{
		const __nv_bfloat16 h = __float2bfloat16_rn(x);
		back = __bfloat162float(h);
		return __bfloat16_as_ushort(h);
	}
};

// x as a high and a low half in the cache's 16-bit type: hi = round(x),
// lo = round(x - hi).
template <typename KV>
__device__ __forceinline__ void split16(float x, uint16_t& hi, uint16_t& lo)
{
	float back, unused;
	hi = Half16<KV>::bits(x, back);
	lo = Half16<KV>::bits(x - back, unused);
}

// The max (or sum) of NR per-lane values across the warp: afterwards lane l
// holds row l >> (5 - log2 NR)'s result (the halving exchange of
// transpose_reduce, with max or add).
template <int NR, bool MAX>
__device__ __forceinline__ float warp_rows(const float (&v)[NR], int lane)
{
	float cur[NR];
#pragma unroll
	for (int r = 0; r < NR; ++r) cur[r] = v[r];
	int n = NR;
#pragma unroll
	for (int mask = 16; mask >= 1; mask >>= 1)
	{
		if (n > 1)
		{
			const int h = n / 2;
			const bool upper = (lane & mask) != 0;
#pragma unroll
			for (int r = 0; r < NR / 2; ++r)
			{
				if (r < h)
				{
					const float send = upper ? cur[r] : cur[r + h];
					const float mine = upper ? cur[r + h] : cur[r];
					const float got = __shfl_xor_sync(0xffffffffu, send, mask);
					cur[r] = MAX ? fmaxf(mine, got) : mine + got;
				}
			}
			n = h;
		}
		else
		{
			const float got = __shfl_xor_sync(0xffffffffu, cur[0], mask);
			cur[0] = MAX ? fmaxf(cur[0], got) : cur[0] + got;
		}
	}
	return cur[0];
}

// The kernel's body. INL: the job table and the CTA starts are the bytes of
// `tab` (a kernel parameter) instead of P.jobs / P.cta_start, and every job
// carries its own tensor maps (`maps` is then NULL).
template <int D, typename KV, int NR, bool INL>
__device__ __forceinline__ void decode_tc_body(const DecodePlan& P, const TcMaps* maps, const unsigned char* tab)
{
	using C = TcCfg<D, NR>;
	constexpr int T = C::T, N = C::N, PW = D + 4;
	constexpr int STAGES = C::STAGES;
	constexpr bool BF = KV::id == KV_BF16;

	extern __shared__ unsigned char smem_raw[];
	unsigned char* smem =
		reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
	float* slot = reinterpret_cast<float*>(smem + C::OFF_SLOT);
	float* red = reinterpret_cast<float*>(smem + C::OFF_RED); // [2][NCW][NR]
	uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
	uint64_t* k_full = bars;                  // [STAGES]
	uint64_t* k_empty = k_full + STAGES;      // [STAGES]
	uint64_t* v_full = k_empty + STAGES;      // [STAGES]
	uint64_t* v_empty = v_full + STAGES;      // [STAGES]
	uint64_t* s_full = v_empty + STAGES;      // [NSB]
	uint64_t* s_empty = s_full + C::NSB;      // [NSB]
	uint64_t* p_full = s_empty + C::NSB;      // [2]
	uint64_t* o_full = p_full + 2;            // [2]
	uint64_t* o_empty = o_full + 2;           // [2]
	uint64_t* q_full = o_empty + 2;           // the slot holds a piece
	uint64_t* q_empty = q_full + 1;           // the slot may be refilled (softmax warps and the append warp)
	uint64_t* q_ready = q_empty + 1;          // the Q operand is written, the piece's patch range is known
	uint64_t* mma_done = q_ready + 1;
	uint64_t* k_patched = mma_done + 1;       // a tile's new K rows are in its stage
	uint64_t* v_patched = k_patched + 1;      // a tile's new V rows are in its stage
	uint64_t* k_land = v_patched + 1;         // a tile holding new rows has landed (the append warp waits,
	uint64_t* v_land = k_land + 1;            // in order: a stage's own barrier may be phases ahead of it)
	uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(v_land + 1);
	// [0] abort, [1] last piece, [2] the piece's tiles, [3] / [4] the first and
	// last of its tiles (CTA-wide index) whose new rows this kernel patches in
	volatile int* flags = reinterpret_cast<volatile int*>(tmem_slot + 2);
	CtaStart* s_start = reinterpret_cast<CtaStart*>(smem + C::OFF_BAR + 384);

	const DevJob* jobs = INL ? reinterpret_cast<const DevJob*>(tab) : P.jobs;
	const CtaStart* starts =
		INL ? reinterpret_cast<const CtaStart*>(tab + ((P.n_jobs * sizeof(DevJob) + 15) & ~size_t(15))) : P.cta_start;
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	if (threadIdx.x == 0)
	{
		*s_start = starts[blockIdx.x];
		for (int s = 0; s < STAGES; ++s)
		{
			mbar_init(&k_full[s], 1);
			mbar_init(&k_empty[s], 1);
			mbar_init(&v_full[s], 1);
			mbar_init(&v_empty[s], 1);
		}
		for (int b = 0; b < C::NSB; ++b)
		{
			mbar_init(&s_full[b], 1);
			mbar_init(&s_empty[b], 32 * NCW); // tile i's S is read by softmax group i % 2
		}
		for (int b = 0; b < 2; ++b)
		{
			mbar_init(&p_full[b], 32 * NCW); // P and O buffer b belong to softmax group b
			mbar_init(&o_full[b], 1);
			mbar_init(&o_empty[b], 32 * NCW);
		}
		mbar_init(q_full, 1);
		mbar_init(q_empty, 2);
		mbar_init(q_ready, NSG * 32 * NCW + 1);
		mbar_init(mma_done, 1);
		mbar_init(k_patched, 1);
		mbar_init(v_patched, 1);
		mbar_init(k_land, 1);
		mbar_init(v_land, 1);
		for (int f = 0; f < 5; ++f) flags[f] = 0;
		fence_barrier_init();
	}
	if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = *tmem_slot;
	const int n_mine = s_start->n_tiles;
	const int* info = reinterpret_cast<const int*>(slot + C::QHEAD - 4);

	if (warp == 0 || warp == 2)
	{
		// ---- TMA: warp 0 the K tiles (and each piece's q slot), warp 2 the V tiles ----
		if (lane == 0 && n_mine > 0)
		{
			const bool is_k = warp == 0;
			uint64_t* full = is_k ? k_full : v_full;
			uint64_t* empty = is_k ? k_empty : v_empty;
			unsigned char* ring = smem + (is_k ? C::OFF_K : C::OFF_V);
			const CtaStart S = *s_start;
			// the first tile goes out before the job is read, from the start record
			// (tensor maps, first row, plane)
			if (S.pre > 0)
			{
				const CUtensorMap* map = reinterpret_cast<const CUtensorMap*>(is_k ? S.k0 : S.v0);
				mbar_arrive_expect_tx(&full[0], TC_TILE);
#pragma unroll
				for (int p = 0; p < C::KP; ++p) tma3(ring + p * C::PANEL, map, 64 * p, S.pad_[0], S.pad_[1], &full[0]);
			}
			Cursor cur;
			cur.job = S.job;
			cur.seg = S.seg;
			cur.tis = S.tis;
			cursor_load<INL>(jobs, P.n_jobs, cur);
			int i = 0, piece = 0, landed = 0; // landed: tiles sent to the land barrier
			bool waited = false;
			for (int left = n_mine; left > 0 && !flags[0];)
			{
				const DevJob& J = jobs[cur.job];
				const int n = min(min(cur.n_tiles - cur.tis, J.chunk - cur.tis % J.chunk), left);
				const int h = cur.seg / J.n_rowgroups, rg = cur.seg % J.n_rowgroups;
				const bool fresh = holds_new_rows(J, cur.tis, n, T);
				if (is_k)
				{
					// the piece's descriptor, q rows, gains and RoPE tables (and, when
					// this kernel appends, the k gains and the new raw k, v rows of
					// its KV head), once the previous piece is done with the slot
					if (piece >= 1 && !mbar_wait_bounded(q_empty, (uint32_t)((piece - 1) & 1), P.err, DEVERR_WAIT_EMPTY))
					{
						flags[0] = 1;
						break;
					}
					const bool append = P.fused && fresh;
					const int G = J.n_head / J.n_kv;
					const int rows = seg_rows(J, rg, NR);
					int* inf = reinterpret_cast<int*>(slot + C::QHEAD - 4);
					inf[0] = n;
					inf[1] = cur.tis;
					inf[2] = cur.seg;
					inf[3] = append;
					const int half = J.n_rot / 2;
					const uint32_t inv_bytes = (uint32_t)((half * 4 + 15) & ~15);
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
					// also releases the info words (and an inline descriptor) above
					mbar_arrive_expect_tx(q_full, bytes - (INL ? (uint32_t)sizeof(DevJob) : 0u));
					if constexpr (!INL) bulk_g2s(slot, &J, (uint32_t)sizeof(DevJob), q_full);
					if (J.q_gamma) bulk_g2s(slot + C::QGAIN, J.q_gamma, (uint32_t)(D * 4), q_full);
					if (inv_bytes) bulk_g2s(slot + C::QINV, J.rope_inv, inv_bytes, q_full);
					if (J.freq_factors) bulk_g2s(slot + C::QFF, J.freq_factors, (uint32_t)(half * 4), q_full);
					for (int r = 0; r < rows;)
					{
						const int gr = rg * NR + r, t = gr / G, g = gr % G;
						const int run = min(G - g, rows - r);
						bulk_g2s(slot + C::QROWS + r * D, J.q + ((size_t)t * J.n_head + (size_t)h * G + g) * D,
						         (uint32_t)(run * D * 4), q_full);
						r += run;
					}
					if (append)
					{
						if (J.k_gamma) bulk_g2s(slot + C::QKG, J.k_gamma, (uint32_t)(D * 4), q_full);
						for (int t = 0; t < J.n_tok; ++t)
						{
							const size_t src = ((size_t)t * J.n_kv + h) * D;
							bulk_g2s(slot + C::QNEW + t * D, J.k + src, (uint32_t)(D * 4), q_full);
							bulk_g2s(slot + C::QNEW + (C::NT + t) * D, J.v + src, (uint32_t)(D * 4), q_full);
						}
					}
				}
				++piece;
				const CUtensorMap* map = static_cast<const CUtensorMap*>(is_k ? J.tmap_k : J.tmap_v);
				if (!map) map = is_k ? &maps->k : &maps->v; // an inline launch's jobs all carry maps
				const int plane = J.plane0 + h;
				for (int k = 0; k < n; ++k, ++i)
				{
					// while K1 appends, the rows it writes come from the preceding grid:
					// wait for it before the tiles that hold them
					if (!P.fused && !waited && holds_new_rows(J, cur.tis + k, 1, T))
					{
						griddep_wait();
						waited = true;
					}
					if (i < S.pre) continue; // issued at the start
					const int s = i % STAGES;
					if (i >= STAGES &&
					    !mbar_wait_bounded(&empty[s], (uint32_t)(((i / STAGES) - 1) & 1), P.err, DEVERR_WAIT_EMPTY))
					{
						flags[0] = 1;
						break;
					}
					if (flags[0]) break;
					const int row0 = ((J.tile_lo + cur.tis + k) * T) % J.rows;
					unsigned char* st = ring + s * TC_TILE;
					// a tile whose new rows the append warp writes lands on its own
					// barrier; the stage's barrier still completes its phase (the MMAs
					// wait for the patched tile instead)
					uint64_t* bar = &full[s];
					if (P.fused && holds_new_rows(J, cur.tis + k, 1, T))
					{
						mbar_arrive(&full[s]);
						bar = is_k ? k_land : v_land;
						++landed;
					}
					mbar_arrive_expect_tx(bar, TC_TILE);
#pragma unroll
					for (int p = 0; p < C::KP; ++p) tma3(st + p * C::PANEL, map, 64 * p, row0, plane, bar);
				}
				left -= n;
				cur.tis += n;
				if (cur.tis >= cur.n_tiles) cursor_next_segment<INL>(jobs, P.n_jobs, cur);
			}
			if (flags[0])
			{
				// do not leave while a copy may still land in this CTA's shared memory
				for (int k = max(0, i - STAGES); k < max(i, S.pre); ++k)
					mbar_wait_bounded(&full[k % STAGES], (uint32_t)((k / STAGES) & 1), nullptr, 0);
				if (is_k && piece > 0) mbar_wait_bounded(q_full, (uint32_t)((piece - 1) & 1), nullptr, 0);
				if (landed > 0) mbar_wait_bounded(is_k ? k_land : v_land, (uint32_t)((landed - 1) & 1), nullptr, 0);
			}
		}
		__syncwarp(); // the whole warp meets the final barrier together
	}
	else if (warp == 1)
	{
		// ---- MMA issue: S_{i+1} = K_{i+1} Q^T, then O_i = V_i^T P_i^T ----
		if (lane == 0 && n_mine > 0)
		{
			constexpr uint32_t ID_QK = tc_idesc(C::MQ, N, BF, false, false);
			constexpr uint32_t ID_PV = tc_idesc(C::MP, N, BF, true, false);
			const uint32_t kb0 = smem_u32(smem + C::OFF_K), vb0 = smem_u32(smem + C::OFF_V);
			const uint32_t qa = smem_u32(smem + C::OFF_Q), pa0 = smem_u32(smem + C::OFF_P);
			// descriptors of the rings' first stages, of Q and of the first P
			// buffer (shared memory stays below 256 KB, so adding an offset to the
			// 14-bit start-address field never carries out of it)
			const uint64_t adesc_k0 = sdesc(kb0, 16, 1024), adesc_v0 = sdesc(vb0, C::PANEL, 1024);
			const uint64_t bdesc_q = sdesc(qa, 16, 1024), bdesc_p0 = sdesc(pa0, 16, 1024);
			bool ok = true;
			int patch_lo = -1, patch_hi = -2, kp = 0, vp = 0; // the piece's patched tiles; patches seen
			// whether tile j's K (or V) is in its stage: landed, or patched by the append warp
			auto k_ready = [&](int j) {
				return j >= patch_lo && j <= patch_hi ? mbar_test(k_patched, (uint32_t)(kp & 1))
				                                      : mbar_test(&k_full[j % STAGES], (uint32_t)((j / STAGES) & 1));
			};
			auto v_ready = [&](int j) {
				return j >= patch_lo && j <= patch_hi ? mbar_test(v_patched, (uint32_t)(vp & 1))
				                                      : mbar_test(&v_full[j % STAGES], (uint32_t)((j / STAGES) & 1));
			};
			// S_j = K_j Q^T into S buffer j % NSB
			auto issue_qk = [&](int j) {
				const int s = j % STAGES, b = j % C::NSB;
				if (j >= patch_lo && j <= patch_hi) ++kp;
				tc_fence_after();
				const uint32_t ts = tmem + b * C::S_COLS;
				// the descriptors of the stage and of Q once; each MMA adds its
				// offset (in 16-byte units) to the start-address field
				const uint64_t ad = adesc_k0 + (uint64_t)((s * TC_TILE) >> 4);
#pragma unroll
				for (int qb = 0; qb < C::NQB; ++qb)
#pragma unroll
					for (int kk = 0; kk < D / 16; ++kk)
						mma_f16(ts + qb * N, ad + (uint64_t)(((kk >> 2) * C::PANEL + qb * C::MQ * 128 + (kk & 3) * 32) >> 4),
						        bdesc_q + (uint64_t)(((kk >> 2) * C::QPANEL + (kk & 3) * 32) >> 4), ID_QK, kk > 0 ? 1u : 0u);
				mma_commit(&s_full[b]);
				mma_commit(&k_empty[s]);
			};
			// O_j = V_j^T P_j^T into O buffer j % 2
			auto issue_pv = [&](int j) {
				const int s = j % STAGES, b = j & 1;
				if (j >= patch_lo && j <= patch_hi) ++vp;
				tc_fence_after();
				const uint32_t to = tmem + C::O_BASE + b * C::O_COLS;
				const uint64_t ad = adesc_v0 + (uint64_t)((s * TC_TILE) >> 4);
				const uint64_t bd = bdesc_p0 + (uint64_t)((b * C::PBYTES) >> 4);
#pragma unroll
				for (int mb = 0; mb < C::NPB; ++mb)
#pragma unroll
					for (int kk = 0; kk < T / 16; ++kk)
						mma_f16(to + mb * N, ad + (uint64_t)((mb * 2 * C::PANEL + kk * 2048) >> 4),
						        bd + (uint64_t)(((kk >> 2) * C::PPANEL + (kk & 3) * 32) >> 4), ID_PV, kk > 0 ? 1u : 0u);
				mma_commit(&o_full[b]);
				mma_commit(&v_empty[s]);
			};
			// Within a piece, whichever is ready first: the next S (its K landed,
			// its buffer read by the softmax; up to NSB - 1 tiles ahead of the
			// softmax) or the next O (its P written, its V landed, its buffer
			// folded). Not across a piece's end: the next piece's Q is written
			// only once this piece is done. A wait without progress gives up after
			// the bounded-wait limit.
			int i = 0;
			for (int piece = 0; ok && i < n_mine; ++piece)
			{
				ok = !flags[0] && mbar_wait_bounded(q_ready, (uint32_t)(piece & 1), P.err, DEVERR_WAIT_FULL);
				if (!ok) break;
				const int n = flags[2];
				patch_lo = flags[3];
				patch_hi = flags[4];
				const int end = i + n;
				int nq = i, np = i;
				uint64_t t_prog = globaltimer_ns();
				for (uint32_t spin = 0; np < end; ++spin)
				{
					bool did = false;
					if (nq < end && nq < np + C::NSB && k_ready(nq) &&
					    (nq < C::NSB || mbar_test(&s_empty[nq % C::NSB], (uint32_t)(((nq / C::NSB) - 1) & 1))))
					{
						issue_qk(nq++);
						did = true;
					}
					if (np < nq && mbar_test(&p_full[np & 1], (uint32_t)((np >> 1) & 1)) && v_ready(np) &&
					    (np < 2 || mbar_test(&o_empty[np & 1], (uint32_t)(((np >> 1) - 1) & 1))))
					{
						issue_pv(np++);
						did = true;
					}
					if (did)
						t_prog = globaltimer_ns();
					else if ((spin & 255u) == 255u && (flags[0] || globaltimer_ns() - t_prog > WAIT_LIMIT_NS))
					{
						if (!flags[0]) atomicCAS(P.err, 0, DEVERR_WAIT_FULL);
						ok = false;
						break;
					}
				}
				i = end;
			}
			if (!ok) flags[0] = 1;
			// every MMA issued has completed before TMEM is freed
			mma_commit(mma_done);
			mbar_wait_bounded(mma_done, 0, nullptr, 0);
		}
		__syncwarp(); // the whole warp meets the final barrier together
	}
	else if (warp == 3)
	{
		// ---- the append warp: for a piece holding the new tokens (when K1 does
		// not run), their K/V rows through attention_forward's per-head steps
		// (model.cpp:1616-1694: K RMSNorm with its gains and RoPE, Gemma 4's V
		// norm), narrowed to the cache type, stored to the cache (first row
		// group only), and written into the landed K and V stages of the tiles
		// that hold them, in place of the rows TMA brought ----
		int i = 0, nl = 0; // nl: patched tiles so far (the land barriers' phases)
		for (int piece = 0; i < n_mine; ++piece)
		{
			bool ok = !flags[0] && mbar_wait_bounded(q_full, (uint32_t)(piece & 1), P.err, DEVERR_WAIT_FULL);
			ok = __all_sync(0xffffffffu, ok);
			if (!ok)
			{
				if (lane == 0)
				{
					flags[0] = 1;
					mbar_arrive(q_ready);
				}
				break;
			}
			const DevJob& J = *reinterpret_cast<const DevJob*>(slot);
			const int n_piece = info[0], tis0 = info[1], seg_local = info[2];
			const bool append = info[3] != 0;
			const int h = seg_local / J.n_rowgroups, rg = seg_local % J.n_rowgroups;
			const int lo = max(J.pos0, J.key_lo), hi = min(J.pos0 + J.n_tok, J.key_hi); // positions appended
			const int key0 = (J.tile_lo + tis0) * T;                                     // the piece's first key
			int plo = -1, phi = -2;
			if (append)
			{
				plo = i + max(0, (lo - key0) / T);
				phi = i + min(n_piece - 1, (hi - 1 - key0) / T);
			}
			if (lane == 0)
			{
				flags[3] = plo;
				flags[4] = phi;
				mbar_arrive(q_ready); // after the softmax warps' writes of flags[2]: the MMA reads both
			}
			// the rows, narrowed, stay in this warp's registers (lane c holds 16-byte
			// chunk c of each), so that the slot goes back to the producer at once
			uint4 krow[C::NT], vrow[C::NT];
			const int n_tok = J.n_tok, pos0 = J.pos0;
			if (append)
			{
				// only the tiles holding the new rows need them (a piece's last,
				// usually): let the softmax warps' q work go first, which the
				// first tile waits for
				if (!mbar_wait_bounded(q_ready, (uint32_t)(piece & 1), P.err, DEVERR_WAIT_FULL) && lane == 0) flags[0] = 1;
				__syncwarp();
				const float* ff = J.freq_factors ? slot + C::QFF : nullptr;
#pragma unroll
				for (int t = 0; t < C::NT; ++t)
				{
					if (t >= n_tok) break;
					float* kb = slot + C::QNEW + t * D;
					float* vb = slot + C::QNEW + (C::NT + t) * D;
					prep_buf(kb, D, J.k_gamma ? slot + C::QKG : nullptr, false, J.eps, true, J.n_rot, J.rope_mode,
					         (float)(pos0 + t) * J.rope_scale, slot + C::QINV, ff);
					narrow_buf<KV>(kb, D);
					prep_buf(vb, D, nullptr, J.v_rmsnorm != 0, J.eps, false, 0, 0, 0.0f, nullptr, nullptr);
					narrow_buf<KV>(vb, D);
					if (lane < D / 8)
					{
						krow[t] = reinterpret_cast<const uint4*>(kb)[lane];
						vrow[t] = reinterpret_cast<const uint4*>(vb)[lane];
					}
				}
			}
			char* const Kc = J.K + (size_t)h * J.head_bytes;
			char* const Vc = J.V + (size_t)h * J.head_bytes;
			const int rows_c = J.rows;
			__syncwarp();
			if (lane == 0) mbar_arrive(q_empty); // done with the slot
			if (append)
			{
				// the append loop (model.cpp:1662-1694): row pos % rows of the cache,
				// by the first row group's piece holding the position
#pragma unroll
				for (int t = 0; t < C::NT; ++t)
				{
					if (t >= n_tok) break;
					const int pos = pos0 + t;
					if (rg == 0 && lane < D / 8 && pos >= lo && pos < hi && pos >= key0 && pos < key0 + n_piece * T)
					{
						const size_t off = (size_t)(pos % rows_c) * D * 2;
						reinterpret_cast<uint4*>(Kc + off)[lane] = krow[t];
						reinterpret_cast<uint4*>(Vc + off)[lane] = vrow[t];
					}
				}
				// the tiles holding the new rows: once each landed, the rows in place
				for (int pi = plo; pi <= phi; ++pi)
				{
					const int s = pi % STAGES;
					const int tkey = key0 + (pi - i) * T; // the tile's first key
					for (int which = 0; which < 2; ++which)
					{
						bool okp = !flags[0] && mbar_wait_bounded(which == 0 ? k_land : v_land, (uint32_t)(nl & 1),
						                                          P.err, DEVERR_WAIT_FULL);
						okp = __all_sync(0xffffffffu, okp);
						if (okp)
						{
							unsigned char* stage = smem + (which == 0 ? C::OFF_K : C::OFF_V) + s * TC_TILE;
#pragma unroll
							for (int t = 0; t < C::NT; ++t)
							{
								if (t >= n_tok) break;
								const int pos = pos0 + t;
								if (pos < lo || pos >= hi || pos < tkey || pos >= tkey + T || lane >= D / 8) continue;
								const int r = pos - tkey, c = lane;
								*reinterpret_cast<uint4*>(stage + (c >> 3) * C::PANEL + r * 128 + (((c ^ r) & 7) << 4)) =
									which == 0 ? krow[t] : vrow[t];
							}
						}
						else if (lane == 0)
							flags[0] = 1;
						asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
						__syncwarp();
						if (lane == 0) mbar_arrive(which == 0 ? k_patched : v_patched);
					}
					++nl;
				}
			}
			i += n_piece;
		}
		__syncwarp();
	}
	else if (warp >= CW0)
	{
		// ---- two softmax groups: group g (warps 4 + 4g .. 7 + 4g) takes the
		// tiles i with i % 2 == g and keeps its own online softmax state; warp
		// cw of a group reaches TMEM lanes 32 cw .. 32 cw + 31 ----
		const int g = (warp - CW0) / NCW;
		const int cw = warp & 3;
		const int gtid = threadIdx.x - CW0 * 32; // 0 .. 255 over both groups
		const int ctid = gtid & (32 * NCW - 1);  // 0 .. 127 within the group
		const int gbar = 2 + g;                  // the group's named barrier
		const uint32_t lane_addr = (uint32_t)(32 * cw) << 16;
		unsigned char* qop = smem + C::OFF_Q;
		float* gred = red + g * 2 * NCW * NR;    // the group's two buffers of per-warp row values
		float* ml1 = red + NSG * 2 * NCW * NR;   // group 1's m, then l, per row
		// this thread's keys of a tile (per Q K^T block) and its head_dim
		// columns of O (per P V block); -1: none (an M = 64 block fills half
		// of each warp's lanes)
		int kx[C::NQB], dx[C::NPB];
#pragma unroll
		for (int qb = 0; qb < C::NQB; ++qb) kx[qb] = C::MQ == 128 ? qb * 128 + 32 * cw + lane : (lane < 16 ? 16 * cw + lane : -1);
#pragma unroll
		for (int mb = 0; mb < C::NPB; ++mb) dx[mb] = C::MP == 128 ? mb * 128 + 32 * cw + lane : (lane < 16 ? 16 * cw + lane : -1);
		int i = 0;
		for (int piece = 0; i < n_mine; ++piece)
		{
			const bool ok = !flags[0] && mbar_wait_bounded(q_full, (uint32_t)(piece & 1), P.err, DEVERR_WAIT_FULL);
			if (named_sync_or(1, NSG * 32 * NCW, !ok)) // every softmax thread takes the same decision
			{
				flags[0] = 1;
				break;
			}
			const DevJob& J = *reinterpret_cast<const DevJob*>(slot);
			const int n_piece = info[0], tis0 = info[1], seg_local = info[2];
			const int G = J.n_head / J.n_kv;
			const int h = seg_local / J.n_rowgroups, rg = seg_local % J.n_rowgroups;
			const int rows = seg_rows(J, rg, NR);
			float* qs = slot + C::QROWS;
			const float* ff = J.freq_factors ? slot + C::QFF : nullptr;
			// attention_forward's per-head q work (model.cpp:1616-1660), a warp per row
			for (int r = warp - CW0; r < rows; r += NSG * NCW)
				prep_buf(qs + r * D, D, J.q_gamma ? slot + C::QGAIN : nullptr, false, J.eps, true, J.n_rot,
				         J.rope_mode, (float)(J.pos0 + (rg * NR + r) / G) * J.rope_scale, slot + C::QINV, ff);
			named_sync(1, NSG * 32 * NCW);
			// the Q operand: row r's high half as operand row r, its low half as
			// row NR + r; padding rows are zero
			for (int idx = gtid; idx < NR * (D / 8); idx += NSG * 32 * NCW)
			{
				const int r = idx / (D / 8), c0 = (idx % (D / 8)) * 8;
				uint16_t hi[8], lo[8];
#pragma unroll
				for (int e = 0; e < 8; ++e)
				{
					const float x = r < rows ? qs[r * D + c0 + e] : 0.0f;
					split16<KV>(x, hi[e], lo[e]);
				}
				unsigned char* panel = qop + (c0 >> 6) * C::QPANEL;
				*reinterpret_cast<uint4*>(panel + swz(r, c0 & 63)) =
					make_uint4(hi[0] | (uint32_t)hi[1] << 16, hi[2] | (uint32_t)hi[3] << 16, hi[4] | (uint32_t)hi[5] << 16,
					           hi[6] | (uint32_t)hi[7] << 16);
				*reinterpret_cast<uint4*>(panel + swz(NR + r, c0 & 63)) =
					make_uint4(lo[0] | (uint32_t)lo[1] << 16, lo[2] | (uint32_t)lo[3] << 16, lo[4] | (uint32_t)lo[5] << 16,
					           lo[6] | (uint32_t)lo[7] << 16);
			}
			// each row's span (model_attn_span) within the launch's keys
			int first[NR], last[NR];
#pragma unroll
			for (int r = 0; r < NR; ++r)
			{
				const int gr = rg * NR + r;
				first[r] = 0;
				last[r] = -1;
				if (r < rows)
				{
					span_of(J.causal, J.window, J.pos0 + gr / G, J.n_seq, first[r], last[r]);
					first[r] = max(first[r], J.key_lo);
					last[r] = min(last[r], J.key_hi - 1);
				}
			}
			const bool softcap = J.softcap > 0.0f;
			const float sl = softcap ? J.scale / J.softcap : J.scale * TC_LOG2E, cl = J.softcap * TC_LOG2E;
			const int key_first = (J.tile_lo + tis0) * T;
			// what the end of the piece needs from the slot
			float* out = J.out;
			const float* gate = J.gate;
			const int n_head = J.n_head, n_tok = J.n_tok, seg = J.seg0 + seg_local, n_pieces = J.n_chunks;
			const int part_slot = J.part0 + seg_local * J.n_chunks + tis0 / J.chunk;
			const int part_first = J.part0 + seg_local * J.n_chunks;
			if (gtid == 0) flags[2] = n_piece;
			asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); // the Q operand, for the MMAs
			named_sync(1, NSG * 32 * NCW);
			if (gtid == 0) mbar_arrive(q_empty); // the slot is no longer read
			tc_fence_before();
			mbar_arrive(q_ready);

			float o[C::NPB][NR], m[NR], lp[NR], alpha_prev[NR];
#pragma unroll
			for (int r = 0; r < NR; ++r)
			{
				m[r] = -CUDART_INF_F;
				lp[r] = 0.0f;
				alpha_prev[r] = 0.0f;
#pragma unroll
				for (int mb = 0; mb < C::NPB; ++mb) o[mb][r] = 0.0f;
			}
			// O of this group's tile j (in TMEM once its P V is done) into o, after
			// the running maximum's correction of the group's tiles before it
			auto fold_o = [&](int j) {
				const int b = j & 1;
				bool okf = !flags[0] && mbar_wait_bounded(&o_full[b], (uint32_t)((j >> 1) & 1), P.err, DEVERR_WAIT_FULL);
				okf = __all_sync(0xffffffffu, okf);
				if (!okf)
				{
					flags[0] = 1;
					mbar_arrive(&o_empty[b]);
					return;
				}
				tc_fence_after();
				float c[C::NPB][N];
#pragma unroll
				for (int mb = 0; mb < C::NPB; ++mb)
					tmem_ld<N>(tmem + lane_addr + C::O_BASE + b * C::O_COLS + mb * N, c[mb]);
				tmem_wait_ld();
				tc_fence_before();
				mbar_arrive(&o_empty[b]);
#pragma unroll
				for (int mb = 0; mb < C::NPB; ++mb)
#pragma unroll
					for (int r = 0; r < NR; ++r) o[mb][r] = fmaf(o[mb][r], alpha_prev[r], c[mb][r] + c[mb][NR + r]);
			};

			int jprev = -1; // the group's previous tile, whose O is folded after this tile's P
			for (int k = g; k < n_piece; k += NSG)
			{
				const int ti = i + k; // this tile's CTA-wide index: its S buffer is ti % NSB, P and O ti % 2
				const int b = ti & 1, sb = ti % C::NSB;
				bool okt = !flags[0] && mbar_wait_bounded(&s_full[sb], (uint32_t)((ti / C::NSB) & 1), P.err, DEVERR_WAIT_FULL);
				okt = __all_sync(0xffffffffu, okt);
				if (!okt) flags[0] = 1;
				float s[C::NQB][NR];
				if (okt)
				{
					tc_fence_after();
					float c[C::NQB][N];
#pragma unroll
					for (int qb = 0; qb < C::NQB; ++qb) tmem_ld<N>(tmem + lane_addr + sb * C::S_COLS + qb * N, c[qb]);
					tmem_wait_ld();
#pragma unroll
					for (int qb = 0; qb < C::NQB; ++qb)
#pragma unroll
						for (int r = 0; r < NR; ++r) s[qb][r] = c[qb][r] + c[qb][NR + r];
				}
				else
				{
#pragma unroll
					for (int qb = 0; qb < C::NQB; ++qb)
#pragma unroll
						for (int r = 0; r < NR; ++r) s[qb][r] = 0.0f;
				}
				tc_fence_before();
				mbar_arrive(&s_empty[sb]);
				// scores in log2 units, soft-capped where asked, masked by each row's span
				const int key_base = key_first + k * T;
				float tmax[NR];
#pragma unroll
				for (int r = 0; r < NR; ++r) tmax[r] = -CUDART_INF_F;
#pragma unroll
				for (int qb = 0; qb < C::NQB; ++qb)
				{
					const int pos = key_base + kx[qb];
#pragma unroll
					for (int r = 0; r < NR; ++r)
					{
						float x = softcap ? tanhf(s[qb][r] * sl) * cl : s[qb][r] * sl;
						if (kx[qb] < 0 || pos < first[r] || pos > last[r]) x = -CUDART_INF_F;
						s[qb][r] = x;
						tmax[r] = fmaxf(tmax[r], x);
					}
				}
				// the tile's row maxima: across the warp, then across the group's four warps
				float* rb = gred + ((ti >> 1) & 1) * NCW * NR;
				{
					const float wm = warp_rows<NR, true>(tmax, lane);
					if ((lane & (32 / NR - 1)) == 0) rb[cw * NR + lane / (32 / NR)] = wm;
				}
				named_sync(gbar, 32 * NCW);
				float alpha[NR], mref[NR];
#pragma unroll
				for (int r = 0; r < NR; ++r)
				{
					float mt = rb[r];
#pragma unroll
					for (int w = 1; w < NCW; ++w) mt = fmaxf(mt, rb[w * NR + r]);
					const float mn = fmaxf(m[r], mt);
					alpha[r] = m[r] == -CUDART_INF_F ? 0.0f : ex2(m[r] - mn);
					m[r] = mn;
					mref[r] = (mn == -CUDART_INF_F ? 0.0f : mn) - P_SHIFT;
				}
				// the group's previous tile's O (its P V also read this P buffer
				// last), then the weights 2^8 exp2(s - m) as high and low halves into
				// P (operand row r, and NR + r)
				if (jprev >= 0) fold_o(jprev);
#pragma unroll
				for (int r = 0; r < NR; ++r) alpha_prev[r] = alpha[r];
				jprev = ti;
				unsigned char* pb = smem + C::OFF_P + b * C::PBYTES;
#pragma unroll
				for (int qb = 0; qb < C::NQB; ++qb)
				{
					if (kx[qb] < 0) continue;
					unsigned char* panel = pb + (kx[qb] >> 6) * C::PPANEL;
					const int col = kx[qb] & 63;
#pragma unroll
					for (int r = 0; r < NR; ++r)
					{
						const float p = s[qb][r] == -CUDART_INF_F ? 0.0f : ex2(s[qb][r] - mref[r]);
						lp[r] = qb == 0 ? fmaf(lp[r], alpha[r], p) : lp[r] + p;
						uint16_t hi, lo;
						split16<KV>(p, hi, lo);
						*reinterpret_cast<uint16_t*>(panel + swz(r, col)) = hi;
						*reinterpret_cast<uint16_t*>(panel + swz(NR + r, col)) = lo;
					}
				}
				if (kx[0] < 0)
				{
#pragma unroll
					for (int r = 0; r < NR; ++r) lp[r] *= alpha[r];
				}
				asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
				tc_fence_before();
				mbar_arrive(&p_full[b]);
			}
			if (jprev >= 0) fold_o(jprev);
			i += n_piece;

			// ---- the piece's end: each group's row sums; group 1 hands its (m, l, o)
			// to group 0 (o through TMEM, lanes as O's), which merges them
			// (nnc_attn_merge's formula) and gives the output or a partial ----
			// not the buffer of the group's last tile (its maxima may still be read)
			float* rs = gred + (jprev >= 0 ? ((jprev + 2) >> 1) & 1 : 0) * NCW * NR;
			{
				const float ws = warp_rows<NR, false>(lp, lane);
				if ((lane & (32 / NR - 1)) == 0) rs[cw * NR + lane / (32 / NR)] = ws;
			}
			named_sync(gbar, 32 * NCW);
			float L[NR];
#pragma unroll
			for (int r = 0; r < NR; ++r)
			{
				float l = rs[r];
#pragma unroll
				for (int w = 1; w < NCW; ++w) l += rs[w * NR + r];
				L[r] = l;
			}
			const uint32_t xaddr = tmem + lane_addr + C::X_BASE;
			if (g == 1)
			{
				float flat[C::X_COLS];
#pragma unroll
				for (int mb = 0; mb < C::NPB; ++mb)
#pragma unroll
					for (int r = 0; r < NR; ++r) flat[mb * NR + r] = o[mb][r];
				tmem_st<C::X_COLS>(xaddr, flat);
				tmem_wait_st();
				if (ctid < NR)
				{
#pragma unroll
					for (int r = 0; r < NR; ++r)
						if (r == ctid)
						{
							ml1[r] = m[r];
							ml1[NR + r] = L[r];
						}
				}
				tc_fence_before();
			}
			named_sync(1, NSG * 32 * NCW);
			if (g == 0)
			{
				tc_fence_after();
				float x1[C::X_COLS];
				tmem_ld<C::X_COLS>(xaddr, x1);
				tmem_wait_ld();
				float M[NR];
#pragma unroll
				for (int r = 0; r < NR; ++r)
				{
					const float m1 = ml1[r], l1 = ml1[NR + r];
					const float mx = fmaxf(m[r], m1);
					const float c0 = m[r] == -CUDART_INF_F ? 0.0f : ex2(m[r] - mx);
					const float c1 = m1 == -CUDART_INF_F ? 0.0f : ex2(m1 - mx);
#pragma unroll
					for (int mb = 0; mb < C::NPB; ++mb) o[mb][r] = fmaf(o[mb][r], c0, x1[mb * NR + r] * c1);
					L[r] = fmaf(L[r], c0, l1 * c1);
					M[r] = mx == -CUDART_INF_F ? -CUDART_INF_F : mx - P_SHIFT;
				}
				const int rows_valid = G * n_tok - rg * NR;
				auto row_off = [&](int R) -> size_t {
					const int gr = rg * NR + R;
					return ((size_t)(gr / G) * n_head + (size_t)h * G + gr % G) * D;
				};
				auto out_row = [&](int R) -> float* { return out + row_off(R); };
				if (n_pieces == 1)
				{
#pragma unroll
					for (int mb = 0; mb < C::NPB; ++mb)
						if (dx[mb] >= 0)
#pragma unroll
							for (int r = 0; r < NR; ++r)
								if (r < rows_valid)
									out_row(r)[dx[mb]] = gated(L[r] > 0.0f ? o[mb][r] / L[r] : 0.0f, gate, row_off(r) + dx[mb]);
				}
				else
				{
					float* part = P.parts + (size_t)part_slot * NR * PW;
#pragma unroll
					for (int mb = 0; mb < C::NPB; ++mb)
						if (dx[mb] >= 0)
#pragma unroll
							for (int r = 0; r < NR; ++r) part[r * PW + dx[mb]] = o[mb][r];
					if (ctid < NR)
					{
#pragma unroll
						for (int r = 0; r < NR; ++r)
							if (r == ctid) *reinterpret_cast<float2*>(part + r * PW + D) = make_float2(M[r], L[r]);
					}
					named_sync(gbar, 32 * NCW);
					if (ctid == 0)
					{
						const int prev = atomic_add_acq_rel(&P.counters[seg], 1);
						flags[1] = prev == n_pieces - 1;
					}
					named_sync(gbar, 32 * NCW);
					if (flags[1])
					{
						// the segment's last piece: fold the pieces in order
						// (nnc_attn_merge), then divide (nnc_attn_finish)
						merge_pieces<D, NR>(P.parts + (size_t)part_first * NR * PW, (size_t)NR * PW, n_pieces, rows_valid,
						                    ctid, 32 * NCW, [&](int R, int d, float4 acc, float Mx, float Lx) {
							                    const float inv = Lx > 0.0f ? 1.0f / Lx : 0.0f;
							                    acc.x *= inv;
							                    acc.y *= inv;
							                    acc.z *= inv;
							                    acc.w *= inv;
							                    *reinterpret_cast<float4*>(out_row(R) + d) = gated4(acc, gate, row_off(R) + d);
						                    });
						if (ctid == 0) P.counters[seg] = 0; // ready for the next launch
					}
				}
				tc_fence_before();
			}
			named_sync(1, NSG * 32 * NCW); // the reduction buffers and the hand-over columns are free again
		}
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 1)
	{
		tc_fence_after();
		tmem_dealloc(tmem, C::TMEM_COLS);
	}
}

template <int D, typename KV, int NR>
__global__ void __launch_bounds__(TC_THREADS, 1) decode_tc_kernel(const DecodePlan P, const __grid_constant__ TcMaps maps)
{
	decode_tc_body<D, KV, NR, false>(P, &maps, nullptr);
}

// A small launch: its job table and CTA starts come with the parameters.
template <int D, typename KV, int NR>
__global__ void __launch_bounds__(TC_THREADS, 1)
	decode_tc_kernel_inline(const DecodePlan P, const __grid_constant__ InlineTable tab)
{
	decode_tc_body<D, KV, NR, true>(P, nullptr, tab.b);
}

template <int D, typename KV, int NR>
int launch_tc(const DecodePlan& P, const void* maps, const InlineTable* tab, cudaStream_t st)
{
	using C = TcCfg<D, NR>;
	static bool configured[2][64] = {};
	int dev = 0;
	cudaGetDevice(&dev);
	if (dev < 0 || dev >= 64) return (int)cudaErrorInvalidDevice;
	if (tab && maps) return (int)cudaErrorInvalidValue; // an inline launch takes the jobs' own maps
	if (!configured[tab != nullptr][dev])
	{
		const cudaError_t e =
			tab ? cudaFuncSetAttribute(decode_tc_kernel_inline<D, KV, NR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
			                           C::SMEM)
			    : cudaFuncSetAttribute(decode_tc_kernel<D, KV, NR>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
		if (e != cudaSuccess) return (int)e;
		configured[tab != nullptr][dev] = true;
	}
	TcMaps m;
	if (maps)
		memcpy(&m, maps, sizeof m);
	else
		memset(&m, 0, sizeof m);
	// after K1 (which then appends the new rows) a programmatic dependent of
	// it: it starts while K1 runs and waits for it before the tiles that hold them
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3((unsigned)P.n_ctas);
	cfg.blockDim = dim3(TC_THREADS);
	cfg.dynamicSmemBytes = C::SMEM;
	cfg.stream = st;
	cudaLaunchAttribute attr[1];
	attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	attr[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = attr;
	cfg.numAttrs = P.fused ? 0 : 1; // appending itself, it follows the stream's previous work in full
	if (tab) return (int)cudaLaunchKernelEx(&cfg, decode_tc_kernel_inline<D, KV, NR>, P, *tab);
	return (int)cudaLaunchKernelEx(&cfg, decode_tc_kernel<D, KV, NR>, P, m);
}

template <typename KV, int NR>
int launch_tc_dims(const DecodePlan& P, const void* maps, const InlineTable* tab, cudaStream_t st)
{
	switch (P.D)
	{
	case 64: return launch_tc<64, KV, NR>(P, maps, tab, st);
	case 128: return launch_tc<128, KV, NR>(P, maps, tab, st);
	case 256: return launch_tc<256, KV, NR>(P, maps, tab, st);
	default: return (int)cudaErrorInvalidValue;
	}
}

} // namespace

int tc_fuse_tokens(int D, int RM)
{
	if (RM == 8) return D == 64 ? TcCfg<64, 8>::NT : D == 128 ? TcCfg<128, 8>::NT : D == 256 ? TcCfg<256, 8>::NT : 0;
	if (RM == 16) return D == 64 ? TcCfg<64, 16>::NT : D == 128 ? TcCfg<128, 16>::NT : D == 256 ? TcCfg<256, 16>::NT : 0;
	return 0;
}

int tc_rows(int D, int kv_type, int rows_needed)
{
	if (kv_type != KV_F16 && kv_type != KV_BF16) return 0;
	if (D != 64 && D != 128 && D != 256) return 0;
	if (rows_needed < 3) return 0; // one or two rows: the CUDA-core kernel
	return rows_needed <= 8 ? 8 : 16;
}

int launch_decode_tc(const DecodePlan& P, const void* maps, void* stream, const InlineTable* tab)
{
	if (P.n_ctas == 0) return 0;
	auto st = static_cast<cudaStream_t>(stream);
	if (P.RM != 8 && P.RM != 16) return (int)cudaErrorInvalidValue;
	if (P.kv_type == KV_F16)
		return P.RM == 8 ? launch_tc_dims<kv_f16, 8>(P, maps, tab, st) : launch_tc_dims<kv_f16, 16>(P, maps, tab, st);
	if (P.kv_type == KV_BF16)
		return P.RM == 8 ? launch_tc_dims<kv_bf16, 8>(P, maps, tab, st)
		                 : launch_tc_dims<kv_bf16, 16>(P, maps, tab, st);
	return (int)cudaErrorInvalidValue;
}

int tc_make_maps(void* kmap, void* vmap, const void* k, const void* v, int kv_type, int D, long long rows,
                 long long planes)
{
	const uint32_t T = (uint32_t)(TC_TILE / (D * 2));
	int e = make_tensor_map(static_cast<CUtensorMap*>(kmap), k, kv_type == KV_BF16, (uint64_t)D, (uint64_t)rows,
	                        (uint64_t)planes, T);
	if (!e)
		e = make_tensor_map(static_cast<CUtensorMap*>(vmap), v, kv_type == KV_BF16, (uint64_t)D, (uint64_t)rows,
		                    (uint64_t)planes, T);
	return e;
}

} // namespace nncu
