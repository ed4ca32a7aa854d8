// plan.cpp -- the plan of one attention launch (host side): which keys each
// CTA of the decode kernel streams.
//
// A segment is one (job, KV head, group of RM query rows) and its keys are
// cut into tiles of T keys (k_decode.cu). The reference splits a query's
// keys into 256-key blocks and merges the blocks' partials in key order
// (model.cpp:1251-1319); here a segment is cut into a few equal chunks of
// whole tiles instead, sized so that the launch's chunks about fill the GPU
// once, and each CTA streams a run of consecutive chunks. Most CTAs then hold
// a single chunk: they stream it without stopping and write one partial (or
// the output itself when the segment has one chunk); the last chunk of a
// segment to finish folds the segment's partials.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>

#include "internal.h"
#include "nncu.h"

namespace nncu
{
namespace
{

// Tiles a CTA issues before it reads its job. One: the piece's q rows, issued
// once the job is read, then queue behind a single tile instead of a full
// ring of them, and the consumers can start on the first tile sooner.
constexpr int PREFETCH_TILES = 1;

// Tiles per SM from which a launch's runs are cut from small chunks.
constexpr long long LONG_RUN = 256;

// The positions a job appends in this launch: its new tokens within its key range.
int append_lo(const DevJob& j) { return j.reuse_kv ? 0 : std::max(j.pos0, j.key_lo); }
int append_hi(const DevJob& j) { return j.reuse_kv ? 0 : std::min(j.pos0 + j.n_tok, j.key_hi); }

bool holds_new_rows(const DevJob& j, int tis, int len, int T)
{
	const int lo = append_lo(j), hi = append_hi(j);
	return lo < hi && (long long)(j.tile_lo + tis) * T <= hi - 1 && (long long)(j.tile_lo + tis + len) * T - 1 >= lo;
}

} // namespace

int plan_launch(DevJob* jobs, int n, int kv_type, int num_sms, DecodePlan& P, CtaStart* starts, int max_starts,
                bool small_chunks, int rows_fixed)
{
	const int D = jobs[0].D;
	const int T = decode_tile_keys(D, kv_type);
	int rows_needed = 1, max_tok = 0;
	for (int i = 0; i < n; ++i)
	{
		rows_needed = std::max(rows_needed, (jobs[i].n_head / jobs[i].n_kv) * jobs[i].n_tok);
		max_tok = std::max(max_tok, jobs[i].n_tok);
	}
	int RM = 1;
	while (RM < rows_needed && RM < decode_rows_max(D)) RM *= 2;
	if (rows_fixed > 0) RM = rows_fixed; // the tensor-core kernel's row groups

	// every job's tiles: the union of its tokens' spans (model_attn_span)
	// within its key range
	long long total = 0;
	int seg = 0;
	for (int i = 0; i < n; ++i)
	{
		DevJob& j = jobs[i];
		int first_min = INT_MAX, last_max = -1;
		for (int t = 0; t < j.n_tok; ++t)
		{
			int f, l;
			nncu_attn_span(j.causal, j.window, j.pos0 + t, j.n_seq, &f, &l);
			f = std::max(f, j.key_lo);
			l = std::min(l, j.key_hi - 1);
			if (l < f) continue;
			first_min = std::min(first_min, f);
			last_max = std::max(last_max, l);
		}
		j.n_rowgroups = ((j.n_head / j.n_kv) * j.n_tok + RM - 1) / RM;
		j.tile_lo = last_max < 0 ? 0 : first_min / T;
		j.n_tiles = last_max < 0 ? 0 : last_max / T - j.tile_lo + 1;
		j.seg0 = seg;
		seg += j.n_kv * j.n_rowgroups;
		total += (long long)j.n_kv * j.n_rowgroups * j.n_tiles;
	}

	// K2 appends the new rows itself (and K1 does not run) when its slots hold
	// every job's new tokens, every new position lies in its job's tiles, and
	// the rows it bulk-copies are 16-byte aligned
	auto aligned = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; };
	int fused = max_tok <= (rows_fixed ? tc_fuse_tokens(D, RM) : decode_fuse_tokens(D, kv_type, RM));
	for (int i = 0; i < n && fused; ++i)
	{
		const DevJob& j = jobs[i];
		const int lo = append_lo(j), hi = append_hi(j);
		if (lo >= hi) continue;
		if (j.n_tiles == 0 || (long long)lo < (long long)j.tile_lo * T ||
		    (long long)hi > (long long)(j.tile_lo + j.n_tiles) * T || !aligned(j.k) || !aligned(j.v) ||
		    !aligned(j.k_gamma))
			fused = 0;
	}

	// chunks: each segment in ceil(n_tiles / C) equal runs of whole tiles
	const int ctas_max = std::max(1, std::min(num_sms, max_starts));
	long long parts = 0, max_chunk = 1;
	auto cut = [&](long long C) {
		parts = 0;
		max_chunk = 1;
		for (int i = 0; i < n; ++i)
		{
			DevJob& j = jobs[i];
			if (j.n_tiles == 0)
			{
				j.chunk = 1;
				j.n_chunks = 0;
				j.part0 = 0;
				continue;
			}
			const int k = (int)((j.n_tiles + C - 1) / C);
			j.chunk = (j.n_tiles + k - 1) / k;
			j.n_chunks = (j.n_tiles + j.chunk - 1) / j.chunk;
			j.part0 = (int)parts;
			if (j.n_chunks > 1) parts += (long long)j.n_kv * j.n_rowgroups * j.n_chunks;
			max_chunk = std::max<long long>(max_chunk, j.chunk);
		}
	};

	// CTAs: runs of consecutive chunks of at most `cap` tiles
	auto pack = [&](long long cap, bool write) -> long long {
		long long ctas = 0, cur = 0;
		for (int i = 0; i < n; ++i)
		{
			const DevJob& j = jobs[i];
			const int segs = j.n_kv * j.n_rowgroups;
			for (int s = 0; s < segs; ++s)
				for (int c = 0; c < j.n_chunks; ++c)
				{
					const int sz = std::min(j.chunk, j.n_tiles - c * j.chunk);
					if (cur > 0 && cur + sz > cap)
					{
						++ctas;
						cur = 0;
					}
					if (cur == 0 && write)
					{
						if (ctas >= max_starts) return LLONG_MAX;
						starts[ctas] = CtaStart{i, s, c * j.chunk, 0, nullptr, nullptr, 0, {0, 0, 0}};
					}
					cur += sz;
					if (write) starts[ctas].n_tiles = (int)cur;
				}
		}
		return cur > 0 ? ctas + 1 : ctas;
	};
	// the smallest run length C (from the tiles per SM up) whose chunks pack
	// into the SMs with runs of at most max(C, largest chunk) tiles. Short
	// runs take whole chunks of about C tiles (growing C, not the runs, keeps
	// a run from holding two big chunks). Long runs (a launch of many tiles
	// per SM) take chunks of about C / 16 tiles, so that a run ends within
	// 1/16 of C wherever the segments' own lengths fall; each chunk is a
	// piece with its own partial, a cost of a few microseconds against
	// the chunk's 64 or more tiles.
	auto chunk_target = [&](long long C) {
		return small_chunks && C >= LONG_RUN ? std::max<long long>(64, C / 16) : C;
	};
	long long C = total > 0 ? (total + ctas_max - 1) / ctas_max : 1;
	for (;;)
	{
		cut(chunk_target(C));
		if (pack(std::max(C, max_chunk), false) <= ctas_max) break;
		C += std::max<long long>(1, C / 64);
	}
	const long long n_ctas = pack(std::max(C, max_chunk), true); // with the chunks of the last cut(C)
	if (n_ctas > max_starts) return set_error(NNCU_ERR_INVALID_ARGUMENT, "decode plan: too many CTAs");

	// each CTA's first tiles, issued before it reads its job: a contiguous run
	// of its first piece (and, while K1 appends, none that holds new rows)
	const size_t es = (size_t)kv_esize(kv_type);
	for (long long c = 0; c < n_ctas; ++c)
	{
		CtaStart& S = starts[c];
		const DevJob& j = jobs[S.job];
		if (rows_fixed)
		{
			// the tensor-core kernel: its first tile by tensor map, row and plane,
			// unless it holds new rows (it waits for K1, or lands for the append)
			if (!j.tmap_k || holds_new_rows(j, S.tis, 1, T)) continue;
			S.k0 = static_cast<const char*>(j.tmap_k);
			S.v0 = static_cast<const char*>(j.tmap_v);
			S.pad_[0] = (int)(((long long)(j.tile_lo + S.tis) * T) % j.rows);
			S.pad_[1] = j.plane0 + S.seg / j.n_rowgroups;
			S.pre = 1;
			continue;
		}
		const int len = std::min({j.chunk - S.tis % j.chunk, j.n_tiles - S.tis, S.n_tiles});
		if (!fused && holds_new_rows(j, S.tis, len, T)) continue;
		const int h = S.seg / j.n_rowgroups;
		const long long row0 = ((long long)(j.tile_lo + S.tis) * T) % j.rows;
		int pre = 0;
		while (pre < std::min(PREFETCH_TILES, len) &&
		       ((long long)(j.tile_lo + S.tis + pre) * T) % j.rows == row0 + (long long)pre * T)
			++pre;
		const size_t off = (size_t)h * (size_t)j.head_bytes + (size_t)row0 * D * es;
		S.k0 = j.K + off;
		S.v0 = j.V + off;
		S.pre = pre;
	}

	P.n_jobs = n;
	P.D = D;
	P.kv_type = kv_type;
	P.RM = RM;
	P.T = T;
	P.n_ctas = (int)n_ctas;
	P.n_segments = seg;
	P.max_tok = max_tok;
	P.fused = fused;
	P.n_parts = parts;
	return NNCU_OK;
}

} // namespace nncu
