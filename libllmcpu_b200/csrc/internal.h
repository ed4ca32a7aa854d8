// internal.h -- what the host side (api.cpp) and the kernels (*.cu) share:
// the per-job device descriptor, the work plan of the decode kernel, and the
// launchers. Plain C++: no CUDA headers are needed to include it.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <vector_types.h>

struct nncu_group;  // split.cpp
struct nncu_weight; // nncu.h

namespace nncu
{

enum
{
	KV_BF16 = 0,
	KV_F32 = 1,
	KV_F16 = 2
};

constexpr int ATTN_BLOCK = 256;                      // MODEL_ATTN_BLOCK (model.h:229)
constexpr unsigned long long WAIT_LIMIT_NS = 2000000000ull; // bounded waits give up after 2 s

// Device error codes written by kernels into the per-cache error word.
enum
{
	DEVERR_NONE = 0,
	DEVERR_WAIT_FULL = 1,  // a consumer's wait for a K/V tile ran out
	DEVERR_WAIT_EMPTY = 2, // the producer's wait for a free stage ran out
	DEVERR_PLAN = 3,       // a tile fell outside every job (a planning bug)
	DEVERR_SPLIT = 4       // a split call's partials did not all arrive on this GPU in time
};

inline int kv_esize(int kv_type) { return kv_type == KV_F32 ? 4 : 2; }

// One attention job (one layer of one sequence) as the kernels see it.
// All pointers are device pointers. The decode kernel bulk-copies it into
// shared memory, hence the 16-byte alignment and size.
struct alignas(16) DevJob
{
	const float* q;           // [n_tok][n_head*D] projections, fp32
	const float* k;           // [n_tok][n_kv*D]
	const float* v;
	float* out;               // [n_tok][n_head*D]
	const float* q_gamma;     // D or null
	const float* k_gamma;     // D or null
	const float* freq_factors; // n_rot/2 or null
	const float* rope_inv;    // n_rot/2, padded to 16 bytes: the fp32 inverse-frequency recurrence
	char* K;                  // this sequence's K slab: [n_kv][rows][D]
	char* V;
	long long head_bytes;     // rows * D * esize
	int rows;                 // allocated rows (a multiple of 256); position p -> row p % rows
	int n_tok, pos0, n_seq;
	int n_head, n_kv, D, n_rot, rope_mode;
	int causal, window, reuse_kv, v_rmsnorm;
	float rope_scale, eps, scale, softcap;
	// the decode plan (filled by plan_launch on the host)
	int tile_lo;          // first tile (absolute, units of T keys) of the union of the tokens' spans
	int n_tiles;          // tiles per segment
	int n_rowgroups;      // segments per KV head (query rows split into groups of RM)
	int seg0;             // this job's first segment (its counters)
	int chunk;            // tiles per chunk: a segment is cut into n_chunks chunks of this many
	int n_chunks;         // (the last may be short); each chunk is one piece with its own partial
	int part0;            // this job's first partial slot: segment s, chunk c at part0 + s * n_chunks + c
	// the keys this launch attends and appends: [key_lo, key_hi) of every
	// query's span (the whole span unless the sequence is split over GPUs)
	int key_lo, key_hi;
	int out_row0;         // split over GPUs: the job's first row in the group's output
	// the tensor-core decode kernel's view of the cache: tensor maps (CUtensorMap,
	// in global memory) over this job's K and V buffers as [planes][rows][D],
	// KV head h of this sequence at plane plane0 + h; NULL: the launch's own maps
	const void* tmap_k;
	const void* tmap_v;
	int plane0;
	const float* gate;    // [n_tok][n_head*D] or null: the output times sigmoid(gate) (Qwen3.5)
};
static_assert(sizeof(DevJob) % 16 == 0, "DevJob is bulk-copied");

// Where one CTA starts: its first tile (job, segment, tile within the
// segment), how many tiles it streams, and the addresses of the first `pre`
// tiles' K and V rows (contiguous runs), which it issues before reading the job.
struct alignas(16) CtaStart
{
	int job, seg, tis, n_tiles;
	const char* k0;
	const char* v0;
	int pre;
	int pad_[3];
};
static_assert(sizeof(CtaStart) == 48, "CtaStart layout");

// A small launch's job table (n DevJobs, then the CTA starts at the next
// 16-byte boundary) passed by value as a kernel parameter, so the launch
// needs no upload and no cross-stream events. With the DecodePlan it makes
// 12 KB of parameters (sm_70 and later take up to 32,764 bytes since CUDA
// 12.1): one job on all 148 SMs (7.3 KB), or the 16 sequences of one layer
// (10.9 KB).
constexpr int INLINE_TABLE_BYTES = 12288 - 320;
struct alignas(16) InlineTable
{
	unsigned char b[INLINE_TABLE_BYTES];
};

constexpr int MAX_WORLD = 8; // GPUs a sequence may be split over (one NVSwitch node)

// One launch of K1 and K2: each CTA streams a run of whole chunks (of one or
// more segments) given by its CtaStart.
struct DecodePlan
{
	const DevJob* jobs;        // device copy of the job table
	const CtaStart* cta_start; // per CTA
	int n_jobs;
	int D, kv_type, RM, T; // head_dim, element type, query rows per segment, keys per tile
	int n_ctas;
	int n_segments;
	int max_tok;            // K1's grid: tokens of the longest job
	int fused;              // 1: K2 appends the new K/V rows itself and K1 does not run
	long long n_parts;      // partial slots in use
	float* parts;   // n_parts slots of RM * (D + 4) floats
	int* counters;  // n_segments, zero between launches
	int* err;       // device error word
	// A sequence split over the GPUs of a group (world > 1; nncu_group, split.cpp):
	// each segment's result over this GPU's keys goes, as a partial, to every
	// GPU's receive buffer and is counted there; at the end of the call each
	// GPU merges, in rank order, the partials that landed in its own memory
	// (split_merge_kernel). All pointers are for this call's parity (calls
	// alternate between two sets), GPU g's at index g.
	int world, rank;
	long long recv_stride;       // floats between two ranks' blocks of a receive buffer
	float* recv[MAX_WORLD];      // [world][segments][RM][D + 4]
	int* arrive[MAX_WORLD];      // [segments] partials arrived, zero between calls
	float* out[MAX_WORLD];       // GPU g's output rows (job i from its out_row0)
	int* poison;                 // this GPU's: set by a merge wait that ran out; every later merge fails
	unsigned long long wait_ns;  // the merge's bounded wait
	int drop_arrivals;           // test injection: this rank's partials are stored but never counted
};
static_assert(sizeof(DecodePlan) + sizeof(InlineTable) <= 12288, "an inline launch's parameters: 12 KB");

// Plan one launch over jobs[0, n) (their D, kv geometry, positions and
// pointers filled): the row group size, every job's tiles, chunks and
// partial slots, whether K2 appends itself, and the per-CTA starts (at most
// max_starts, at most num_sms). With small_chunks, launches of many tiles
// per SM are cut finer for balance (more partial slots). Host code;
// allocates nothing.
int plan_launch(DevJob* jobs, int n, int kv_type, int num_sms, DecodePlan& P, CtaStart* starts, int max_starts,
                bool small_chunks = true, int rows_fixed = 0);

// The tensor-core decode kernel (k_decode_tc.cu): 16-bit caches, head_dim
// 64, 128 or 256, several query rows per KV head (tc_rows(): 8 or 16 per
// segment, 0 when the launch does not suit it). Launched after K1 (which
// appends the new rows) as its programmatic dependent. `maps`: two
// CUtensorMaps (K, V) for jobs whose tmap_k / tmap_v are NULL, or NULL.
int tc_rows(int D, int kv_type, int rows_needed);
int tc_fuse_tokens(int D, int RM); // new tokens the tensor-core kernel appends itself (0: K1 must)
int launch_decode_tc(const DecodePlan& plan, const void* maps, void* stream, const InlineTable* tab = nullptr);
// The tensor maps of a 16-bit cache buffer [planes][rows][D] in the kernel's
// tile form (host side; 128 bytes each, 64-byte aligned).
constexpr int TENSOR_MAP_BYTES = 128;
int tc_make_maps(void* kmap, void* vmap, const void* k, const void* v, int kv_type, int D, long long rows,
                 long long planes);

// One causal prefill on the tensor cores (k_prefill.cu): bf16 cache, head_dim 128.
struct PrefillPlan
{
	int n_tok, pos0, n_seq, n_head, n_kv, window, q_pairs; // q_pairs: CTAs per head (256 query rows each)
	float scale, log2e, softcap;
	float* out; // [n_tok][n_head * 128]
	const float* gate; // like out, or null
	int* err;   // device error word
};
bool prefill_supported(int D, int kv_type);
size_t prefill_qbuf_bytes(int n_tok, int n_head);
// The prefill's per-head work: q rows normed and rotated into `qbuf` (bf16,
// head-major), k and v rows appended to the cache. j is the host copy of the job.
int launch_prefill_prep(const DevJob& j, void* qbuf, void* stream);
// The attention of every row over its causal span into j.out (after the prep).
int launch_prefill(const DevJob& j, void* qbuf, int* err, void* stream);

// A list of copies done by one kernel launch (k_prep.cu): each entry's
// bytes from src to dst, either side device memory or the device's mapping
// of registered (pinned) host memory, cut into COPY_CHUNK pieces, one CTA
// each (cta0: the entry's first CTA, filled in by launch_copy_list). At most
// COPY_LIST_MAX entries travel as the launch's parameter.
struct CopyEntry
{
	const void* src;
	void* dst;
	uint64_t bytes;
	uint32_t cta0;
};
constexpr int COPY_LIST_MAX = 120; // 8 + 120 x 32 bytes of parameter
constexpr uint64_t COPY_CHUNK = 64 << 10;
struct CopyList
{
	int n;
	CopyEntry e[COPY_LIST_MAX];
};
int launch_copy_list(CopyList& l, void* stream);

// Record a failure for nncu_last_error() (api.cpp); return `status`.
int set_error(int status, const char* msg);
int set_cuda_error(int cuda_status, const char* what);

// The pointers of one job that the kernels read with bulk copies or write
// with 16-byte vector stores, checked before anything is launched: a
// misaligned one is refused with NNCU_ERR_INVALID_ARGUMENT (a bulk copy from
// it would fault the GPU). NULL pointers pass (the caller checks which may be
// NULL). `job` numbers the message; `what` names the call.
struct JobPointers
{
	const void* q;
	const void* k;
	const void* v;
	const void* out;
	const void* q_gamma;
	const void* k_gamma;
	const void* freq_factors;
	const void* k_cache;
	const void* v_cache;
};
int check_alignment(const JobPointers& p, int job, const char* what);
// Count kernels launched outside api.cpp (nncu_launch_count).
void note_launches(int n);

// Launchers (implemented in the .cu files). Each returns a cudaError_t value.
int launch_prep(const DecodePlan& plan, void* stream);
// The decode kernel; with `tab`, its job table and CTA starts travel in the
// launch's parameters (a fused launch whose table fits) and plan.jobs /
// plan.cta_start are not read.
int launch_decode(const DecodePlan& plan, void* stream, const InlineTable* tab = nullptr);
int launch_split_wait(const DecodePlan& plan, void* stream); // a split call's end: the world's partials merged here

// Fill the split fields of a plan from a group (split.cpp): its peers'
// buffers for this call's parity; checks that the call fits the group.
int group_prepare(nncu_group* g, DecodePlan& P, int n_rows);
int group_device(const nncu_group* g);
bool decode_supported(int D, int kv_type);
int decode_tile_keys(int D, int kv_type);
int decode_rows_max(int D);
int decode_fuse_tokens(int D, int kv_type, int RM); // new tokens K2 can append itself (0: K1 must)

// Unit-seam kernels (nn_ops.h equivalents).
int launch_attn_block(const float* q, size_t q_stride, const void* K, const void* V, int kv_type, size_t kv_stride,
                      size_t n_keys, size_t head_dim, size_t n_heads, float scale, float softcap, float* part,
                      void* stream);
int launch_attn_merge(float* acc, const float* part, size_t head_dim, size_t n_heads, void* stream);
int launch_attn_finish(float* out, size_t out_stride, const float* acc, size_t head_dim, size_t n_heads,
                       void* stream);
int launch_rmsnorm(float* y, const float* x, size_t n_groups, size_t dim, const float* gamma, float eps,
                   void* stream);
int launch_rope(float* x, uint32_t n_tok, uint32_t n_heads, uint32_t head_dim, uint32_t n_rot, int32_t pos0,
                float pos_scale, const float* rope_inv, int mode, const float* freq_factors, void* stream);
int launch_softcap(float* y, const float* x, size_t n, float cap, void* stream);

// attention_forward's projections (k_gemv.cu): a weight's shape and pointers
// checked against what the layer needs; batched gemvs with the optional
// query / gate split and bias (GemvArgs); block sums for Q4_S weights.
int check_weight(const nncu_weight& w, uint32_t rows, uint32_t cols, const char* name);
struct Projection
{
	const nncu_weight* w;
	float* Y;
	size_t y_stride;
	float* Y2;          // with split > 0: the second half-rows of each pair (the gate)
	uint32_t split;
	const float* bias;  // or NULL
};
// up to three projections of the same vectors, one launch per weight format
int launch_projections(const Projection* p, int n, const float* X, size_t x_stride, const float* XSUM,
                       size_t xsum_stride, uint32_t n_batch, void* stream);
int launch_block_sums(const float* x, float* out, size_t n, void* stream);

} // namespace nncu
