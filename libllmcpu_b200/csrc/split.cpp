// split.cpp -- one long sequence's attention split over the GPUs of a node.
//
// BASELINE config 5 (131,073 keys of one sequence, one new token): each GPU
// holds and reads one 256-aligned range of the keys, and the per-range
// partials (o, m, l) are merged by log-sum-exp in rank order, the reference's
// nnc_attn_merge over blocks (nn_ops.cpp:461-482) with the blocks grouped by
// GPU. The partials cross NVLink inside the attention kernel itself: a
// segment's partial is stored straight into every GPU's receive buffer (peer
// stores through CUDA IPC mappings) and counted on a system-scope counter per
// segment there. A kernel at the end of each call waits, bounded, on each
// GPU until the world's partials of every segment have landed in its own
// memory, and merges them into that GPU's output with local loads and
// stores.
//
// A merge whose wait runs out marks this GPU's group as poisoned: its
// counters may then be met late by the slow rank's arrival, so every later
// merge on this GPU fails (NNCU_ERR_TIMEOUT through nncu_sync) instead of
// merging stale partials, until every rank has called nncu_group_reset at a
// common step boundary (no call of the group in flight on any GPU).
//
// One process per GPU. The caller exchanges the groups' memory handles out of
// band (torch.distributed in the Python binding) and opens each peer's.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstring>

#include "internal.h"
#include "nncu.h"

struct nncu_group
{
	int device = 0, rank = 0, world = 1, max_rows = 0, head_dim = 0;
	long long cap_rows = 0; // partial rows per rank per parity
	char* base = nullptr;   // this GPU's shared block
	char* peer[nncu::MAX_WORLD] = {};
	bool opened[nncu::MAX_WORLD] = {};
	size_t off_recv = 0, off_arrive = 0, off_state = 0, off_out = 0, bytes = 0;
	int calls = 0;
	unsigned long long wait_ns = nncu::WAIT_LIMIT_NS;
	int drop_next = 0; // test injection: calls whose arrivals this rank drops
};

namespace
{

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

struct Guard
{
	int prev = -1;
	explicit Guard(int dev)
	{
		if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
		if (prev != dev) cudaSetDevice(dev);
	}
	~Guard()
	{
		if (prev >= 0) cudaSetDevice(prev);
	}
};

} // namespace

extern "C" int nncu_group_create(int32_t device, int32_t rank, int32_t world, int32_t max_rows, int32_t head_dim,
                                 nncu_group** out)
{
	using namespace nncu;
	if (!out) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL output");
	*out = nullptr;
	if (world < 2 || world > MAX_WORLD || rank < 0 || rank >= world)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "a group has 2 to 8 ranks and rank < world");
	if (max_rows <= 0 || !decode_supported(head_dim, KV_F32))
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "max_rows must be positive and head_dim 64, 128, 256 or 512");
	Guard dg(device);
	auto* g = new nncu_group;
	g->device = device;
	g->rank = rank;
	g->world = world;
	g->max_rows = max_rows;
	g->head_dim = head_dim;
	// a segment's partial block holds its RM rows, the last row group of each
	// KV head padded: room for the output rows plus that padding
	g->cap_rows = (long long)max_rows + 32LL * 64;
	const size_t pw = (size_t)head_dim + 4;
	const size_t recv = 2 * (size_t)world * (size_t)g->cap_rows * pw * sizeof(float);
	const size_t arrive = 2 * (size_t)g->cap_rows * sizeof(int);
	g->off_recv = 0;
	g->off_arrive = up256(recv);
	g->off_state = g->off_arrive + up256(arrive); // [0]: the poison word
	g->off_out = g->off_state + 256;
	g->bytes = g->off_out + up256((size_t)max_rows * head_dim * sizeof(float));
	cudaError_t e = cudaMalloc(&g->base, g->bytes);
	if (e == cudaSuccess) e = cudaMemset(g->base, 0, g->bytes);
	if (e == cudaSuccess) e = cudaDeviceSynchronize();
	if (e != cudaSuccess)
	{
		if (g->base) cudaFree(g->base);
		delete g;
		return set_cuda_error((int)e, "group memory");
	}
	g->peer[rank] = g->base;
	g->opened[rank] = true;
	*out = g;
	return NNCU_OK;
}

extern "C" int nncu_group_handle(const nncu_group* g, void* handle)
{
	using namespace nncu;
	if (!g || !handle) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL argument");
	static_assert(sizeof(cudaIpcMemHandle_t) <= NNCU_GROUP_HANDLE_BYTES, "handle size");
	Guard dg(g->device);
	cudaIpcMemHandle_t h;
	const cudaError_t e = cudaIpcGetMemHandle(&h, g->base);
	if (e != cudaSuccess) return set_cuda_error((int)e, "cudaIpcGetMemHandle");
	std::memset(handle, 0, NNCU_GROUP_HANDLE_BYTES);
	std::memcpy(handle, &h, sizeof h);
	return NNCU_OK;
}

extern "C" int nncu_group_open(nncu_group* g, int32_t peer, const void* handle)
{
	using namespace nncu;
	if (!g || !handle) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL argument");
	if (peer < 0 || peer >= g->world || peer == g->rank)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "peer out of range (or this rank)");
	if (g->opened[peer]) return set_error(NNCU_ERR_INVALID_ARGUMENT, "peer already open");
	Guard dg(g->device);
	cudaIpcMemHandle_t h;
	std::memcpy(&h, handle, sizeof h);
	void* p = nullptr;
	const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
	if (e != cudaSuccess) return set_cuda_error((int)e, "cudaIpcOpenMemHandle");
	g->peer[peer] = static_cast<char*>(p);
	g->opened[peer] = true;
	return NNCU_OK;
}

extern "C" float* nncu_group_output(const nncu_group* g)
{
	return g ? reinterpret_cast<float*>(g->base + g->off_out) : nullptr;
}

extern "C" int nncu_group_copy_output(const nncu_group* g, float* dst, size_t n_floats, void* stream)
{
	using namespace nncu;
	if (!g || (!dst && n_floats)) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL argument");
	if (n_floats > (size_t)g->max_rows * g->head_dim)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "more floats than the group's output holds");
	Guard dg(g->device);
	const cudaError_t e = cudaMemcpyAsync(dst, g->base + g->off_out, n_floats * sizeof(float), cudaMemcpyDefault,
	                                      static_cast<cudaStream_t>(stream));
	if (e != cudaSuccess) return set_cuda_error((int)e, "group output copy");
	return NNCU_OK;
}

extern "C" int nncu_group_set_timeout(nncu_group* g, uint32_t ms)
{
	using namespace nncu;
	if (!g) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL group");
	if (ms == 0 || ms > 60000) return set_error(NNCU_ERR_INVALID_ARGUMENT, "the timeout must be 1 to 60000 ms");
	g->wait_ns = (unsigned long long)ms * 1000000ull;
	return NNCU_OK;
}

extern "C" int nncu_group_reset(nncu_group* g)
{
	using namespace nncu;
	if (!g) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL group");
	Guard dg(g->device);
	// every kernel of this GPU that could still count into the block is done
	cudaError_t e = cudaDeviceSynchronize();
	if (e == cudaSuccess) e = cudaMemset(g->base + g->off_arrive, 0, g->off_out - g->off_arrive);
	if (e == cudaSuccess) e = cudaDeviceSynchronize();
	if (e != cudaSuccess) return set_cuda_error((int)e, "group reset");
	g->calls = 0;
	g->drop_next = 0;
	return NNCU_OK;
}

extern "C" int nncu_group_inject_drop(nncu_group* g, int32_t n_calls)
{
	using namespace nncu;
	if (!g || n_calls < 0) return set_error(NNCU_ERR_INVALID_ARGUMENT, "NULL group or negative count");
	g->drop_next = n_calls;
	return NNCU_OK;
}

extern "C" void nncu_group_free(nncu_group* g)
{
	if (!g) return;
	Guard dg(g->device);
	cudaDeviceSynchronize();
	for (int r = 0; r < g->world; ++r)
		if (r != g->rank && g->opened[r]) cudaIpcCloseMemHandle(g->peer[r]);
	if (g->base) cudaFree(g->base);
	delete g;
}

namespace nncu
{

int group_prepare(nncu_group* g, DecodePlan& P, int n_rows)
{
	for (int r = 0; r < g->world; ++r)
		if (!g->opened[r]) return set_error(NNCU_ERR_INVALID_ARGUMENT, "the group has a peer not yet opened");
	if (P.D != g->head_dim) return set_error(NNCU_ERR_INVALID_ARGUMENT, "head_dim differs from the group's");
	if (n_rows > g->max_rows) return set_error(NNCU_ERR_INVALID_ARGUMENT, "more output rows than the group holds");
	if ((long long)P.n_segments * P.RM > g->cap_rows)
		return set_error(NNCU_ERR_INVALID_ARGUMENT, "more partial rows than the group holds");
	const int parity = g->calls & 1;
	const size_t pw = (size_t)g->head_dim + 4;
	P.world = g->world;
	P.rank = g->rank;
	P.recv_stride = g->cap_rows * (long long)pw;
	for (int r = 0; r < g->world; ++r)
	{
		char* b = g->peer[r];
		P.recv[r] = reinterpret_cast<float*>(b + g->off_recv) + (size_t)parity * g->world * P.recv_stride;
		P.arrive[r] = reinterpret_cast<int*>(b + g->off_arrive) + (size_t)parity * g->cap_rows;
		P.out[r] = reinterpret_cast<float*>(b + g->off_out);
	}
	P.poison = reinterpret_cast<int*>(g->base + g->off_state);
	P.wait_ns = g->wait_ns;
	P.drop_arrivals = 0;
	if (g->drop_next > 0)
	{
		P.drop_arrivals = 1;
		--g->drop_next;
	}
	++g->calls;
	return NNCU_OK;
}

int group_device(const nncu_group* g) { return g->device; }

} // namespace nncu
