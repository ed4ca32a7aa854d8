// api.cpp -- the host side of libnncu: the C ABI declared in include/nncu.h.
//
//  * errors: libnnc's convention (a status return plus a per-thread message,
//    runtime.h:29-46 / nnc.h:62-69), never an exception across the ABI;
//  * the HBM K/V cache: model_kv_init's sizing rules (model.cpp:1891-2040)
//    and model_kv_rewind (model.cpp:2137-2143) over device buffers laid out
//    [n_seq][n_kv][rows][head_dim];
//  * the attention op: validation, the decode work plan (stream-K over
//    256-aligned key tiles), pinned staging for the host-pointer calls, and
//    the launches of K1 (k_prep.cu) and K2+K3 (k_decode.cu).
#include "nncu.h"

#include <cuda_runtime.h>
#include <vector_functions.h>

#include <algorithm>
#include <atomic>
#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <tuple>
#include <string>
#include <vector>

#include "internal.h"

using namespace nncu;

// ---- errors -------------------------------------------------------------------

namespace
{
thread_local int t_status = NNCU_OK;
int cuda_fail(cudaError_t e, const char* what);
thread_local char t_msg[512] = "";

int fail(int status, const char* fmt, ...)
{
	t_status = status;
	va_list ap;
	va_start(ap, fmt);
	std::vsnprintf(t_msg, sizeof t_msg, fmt, ap);
	va_end(ap);
	return status;
}

} // namespace

// The same per-thread status and message for the library's other files.
int nncu::set_error(int status, const char* msg)
{
	return fail(status, "%s", msg);
}

// Every (q rows, the gains, the frequency
// factors, the new k and v rows, the cache) or writes with 16-byte stores
// (the output) must be 16-byte aligned; a misaligned one would fault the GPU
// instead of failing the call, so it is refused here, before any launch.
int nncu::check_alignment(const JobPointers& p, int job, const char* what)
{
	const struct
	{
		const void* ptr;
		const char* name;
	} ptrs[] = {{p.q, "q"},
	            {p.k, "k"},
	            {p.v, "v"},
	            {p.out, "out"},
	            {p.q_gamma, "q_gamma"},
	            {p.k_gamma, "k_gamma"},
	            {p.freq_factors, "freq_factors"},
	            {p.k_cache, "k_cache"},
	            {p.v_cache, "v_cache"}};
	for (const auto& e : ptrs)
		if (reinterpret_cast<uintptr_t>(e.ptr) & 15u)
			return fail(NNCU_ERR_INVALID_ARGUMENT, "%s: job %d: %s (%p) is not 16-byte aligned", what, job, e.name,
			            e.ptr);
	return NNCU_OK;
}

int nncu::set_cuda_error(int cuda_status, const char* what)
{
	return cuda_fail(static_cast<cudaError_t>(cuda_status), what);
}

namespace
{
int cuda_fail(cudaError_t e, const char* what)
{
	if (e == cudaErrorMemoryAllocation)
		return fail(NNCU_ERR_OUT_OF_MEMORY, "%s: out of device memory", what);
	return fail(NNCU_ERR_DEVICE, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

#define CU(call, what)                                                                                                \
	do                                                                                                                \
	{                                                                                                                 \
		cudaError_t e_ = (call);                                                                                      \
		if (e_ != cudaSuccess) return cuda_fail(e_, what);                                                             \
	} while (0)

struct DeviceGuard
{
	int prev = -1;
	explicit DeviceGuard(int dev)
	{
		cudaGetDevice(&prev);
		if (prev != dev) cudaSetDevice(dev);
	}
	~DeviceGuard()
	{
		if (prev >= 0) cudaSetDevice(prev);
	}
};

// A device allocation that grows on demand.
struct DevBuf
{
	void* p = nullptr;
	size_t cap = 0;
	cudaError_t reserve(size_t bytes)
	{
		if (bytes <= cap) return cudaSuccess;
		if (p) cudaFree(p);
		p = nullptr;
		cap = 0;
		const size_t want = std::max(bytes, (size_t)4096);
		cudaError_t e = cudaMalloc(&p, want);
		if (e == cudaSuccess) cap = want;
		return e;
	}
	void release()
	{
		if (p) cudaFree(p);
		p = nullptr;
		cap = 0;
	}
};

struct HostBuf
{
	void* p = nullptr;
	size_t cap = 0;
	cudaError_t reserve(size_t bytes)
	{
		if (bytes <= cap) return cudaSuccess;
		if (p) cudaFreeHost(p);
		p = nullptr;
		cap = 0;
		const size_t want = std::max(bytes, (size_t)4096);
		cudaError_t e = cudaMallocHost(&p, want);
		if (e == cudaSuccess) cap = want;
		return e;
	}
	void release()
	{
		if (p) cudaFreeHost(p);
		p = nullptr;
		cap = 0;
	}
};

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ---- registered host buffers (nncu_host_register) ----------------------------
// Ranges of host memory the caller pinned through the library, keyed by
// their start: a synchronous call whose every host buffer lies inside them
// moves its inputs and outputs with kernels reading and writing the
// device's mapping of that memory, instead of host copies through staging.
struct Registered
{
	size_t bytes;
	char* dev; // the device's address of the range's first byte
};
std::mutex g_reg_mu;
std::map<uintptr_t, Registered> g_reg;

// The device address of [p, p + bytes) if it lies inside one registered
// range; nullptr otherwise.
void* mapped(const void* p, size_t bytes)
{
	const uintptr_t a = reinterpret_cast<uintptr_t>(p);
	std::lock_guard<std::mutex> g(g_reg_mu);
	auto it = g_reg.upper_bound(a);
	if (it == g_reg.begin()) return nullptr;
	--it;
	if (a + bytes > it->first + it->second.bytes) return nullptr;
	return it->second.dev + (a - it->first);
}


// ---- the phase profiler (nnc_perf_*, runtime.h:147-195, on CUDA events) ----
std::atomic<uint64_t> g_launches{0};
std::atomic<bool> g_perf_on{false};
std::mutex g_perf_mu;
struct PerfPending
{
	int slot;
	cudaEvent_t a, b;
	uint64_t bytes;
};
std::vector<PerfPending> g_perf_pending;
std::vector<cudaEvent_t> g_perf_free;
nncu_perf_phase g_perf[NNCU_PERF_COUNT];
std::string g_perf_text;

cudaEvent_t perf_event()
{
	if (!g_perf_free.empty())
	{
		cudaEvent_t e = g_perf_free.back();
		g_perf_free.pop_back();
		return e;
	}
	cudaEvent_t e = nullptr;
	cudaEventCreate(&e);
	return e;
}

// Brackets one launch: records an event before and after it on `st` when the
// profiler is on, and counts the launch either way.
struct PerfScope
{
	int slot;
	uint64_t bytes;
	cudaStream_t st;
	cudaEvent_t a = nullptr;
	PerfScope(int slot_, uint64_t bytes_, cudaStream_t st_) : slot(slot_), bytes(bytes_), st(st_)
	{
		if (g_perf_on.load(std::memory_order_relaxed))
		{
			std::lock_guard<std::mutex> lk(g_perf_mu);
			a = perf_event();
			if (a) cudaEventRecord(a, st);
		}
	}
	~PerfScope()
	{
		g_launches.fetch_add(1, std::memory_order_relaxed);
		if (!a) return;
		std::lock_guard<std::mutex> lk(g_perf_mu);
		cudaEvent_t b = perf_event();
		if (!b) return;
		cudaEventRecord(b, st);
		g_perf_pending.push_back({slot, a, b, bytes});
	}
};
} // namespace

void nncu::note_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

// ---- the cache object ---------------------------------------------------------------

struct Buffer
{
	int rows = 0;       // logical rows (model_kv_buffer::rows)
	int rows_alloc = 0; // allocated rows: a multiple of 256 (rings already are)
	int window = 0;     // a ring's window; 0 for a full buffer
	size_t seq_bytes = 0;
	void* k = nullptr;
	void* v = nullptr;
	void* tmaps = nullptr; // the tensor-core kernel's maps over k and v (device memory, made on first use)
};

struct nncu_kv
{
	int device = 0;
	int n_layer = 0, n_seq = 1, n_ctx = 0, n_batch = 1, kv_type = KV_BF16;
	bool causal = true;
	int num_sms = 148;
	std::vector<nncu_layer_desc> layers;
	std::vector<int> kv_buf; // layer -> buffer index
	std::vector<Buffer> bufs;
	std::vector<int> cur_pos, kv_written; // per sequence
	int max_rewind = INT_MAX;
	size_t bytes = 0;

	cudaStream_t stream = nullptr; // the host-pointer calls' stream
	int* err_dev = nullptr;        // device error word (bounded waits)
	DevBuf stage_dev, parts, counters, qbuf;
	DevBuf fwd; // attention_forward's q / gate / k / v / attention rows and block sums
	std::vector<nncu_attn_job> fwd_jobs;
	HostBuf stage_host;
	// The job tables go up on their own stream through a ring of slots, so
	// the upload of one call's table overlaps the previous call's kernels
	// instead of sitting between them in the launching stream.
	struct JobSlot
	{
		DevBuf dev;
		HostBuf host;
		cudaEvent_t up = nullptr;   // the upload from `host` into `dev` is done
		cudaEvent_t used = nullptr; // the kernels that read `dev` are done
		bool ever = false;
	};
	static constexpr int JOB_SLOTS = 4;
	JobSlot slots[JOB_SLOTS];
	int slot_next = 0;
	cudaStream_t up = nullptr; // the upload stream
	cudaEvent_t done = nullptr;          // the last submission's kernels have finished: calls on one
	                                     // cache are ordered on the device whatever their streams
	cudaStream_t last_stream = nullptr;  // the stream `done` was recorded on
	bool any_call = false;
	std::map<std::pair<uint32_t, int>, float*> rope_tables;
	std::vector<DevJob> jobs_tmp;
	std::vector<CtaStart> starts_tmp;
	int counters_n = 0;
	bool no_tc = false; // keep 16-bit multi-row launches on the CUDA-core kernel (nncu_kv_set_option)

	~nncu_kv()
	{
		DeviceGuard g(device);
		if (stream) cudaStreamSynchronize(stream);
		for (auto& b : bufs)
		{
			if (b.k) cudaFree(b.k);
			if (b.v) cudaFree(b.v);
			if (b.tmaps) cudaFree(b.tmaps);
		}
		for (auto& kv : rope_tables) cudaFree(kv.second);
		if (err_dev) cudaFree(err_dev);
		for (auto& sl : slots)
		{
			sl.dev.release();
			sl.host.release();
			if (sl.up) cudaEventDestroy(sl.up);
			if (sl.used) cudaEventDestroy(sl.used);
		}
		stage_dev.release();
		qbuf.release();
		fwd.release();
		parts.release();
		counters.release();
		stage_host.release();
		if (done) cudaEventDestroy(done);
		if (stream) cudaStreamDestroy(stream);
		if (up) cudaStreamDestroy(up);
	}
};

// ---- small host functions --------------------------------------------------------

extern "C" {

const char* nncu_status_string(int status)
{
	switch (status)
	{
	case NNCU_OK: return "ok";
	case NNCU_ERR_INVALID_ARGUMENT: return "invalid argument";
	case NNCU_ERR_UNSUPPORTED: return "no usable sm_100 device";
	case NNCU_ERR_OUT_OF_MEMORY: return "out of memory";
	case NNCU_ERR_CONTEXT_FULL: return "context full";
	case NNCU_ERR_DEVICE: return "CUDA error";
	case NNCU_ERR_TIMEOUT: return "a bounded wait timed out";
	default: return "unknown status";
	}
}

const char* nncu_last_error(void) { return t_msg; }
int nncu_last_status(void) { return t_status; }
void nncu_clear_error(void)
{
	t_status = NNCU_OK;
	t_msg[0] = 0;
}

const char* nncu_version(void) { return "libnncu 0.1 (sm_100a)"; }

int nncu_device_check(int device)
{
	int n = 0;
	cudaError_t e = cudaGetDeviceCount(&n);
	if (e != cudaSuccess || n == 0) return fail(NNCU_ERR_UNSUPPORTED, "no CUDA device is visible");
	if (device < 0 || device >= n) return fail(NNCU_ERR_INVALID_ARGUMENT, "device %d does not exist (%d visible)", device, n);
	cudaDeviceProp prop;
	CU(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
	if (prop.major != 10)
		return fail(NNCU_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build is for sm_100a (B200)", device, prop.major,
		            prop.minor);
	return NNCU_OK;
}

void nncu_attn_span(int causal, int window, int pos, int n_seq, int* first, int* last)
{
	// model.cpp:2300-2316
	if (causal)
	{
		*first = (window > 0 && pos + 1 > window) ? pos + 1 - window : 0;
		*last = std::min(pos, n_seq - 1);
		return;
	}
	*first = 0;
	*last = n_seq - 1;
	if (window > 0)
	{
		const int half = window / 2;
		*first = std::max(0, pos - half);
		*last = std::min(n_seq - 1, pos + half);
	}
}

} // extern "C"

// ---- rope tables ----------------------------------------------------------------------

namespace
{
// The inverse frequencies of nnc_rope_f32 (nn_ops.cpp:1844-1856): the fp32
// recurrence inv *= base^(-2/n_rot), formed on the host with the same libm
// and the same fp32 operations, so the device multiplies exactly these values.
void rope_inv_table(float base, int n_rot, std::vector<float>& out)
{
	const int half = n_rot / 2;
	out.resize(half);
	const float ratio = std::pow(base, -2.0f / static_cast<float>(n_rot));
	float inv = 1.0f;
	for (int i = 0; i < half; ++i)
	{
		out[i] = inv;
		inv *= ratio;
	}
}

int rope_table(nncu_kv* kv, float base, int n_rot, const float** out)
{
	*out = nullptr;
	if (n_rot <= 0) return NNCU_OK;
	uint32_t bits;
	std::memcpy(&bits, &base, 4);
	auto key = std::make_pair(bits, n_rot);
	auto it = kv->rope_tables.find(key);
	if (it != kv->rope_tables.end())
	{
		*out = it->second;
		return NNCU_OK;
	}
	std::vector<float> tab;
	rope_inv_table(base, n_rot, tab);
	tab.resize((tab.size() + 3) & ~size_t(3), 0.0f); // whole 16-byte pieces: the decode kernel bulk-copies it
	float* d = nullptr;
	CU(cudaMalloc(&d, tab.size() * sizeof(float)), "rope table");
	cudaError_t e = cudaMemcpy(d, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice);
	if (e != cudaSuccess)
	{
		cudaFree(d);
		return cuda_fail(e, "rope table upload");
	}
	kv->rope_tables[key] = d;
	*out = d;
	return NNCU_OK;
}
} // namespace

// ---- the cache ----------------------------------------------------------------------------

namespace
{
// model_kv_init's checks and sizing (model.cpp:1891-1962), device-free.
int kv_layout(const nncu_layer_desc* layers, int32_t n_layer, const nncu_kv_params* p, std::vector<int>& kv_buf,
              std::vector<Buffer>& bufs, int& max_rewind)
{
	if (!layers || !p || n_layer <= 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "no layers");
	if (p->n_ctx <= 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "the context size must be positive");
	if (p->n_seq <= 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "n_seq must be positive");
	if (p->kv_type != KV_BF16 && p->kv_type != KV_F32 && p->kv_type != KV_F16)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "unknown K/V type %d", p->kv_type);
	for (int li = 0; li < n_layer; ++li)
	{
		const nncu_layer_desc& L = layers[li];
		if (L.n_kv <= 0 || L.head_dim <= 0 || L.head_dim > 512 || L.window < 0)
			return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d: bad shape (n_kv %d, head_dim %d, window %d)", li, L.n_kv,
			            L.head_dim, L.window);
		if (L.kv_layer < 0 || L.kv_layer >= n_layer)
			return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d: kv_layer %d out of range", li, L.kv_layer);
		const nncu_layer_desc& O = layers[L.kv_layer];
		if (O.kv_layer != L.kv_layer)
			return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d reads layer %d, which owns no cache", li, L.kv_layer);
		if (p->causal && (O.n_kv != L.n_kv || O.head_dim != L.head_dim))
			return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d reads a cache of another shape", li);
	}
	const size_t es = kv_esize(p->kv_type);
	const int nb = p->n_batch > 0 ? p->n_batch : 1;
	kv_buf.assign(n_layer, 0);
	max_rewind = INT_MAX;
	if (!p->causal)
	{
		// a bidirectional model: one n_ctx-row buffer that every layer rewrites
		bufs.assign(1, Buffer{});
		Buffer& b = bufs[0];
		b.rows = p->n_ctx;
		b.rows_alloc = (int)align_up((size_t)p->n_ctx, ATTN_BLOCK);
		size_t max_head = 0;
		for (int li = 0; li < n_layer; ++li) max_head = std::max(max_head, (size_t)layers[li].n_kv * layers[li].head_dim);
		b.seq_bytes = max_head * b.rows_alloc * es;
		return NNCU_OK;
	}
	// a sliding layer's buffer becomes a ring when that saves memory and every
	// layer reading it slides the same way
	std::vector<int> ring_window(n_layer, 0);
	std::vector<bool> can_ring(n_layer, true);
	for (int li = 0; li < n_layer; ++li)
	{
		const nncu_layer_desc& L = layers[li];
		const int owner = L.kv_layer;
		if (L.window == 0) can_ring[owner] = false;
		else if (ring_window[owner] == 0) ring_window[owner] = L.window;
		else if (ring_window[owner] != L.window) can_ring[owner] = false;
	}
	bufs.assign(n_layer, Buffer{});
	for (int li = 0; li < n_layer; ++li)
	{
		const nncu_layer_desc& L = layers[li];
		kv_buf[li] = L.kv_layer;
		if (L.kv_layer != li) continue;
		Buffer& b = bufs[li];
		const int w = ring_window[li];
		const int ring = (int)align_up((size_t)w + nb, ATTN_BLOCK);
		const bool is_ring = can_ring[li] && w > 0 && ring < p->n_ctx;
		b.rows = is_ring ? ring : p->n_ctx;
		b.rows_alloc = (int)align_up((size_t)b.rows, ATTN_BLOCK);
		b.window = is_ring ? w : 0;
		if (b.window) max_rewind = std::min(max_rewind, b.rows - b.window);
		b.seq_bytes = (size_t)L.n_kv * L.head_dim * b.rows_alloc * es;
	}
	return NNCU_OK;
}
} // namespace

extern "C" int nncu_kv_plan(const nncu_layer_desc* layers, int32_t n_layer, const nncu_kv_params* p,
                            nncu_kv_layer_info* per_layer, int32_t* max_rewind, size_t* bytes)
{
	std::vector<int> kv_buf;
	std::vector<Buffer> bufs;
	int mr = INT_MAX;
	int rc = kv_layout(layers, n_layer, p, kv_buf, bufs, mr);
	if (rc != NNCU_OK) return rc;
	const size_t es = kv_esize(p->kv_type);
	size_t total = 0;
	for (const auto& b : bufs)
		if (b.rows) total += 2 * b.seq_bytes * p->n_seq;
	if (per_layer)
		for (int li = 0; li < n_layer; ++li)
		{
			const Buffer& b = bufs[kv_buf[li]];
			nncu_kv_layer_info& o = per_layer[li];
			o.buffer = kv_buf[li];
			o.rows = b.rows;
			o.window = b.window;
			o.n_kv = layers[li].n_kv;
			o.head_dim = layers[li].head_dim;
			o.kv_type = p->kv_type;
			o.head_bytes = (size_t)b.rows_alloc * layers[li].head_dim * es;
			o.seq_bytes = b.seq_bytes;
			o.k = nullptr;
			o.v = nullptr;
		}
	if (max_rewind) *max_rewind = mr;
	if (bytes) *bytes = total;
	return NNCU_OK;
}

extern "C" int nncu_kv_create(const nncu_layer_desc* layers, int32_t n_layer, const nncu_kv_params* p, nncu_kv** out)
{
	if (!out) return fail(NNCU_ERR_INVALID_ARGUMENT, "out is NULL");
	*out = nullptr;
	std::vector<int> kv_buf;
	std::vector<Buffer> bufs;
	int max_rewind = INT_MAX;
	int rc = kv_layout(layers, n_layer, p, kv_buf, bufs, max_rewind);
	if (rc != NNCU_OK) return rc;
	rc = nncu_device_check(p->device);
	if (rc != NNCU_OK) return rc;

	nncu_kv* kv = new (std::nothrow) nncu_kv();
	if (!kv) return fail(NNCU_ERR_OUT_OF_MEMORY, "out of host memory");
	DeviceGuard guard(p->device);
	kv->device = p->device;
	kv->n_layer = n_layer;
	kv->n_seq = p->n_seq;
	kv->n_ctx = p->n_ctx;
	kv->n_batch = p->n_batch > 0 ? p->n_batch : 1;
	kv->kv_type = p->kv_type;
	kv->causal = p->causal != 0;
	kv->layers.assign(layers, layers + n_layer);
	kv->kv_buf = kv_buf;
	kv->bufs = bufs;
	kv->max_rewind = max_rewind;
	kv->cur_pos.assign(p->n_seq, 0);
	kv->kv_written.assign(p->n_seq, 0);
	cudaDeviceGetAttribute(&kv->num_sms, cudaDevAttrMultiProcessorCount, p->device);

	auto fail_free = [&](int status) {
		delete kv;
		return status;
	};
	for (auto& b : kv->bufs)
	{
		if (b.rows == 0) continue;
		const size_t n = b.seq_bytes * kv->n_seq;
		cudaError_t e = cudaMalloc(&b.k, n);
		if (e == cudaSuccess) e = cudaMalloc(&b.v, n);
		if (e == cudaSuccess) e = cudaMemset(b.k, 0, n);
		if (e == cudaSuccess) e = cudaMemset(b.v, 0, n);
		if (e != cudaSuccess)
		{
			cudaGetLastError();
			const int st = e == cudaErrorMemoryAllocation
			                   ? fail(NNCU_ERR_OUT_OF_MEMORY, "out of memory allocating a %d-token context", p->n_ctx)
			                   : cuda_fail(e, "K/V allocation");
			return fail_free(st);
		}
		kv->bytes += 2 * n;
	}
	cudaError_t e = cudaStreamCreateWithFlags(&kv->stream, cudaStreamNonBlocking);
	if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&kv->up, cudaStreamNonBlocking);
	for (auto& sl : kv->slots)
	{
		if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sl.up, cudaEventDisableTiming);
		if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sl.used, cudaEventDisableTiming);
	}
	if (e == cudaSuccess) e = cudaMalloc(&kv->err_dev, sizeof(int));
	if (e == cudaSuccess) e = cudaMemset(kv->err_dev, 0, sizeof(int));
	if (e == cudaSuccess) e = cudaEventCreateWithFlags(&kv->done, cudaEventDisableTiming);
	if (e != cudaSuccess) return fail_free(cuda_fail(e, "cache set-up"));
	*out = kv;
	return NNCU_OK;
}

extern "C" void nncu_kv_free(nncu_kv* kv) { delete kv; }

extern "C" int nncu_kv_set_tensor_cores(nncu_kv* kv, int enabled)
{
	if (!kv) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL cache");
	kv->no_tc = enabled == 0;
	return NNCU_OK;
}

extern "C" int nncu_kv_layer(const nncu_kv* kv, int32_t layer, nncu_kv_layer_info* out)
{
	if (!kv || !out) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL argument");
	if (layer < 0 || layer >= kv->n_layer) return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d out of range", layer);
	const nncu_layer_desc& L = kv->layers[layer];
	const int bi = kv->kv_buf[layer];
	const Buffer& b = kv->bufs[bi];
	const size_t es = kv_esize(kv->kv_type);
	out->buffer = bi;
	out->rows = b.rows;
	out->window = b.window;
	out->n_kv = L.n_kv;
	out->head_dim = L.head_dim;
	out->kv_type = kv->kv_type;
	out->head_bytes = (size_t)b.rows_alloc * L.head_dim * es;
	out->seq_bytes = b.seq_bytes;
	out->k = b.k;
	out->v = b.v;
	return NNCU_OK;
}

extern "C" int nncu_kv_get_state(const nncu_kv* kv, int32_t seq, nncu_kv_state* out)
{
	if (!kv || !out) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL argument");
	if (seq < 0 || seq >= kv->n_seq) return fail(NNCU_ERR_INVALID_ARGUMENT, "sequence %d out of range", seq);
	out->cur_pos = kv->cur_pos[seq];
	out->kv_written = kv->kv_written[seq];
	out->max_rewind = kv->max_rewind;
	out->n_ctx = kv->n_ctx;
	out->bytes = kv->bytes;
	return NNCU_OK;
}

extern "C" int nncu_kv_rewind(nncu_kv* kv, int32_t seq, int32_t pos)
{
	// model_kv_rewind (model.cpp:2137-2143)
	if (!kv) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL cache");
	if (seq < 0 || seq >= kv->n_seq) return fail(NNCU_ERR_INVALID_ARGUMENT, "sequence %d out of range", seq);
	if (pos < 0 || pos > kv->cur_pos[seq])
		return fail(NNCU_ERR_INVALID_ARGUMENT, "cannot rewind to %d: the cache is at %d", pos, kv->cur_pos[seq]);
	if (pos > 0 && kv->kv_written[seq] - pos > kv->max_rewind)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "cannot rewind to %d: a ring holds only %d positions below %d", pos,
		            kv->max_rewind, kv->kv_written[seq]);
	kv->cur_pos[seq] = pos;
	return NNCU_OK;
}

extern "C" int nncu_kv_commit(nncu_kv* kv, int32_t seq, int32_t pos0, int32_t n_tok)
{
	// the end of model_forward (model.cpp:2130-2133)
	if (!kv) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL cache");
	if (seq < 0 || seq >= kv->n_seq) return fail(NNCU_ERR_INVALID_ARGUMENT, "sequence %d out of range", seq);
	if (pos0 < 0 || n_tok < 0 || pos0 + n_tok > kv->n_ctx)
		return fail(NNCU_ERR_CONTEXT_FULL, "positions %d..%d exceed the context of %d", pos0, pos0 + n_tok, kv->n_ctx);
	kv->cur_pos[seq] = pos0 + n_tok;
	kv->kv_written[seq] = std::max(pos0 == 0 ? 0 : kv->kv_written[seq], kv->cur_pos[seq]);
	return NNCU_OK;
}

namespace
{
int kv_rows_copy(const nncu_kv* kv, int32_t layer, int32_t seq, int32_t pos0, int32_t n, const void* k_src,
                 const void* v_src, void* k_dst, void* v_dst, bool to_device)
{
	if (!kv) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL cache");
	if (layer < 0 || layer >= kv->n_layer) return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d out of range", layer);
	if (seq < 0 || seq >= kv->n_seq) return fail(NNCU_ERR_INVALID_ARGUMENT, "sequence %d out of range", seq);
	if (pos0 < 0 || n < 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "negative position or count");
	const nncu_layer_desc& L = kv->layers[layer];
	const Buffer& b = kv->bufs[kv->kv_buf[layer]];
	if (n > b.rows) return fail(NNCU_ERR_INVALID_ARGUMENT, "%d rows do not fit a buffer of %d", n, b.rows);
	if (!b.window && pos0 + n > b.rows)
		return fail(NNCU_ERR_CONTEXT_FULL, "positions up to %d exceed the buffer's %d rows", pos0 + n, b.rows);
	DeviceGuard g(kv->device);
	const size_t es = kv_esize(kv->kv_type);
	const size_t D = L.head_dim, row_bytes = D * es, host_pitch = (size_t)L.n_kv * row_bytes;
	const size_t head_bytes = (size_t)b.rows_alloc * row_bytes;
	int done = 0;
	while (done < n)
	{
		const int p = pos0 + done;
		const int row = p % b.rows_alloc;
		const int run = std::min(n - done, b.rows_alloc - row); // rows up to the ring's end
		for (int h = 0; h < L.n_kv; ++h)
		{
			const size_t dev_off = (size_t)seq * b.seq_bytes + (size_t)h * head_bytes + (size_t)row * row_bytes;
			const size_t host_off = (size_t)done * host_pitch + (size_t)h * row_bytes;
			for (int which = 0; which < 2; ++which)
			{
				if (to_device)
				{
					const char* src = static_cast<const char*>(which ? v_src : k_src);
					char* dst = static_cast<char*>(which ? b.v : b.k);
					if (!src) continue;
					CU(cudaMemcpy2D(dst + dev_off, row_bytes, src + host_off, host_pitch, row_bytes, run,
					                cudaMemcpyDefault),
					   "cache write");
				}
				else
				{
					const char* src = static_cast<const char*>(which ? b.v : b.k);
					char* dst = static_cast<char*>(which ? v_dst : k_dst);
					if (!dst) continue;
					CU(cudaMemcpy2D(dst + host_off, host_pitch, src + dev_off, row_bytes, row_bytes, run,
					                cudaMemcpyDefault),
					   "cache read");
				}
			}
		}
		done += run;
	}
	return NNCU_OK;
}
} // namespace

extern "C" int nncu_kv_write_rows(nncu_kv* kv, int32_t layer, int32_t seq, int32_t pos0, int32_t n, const void* k_rows,
                                  const void* v_rows)
{
	return kv_rows_copy(kv, layer, seq, pos0, n, k_rows, v_rows, nullptr, nullptr, true);
}

extern "C" int nncu_kv_read_rows(const nncu_kv* kv, int32_t layer, int32_t seq, int32_t pos0, int32_t n, void* k_rows,
                                 void* v_rows)
{
	return kv_rows_copy(kv, layer, seq, pos0, n, nullptr, nullptr, k_rows, v_rows, false);
}

// ---- the attention op ----------------------------------------------------------------------

namespace
{

int validate_job(const nncu_kv* kv, const nncu_attn_job& j)
{
	const nncu_attn_params& p = j.p;
	if (j.layer < 0 || j.layer >= kv->n_layer) return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d out of range", j.layer);
	if (j.seq < 0 || j.seq >= kv->n_seq) return fail(NNCU_ERR_INVALID_ARGUMENT, "sequence %d out of range", j.seq);
	const nncu_layer_desc& L = kv->layers[j.layer];
	const Buffer& b = kv->bufs[kv->kv_buf[j.layer]];
	if (p.n_kv != L.n_kv || p.head_dim != L.head_dim)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d: n_kv %d / head_dim %d do not match the cache's %d / %d",
		            j.layer, p.n_kv, p.head_dim, L.n_kv, L.head_dim);
	if (p.n_head <= 0 || p.n_head % p.n_kv != 0)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "n_head %d is not a multiple of n_kv %d", p.n_head, p.n_kv);
	if (!decode_supported(p.head_dim, kv->kv_type))
		return fail(NNCU_ERR_INVALID_ARGUMENT, "head_dim %d: the device path takes 64, 128, 256 or 512", p.head_dim);
	if (p.n_tok <= 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "n_tok must be positive");
	if (p.n_tok > kv->n_batch)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "%d tokens exceed the cache's batch of %d", p.n_tok, kv->n_batch);
	if (p.pos0 < 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "negative position");
	if (p.pos0 + p.n_tok > kv->n_ctx)
		return fail(NNCU_ERR_CONTEXT_FULL, "positions %d..%d exceed the context of %d", p.pos0, p.pos0 + p.n_tok - 1,
		            kv->n_ctx);
	if (p.n_seq <= 0 || p.n_seq > kv->n_ctx) return fail(NNCU_ERR_INVALID_ARGUMENT, "n_seq %d out of range", p.n_seq);
	if (p.n_rot < 0 || p.n_rot > p.head_dim || (p.n_rot & 1))
		return fail(NNCU_ERR_INVALID_ARGUMENT, "n_rot %d must be even and at most head_dim", p.n_rot);
	if (p.rope_mode != NNCU_ROPE_NEOX && p.rope_mode != NNCU_ROPE_NORM)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "unknown rope mode %d", p.rope_mode);
	if (p.freq_factors && p.n_rot % 8)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "freq_factors need n_rot to be a multiple of 8 (it is %d)", p.n_rot);
	if (p.window < 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "negative window");
	if ((p.reuse_kv != 0) != (L.kv_layer != j.layer))
		return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d: reuse_kv %d disagrees with the cache (it reads layer %d)",
		            j.layer, p.reuse_kv, L.kv_layer);
	if (b.window && (!p.causal || p.window != b.window))
		return fail(NNCU_ERR_INVALID_ARGUMENT, "layer %d: a ring of window %d cannot serve window %d", j.layer, b.window,
		            p.window);
	if (!p.causal && p.pos0 + p.n_tok > p.n_seq)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "bidirectional: queries beyond the %d keys", p.n_seq);
	if (p.softcap < 0.0f || !(p.scale == p.scale)) return fail(NNCU_ERR_INVALID_ARGUMENT, "bad scale or softcap");
	return NNCU_OK;
}

// Jobs of one submission run concurrently: none may read a (buffer,
// sequence) another of them appends to, and no two may append to the same one.
int check_conflicts(const nncu_kv* kv, const nncu_attn_job* jobs, int n)
{
	if (n < 2) return NNCU_OK;
	std::map<std::pair<int, int>, std::pair<int, int>> use; // (buffer, seq) -> (jobs, appenders)
	for (int i = 0; i < n; ++i)
	{
		auto& u = use[{kv->kv_buf[jobs[i].layer], jobs[i].seq}];
		u.first += 1;
		u.second += jobs[i].p.reuse_kv ? 0 : 1;
	}
	for (const auto& kvp : use)
		if (kvp.second.second > 0 && kvp.second.first > 1)
			return fail(NNCU_ERR_INVALID_ARGUMENT,
			            "jobs of one call share buffer %d of sequence %d while one of them appends to it; "
			            "submit them in separate calls",
			            kvp.first.first, kvp.first.second);
	return NNCU_OK;
}

// The tensor maps of buffer `bi` for the tensor-core decode kernel, made
// once: [n_seq * n_kv planes][rows][head_dim] over its K and its V. They are
// never rewritten, so the kernels may cache them.
int buffer_tmaps(nncu_kv* kv, int bi, int D, int n_kv, const void** out)
{
	Buffer& b = kv->bufs[bi];
	if (!b.tmaps)
	{
		alignas(64) unsigned char h[2 * TENSOR_MAP_BYTES];
		int e = tc_make_maps(h, h + TENSOR_MAP_BYTES, b.k, b.v, kv->kv_type, D, b.rows_alloc,
		                     (long long)kv->n_seq * n_kv);
		if (e) return cuda_fail((cudaError_t)e, "tensor maps of the cache");
		void* dmem = nullptr;
		CU(cudaMalloc(&dmem, sizeof h), "tensor maps");
		cudaError_t ce = cudaMemcpy(dmem, h, sizeof h, cudaMemcpyHostToDevice);
		if (ce != cudaSuccess)
		{
			cudaFree(dmem);
			return cuda_fail(ce, "tensor maps upload");
		}
		b.tmaps = dmem;
	}
	*out = b.tmaps;
	return NNCU_OK;
}

// Turn one public job into a DevJob (device pointers already resolved).
void fill_devjob(nncu_kv* kv, const nncu_attn_job& j, DevJob& d)
{
	const nncu_attn_params& p = j.p;
	const Buffer& b = kv->bufs[kv->kv_buf[j.layer]];
	const size_t es = kv_esize(kv->kv_type);
	std::memset(&d, 0, sizeof d);
	d.q = j.q;
	d.k = j.k;
	d.v = j.v;
	d.out = j.out;
	d.q_gamma = p.q_gamma;
	d.k_gamma = p.k_gamma;
	d.freq_factors = p.freq_factors;
	d.gate = p.gate;
	d.K = static_cast<char*>(b.k) + (size_t)j.seq * b.seq_bytes;
	d.V = static_cast<char*>(b.v) + (size_t)j.seq * b.seq_bytes;
	d.head_bytes = (long long)b.rows_alloc * p.head_dim * es;
	d.rows = b.rows_alloc;
	d.n_tok = p.n_tok;
	d.pos0 = p.pos0;
	d.n_seq = p.n_seq;
	d.n_head = p.n_head;
	d.n_kv = p.n_kv;
	d.D = p.head_dim;
	d.n_rot = p.n_rot;
	d.rope_mode = p.rope_mode;
	d.causal = p.causal != 0;
	d.window = p.window;
	d.reuse_kv = p.reuse_kv != 0;
	d.v_rmsnorm = p.v_rmsnorm != 0;
	d.rope_scale = p.rope_scale;
	d.eps = p.eps;
	d.scale = p.scale;
	d.softcap = p.softcap;
	d.key_lo = 0;
	d.key_hi = INT_MAX;
	d.plane0 = j.seq * p.n_kv;
}

// The tensor maps of every job that the tensor-core decode kernel could take
// (16-bit cache, head_dim 64, 128 or 256).
int attach_tmaps(nncu_kv* kv, std::vector<DevJob>& jobs, const nncu_attn_job* pub)
{
	if (kv->kv_type == KV_F32) return NNCU_OK;
	for (size_t i = 0; i < jobs.size(); ++i)
	{
		const int D = jobs[i].D;
		if (D != 64 && D != 128 && D != 256) continue;
		const void* maps = nullptr;
		int rc = buffer_tmaps(kv, kv->kv_buf[pub[i].layer], D, pub[i].p.n_kv, &maps);
		if (rc != NNCU_OK) return rc;
		jobs[i].tmap_k = maps;
		jobs[i].tmap_v = static_cast<const char*>(maps) + TENSOR_MAP_BYTES;
	}
	return NNCU_OK;
}

// Launch K1 and K2 for jobs whose DevJob pointers are all device pointers,
// on `st`.
// A long causal batch on a bf16 cache of head_dim 128 (a prefill) runs on
// the tensor cores: one kernel does every head's norm and RoPE and appends
// the k, v rows, then the attention of every row (k_prefill.cu).
bool prefill_eligible(const nncu_kv* kv, const DevJob& j, const nncu_attn_job& pub)
{
	const Buffer& b = kv->bufs[kv->kv_buf[pub.layer]];
	// the prep kernel rotates NEOX pairs within a lane: n_rot / 2 of 32 or 64
	const bool rope_ok = j.rope_mode != NNCU_ROPE_NEOX || j.n_rot == 0 || j.n_rot == 64 || j.n_rot == 128;
	return prefill_supported(j.D, kv->kv_type) && j.causal && j.n_tok >= 128 && b.window == 0 && j.key_lo == 0 &&
	       j.key_hi == INT_MAX && rope_ok;
}

int run_prefill(nncu_kv* kv, const DevJob& j, cudaStream_t st)
{
	CU(kv->qbuf.reserve(prefill_qbuf_bytes(j.n_tok, j.n_head)), "prefill q scratch");
	const size_t es = kv_esize(kv->kv_type);
	const uint64_t kvb = j.reuse_kv ? 0 : (uint64_t)j.n_tok * j.n_kv * j.D;
	const uint64_t keys = (uint64_t)std::min(j.n_seq, j.pos0 + j.n_tok);
	int e = 0;
	{
		PerfScope ps(NNCU_PERF_ATTN_ROPE, kvb * (8 + 2 * es) + (uint64_t)j.n_tok * j.n_head * j.D * 6, st);
		e = launch_prefill_prep(j, kv->qbuf.p, st);
	}
	if (e) return cuda_fail((cudaError_t)e, "prefill norm, RoPE, append launch");
	{
		PerfScope ps(NNCU_PERF_ATTN_CORE,
		             keys * j.n_kv * j.D * es * 2 + (uint64_t)j.n_tok * j.n_head * j.D * (2 + 4), st);
		e = launch_prefill(j, kv->qbuf.p, kv->err_dev, st);
	}
	if (e) return cuda_fail((cudaError_t)e, "prefill attention launch");
	return NNCU_OK;
}

// A synchronous call's pinned staging block: the job table is written at
// `lead` (after the inputs) and goes up with the inputs in one transfer on
// the launching stream, instead of through the job slots.
struct Staged
{
	char* host;
	char* dev;
	size_t lead; // bytes before the table (16-byte aligned), uploaded with it
	size_t cap;  // room for the table
	size_t done; // bytes at the start already uploaded on the launching stream
};

// A synchronous call's inputs of at least this many bytes go up in groups
// of about this size, each group's upload overlapping the host copy of the
// next.
constexpr size_t STAGE_GROUP_BYTES = 512 << 10;
// A synchronous call moves its data with the copy kernels (registered host
// buffers) only from this many bytes in and out: below it, two more launches
// cost more than the host copies they replace.
constexpr size_t MAP_MIN_BYTES = 128 << 10;

// The rest of the staged inputs, [done, end), up on `st`.
cudaError_t staged_upload(const Staged* sg, size_t end, cudaStream_t st)
{
	if (end <= sg->done) return cudaSuccess;
	return cudaMemcpyAsync(sg->dev + sg->done, sg->host + sg->done, end - sg->done, cudaMemcpyHostToDevice, st);
}

int run_jobs(nncu_kv* kv, std::vector<DevJob>& jobs, const nncu_attn_job* pub, cudaStream_t st,
             nncu_group* group = nullptr, const Staged* staged = nullptr)
{
	int n = (int)jobs.size();
	for (int i = 0; i < n; ++i)
	{
		int rc = rope_table(kv, pub[i].p.freq_base, pub[i].p.n_rot, &jobs[i].rope_inv);
		if (rc != NNCU_OK) return rc;
	}
	if (!group)
	{
		int rc = attach_tmaps(kv, jobs, pub);
		if (rc != NNCU_OK) return rc;
	}
	// Every job of one launch shares head_dim (the kernels are specialised on it).
	for (int i = 1; i < n; ++i)
		if (jobs[i].D != jobs[0].D)
			return fail(NNCU_ERR_INVALID_ARGUMENT, "jobs of one call must share head_dim (%d vs %d)", jobs[i].D,
			            jobs[0].D);
	// the partials and counters are the cache's: a call on another stream than
	// the previous one waits for it on the device
	if (kv->any_call && kv->last_stream != st)
		CU(cudaStreamWaitEvent(st, kv->done, 0), "order after the previous call");
	// prefills one by one on the tensor cores; the rest together below
	if (!group)
	{
		int keep = 0;
		for (int i = 0; i < n; ++i)
		{
			if (prefill_eligible(kv, jobs[i], pub[i]))
			{
				int rc = run_prefill(kv, jobs[i], st);
				if (rc != NNCU_OK) return rc;
			}
			else
				jobs[keep++] = jobs[i];
		}
		jobs.resize(keep);
		n = keep;
		if (n == 0)
		{
			if (staged) CU(staged_upload(staged, staged->lead, st), "input upload");
			CU(cudaEventRecord(kv->done, st), "completion event");
			kv->last_stream = st;
			kv->any_call = true;
			return NNCU_OK;
		}
	}
	// several query rows per KV head on a 16-bit cache: the tensor-core kernel
	int rows_needed = 1;
	bool maps = true;
	for (int i = 0; i < n; ++i)
	{
		rows_needed = std::max(rows_needed, (jobs[i].n_head / jobs[i].n_kv) * jobs[i].n_tok);
		maps = maps && jobs[i].tmap_k != nullptr;
	}
	const int tc = !group && maps && !kv->no_tc ? tc_rows(jobs[0].D, kv->kv_type, rows_needed) : 0;
	DecodePlan P{};
	kv->starts_tmp.resize((size_t)kv->num_sms);
	int rc = plan_launch(jobs.data(), n, kv->kv_type, kv->num_sms, P, kv->starts_tmp.data(), kv->num_sms, true, tc);
	if (rc != NNCU_OK) return rc;
	P.err = kv->err_dev;
	P.world = 1;
	if (group)
	{
		// every GPU of the split sends a partial for every segment: each needs keys
		int n_rows = 0;
		for (int i = 0; i < n; ++i)
		{
			if (jobs[i].n_tiles == 0)
				return fail(NNCU_ERR_INVALID_ARGUMENT, "split: job %d sees no key in [%d, %d) on this GPU", i,
				            jobs[i].key_lo, jobs[i].key_hi);
			n_rows += jobs[i].n_tok * jobs[i].n_head;
		}
		rc = group_prepare(group, P, n_rows);
		if (rc != NNCU_OK) return rc;
	}
	// scratch for partials and the per-segment counters
	const size_t part_floats = (size_t)std::max<long long>(P.n_parts, 1) * P.RM * (P.D + 4);
	CU(kv->parts.reserve(part_floats * sizeof(float)), "partials scratch");
	if (P.n_segments > kv->counters_n)
	{
		CU(kv->counters.reserve((size_t)P.n_segments * sizeof(int)), "counters");
		CU(cudaMemsetAsync(kv->counters.p, 0, kv->counters.cap, st), "counters clear");
		kv->counters_n = (int)(kv->counters.cap / sizeof(int));
	}
	P.parts = static_cast<float*>(kv->parts.p);
	P.counters = static_cast<int*>(kv->counters.p);
	const size_t jb = align_up((size_t)n * sizeof(DevJob), 16);
	const size_t sb = (size_t)P.n_ctas * sizeof(CtaStart);
	nncu_kv::JobSlot* used = nullptr;
	InlineTable tab_inline;
	const InlineTable* tab = nullptr;
	if (!group && !staged && P.fused && jb + sb <= (size_t)INLINE_TABLE_BYTES)
	{
		// small enough to travel with the launch: no upload, no events
		std::memcpy(tab_inline.b, jobs.data(), (size_t)n * sizeof(DevJob));
		std::memcpy(tab_inline.b + jb, kv->starts_tmp.data(), sb);
		tab = &tab_inline;
	}
	else if (staged && jb + sb <= staged->cap)
	{
		std::memcpy(staged->host + staged->lead, jobs.data(), (size_t)n * sizeof(DevJob));
		std::memcpy(staged->host + staged->lead + jb, kv->starts_tmp.data(), sb);
		CU(staged_upload(staged, staged->lead + jb + sb, st), "input and job table upload");
		P.jobs = reinterpret_cast<const DevJob*>(staged->dev + staged->lead);
		P.cta_start = reinterpret_cast<const CtaStart*>(staged->dev + staged->lead + jb);
	}
	else
	{
		if (staged) CU(staged_upload(staged, staged->lead, st), "input upload");
		auto& slot = kv->slots[kv->slot_next];
		used = &slot;
		kv->slot_next = (kv->slot_next + 1) % nncu_kv::JOB_SLOTS;
		// its pinned copy was read (usually long since: a query is cheaper than a wait)
		cudaError_t q = cudaEventQuery(slot.up);
		if (q == cudaErrorNotReady) q = cudaEventSynchronize(slot.up);
		CU(q, "job table reuse");
		CU(slot.host.reserve(jb + sb), "job table (host)");
		if (slot.dev.cap < jb + sb)
		{
			CU(cudaStreamSynchronize(kv->up), "job table growth");
			CU(slot.dev.reserve(jb + sb), "job table (device)");
		}
		std::memcpy(slot.host.p, jobs.data(), (size_t)n * sizeof(DevJob));
		std::memcpy(static_cast<char*>(slot.host.p) + jb, kv->starts_tmp.data(), sb);
		// upload on the side stream once the kernels that last read this slot are
		// done; the launching stream waits only for the upload itself
		if (slot.ever) CU(cudaStreamWaitEvent(kv->up, slot.used, 0), "job table slot reuse");
		CU(cudaMemcpyAsync(slot.dev.p, slot.host.p, jb + sb, cudaMemcpyHostToDevice, kv->up), "job table upload");
		CU(cudaEventRecord(slot.up, kv->up), "job table event");
		CU(cudaStreamWaitEvent(st, slot.up, 0), "job table ready");
		P.jobs = static_cast<const DevJob*>(slot.dev.p);
		P.cta_start = reinterpret_cast<const CtaStart*>(static_cast<const char*>(slot.dev.p) + jb);
	}
	// algorithmic bytes: K1 reads k, v and writes the appended rows; K2 reads
	// the K/V rows of every key attended (once per KV head), q, and writes the output.
	// Jobs whose queries see no key at all produce zeros, as nnc_attn_finish does for l = 0.
	uint64_t rope_bytes = 0, core_bytes = 0;
	const size_t es = kv_esize(kv->kv_type);
	for (int i = 0; i < n; ++i)
	{
		const DevJob& j = jobs[i];
		const uint64_t qb = (uint64_t)j.n_tok * j.n_head * j.D * 4;
		const uint64_t kvb = j.reuse_kv ? 0 : (uint64_t)j.n_tok * j.n_kv * j.D;
		rope_bytes += kvb * 4 * 2 + kvb * es * 2;
		if (j.n_tiles == 0)
		{
			CU(cudaMemsetAsync(j.out, 0, qb, st), "empty output");
			continue;
		}
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
		core_bytes += (uint64_t)(last_max - first_min + 1) * j.n_kv * j.D * es * 2 + 2 * qb;
	}
	// K1 then K2, or K2 alone when it appends the new rows itself. After K1,
	// K2 is a programmatic dependent of it: its CTAs become resident while K1
	// runs and start streaming at once.
	int e = 0;
	if (!P.fused)
	{
		PerfScope ps(NNCU_PERF_ATTN_ROPE, rope_bytes, st);
		e = launch_prep(P, st);
	}
	if (e) return cuda_fail((cudaError_t)e, "K1 (norm, RoPE, append) launch");
	{
		PerfScope ps(NNCU_PERF_ATTN_CORE, core_bytes, st);
		e = tc ? launch_decode_tc(P, nullptr, st, tab) : launch_decode(P, st, tab);
	}
	if (e) return cuda_fail((cudaError_t)e, "K2 (attention) launch");
	if (group)
	{
		e = launch_split_wait(P, st);
		if (e) return cuda_fail((cudaError_t)e, "split wait launch");
	}
	if (used)
	{
		CU(cudaEventRecord(used->used, st), "job table slot event");
		used->ever = true;
	}
	CU(cudaEventRecord(kv->done, st), "completion event");
	kv->last_stream = st;
	kv->any_call = true;
	return NNCU_OK;
}

// The device error word `h` read back: a kernel's wait that timed out voids
// the call's output; the word is cleared for the next call.
int device_error_status(nncu_kv* kv, int h)
{
	if (h != 0)
	{
		cudaMemset(kv->err_dev, 0, sizeof(int));
		return fail(NNCU_ERR_TIMEOUT, "a kernel's bounded wait timed out (code %d); the output is void", h);
	}
	return NNCU_OK;
}

int check_device_error(nncu_kv* kv)
{
	int h = 0;
	CU(cudaMemcpy(&h, kv->err_dev, sizeof(int), cudaMemcpyDeviceToHost), "error word");
	return device_error_status(kv, h);
}

size_t fbytes(size_t n) { return align_up(n * sizeof(float), 256); }

JobPointers job_pointers(const nncu_attn_job& j)
{
	JobPointers p{};
	p.q = j.q;
	p.k = j.p.reuse_kv ? nullptr : j.k;
	p.v = j.p.reuse_kv ? nullptr : j.v;
	p.out = j.out;
	p.q_gamma = j.p.q_gamma;
	p.k_gamma = j.p.k_gamma;
	p.freq_factors = j.p.freq_factors;
	return p;
}

} // namespace

extern "C" int nncu_attention_batch_dev(nncu_kv* kv, const nncu_attn_job* jobs, int32_t n_jobs, void* stream)
{
	if (!kv || !jobs || n_jobs <= 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "no jobs");
	int rc = NNCU_OK;
	for (int i = 0; i < n_jobs; ++i)
	{
		rc = validate_job(kv, jobs[i]);
		if (rc != NNCU_OK) return rc;
		if (!jobs[i].q || !jobs[i].out || (!jobs[i].p.reuse_kv && (!jobs[i].k || !jobs[i].v)))
			return fail(NNCU_ERR_INVALID_ARGUMENT, "job %d: NULL input or output", i);
		rc = check_alignment(job_pointers(jobs[i]), i, "nncu_attention_batch_dev");
		if (rc != NNCU_OK) return rc;
	}
	rc = check_conflicts(kv, jobs, n_jobs);
	if (rc != NNCU_OK) return rc;
	DeviceGuard g(kv->device);
	kv->jobs_tmp.resize(n_jobs);
	for (int i = 0; i < n_jobs; ++i) fill_devjob(kv, jobs[i], kv->jobs_tmp[i]);
	return run_jobs(kv, kv->jobs_tmp, jobs, static_cast<cudaStream_t>(stream));
}

namespace
{

// attention_forward for n sequences of one layer: x and y hold their tokens
// one sequence after another; the gemvs run over all the tokens at once (one
// pass over the weights for the whole batch), the attention takes one job per
// sequence.
int forward_impl(nncu_kv* kv, int32_t layer, int32_t n, const int32_t* seqs, const nncu_attn_params* ps,
                 const nncu_attn_weights* w, const float* x, float* y, cudaStream_t st)
{
	if (!kv || !ps || !w || !x || !y || n <= 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL argument or no sequences");
	const nncu_attn_params& p0 = ps[0];
	std::vector<nncu_attn_job>& jobs = kv->fwd_jobs;
	jobs.assign((size_t)n, nncu_attn_job{});
	uint32_t n_tok = 0;
	for (int i = 0; i < n; ++i)
	{
		const nncu_attn_params& p = ps[i];
		if (p.gate) return fail(NNCU_ERR_INVALID_ARGUMENT, "the gate comes from the q projection: p->gate must be NULL");
		if (p.n_head != p0.n_head || p.n_kv != p0.n_kv || p.head_dim != p0.head_dim || p.reuse_kv != p0.reuse_kv)
			return fail(NNCU_ERR_INVALID_ARGUMENT, "sequence %d: the layer's heads differ from the first sequence's", i);
		for (int j = 0; j < i; ++j)
			if (seqs[j] == seqs[i]) return fail(NNCU_ERR_INVALID_ARGUMENT, "sequence %d appears twice", seqs[i]);
		jobs[i].layer = layer;
		jobs[i].seq = seqs[i];
		jobs[i].p = p;
		const int rc = validate_job(kv, jobs[i]);
		if (rc != NNCU_OK) return rc;
		n_tok += (uint32_t)p.n_tok;
	}
	const bool reuse = p0.reuse_kv != 0, gated = w->gated != 0;
	const uint32_t hd = (uint32_t)p0.head_dim;
	const uint32_t q_dim = (uint32_t)p0.n_head * hd, kv_dim = (uint32_t)p0.n_kv * hd, n_embd = w->o.rows;
	if (n_embd == 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "o: no rows");
	int rc = check_weight(w->q, (gated ? 2 : 1) * q_dim, n_embd, "q");
	if (rc == NNCU_OK && !reuse) rc = check_weight(w->k, kv_dim, n_embd, "k");
	if (rc == NNCU_OK && !reuse && w->v.data) rc = check_weight(w->v, kv_dim, n_embd, "v");
	if (rc == NNCU_OK) rc = check_weight(w->o, n_embd, q_dim, "o");
	if (rc != NNCU_OK) return rc;
	const size_t io = (size_t)n_tok * n_embd * sizeof(float);
	const char *xb = reinterpret_cast<const char*>(x), *yb = reinterpret_cast<const char*>(y);
	if (xb < yb + io && yb < xb + io) return fail(NNCU_ERR_INVALID_ARGUMENT, "x and y overlap");

	// V is the raw K projection without a v_proj; with a K bias it is a
	// second, unbiased K gemv (the reference copies V before adding biases)
	const bool v_own = !reuse && (w->v.data || w->k_bias);
	// Q4_S weights need the activations' block sums: one token's are formed
	// inside the gemv (no launch); several tokens' once, by a block-sum launch
	// (the gemv runs once per token and would form them every time)
	const bool q4_in = n_tok > 1 && (w->q.type == NNCU_W_Q4_S ||
	                                 (!reuse && (w->k.type == NNCU_W_Q4_S || (w->v.data && w->v.type == NNCU_W_Q4_S))));
	const bool q4_out = n_tok > 1 && w->o.type == NNCU_W_Q4_S;
	auto up64 = [](size_t v) { return (v + 63) & ~size_t(63); }; // 256-byte slots
	const size_t n_q = up64((size_t)n_tok * q_dim), n_kvr = up64((size_t)n_tok * kv_dim);
	const size_t o_q = 0, o_g = o_q + n_q, o_k = o_g + (gated ? n_q : 0), o_v = o_k + (reuse ? 0 : n_kvr);
	const size_t o_a = o_v + (v_own ? n_kvr : 0), o_xs = o_a + n_q;
	const size_t o_as = o_xs + (q4_in ? up64((size_t)n_tok * (n_embd / 32)) : 0);
	const size_t total = o_as + (q4_out ? up64((size_t)n_tok * (q_dim / 32)) : 0);

	DeviceGuard g(kv->device);
	// the scratch is the cache's: wait for the previous call on another stream
	if (kv->any_call && kv->last_stream != st)
		CU(cudaStreamWaitEvent(st, kv->done, 0), "order after the previous call");
	CU(kv->fwd.reserve(total * sizeof(float)), "attention_forward scratch");
	float* f = static_cast<float*>(kv->fwd.p);
	float *q = f + o_q, *gate = gated ? f + o_g : nullptr, *k = f + o_k, *v = v_own ? f + o_v : k, *attn = f + o_a;
	float* xs = q4_in ? f + o_xs : nullptr;
	float* as = q4_out ? f + o_as : nullptr;

	int e = 0;
	if (q4_in) e = launch_block_sums(x, xs, (size_t)n_tok * n_embd, st);
	// q, k and v in one launch per weight format
	Projection proj[3];
	int n_proj = 0;
	proj[n_proj++] = Projection{&w->q, q, q_dim, gate, gated ? hd : 0, w->q_bias};
	if (!reuse) proj[n_proj++] = Projection{&w->k, k, kv_dim, nullptr, 0, w->k_bias};
	if (v_own)
		proj[n_proj++] = Projection{w->v.data ? &w->v : &w->k, v, kv_dim, nullptr, 0, w->v.data ? w->v_bias : nullptr};
	if (!e) e = launch_projections(proj, n_proj, x, n_embd, xs, n_embd / 32, n_tok, st);
	if (e) return cuda_fail((cudaError_t)e, "attention_forward projections");

	size_t row = 0; // the sequence's first token among all
	for (int i = 0; i < n; ++i)
	{
		nncu_attn_job& j = jobs[i];
		j.p.gate = gate ? gate + row * q_dim : nullptr;
		j.q = q + row * q_dim;
		j.k = reuse ? nullptr : k + row * kv_dim;
		j.v = reuse ? nullptr : v + row * kv_dim;
		j.out = attn + row * q_dim;
		row += (size_t)j.p.n_tok;
	}
	rc = nncu_attention_batch_dev(kv, jobs.data(), n, st);
	if (rc != NNCU_OK) return rc;

	if (q4_out) e = launch_block_sums(attn, as, (size_t)n_tok * q_dim, st);
	const Projection po{&w->o, y, n_embd, nullptr, 0, nullptr};
	if (!e) e = launch_projections(&po, 1, attn, q_dim, as, q_dim / 32, n_tok, st);
	if (e) return cuda_fail((cudaError_t)e, "attention_forward output projection");
	CU(cudaEventRecord(kv->done, st), "completion event");
	kv->last_stream = st;
	kv->any_call = true;
	return NNCU_OK;
}

} // namespace

// attention_forward (model.cpp:1559-1768) on the device: the reference's
// sequence of gemv_batch calls, bias adds and the attention, with the
// query / gate split and the biases folded into the q / k / v gemvs'
// stores, and norms, RoPE, append, attend and the gate inside the attention
// kernels of nncu_attention_batch_dev.
extern "C" int nncu_attention_forward_dev(nncu_kv* kv, int32_t layer, int32_t seq, const nncu_attn_params* p,
                                          const nncu_attn_weights* w, const float* x, float* y, void* stream)
{
	return forward_impl(kv, layer, 1, &seq, p, w, x, y, static_cast<cudaStream_t>(stream));
}

extern "C" int nncu_attention_forward_batch_dev(nncu_kv* kv, int32_t layer, int32_t n_seqs, const int32_t* seqs,
                                                const nncu_attn_params* params, const nncu_attn_weights* w,
                                                const float* x, float* y, void* stream)
{
	if (!seqs) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL sequence list");
	return forward_impl(kv, layer, n_seqs, seqs, params, w, x, y, static_cast<cudaStream_t>(stream));
}

extern "C" int nncu_attention_split_dev(nncu_kv* kv, nncu_group* group, const nncu_attn_job* jobs, int32_t n_jobs,
                                        int32_t key_lo, int32_t key_hi, void* stream)
{
	if (!kv || !group || !jobs || n_jobs <= 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "no jobs or no group");
	if (group_device(group) != kv->device) return fail(NNCU_ERR_INVALID_ARGUMENT, "group and cache on different GPUs");
	if (key_lo < 0 || key_hi <= key_lo || key_lo % ATTN_BLOCK)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "split: keys [%d, %d) must be a non-empty range from a 256-key block",
		            key_lo, key_hi);
	for (int i = 0; i < n_jobs; ++i)
	{
		int rc = validate_job(kv, jobs[i]);
		if (rc != NNCU_OK) return rc;
		if (!jobs[i].q || (!jobs[i].p.reuse_kv && (!jobs[i].k || !jobs[i].v)))
			return fail(NNCU_ERR_INVALID_ARGUMENT, "job %d: NULL input", i);
		JobPointers jp = job_pointers(jobs[i]);
		jp.out = nullptr; // the merged rows land in the group's output
		rc = check_alignment(jp, i, "nncu_attention_split_dev");
		if (rc != NNCU_OK) return rc;
	}
	int rc = check_conflicts(kv, jobs, n_jobs);
	if (rc != NNCU_OK) return rc;
	DeviceGuard g(kv->device);
	kv->jobs_tmp.resize(n_jobs);
	int row = 0;
	for (int i = 0; i < n_jobs; ++i)
	{
		fill_devjob(kv, jobs[i], kv->jobs_tmp[i]);
		kv->jobs_tmp[i].key_lo = key_lo;
		kv->jobs_tmp[i].key_hi = key_hi;
		kv->jobs_tmp[i].out_row0 = row;
		kv->jobs_tmp[i].out = nullptr; // the merged rows land in the group's output
		row += jobs[i].p.n_tok * jobs[i].p.n_head;
	}
	return run_jobs(kv, kv->jobs_tmp, jobs, static_cast<cudaStream_t>(stream), group);
}

extern "C" int nncu_host_register(void* p, size_t bytes)
{
	if (!p || !bytes) return fail(NNCU_ERR_INVALID_ARGUMENT, "nothing to register");
	const uintptr_t a = reinterpret_cast<uintptr_t>(p);
	{
		std::lock_guard<std::mutex> g(g_reg_mu);
		auto it = g_reg.upper_bound(a + bytes - 1);
		if (it != g_reg.begin() && std::prev(it)->first + std::prev(it)->second.bytes > a)
			return fail(NNCU_ERR_INVALID_ARGUMENT, "host range %p+%zu overlaps a registered one", p, bytes);
	}
	cudaError_t e = cudaHostRegister(p, bytes, cudaHostRegisterMapped | cudaHostRegisterPortable);
	if (e != cudaSuccess) return cuda_fail(e, "cudaHostRegister");
	void* dev = nullptr;
	e = cudaHostGetDevicePointer(&dev, p, 0);
	if (e != cudaSuccess)
	{
		cudaHostUnregister(p);
		return cuda_fail(e, "cudaHostGetDevicePointer");
	}
	std::lock_guard<std::mutex> g(g_reg_mu);
	g_reg[a] = Registered{bytes, static_cast<char*>(dev)};
	return NNCU_OK;
}

extern "C" int nncu_host_unregister(void* p)
{
	{
		std::lock_guard<std::mutex> g(g_reg_mu);
		auto it = g_reg.find(reinterpret_cast<uintptr_t>(p));
		if (it == g_reg.end()) return fail(NNCU_ERR_INVALID_ARGUMENT, "%p was not registered", p);
		g_reg.erase(it);
	}
	CU(cudaHostUnregister(p), "cudaHostUnregister");
	return NNCU_OK;
}

extern "C" int nncu_attention_batch(nncu_kv* kv, const nncu_attn_job* jobs, int32_t n_jobs)
{
	if (!kv || !jobs || n_jobs <= 0) return fail(NNCU_ERR_INVALID_ARGUMENT, "no jobs");
	// Stage every input in one pinned block, copy it up in one transfer, run,
	// and bring every output back in one transfer.
	// per job: q, k, v, the q and k gains, the frequency factors, the gate
	constexpr int NIN = 7;
	std::vector<size_t> in_off(n_jobs * NIN), out_off(n_jobs);
	size_t in_bytes = 0, out_bytes = 0;
	for (int i = 0; i < n_jobs; ++i)
	{
		int rc = validate_job(kv, jobs[i]);
		if (rc != NNCU_OK) return rc;
		const nncu_attn_params& p = jobs[i].p;
		if (!jobs[i].q || !jobs[i].out || (!p.reuse_kv && (!jobs[i].k || !jobs[i].v)))
			return fail(NNCU_ERR_INVALID_ARGUMENT, "job %d: NULL input or output", i);
		const size_t qn = (size_t)p.n_tok * p.n_head * p.head_dim, kn = (size_t)p.n_tok * p.n_kv * p.head_dim;
		const size_t sizes[NIN] = {qn, p.reuse_kv ? 0 : kn, p.reuse_kv ? 0 : kn, p.q_gamma ? (size_t)p.head_dim : 0,
		                           p.k_gamma ? (size_t)p.head_dim : 0, p.freq_factors ? (size_t)p.n_rot / 2 : 0,
		                           p.gate ? qn : 0};
		for (int s = 0; s < NIN; ++s)
		{
			in_off[i * NIN + s] = in_bytes;
			in_bytes += fbytes(sizes[s]);
		}
		out_off[i] = out_bytes;
		out_bytes += fbytes(qn);
	}
	int rc0 = check_conflicts(kv, jobs, n_jobs);
	if (rc0 != NNCU_OK) return rc0;
	DeviceGuard g(kv->device);
	// the block: inputs, the job table (it goes up with them), outputs, and
	// (pinned side only) the error word, which comes back with the outputs
	const size_t table_cap =
		align_up(align_up((size_t)n_jobs * sizeof(DevJob), 16) + (size_t)kv->num_sms * sizeof(CtaStart), 256);
	const size_t out_base = in_bytes + table_cap;
	CU(kv->stage_host.reserve(out_base + out_bytes + 256), "pinned staging");
	CU(kv->stage_dev.reserve(out_base + out_bytes), "device staging");
	CU(cudaStreamSynchronize(kv->stream), "staging reuse");
	char* hs = static_cast<char*>(kv->stage_host.p);
	char* ds = static_cast<char*>(kv->stage_dev.p);
	std::vector<nncu_attn_job> dj(jobs, jobs + n_jobs);
	// Every host buffer registered (and enough bytes to pay for two more
	// launches): a kernel gathers the inputs through the device's mapping of
	// the caller's memory and another scatters the outputs back; no host copy.
	CopyList gather, scatter;
	gather.n = scatter.n = 0;
	bool use_map = in_bytes + out_bytes >= MAP_MIN_BYTES;
	for (int i = 0; i < n_jobs && use_map; ++i)
	{
		const nncu_attn_params& p = jobs[i].p;
		const size_t qn = (size_t)p.n_tok * p.n_head * p.head_dim, kn = (size_t)p.n_tok * p.n_kv * p.head_dim;
		const float* srcs[NIN] = {jobs[i].q, jobs[i].k, jobs[i].v, p.q_gamma, p.k_gamma, p.freq_factors, p.gate};
		const size_t sizes[NIN] = {qn, p.reuse_kv ? 0 : kn, p.reuse_kv ? 0 : kn, p.q_gamma ? (size_t)p.head_dim : 0,
		                           p.k_gamma ? (size_t)p.head_dim : 0, p.freq_factors ? (size_t)p.n_rot / 2 : 0,
		                           p.gate ? qn : 0};
		for (int s = 0; s < NIN && use_map; ++s)
		{
			if (!sizes[s]) continue;
			const void* src = mapped(srcs[s], sizes[s] * sizeof(float));
			use_map = src && gather.n < COPY_LIST_MAX;
			if (use_map) gather.e[gather.n++] = {src, ds + in_off[i * NIN + s], sizes[s] * sizeof(float), 0};
		}
		void* dst = use_map ? mapped(jobs[i].out, qn * sizeof(float)) : nullptr;
		use_map = dst && scatter.n < COPY_LIST_MAX;
		if (use_map) scatter.e[scatter.n++] = {ds + out_base + out_off[i], dst, qn * sizeof(float), 0};
	}
	struct CopyTask
	{
		void* dst;
		const void* src;
		size_t bytes;
	};
	std::vector<CopyTask> ins;
	ins.reserve((size_t)n_jobs * NIN);
	for (int i = 0; i < n_jobs; ++i)
	{
		const nncu_attn_params& p = jobs[i].p;
		const size_t qn = (size_t)p.n_tok * p.n_head * p.head_dim, kn = (size_t)p.n_tok * p.n_kv * p.head_dim;
		const float* srcs[NIN] = {jobs[i].q, jobs[i].k, jobs[i].v, p.q_gamma, p.k_gamma, p.freq_factors, p.gate};
		const size_t sizes[NIN] = {qn, p.reuse_kv ? 0 : kn, p.reuse_kv ? 0 : kn, p.q_gamma ? (size_t)p.head_dim : 0,
		                           p.k_gamma ? (size_t)p.head_dim : 0, p.freq_factors ? (size_t)p.n_rot / 2 : 0,
		                           p.gate ? qn : 0};
		const float* dptr[NIN];
		for (int s = 0; s < NIN; ++s)
		{
			dptr[s] = sizes[s] ? reinterpret_cast<const float*>(ds + in_off[i * NIN + s]) : nullptr;
			if (sizes[s]) ins.push_back({hs + in_off[i * NIN + s], srcs[s], sizes[s] * sizeof(float)});
		}
		dj[i].q = dptr[0];
		dj[i].k = dptr[1];
		dj[i].v = dptr[2];
		dj[i].p.q_gamma = dptr[3];
		dj[i].p.k_gamma = dptr[4];
		dj[i].p.freq_factors = dptr[5];
		dj[i].p.gate = dptr[6];
		dj[i].out = reinterpret_cast<float*>(ds + out_base + out_off[i]);
	}
	kv->jobs_tmp.resize(n_jobs);
	bool prefill = false; // a prefill launches before the plan: the inputs go up first
	for (int i = 0; i < n_jobs; ++i)
	{
		fill_devjob(kv, dj[i], kv->jobs_tmp[i]);
		prefill = prefill || prefill_eligible(kv, kv->jobs_tmp[i], dj[i]);
	}
	// Into the pinned block: a large batch goes up in a few groups, each
	// group's upload overlapping the next group's host copy; a small one goes
	// up with the job table in one transfer.
	size_t uploaded = 0;
	if (use_map)
	{
		CU((cudaError_t)launch_copy_list(gather, kv->stream), "input gather");
		uploaded = in_bytes;
	}
	else if (prefill || in_bytes >= STAGE_GROUP_BYTES)
	{
		size_t first = 0, group_end = 0;
		for (size_t t = 0; t < ins.size(); ++t)
		{
			const size_t end = static_cast<char*>(ins[t].dst) - hs + ins[t].bytes;
			if (end - group_end < STAGE_GROUP_BYTES && t + 1 < ins.size()) continue;
			for (size_t c = first; c <= t; ++c) std::memcpy(ins[c].dst, ins[c].src, ins[c].bytes);
			const size_t up_to = t + 1 < ins.size() ? end : in_bytes;
			CU(cudaMemcpyAsync(ds + uploaded, hs + uploaded, up_to - uploaded, cudaMemcpyHostToDevice, kv->stream),
			   "input upload");
			uploaded = group_end = up_to;
			first = t + 1;
		}
	}
	else
		for (const CopyTask& c : ins) std::memcpy(c.dst, c.src, c.bytes);
	const Staged staged{hs, ds, in_bytes, table_cap, uploaded};
	int rc = run_jobs(kv, kv->jobs_tmp, dj.data(), kv->stream, nullptr, prefill ? nullptr : &staged);
	if (rc != NNCU_OK) return rc;
	if (use_map)
		CU((cudaError_t)launch_copy_list(scatter, kv->stream), "output scatter");
	else
		CU(cudaMemcpyAsync(hs + out_base, ds + out_base, out_bytes, cudaMemcpyDeviceToHost, kv->stream),
		   "output download");
	int* err_h = reinterpret_cast<int*>(hs + out_base + out_bytes);
	CU(cudaMemcpyAsync(err_h, kv->err_dev, sizeof(int), cudaMemcpyDeviceToHost, kv->stream), "error word");
	CU(cudaStreamSynchronize(kv->stream), "attention");
	rc = device_error_status(kv, *err_h);
	if (rc != NNCU_OK) return rc;
	if (!use_map)
		for (int i = 0; i < n_jobs; ++i)
		{
			const nncu_attn_params& p = jobs[i].p;
			std::memcpy(jobs[i].out, hs + out_base + out_off[i],
			            (size_t)p.n_tok * p.n_head * p.head_dim * sizeof(float));
		}
	return NNCU_OK;
}

extern "C" int nncu_sync(nncu_kv* kv, void* stream)
{
	if (!kv) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL cache");
	DeviceGuard g(kv->device);
	CU(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "stream");
	return check_device_error(kv);
}

extern "C" int nncu_attention(nncu_kv* kv, int32_t layer, int32_t seq, const nncu_attn_params* p, const float* q,
                              const float* k, const float* v, float* out)
{
	if (!p) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL parameters");
	nncu_attn_job j{};
	j.layer = layer;
	j.seq = seq;
	j.p = *p;
	j.q = q;
	j.k = k;
	j.v = v;
	j.out = out;
	return nncu_attention_batch(kv, &j, 1);
}

// ---- unit seam on device pointers ----------------------------------------------------------------

namespace
{
int launched(int e, const char* what)
{
	if (e) return cuda_fail((cudaError_t)e, what);
	g_launches.fetch_add(1, std::memory_order_relaxed);
	return NNCU_OK;
}
} // namespace

extern "C" int nncu_attn_block_dev(const float* q, size_t q_stride, const void* K, const void* V, int kv_type,
                                   size_t kv_stride, size_t n_keys, size_t head_dim, size_t n_heads, float scale,
                                   float softcap, float* part, void* stream)
{
	if (kv_type != KV_F32 && kv_type != KV_BF16 && kv_type != KV_F16)
		return fail(NNCU_ERR_INVALID_ARGUMENT, "unknown K/V type %d", kv_type);
	if (head_dim == 0 || head_dim > 512) return fail(NNCU_ERR_INVALID_ARGUMENT, "head_dim %zu out of range", head_dim);
	if (n_keys == 0 || n_heads == 0) return NNCU_OK; // nnc_attn_block returns without writing
	if (!q || !K || !V || !part) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL pointer");
	return launched(launch_attn_block(q, q_stride, K, V, kv_type, kv_stride, n_keys, head_dim, n_heads, scale, softcap,
	                                  part, stream),
	                "attn_block");
}

extern "C" int nncu_attn_merge_dev(float* acc, const float* part, size_t head_dim, size_t n_heads, void* stream)
{
	if (!acc || !part) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL pointer");
	return launched(launch_attn_merge(acc, part, head_dim, n_heads, stream), "attn_merge");
}

extern "C" int nncu_attn_finish_dev(float* out, size_t out_stride, const float* acc, size_t head_dim, size_t n_heads,
                                    void* stream)
{
	if (!out || !acc) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL pointer");
	return launched(launch_attn_finish(out, out_stride, acc, head_dim, n_heads, stream), "attn_finish");
}

extern "C" int nncu_rmsnorm_gamma_multi_dev(float* y, const float* x, size_t n_groups, size_t dim, const float* gamma,
                                            float eps, void* stream)
{
	if (!y || !x || !gamma) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL pointer");
	return launched(launch_rmsnorm(y, x, n_groups, dim, gamma, eps, stream), "rmsnorm_gamma_multi");
}

extern "C" int nncu_rmsnorm_dev(float* y, const float* x, size_t n_groups, size_t dim, float eps, void* stream)
{
	if (!y || !x) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL pointer");
	return launched(launch_rmsnorm(y, x, n_groups, dim, nullptr, eps, stream), "rmsnorm");
}

namespace
{
std::mutex g_rope_mu;
std::map<std::tuple<int, uint32_t, int>, float*> g_rope_unit; // (device, base bits, n_rot) -> table
} // namespace

extern "C" int nncu_rope_dev(float* x, uint32_t n_tok, uint32_t n_heads, uint32_t head_dim, uint32_t n_rot,
                             int32_t pos0, float pos_scale, float freq_base, int mode, const float* freq_factors,
                             void* stream)
{
	if (!x) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL pointer");
	if (n_rot & 1u) return fail(NNCU_ERR_INVALID_ARGUMENT, "nnc_rope_f32: n_rot must be even");
	if (n_rot > head_dim || n_rot / 2 > 256) return fail(NNCU_ERR_INVALID_ARGUMENT, "n_rot %u out of range", n_rot);
	if (mode != NNCU_ROPE_NEOX && mode != NNCU_ROPE_NORM) return fail(NNCU_ERR_INVALID_ARGUMENT, "unknown rope mode");
	if (n_rot == 0) return NNCU_OK;
	int dev = 0;
	cudaGetDevice(&dev);
	uint32_t bits;
	std::memcpy(&bits, &freq_base, 4);
	float* tab = nullptr;
	{
		std::lock_guard<std::mutex> lk(g_rope_mu);
		auto key = std::make_tuple(dev, bits, (int)n_rot);
		auto it = g_rope_unit.find(key);
		if (it == g_rope_unit.end())
		{
			std::vector<float> h;
			rope_inv_table(freq_base, (int)n_rot, h);
			CU(cudaMalloc(&tab, h.size() * sizeof(float)), "rope table");
			CU(cudaMemcpy(tab, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice), "rope table upload");
			g_rope_unit[key] = tab;
		}
		else
			tab = it->second;
	}
	return launched(launch_rope(x, n_tok, n_heads, head_dim, n_rot, pos0, pos_scale, tab, mode, freq_factors, stream),
	                "rope");
}

extern "C" int nncu_softcap_dev(float* y, const float* x, size_t n, float cap, void* stream)
{
	if (!y || !x) return fail(NNCU_ERR_INVALID_ARGUMENT, "NULL pointer");
	if (!(cap > 0.0f)) return fail(NNCU_ERR_INVALID_ARGUMENT, "the cap must be positive");
	return launched(launch_softcap(y, x, n, cap, stream), "softcap");
}

// ---- profiling ---------------------------------------------------------------------------------

extern "C" void nncu_perf_enable(int enabled) { g_perf_on.store(enabled != 0); }

extern "C" void nncu_perf_reset(void)
{
	std::lock_guard<std::mutex> lk(g_perf_mu);
	for (auto& p : g_perf_pending)
	{
		cudaEventSynchronize(p.b);
		g_perf_free.push_back(p.a);
		g_perf_free.push_back(p.b);
	}
	g_perf_pending.clear();
	for (auto& ph : g_perf) ph = nncu_perf_phase{0.0, 0, 0};
}

extern "C" int nncu_perf_read(nncu_perf_phase* out)
{
	std::lock_guard<std::mutex> lk(g_perf_mu);
	for (auto& p : g_perf_pending)
	{
		float ms = 0.0f;
		cudaError_t e = cudaEventSynchronize(p.b);
		if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, p.a, p.b);
		if (e != cudaSuccess) return cuda_fail(e, "profiler events");
		g_perf[p.slot].ms += ms;
		g_perf[p.slot].calls += 1;
		g_perf[p.slot].bytes += p.bytes;
		g_perf_free.push_back(p.a);
		g_perf_free.push_back(p.b);
	}
	g_perf_pending.clear();
	if (out)
		for (int i = 0; i < NNCU_PERF_COUNT; ++i) out[i] = g_perf[i];
	return NNCU_OK;
}

extern "C" const char* nncu_perf_report(const char* title, int32_t n_tokens)
{
	nncu_perf_phase ph[NNCU_PERF_COUNT];
	if (nncu_perf_read(ph) != NNCU_OK) return "profiler unavailable";
	static const char* names[NNCU_PERF_COUNT] = {"attn_rope", "attn_core"};
	double total = 0.0;
	for (const auto& p : ph) total += p.ms;
	char line[256];
	std::lock_guard<std::mutex> lk(g_perf_mu);
	g_perf_text = std::string(title ? title : "nncu") + "\n";
	g_perf_text += "phase           ms       %     calls    us/call     GB/s\n";
	for (int i = 0; i < NNCU_PERF_COUNT; ++i)
	{
		const nncu_perf_phase& p = ph[i];
		const double us = p.calls ? 1000.0 * p.ms / (double)p.calls : 0.0;
		const double gbs = p.ms > 0.0 ? (double)p.bytes / (p.ms * 1e-3) / 1e9 : 0.0;
		std::snprintf(line, sizeof line, "%-10s %9.3f %7.1f %9lld %10.2f %8.1f\n", names[i], p.ms,
		              total > 0 ? 100.0 * p.ms / total : 0.0, (long long)p.calls, us, gbs);
		g_perf_text += line;
	}
	if (n_tokens > 0)
	{
		std::snprintf(line, sizeof line, "per token: %.3f ms\n", total / n_tokens);
		g_perf_text += line;
	}
	return g_perf_text.c_str();
}

extern "C" uint64_t nncu_launch_count(void) { return g_launches.load(); }
