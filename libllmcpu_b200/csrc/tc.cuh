// tc.cuh -- the 5th-generation tensor core (tcgen05) and tensor-map TMA
// primitives shared by the tensor-core kernels (prefill, 16-bit decode),
// written as inline PTX for sm_100a.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace nncu
{

// Instruction descriptor of tcgen05.mma kind::f16 with fp32 accumulation:
// A and B both bf16 (or both f16), M x N, each operand K-major or MN-major.
constexpr uint32_t tc_idesc(int M, int N, bool bf16, bool a_mn_major, bool b_mn_major)
{
	return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn_major ? 1u : 0u) << 15) |
	       ((b_mn_major ? 1u : 0u) << 16) | (((uint32_t)N >> 3) << 17) | (((uint32_t)M >> 4) << 24);
}

// Shared memory matrix descriptor, 128-byte swizzle (layout type 2),
// version 1: start address, leading and stride byte offsets (16-byte units).
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
	return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
	       ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t id, uint32_t acc)
{
	asm volatile(
		"{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
		"tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
		"l"(adesc), "l"(bdesc), "r"(id), "r"(acc)
		: "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar)
{
	asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
	             : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v)
{
	uint32_t r[32];
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
	             "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
	             "[%32];"
	             : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
	               "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
	               "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
	               "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
	               "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
	             : "r"(taddr)
	             : "memory");
#pragma unroll
	for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v)
{
	asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
	             "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, "
	             "%31, %32};" ::"r"(taddr),
	             "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
	             "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
	             "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
	             "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
	             "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
	             "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
	             "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
	             "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
	             "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
	             "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
	             "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
	             : "memory");
}

// 8, 16 or 32 consecutive fp32 columns into this thread's TMEM lane.
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const float* v)
{
	static_assert(N == 8 || N == 16 || N == 32, "8, 16 or 32 columns");
	if constexpr (N == 32)
		tmem_st32(taddr, v);
	else if constexpr (N == 8)
		asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
		             "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
		             "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
		             "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
		             : "memory");
	else
		asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
		             "%12, %13, %14, %15, %16};" ::"r"(taddr),
		             "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
		             "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
		             "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
		             "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
		             "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
		             "r"(__float_as_uint(v[15]))
		             : "memory");
}

// 8 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v)
{
	uint32_t r[8];
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
	             : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
	             : "r"(taddr)
	             : "memory");
#pragma unroll
	for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// One box of a 3-D tensor map (x along head_dim, y rows, z head) into shared
// memory, completing on `bar`. x is 0 or 64: 128-byte aligned.
__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar)
{
	asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
	             "%4}], [%5];" ::"r"(smem_u32(dst)),
	             "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
	             : "memory");
}


// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v)
{
	uint32_t r[16];
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, "
	             "%13, %14, %15}, [%16];"
	             : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
	               "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
	               "=r"(r[15])
	             : "r"(taddr)
	             : "memory");
#pragma unroll
	for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v);

// N (8, 16 or 32) consecutive fp32 columns of this thread's TMEM lane.
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float* v)
{
	static_assert(N == 8 || N == 16 || N == 32, "8, 16 or 32 columns");
	if constexpr (N == 8)
		tmem_ld8(taddr, v);
	else if constexpr (N == 16)
		tmem_ld16(taddr, v);
	else
		tmem_ld32(taddr, v);
}

// A 3-D tensor map (host side) over a head-major 16-bit array [planes][rows][D]
// with a box of 64 elements x box_rows rows x 1 plane, 128-byte swizzled:
// the operand layout the tensor-core kernels describe with sdesc. Returns a
// cudaError_t value.
int make_tensor_map(CUtensorMap* map, const void* base, bool bf16, uint64_t D, uint64_t rows, uint64_t planes,
                    uint32_t box_rows);

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols)
{
	asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
	             : "memory");
	asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols)
{
	asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

} // namespace nncu
