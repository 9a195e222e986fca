// SPDX-License-Identifier: Apache-2.0
//
// kllm_umma.cuh - sm_100a tensor-core plumbing shared by the tcgen05 kernels:
// UMMA shared-memory descriptors (128-byte swizzle), tcgen05.mma issue from
// shared memory or TMEM, commit to an mbarrier, TMEM loads and stores, 2D/3D
// TMA tensor loads (no multicast), and the driver's tensor-map encoder.
#pragma once

#include "kllm_device.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace kllm {
namespace {

// UMMA shared-memory descriptor, SWIZZLE_128B, sm_100 format
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
	return (uint64_t)((saddr >> 4) & 0x3FFFu) |
	       ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
	       ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) |
	       (1ull << 46) |   // descriptor version for sm_100
	       (2ull << 61);    // SWIZZLE_128B
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, shape M x N, A
// K-major, B K-major or MN-major
__device__ __forceinline__ uint32_t umma_idesc_bf16(int m, int n, bool b_mn_major)
{
	return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
	       ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b,
					 uint32_t idesc, uint32_t accumulate)
{
	asm volatile("{\n\t.reg .pred p;\n\t"
		     "setp.ne.b32 p, %4, 0;\n\t"
		     "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
		     :: "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// Same, with A read from tensor memory (M = 128 rows in lanes 0..127, K
// packed two bf16 per 32-bit column, the lower half first).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
					    uint32_t idesc, uint32_t accumulate)
{
	asm volatile("{\n\t.reg .pred p;\n\t"
		     "setp.ne.b32 p, %4, 0;\n\t"
		     "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
		     :: "r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
	asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
		     :: "r"(smem_u32(bar)) : "memory");
}

// true in exactly one lane of the (fully active) warp
__device__ __forceinline__ bool elect_one()
{
	uint32_t is;
	asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
		     : "=r"(is));
	return is != 0;
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Issue-only forms: the caller waits (tcgen05.wait::ld / ::st) before using
// the loaded registers / before signalling that the stores are visible.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16])
{
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
		     "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
		     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
		       "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
		       "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
		     : "r"(taddr) : "memory");
}

__device__ __forceinline__ void tmem_st16_nowait(uint32_t taddr, const float (&v)[16])
{
	asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
		     "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
		     :: "r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]),
		        "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]),
		        "f"(v[13]), "f"(v[14]), "f"(v[15])
		     : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane. Load and wait are
// one asm statement, so no use of the registers can be scheduled before the
// wait.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16])
{
	uint32_t r[16];
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
		     "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
		     "tcgen05.wait::ld.sync.aligned;"
		     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
		       "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
		       "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
		     : "r"(taddr) : "memory");
#pragma unroll
	for (int i = 0; i < 16; ++i)
		v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16])
{
	asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
		     "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
		     :: "r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]),
		        "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]),
		        "f"(v[13]), "f"(v[14]), "f"(v[15])
		     : "memory");
	asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
					    uint64_t *bar)
{
	asm volatile(
	    "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
	    " [%0], [%1, {%2, %3}], [%4];"
	    :: "r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
	    : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y,
					    int z, uint64_t *bar)
{
	asm volatile(
	    "cp.async.bulk.tensor.3d.shared::cta.global.mbarrier::complete_tx::bytes"
	    " [%0], [%1, {%2, %3, %4}], [%5];"
	    :: "r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
	    : "memory");
}

// x32 form: 32 consecutive fp32 columns of this thread's TMEM lane, load
// and wait in one asm statement.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
	uint32_t r[32];
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
		     "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
		     "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
		     "tcgen05.wait::ld.sync.aligned;"
		     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
		       "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
		       "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
		       "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
		       "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
		       "=r"(r[30]), "=r"(r[31])
		     : "r"(taddr) : "memory");
#pragma unroll
	for (int i = 0; i < 32; ++i)
		v[i] = __uint_as_float(r[i]);
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode()
{
	static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
	if (!fn) {
		cudaDriverEntryPointQueryResult q;
		void *p = nullptr;
		if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
			    cudaSuccess &&
		    q == cudaDriverEntryPointSuccess)
			fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
	}
	return fn;
}

}  // namespace
}  // namespace kllm
