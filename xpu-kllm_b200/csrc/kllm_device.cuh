// SPDX-License-Identifier: Apache-2.0
// kllm_device.cuh - sm_100a device primitives shared by the kernels:
// mbarrier + bulk-copy (TMA engine) staging, warp MMA fragments, and the
// in-register MX-FP8 (E4M3 payload x E4M3 scale per 8 elements) dequant.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "kllm_internal.h"

namespace kllm {

// ---------------------------------------------------------------------------
// mbarrier + cp.async.bulk (global -> shared through the TMA engine)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
	return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
	asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;"
		     :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
	asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
	asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
		     :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
	asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
		     :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity)
{
	uint32_t ok;
	asm volatile("{\n\t.reg .pred p;\n\t"
		     "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
		     "selp.u32 %0, 1, 0, p;\n\t}"
		     : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
	return ok != 0;
}

// try_wait that may suspend the thread for up to hint_ns nanoseconds (it
// resumes as soon as the phase completes), so a waiting warp costs almost no
// issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity,
						    uint32_t hint_ns)
{
	uint32_t ok;
	asm volatile("{\n\t.reg .pred p;\n\t"
		     "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
		     "selp.u32 %0, 1, 0, p;\n\t}"
		     : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns) : "memory");
	return ok != 0;
}

// 2^x by the hardware approximation (relative error about 2^-22; results
// below 2^-126 flush to zero).
__device__ __forceinline__ float ex2_approx(float x)
{
	float y;
	asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
	return y;
}

// Bounded wait: each try_wait suspends for a hardware-bounded interval, so
// kMaxTries bounds the wait to well under a minute. Returns false on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity)
{
	constexpr uint32_t kMaxTries = 1u << 24;
	for (uint32_t i = 0; i < kMaxTries; ++i)
		if (mbar_try_wait(bar, parity))
			return true;
	return false;
}

// True when [p, p + bytes) lies inside one registered arena, or when no
// arena is registered (the check is off).
__device__ __forceinline__ bool in_arenas(const kllm_arenas &ar, unsigned long long p,
					  unsigned long long bytes)
{
	if (ar.count <= 0)
		return true;
	bool ok = false;
	for (int r = 0; r < ar.count && r < KLLM_MAX_ARENAS; ++r)
		ok |= p >= ar.lo[r] && p + bytes <= ar.hi[r] && p + bytes >= p;
	return ok;
}

// Programmatic dependent launch. In a kernel launched with programmatic
// stream serialization, grid_dependency_wait() returns once the previous
// kernel on the stream has completed and its writes are visible;
// grid_launch_dependents() lets the next such kernel start launching. Both
// are no-ops in a kernel launched normally.
__device__ __forceinline__ void grid_dependency_wait()
{
	asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void grid_launch_dependents()
{
	asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_ns()
{
	uint64_t t;
	asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
	return t;
}

// Wait bounded by wall time (nanoseconds of the global timer) rather than
// by a try count, for waits that complete in microseconds when healthy.
__device__ __forceinline__ bool mbar_wait_ns(uint64_t *bar, uint32_t parity, uint64_t limit_ns)
{
	if (mbar_try_wait(bar, parity))
		return true;
	const uint64_t t0 = global_ns();
	while (!mbar_try_wait(bar, parity))
		if (global_ns() - t0 > limit_ns)
			return false;
	return true;
}

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src,
					 uint32_t bytes, uint64_t *bar)
{
	asm volatile(
	    "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes"
	    " [%0], [%1], %2, [%3];"
	    :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
	    : "memory");
}

// Same, with an L2 evict-first policy: KV pages are streamed exactly once.
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src,
						uint32_t bytes, uint64_t *bar,
						uint64_t policy)
{
	asm volatile(
	    "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
	    " [%0], [%1], %2, [%3], %4;"
	    :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)),
	       "l"(policy)
	    : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy()
{
	uint64_t pol;
	asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;"
		     : "=l"(pol));
	return pol;
}

// ---------------------------------------------------------------------------
// warp MMA (m16n8k16, bf16 in, fp32 accumulate) and fragment transpose
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0,
					 uint32_t a1, uint32_t a2, uint32_t a3,
					 uint32_t b0, uint32_t b1)
{
	asm volatile(
	    "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
	    "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
	    : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
	    : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 8x8 b16 matrix held one row-pair per lane (row lane/4, cols 2*(lane%4)+{0,1})
// -> its transpose in the same layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x)
{
	uint32_t y;
	asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;"
		     : "=r"(y) : "r"(x));
	return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
	__nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
	return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0,
					uint32_t a1, uint32_t a2, uint32_t a3,
					uint32_t b0, uint32_t b1)
{
	asm volatile(
	    "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
	    "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
	    : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
	    : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi)
{
	__half2 v = __floats2half2_rn(lo, hi);
	return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ uint32_t f16x2_mul(uint32_t a, uint32_t b)
{
	uint32_t d;
	asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
	return d;
}

// Two E4M3 codes (bytes 0, 1 of the low or high half of w) -> f16x2, exact
// (every E4M3 value is an f16 value); byte 0 lands in the low half.
__device__ __forceinline__ uint32_t e4m3x2_lo_to_f16x2(uint32_t w)
{
	uint32_t d;
	asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\t"
	    "cvt.rn.f16x2.e4m3x2 %0, l;\n\t}" : "=r"(d) : "r"(w));
	return d;
}

__device__ __forceinline__ uint32_t e4m3x2_hi_to_f16x2(uint32_t w)
{
	uint32_t d;
	asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %1;\n\t"
	    "cvt.rn.f16x2.e4m3x2 %0, h;\n\t}" : "=r"(d) : "r"(w));
	return d;
}

// f16x2 (both halves) of e4m3(code) / 4: the MX-FP8 decode scale. With the
// 2^-2 factor, payload x scale <= 448 * 448 / 4 = 50176 stays an f16 value;
// products of at least 2^-14 are exact, smaller ones are rounded to the f16
// subnormal step 2^-24 (2^-22 after the factor is undone).
__device__ __forceinline__ uint32_t mx_scale_lut_entry_f16(uint32_t code)
{
	const uint32_t e = (code >> 3) & 0xFu, m = code & 0x7u;
	// (8 + m) * 2^(e - 10) for e > 0, m * 2^-9 for e == 0; then / 4
	const float v = e ? (float)(8u + m) * __uint_as_float((e + 115u) << 23)
			  : (float)m * __uint_as_float(116u << 23);
	const uint32_t h = pack_f16x2(v, v);
	return (code & 0x80u) ? (h | 0x80008000u) : h;
}

// One E4M3 code as the reference decodes it (userspace/compute/mx_dequant.h:
// 30-55): bias 7, subnormals m/8 * 2^-6, and exponent 15 with mantissa 7
// (0x7F / 0xFF) as +-480 rather than NaN. Exact in fp32.
__device__ __forceinline__ float e4m3_ref_to_f32(uint32_t code)
{
	const uint32_t e = (code >> 3) & 0xFu, m = code & 0x7u;
	const float v = e ? __uint_as_float(((e + 120u) << 23) | (m << 20))
			  : (float)m * __uint_as_float(118u << 23);
	return (code & 0x80u) ? -v : v;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b)
{
	uint32_t d;
	asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
	return d;
}

// ---------------------------------------------------------------------------
// MX-FP8 dequant
//
// An E4M3 code s.eeee.mmm placed into a bf16 as s.0000eeee.mmm0000 reads as
// value * 2^-120 exactly (exponent field e with bias 127 instead of 7; e = 0
// lands on the bf16 subnormals, matching E4M3 subnormals, and 0x7F gives
// 480 * 2^-120 as the reference decoder does, userspace/compute/mx_dequant.h:
// 30-55). Multiplying by the scale pre-biased by 2^112 then yields
// payload * scale * 2^-8: both factors carry at most 4 significant bits, so
// the product (<= 8 bits, 2^-26 .. 2^9.8 after the bias) is exact in bf16.
// The 2^-8 is folded into the softmax scale (QK) and the final
// normalisation (PV).
// ---------------------------------------------------------------------------

constexpr float kMxUnbias = 256.0f;  // undoes the 2^-8 above

// bytes (0,1) [hi = false] or (2,3) [hi = true] of w -> bf16x2 of e4m3*2^-120
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2_raw(uint32_t w, bool hi)
{
	uint32_t x = __byte_perm(w, 0u, hi ? 0x3424u : 0x1404u);  // [0,b0,0,b1]
	return ((x & 0x7F007F00u) >> 4) | (x & 0x80008000u);
}

// Four E4M3 bytes of w (b0..b3, low to high) -> two bf16x2 words of
// e4m3 * 2^-120: lo = (b0, b1), hi = (b2, b3). Per byte the bf16 low byte is
// (b & 0x0F) << 4 and the high byte is (b & 0x80) | (b >> 4 & 0x07); both are
// built for all four bytes at once and interleaved with two byte permutes.
// k16 = 16 and k2p28 = 2^28 are passed as runtime values so the shifts are
// issued as integer multiplies (FMA pipe), keeping the ALU pipe free.
__device__ __forceinline__ void e4m3x4_to_bf16x2_raw(uint32_t w, uint32_t k16,
						     uint32_t k2p28, uint32_t &lo,
						     uint32_t &hi)
{
	const uint32_t l = (w & 0x0F0F0F0Fu) * k16;
	const uint32_t h = __umulhi(w & 0x70707070u, k2p28) | (w & 0x80808080u);
	lo = __byte_perm(l, h, 0x5140u);
	hi = __byte_perm(l, h, 0x7362u);
}

// bf16 bits of e4m3(code) * 2^112 (the pre-biased scale), duplicated into
// both halves of a word.
__device__ __forceinline__ uint32_t mx_scale_lut_entry(uint32_t code)
{
	uint32_t sign = (code & 0x80u) << 24;
	uint32_t e = (code >> 3) & 0xFu, m = code & 0x7u;
	uint32_t fbits;
	if (e != 0) {
		// 2^(e-7) * (1 + m/8) * 2^112 -> exponent field e - 7 + 112 + 127
		fbits = ((e + 232u) << 23) | (m << 20);
	} else if (m != 0) {
		// m * 2^-9 * 2^112 = m * 2^103
		fbits = __float_as_uint((float)m) + (103u << 23);
	} else {
		fbits = 0u;
	}
	uint32_t b = (fbits | sign) >> 16;  // exact: <= 4 significant bits
	return b | (b << 16);
}

}  // namespace kllm
