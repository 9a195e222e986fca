// SPDX-License-Identifier: Apache-2.0
//
// prefill.cu - chunked prefill attention on sm_100a tensor cores (tcgen05).
//
// For every sequence, the queries of its current chunk attend causally to
// the sequence's cached context (read from the paged KV cache, MX-FP8 or
// BF16, through the block table) followed by the chunk's own keys (BF16,
// read directly). The reference has no prefill or masked attention; the
// semantics are those of its CPU attention (userspace/compute/ace_attention.c:
// 85-134) applied row by row with keys [0, position].
//
// One CTA (4 warps) per (sequence, kv head, block of 128/G chunk positions).
// Its 128 matrix rows are (query head of the group, position): row r = h *
// (128/G) + p, so the K/V tiles are shared by the G heads of the group.
// Per 128-key block:
//   S[128 x 128] = Q . K^T          tcgen05.mma kind::f16, D in TMEM
//   P = exp2(S*scale - m)           each thread owns one row (TMEM lane)
//   O[128 x 128] += P . V           tcgen05.mma, A = P (smem), B = V (MN-major)
// P enters the product as two bf16 terms (P_hi + P_lo, residual ~2^-17 |P|),
// issued as one K = 256 accumulation over the same V tile.
// Q, K, V and P live in shared memory in the 128-byte-swizzled K-major
// (V: MN-major) canonical layouts. Chunk K/V tiles arrive by TMA tensor
// copies; cached-context tiles are dequantised into the same layout by the
// threads (MX: exact bf16 values, see kllm_device.cuh).

#include "kllm_device.cuh"
#include "kllm_internal.h"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <math_constants.h>

namespace kllm {
namespace {

constexpr int kRows = 128;          // MMA M: TMEM lanes, one thread each
constexpr int kKeys = 128;          // keys per block (MMA N of S, K of PV)
constexpr int kD = 128;             // head_dim
constexpr int kHalf = 64;           // bf16 elements per 128-byte swizzle row
constexpr int kTileBytes = kRows * kD * 2;    // 32 KB: one [128 x 128] bf16 tile
constexpr int kHalfBytes = kTileBytes / 2;    // 16 KB: one 64-column half
constexpr float kLazyLog2 = 8.f;
constexpr uint64_t kWaitNs = 200000000ull;  // 200 ms: a healthy wait takes microseconds

struct PrefillSmem {
	// each tile: two 64-column halves of 128 rows x 128 B, SW128
	uint8_t q[kTileBytes];
	uint8_t k[kTileBytes];
	uint8_t v[kTileBytes];
	uint8_t p[kTileBytes];    // P rounded to bf16
	uint8_t pl[kTileBytes];   // P - bf16(P), rounded to bf16
	uint64_t tma_bar, s_bar, pv_bar;
	uint32_t tmem_base;
	int wait_ok;
	uint32_t key_ok[kKeys / 32];
	uint32_t lut[260];   // 256 scale entries + dequant multiplier constants
};

__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk16)
{
	// byte offset of 16-byte chunk `chunk16` (0..7) of row `row` inside one
	// 64-column half: rows of 128 B, chunk index XOR-ed with row % 8
	return (uint32_t)row * 128u + (uint32_t)((chunk16 ^ (row & 7)) << 4);
}

// UMMA shared-memory descriptor, SWIZZLE_128B, sm_100 format
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
	return (uint64_t)((saddr >> 4) & 0x3FFFu) |
	       ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
	       ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) |
	       (1ull << 46) |   // descriptor version for sm_100
	       (2ull << 61);    // SWIZZLE_128B
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, M = 128, N = 128
__device__ __forceinline__ uint32_t umma_idesc(bool b_mn_major)
{
	return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
	       ((uint32_t)(kKeys >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b,
					 uint32_t idesc, uint32_t accumulate)
{
	asm volatile("{\n\t.reg .pred p;\n\t"
		     "setp.ne.b32 p, %4, 0;\n\t"
		     "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
		     :: "r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
	asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
		     :: "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
	uint32_t r[32];
	asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
		     "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
		     "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
		     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
		       "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
		       "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
		       "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
		       "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
		       "=r"(r[30]), "=r"(r[31])
		     : "r"(taddr));
	asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
	for (int i = 0; i < 32; ++i)
		v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32])
{
	asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
		     "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
		     "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
		     :: "r"(taddr), "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]),
		        "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]),
		        "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
		        "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]),
		        "f"(v[25]), "f"(v[26]), "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]),
		        "f"(v[31])
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

struct DevEntry {
	unsigned long long k, v;
	int valid;
	int pad;
};

// Writes one 128-element bf16 row (given as 64 packed words) into a tile.
__device__ __forceinline__ void store_row(uint8_t *tile, int row, const uint32_t (&w)[64])
{
#pragma unroll
	for (int half = 0; half < 2; ++half)
#pragma unroll
		for (int c = 0; c < 8; ++c)
			*reinterpret_cast<uint4 *>(tile + half * kHalfBytes + sw128_offset(row, c)) =
			    make_uint4(w[half * 32 + c * 4], w[half * 32 + c * 4 + 1],
				       w[half * 32 + c * 4 + 2], w[half * 32 + c * 4 + 3]);
}

// One key row of the cached context (kv head kvh), as 128 exact bf16
// values; zeros when the token has no valid page.
__device__ __forceinline__ bool load_cached_row(const kllm_prefill_args &a, const uint32_t *lut,
						int seq, int kvh, int kpos, int which,
						uint32_t (&w)[64])
{
	const int bs = a.block_size;
	const int page = kpos / bs, slot = kpos - page * bs;
	const DevEntry *e = reinterpret_cast<const DevEntry *>(a.table) +
			    (size_t)seq * a.max_blocks + (page < a.max_blocks ? page : 0);
	const unsigned long long kp = e->k, vp = e->v;
	if (page >= a.max_blocks || !e->valid || !kp) {
#pragma unroll
		for (int i = 0; i < 64; ++i)
			w[i] = 0u;
		return false;
	}
	const uint8_t *base = reinterpret_cast<const uint8_t *>(which ? vp : kp) + a.layer_off;
	if (a.kv_dtype == 1) {
		const size_t sec = (size_t)bs * kD * 9 / 8;
		const uint8_t *pay = base + (size_t)kvh * sec + (size_t)slot * kD;
		const uint8_t *scl = base + (size_t)kvh * sec + (size_t)bs * kD + (size_t)slot * (kD / 8);
		const uint4 sc = *reinterpret_cast<const uint4 *>(scl);
		const uint32_t scw[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
		for (int i = 0; i < 8; ++i) {  // 16 payload bytes = 2 scale blocks
			const uint4 pv = *reinterpret_cast<const uint4 *>(pay + 16 * i);
			const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
			for (int j = 0; j < 4; ++j) {
				const int blk = 2 * i + (j >> 1);
				const uint32_t s = lut[__byte_perm(scw[blk >> 2], 0u, 0x4440u | (blk & 3))];
				uint32_t lo, hi;
				e4m3x4_to_bf16x2_raw(pw[j], lut[256], lut[257], lo, hi);
				// value * 2^-8 in bf16; exact, undone by scaling P by 2^8
				w[8 * i + 2 * j] = bf16x2_mul(lo, s);
				w[8 * i + 2 * j + 1] = bf16x2_mul(hi, s);
			}
		}
	} else {
		const size_t sec = (size_t)bs * kD * 2;
		const uint4 *src = reinterpret_cast<const uint4 *>(base + (size_t)kvh * sec +
								  (size_t)slot * kD * 2);
#pragma unroll
		for (int i = 0; i < 16; ++i) {
			const uint4 v = src[i];
			w[4 * i] = v.x;
			w[4 * i + 1] = v.y;
			w[4 * i + 2] = v.z;
			w[4 * i + 3] = v.w;
		}
	}
	return true;
}

template <int G>
__global__ void __launch_bounds__(128, 1)
prefill_kernel(const kllm_prefill_args a, const __grid_constant__ CUtensorMap tm_k,
	       const __grid_constant__ CUtensorMap tm_v)
{
	constexpr int BQ = kRows / G;  // chunk positions per CTA
	extern __shared__ __align__(1024) uint8_t smem_raw[];
	PrefillSmem &sm = *reinterpret_cast<PrefillSmem *>(
	    (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);

	const int tid = threadIdx.x, warp = tid >> 5;
	const int qb = blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
	const int t0 = a.cu_seqlens[seq];
	const int clen = a.cu_seqlens[seq + 1] - t0;        // chunk length
	const int ctx = max(a.ctx_lens[seq], 0);             // cached tokens before it
	if (qb * BQ >= clen)
		return;
	const int ctx_cap = min(ctx, a.max_blocks * a.block_size);

	// ---- setup: barriers, LUT, TMEM ----------------------------------------
	if (tid == 0) {
		mbar_init(&sm.tma_bar, 1);
		mbar_init(&sm.s_bar, 1);
		mbar_init(&sm.pv_bar, 1);
		fence_mbar_init();
	}
	for (int i = tid; i < 256; i += 128)
		sm.lut[i] = mx_scale_lut_entry((uint32_t)i);
	if (tid == 0) {
		sm.lut[256] = 16u;
		sm.lut[257] = 1u << 28;
	}
	if (warp == 0) {
		asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
			     :: "r"(smem_u32(&sm.tmem_base)), "r"(256u));
		asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
	}

	// ---- Q tile: row r = head h of the group, position p ------------------
	const int h = tid / BQ, p = tid % BQ;          // this thread's row = tid
	const int qpos = qb * BQ + p;                  // position inside the chunk
	const bool row_live = qpos < clen;
	{
		uint32_t w[64];
		if (row_live) {
			const uint4 *src = reinterpret_cast<const uint4 *>(
			    reinterpret_cast<const uint8_t *>(a.q) +
			    (((size_t)(t0 + qpos) * a.num_heads + (size_t)kvh * G + h) * kD) * 2);
#pragma unroll
			for (int i = 0; i < 16; ++i) {
				const uint4 v = src[i];
				w[4 * i] = v.x;
				w[4 * i + 1] = v.y;
				w[4 * i + 2] = v.z;
				w[4 * i + 3] = v.w;
			}
		} else {
#pragma unroll
			for (int i = 0; i < 64; ++i)
				w[i] = 0u;
		}
		store_row(sm.q, tid, w);
	}
	fence_async_smem();
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = sm.tmem_base;
	const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
	const uint32_t tS = t_lane, tO = t_lane + 128;

	// zero O in TMEM
	{
		float z[32];
#pragma unroll
		for (int i = 0; i < 32; ++i)
			z[i] = 0.f;
#pragma unroll
		for (int c = 0; c < 4; ++c)
			tmem_st32(tO + 32 * c, z);
	}

	const uint32_t sq = smem_u32(sm.q), sk = smem_u32(sm.k), sv = smem_u32(sm.v),
		       sp = smem_u32(sm.p), spl = smem_u32(sm.pl);
	const uint32_t id_s = umma_idesc(false), id_pv = umma_idesc(true);
	float m_ref = -CUDART_INF_F, l_sum = 0.f;
	bool ok = true;
	uint32_t phase_s = 0, phase_pv = 0, phase_tma = 0;

	const int n_prior = (ctx_cap + kKeys - 1) / kKeys;
	const int last_q = min(qb * BQ + BQ, clen) - 1;    // last chunk position here
	const int n_chunk = last_q / kKeys + 1;

	for (int blk = 0; blk < n_prior + n_chunk && ok; ++blk) {
		const bool prior = blk < n_prior;
		const int kbase = prior ? blk * kKeys : (blk - n_prior) * kKeys;  // key offset
		// ---- stage K and V -----------------------------------------------------
		if (prior) {
			uint32_t w[64];
			const int kpos = kbase + tid;
			bool live = kpos < ctx_cap;
			bool okk = live && load_cached_row(a, sm.lut, seq, kvh, kpos, 0, w);
			if (!okk) {
#pragma unroll
				for (int i = 0; i < 64; ++i)
					w[i] = 0u;
			}
			store_row(sm.k, tid, w);
			if (okk)
				load_cached_row(a, sm.lut, seq, kvh, kpos, 1, w);
			store_row(sm.v, tid, w);
			const uint32_t ball = __ballot_sync(0xffffffffu, okk);
			if ((tid & 31) == 0)
				sm.key_ok[warp] = ball;
			fence_async_smem();
		} else if (tid == 0) {
			mbar_arrive_expect_tx(&sm.tma_bar, 4 * kHalfBytes);
			const int y = t0 + kbase;
			for (int half = 0; half < 2; ++half) {
				tma_load_2d(sm.k + half * kHalfBytes, &tm_k, kvh * kD + half * kHalf, y, &sm.tma_bar);
				tma_load_2d(sm.v + half * kHalfBytes, &tm_v, kvh * kD + half * kHalf, y, &sm.tma_bar);
			}
		}
		if (!prior) {
			if (tid == 0)
				sm.wait_ok = mbar_wait_ns(&sm.tma_bar, phase_tma, kWaitNs);
			phase_tma ^= 1u;
		}
		tc_fence_before();
		__syncthreads();
		if (!prior && !sm.wait_ok) {
			ok = false;
			break;
		}
		tc_fence_after();

		// ---- S = Q K^T ---------------------------------------------------------
		if (tid == 0) {
#pragma unroll
			for (int kk = 0; kk < kD / 16; ++kk) {
				const uint32_t off = (uint32_t)(kk >> 2) * kHalfBytes + (uint32_t)(kk & 3) * 32u;
				umma_f16(tS, umma_desc(sq + off, 16u, 1024u), umma_desc(sk + off, 16u, 1024u),
					 id_s, kk > 0);
			}
			umma_commit(&sm.s_bar);
		}
		if (tid == 0)
			sm.wait_ok = mbar_wait_ns(&sm.s_bar, phase_s, kWaitNs);
		phase_s ^= 1u;
		__syncthreads();
		if (!sm.wait_ok) {
			ok = false;
			break;
		}
		tc_fence_after();

		// ---- softmax on this row ---------------------------------------------
		// key j of the block is valid for this row when it exists and, for chunk
		// keys, lies at or before the row's position (causal)
		const float sl2 = a.scale_log2 * (prior && a.kv_dtype == 1 ? 256.f : 1.f);
		auto key_valid = [&](int j) -> bool {
			if (!row_live)
				return false;
			if (prior)
				return (sm.key_ok[j >> 5] >> (j & 31)) & 1u;
			const int kp = kbase + j;
			return kp < clen && kp <= qpos;
		};
		float mx = -CUDART_INF_F;
#pragma unroll
		for (int c = 0; c < 4; ++c) {
			float v[32];
			tmem_ld32(tS + 32 * c, v);
#pragma unroll
			for (int i = 0; i < 32; ++i)
				if (key_valid(32 * c + i))
					mx = fmaxf(mx, v[i] * sl2);
		}
		// Raise the reference max where a row exceeds it by more than the
		// slack. tcgen05.ld/st are warp-collective, so the O rescale runs for
		// the whole warp when any of its rows needs it (factor 1 elsewhere).
		const bool raise = mx > m_ref + kLazyLog2;
		if (__any_sync(0xffffffffu, raise)) {
			const float f = raise ? exp2f(m_ref - mx) : 1.f;
#pragma unroll
			for (int c = 0; c < 4; ++c) {
				float v[32];
				tmem_ld32(tO + 32 * c, v);
#pragma unroll
				for (int i = 0; i < 32; ++i)
					v[i] *= f;
				tmem_st32(tO + 32 * c, v);
			}
			if (raise) {
				l_sum *= f;
				m_ref = mx;
			}
		}
		const float pscale = prior && a.kv_dtype == 1 ? 256.f : 1.f;  // undo the V bias
#pragma unroll
		for (int c = 0; c < 4; ++c) {
			float v[32];
			tmem_ld32(tS + 32 * c, v);
			uint32_t pk[16], pr[16];
#pragma unroll
			for (int i = 0; i < 16; ++i) {
				const int j0 = 32 * c + 2 * i;
				const float p0 = key_valid(j0) ? exp2f(v[2 * i] * sl2 - m_ref) : 0.f;
				const float p1 = key_valid(j0 + 1) ? exp2f(v[2 * i + 1] * sl2 - m_ref) : 0.f;
				l_sum += p0 + p1;
				const float q0 = p0 * pscale, q1 = p1 * pscale;
				pk[i] = pack_bf16x2(q0, q1);
				pr[i] = pack_bf16x2(q0 - __uint_as_float(pk[i] << 16),
						    q1 - __uint_as_float(pk[i] & 0xFFFF0000u));
			}
			// keys 32c..32c+31 = half c/2, 16-byte chunks 4*(c%2) .. +3
#pragma unroll
			for (int j = 0; j < 4; ++j) {
				const uint32_t off = (c >> 1) * kHalfBytes + sw128_offset(tid, 4 * (c & 1) + j);
				*reinterpret_cast<uint4 *>(sm.p + off) =
				    make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
				*reinterpret_cast<uint4 *>(sm.pl + off) =
				    make_uint4(pr[4 * j], pr[4 * j + 1], pr[4 * j + 2], pr[4 * j + 3]);
			}
		}
		fence_async_smem();
		tc_fence_before();
		__syncthreads();
		tc_fence_after();

		// ---- O += P V ------------------------------------------------------------
		if (tid == 0) {
#pragma unroll
			for (int kk = 0; kk < 2 * kKeys / 16; ++kk) {
				const int k8 = kk & 7;   // kk < 8: P_hi, else P_lo
				const uint32_t poff = (uint32_t)(k8 >> 2) * kHalfBytes + (uint32_t)(k8 & 3) * 32u;
				const uint32_t voff = (uint32_t)k8 * 2048u;
				umma_f16(tO, umma_desc((kk < 8 ? sp : spl) + poff, 16u, 1024u),
					 umma_desc(sv + voff, (uint32_t)kHalfBytes, 1024u), id_pv, 1u);
			}
			umma_commit(&sm.pv_bar);
		}
		if (tid == 0)
			sm.wait_ok = mbar_wait_ns(&sm.pv_bar, phase_pv, kWaitNs);
		phase_pv ^= 1u;
		__syncthreads();
		if (!sm.wait_ok) {
			ok = false;
			break;
		}
		tc_fence_after();
	}

	// ---- epilogue: O / l -> bf16 ----------------------------------------------
	// (every lane loads: tcgen05.ld is warp-collective; live rows store)
	if (ok) {
		const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
		uint4 *dst = reinterpret_cast<uint4 *>(
		    reinterpret_cast<uint8_t *>(a.out) +
		    (((size_t)(t0 + (row_live ? qpos : 0)) * a.num_heads + (size_t)kvh * G + h) *
		     kD) * 2);
#pragma unroll
		for (int c = 0; c < 4; ++c) {
			float v[32];
			tmem_ld32(tO + 32 * c, v);
			if (!row_live)
				continue;
#pragma unroll
			for (int i = 0; i < 4; ++i)
				dst[4 * c + i] = make_uint4(
				    pack_bf16x2(v[8 * i] * inv, v[8 * i + 1] * inv),
				    pack_bf16x2(v[8 * i + 2] * inv, v[8 * i + 3] * inv),
				    pack_bf16x2(v[8 * i + 4] * inv, v[8 * i + 5] * inv),
				    pack_bf16x2(v[8 * i + 6] * inv, v[8 * i + 7] * inv));
		}
	} else if (tid == 0 && a.err) {
		atomicOr(a.err, KLLM_ERR_TIMEOUT_BIT);
	}
	tc_fence_before();
	__syncthreads();
	if (warp == 0)
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
			     :: "r"(tmem), "r"(256u));
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

// [num_tokens][num_kv_heads * 128] bf16, box 64 x 128 rows, 128-byte swizzle
bool make_map(CUtensorMap *m, const void *base, int num_tokens, int hkv)
{
	auto enc = get_encode();
	if (!enc)
		return false;
	cuuint64_t dims[2] = {(cuuint64_t)hkv * kD, (cuuint64_t)num_tokens};
	cuuint64_t strides[1] = {(cuuint64_t)hkv * kD * 2};
	cuuint32_t box[2] = {(cuuint32_t)kHalf, (cuuint32_t)kKeys};
	cuuint32_t estr[2] = {1, 1};
	return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
		   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
		   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
		   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int G>
int launch_g(const kllm_prefill_args &a, const CUtensorMap &mk, const CUtensorMap &mv,
	     cudaStream_t st)
{
	const size_t smem = sizeof(PrefillSmem) + 1024;
	cudaError_t e = cudaFuncSetAttribute(prefill_kernel<G>,
					     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
	if (e != cudaSuccess)
		return (int)e;
	constexpr int BQ = kRows / G;
	dim3 grid((a.max_chunk + BQ - 1) / BQ, a.num_kv_heads, a.num_seqs);
	prefill_kernel<G><<<grid, 128, smem, st>>>(a, mk, mv);
	return (int)cudaGetLastError();
}

}  // namespace
}  // namespace kllm

using namespace kllm;

extern "C" int kllm_prefill_launch(const struct kllm_prefill_args *a, void *stream)
{
	if (a->head_dim != kD)
		return (int)cudaErrorInvalidValue;
	CUtensorMap mk, mv;
	if (!make_map(&mk, a->k, a->num_tokens, a->num_kv_heads) ||
	    !make_map(&mv, a->v, a->num_tokens, a->num_kv_heads))
		return (int)cudaErrorInvalidValue;
	cudaStream_t st = static_cast<cudaStream_t>(stream);
	switch (a->num_heads / a->num_kv_heads) {
	case 1: return launch_g<1>(*a, mk, mv, st);
	case 2: return launch_g<2>(*a, mk, mv, st);
	case 4: return launch_g<4>(*a, mk, mv, st);
	case 8: return launch_g<8>(*a, mk, mv, st);
	default: return (int)cudaErrorInvalidValue;
	}
}
