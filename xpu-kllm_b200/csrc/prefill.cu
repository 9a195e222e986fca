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
// One CTA per (sequence, kv head, 2 x 128/G chunk positions) holds two query
// tiles A and B of 128 MMA rows each (row r = p * G + h: position p, head h
// of the group, as a TMA box {64 dims, G heads, 128/G tokens} lands them),
// which share every K/V block. Per 128-key block j:
//   S_t = Q_t . K_j^T        tcgen05.mma kind::f16, Q and K in shared memory
//   P_t = exp2(S_t*c - m)    one softmax thread per row (TMEM lane), written
//                            back over S_t as bf16 hi + lo
//   O_t += P_t . V_j         tcgen05.mma with A = P_t read from TMEM, in two
//                            halves: keys 0-63 start as soon as the softmax
//                            has written them, while it finishes 64-127
// Warp roles (13 warps):
//   0-3 / 4-7  softmax of tile A / B (warp w reads TMEM lanes 32 (w % 4) ..)
//   8-11       producer: Q tiles, then per block either TMA tensor copies of
//              the chunk's K/V or the exact dequant of cached pages
//   12         TMEM allocation and MMA issue (one lane)
// K/V blocks go through a 2-stage ring, so the tensor core runs one tile's
// PV and next S while the other tile's softmax runs. TMEM: S_A, S_B, O_A,
// O_B, 128 fp32 columns each. Every wait is bounded in wall time and can be
// aborted; a timeout sets KLLM_ERR_TIMEOUT, drains the CTA's own copies and
// MMAs, frees TMEM and leaves the CTA.

#include "kllm_device.cuh"
#include "kllm_internal.h"
#include "kllm_umma.cuh"

#include <cstdio>
#include <cstdlib>
#include <math_constants.h>

namespace kllm {
namespace {

constexpr int kRows = 128;          // MMA M: TMEM lanes, one thread each
constexpr int kKeys = 128;          // keys per block (MMA N of S, K of PV)
constexpr int kD = 128;             // head_dim
constexpr int kHalf = 64;           // bf16 elements per 128-byte swizzle row
constexpr int kTileBytes = kRows * kD * 2;    // 32 KB: one [128 x 128] bf16 tile
constexpr int kHalfBytes = kTileBytes / 2;    // 16 KB: one 64-column half
// With the row's block max known before P is written, the reference is
// raised whenever a block max exceeds it by 2^8 (P <= 256, x 2^8 on cached
// MX blocks); that costs one O rescale.
constexpr float kRaiseLog2 = 8.f;
#ifndef KLLM_PF_WAIT_HINT
#define KLLM_PF_WAIT_HINT 20000   // try_wait suspend hint, ns (0: plain try_wait)
#endif
constexpr uint64_t kWaitNs = 200000000ull;  // 200 ms: a healthy wait takes microseconds

constexpr int kStages = 2;
constexpr int kWarpsSoftmax = 8, kWarpMma = 8, kWarpProducer0 = 9;
constexpr int kProducerThreads = 96;
constexpr int kThreads = 12 * 32;

struct PrefillSmem {
	// tiles: two 64-column halves of 128 rows x 128 B, SW128
	uint8_t q[2][kTileBytes];
	uint8_t k[kStages][kTileBytes];
	uint8_t v[kStages][kTileBytes];
	uint64_t q_full;
	// K and V stages fill and drain separately: K(j) is free once both tiles'
	// S(j) are done, V(j) (and the key mask, read by the softmax of block j)
	// once both PV(j) are issued after the softmax
	uint64_t k_full[kStages], k_empty[kStages], v_full[kStages], v_empty[kStages];
	// p_half: P of keys 0-63 written (the PV of that half may start while
	// the softmax finishes keys 64-127); p_full: all of P written
	uint64_t s_full[2], p_half[2], p_full[2], o_full[2];
	uint64_t drain;
	uint32_t tmem_base;
	int abort;
	int prod_ok[2];      // producer go / stop, double-buffered by block parity
	uint32_t key_ok[kStages][kKeys / 32];
	uint32_t lut[260];   // 256 scale entries + dequant multiplier constants
};

__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk16)
{
	// byte offset of 16-byte chunk `chunk16` (0..7) of row `row` inside one
	// 64-column half: rows of 128 B, chunk index XOR-ed with row % 8
	return (uint32_t)row * 128u + (uint32_t)((chunk16 ^ (row & 7)) << 4);
}

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, M = 128, N = 128
__device__ __forceinline__ uint32_t umma_idesc(bool b_mn_major)
{
	return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
	       ((uint32_t)(kKeys >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
}

struct DevEntry {
	unsigned long long k, v;
	int valid;
	int pad;
};

// Writes half `half` (elements 64*half .. +63, as 32 packed words) of row
// `row` into a tile: that half's 128-byte swizzled row.
__device__ __forceinline__ void store_half_row(uint8_t *tile, int row, int half,
					       const uint32_t (&w)[32])
{
#pragma unroll
	for (int c = 0; c < 8; ++c)
		*reinterpret_cast<uint4 *>(tile + half * kHalfBytes + sw128_offset(row, c)) =
		    make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Page base (K if which == 0, else V) holding cached token kpos of the
// sequence's kv head section, or null when the token has no valid page.
__device__ __forceinline__ const uint8_t *cached_section(const kllm_prefill_args &a, int seq,
							 int kvh, int kpos, int which, int &slot)
{
	const int bs = a.block_size;
	const int page = kpos / bs;
	slot = kpos - page * bs;
	if (page >= a.max_blocks)
		return nullptr;
	const DevEntry *e = reinterpret_cast<const DevEntry *>(a.table) +
			    (size_t)seq * a.max_blocks + page;
	const unsigned long long kp = e->k, vp = e->v;
	if (!e->valid || !kp)
		return nullptr;
	const size_t sec = a.kv_dtype == 1 ? (size_t)bs * kD * 9 / 8 : (size_t)bs * kD * 2;
	const unsigned long long p = (which ? vp : kp) + a.layer_off + (size_t)kvh * sec;
	if (!in_arenas(a.arenas, p, sec)) {   // outside the registered arenas: skipped
		if (a.err)
			atomicOr(a.err, KLLM_ERR_PAGE_RANGE_BIT);
		return nullptr;
	}
	return reinterpret_cast<const uint8_t *>(p);
}

// 64 MX elements (4 x 16 payload bytes, 8 scale bytes) -> 64 exact bf16
// values x 2^-8, as 32 packed words.
__device__ __forceinline__ void mx_dequant_half(const uint32_t *lut, const uint4 *pay, uint2 sc,
						uint32_t (&w)[32])
{
	const uint32_t scw[2] = {sc.x, sc.y};
#pragma unroll
	for (int i = 0; i < 4; ++i) {  // 16 payload bytes = 2 scale blocks
		const uint32_t pw[4] = {pay[i].x, pay[i].y, pay[i].z, pay[i].w};
#pragma unroll
		for (int j = 0; j < 4; ++j) {
			const int blk = 2 * i + (j >> 1);
			const uint32_t s = lut[__byte_perm(scw[blk >> 2], 0u, 0x4440u | (blk & 3))];
			uint32_t lo, hi;
			e4m3x4_to_bf16x2_raw(pw[j], lut[256], lut[257], lo, hi);
			w[8 * i + 2 * j] = bf16x2_mul(lo, s);
			w[8 * i + 2 * j + 1] = bf16x2_mul(hi, s);
		}
	}
}

// Half `half` of one cached key/value row as 64 exact bf16 values (MX:
// value x 2^-8, undone by the caller's scaling).
__device__ __forceinline__ void load_cached_half(const kllm_prefill_args &a, const uint32_t *lut,
						 const uint8_t *sec, int slot, int half,
						 uint32_t (&w)[32])
{
	if (a.kv_dtype == 1) {
		const uint8_t *pay = sec + (size_t)slot * kD + 64 * half;
		const uint2 sc = *reinterpret_cast<const uint2 *>(
		    sec + (size_t)a.block_size * kD + (size_t)slot * (kD / 8) + 8 * half);
		const uint32_t scw[2] = {sc.x, sc.y};
#pragma unroll
		for (int i = 0; i < 4; ++i) {  // 16 payload bytes = 2 scale blocks
			const uint4 pv = *reinterpret_cast<const uint4 *>(pay + 16 * i);
			const uint32_t pw[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
			for (int j = 0; j < 4; ++j) {
				const int blk = 2 * i + (j >> 1);
				const uint32_t s = lut[__byte_perm(scw[blk >> 2], 0u, 0x4440u | (blk & 3))];
				uint32_t lo, hi;
				e4m3x4_to_bf16x2_raw(pw[j], lut[256], lut[257], lo, hi);
				w[8 * i + 2 * j] = bf16x2_mul(lo, s);
				w[8 * i + 2 * j + 1] = bf16x2_mul(hi, s);
			}
		}
	} else {
		const uint4 *src = reinterpret_cast<const uint4 *>(sec + (size_t)slot * kD * 2 +
								  128 * half);
#pragma unroll
		for (int i = 0; i < 8; ++i) {
			const uint4 v = src[i];
			w[4 * i] = v.x;
			w[4 * i + 1] = v.y;
			w[4 * i + 2] = v.z;
			w[4 * i + 3] = v.w;
		}
	}
}

// Bounded wait that gives up early once another role of the CTA aborted.
__device__ __forceinline__ bool wait_or_abort(PrefillSmem &sm, uint64_t *bar, uint32_t parity,
					      const kllm_prefill_args &a)
{
	if (mbar_try_wait(bar, parity))
		return true;
	const uint64_t t0 = global_ns();
	for (uint32_t n = 0;; ++n) {
#if KLLM_PF_WAIT_HINT > 0
		if (mbar_try_wait_sleep(bar, parity, KLLM_PF_WAIT_HINT))
			return true;
#else
		if (mbar_try_wait(bar, parity))
			return true;
		if (n & 31u)
			continue;   // the clock and the abort flag every 32 tries
#endif
		if (*reinterpret_cast<volatile int *>(&sm.abort))
			return false;
		if (global_ns() - t0 > kWaitNs) {
			*reinterpret_cast<volatile int *>(&sm.abort) = 1;
			if (a.err)
				atomicOr(a.err, KLLM_ERR_TIMEOUT_BIT);
			return false;
		}
	}
}

// Blocks of a tile whose last chunk position is `last` (-1: empty tile).
__device__ __forceinline__ int tile_blocks(int n_prior, int last)
{
	return last < 0 ? 0 : n_prior + last / kKeys + 1;
}

// p of one 16-key group -> bf16 hi/lo pairs: hi in w[0..7], lo in w[8..15]
__device__ __forceinline__ void pack_p_pair(float q0, float q1, float &whi, float &wlo)
{
	const uint32_t hi = pack_bf16x2(q0, q1);
	const uint32_t lo = pack_bf16x2(q0 - __uint_as_float(hi << 16),
					q1 - __uint_as_float(hi & 0xFFFF0000u));
	whi = __uint_as_float(hi);
	wlo = __uint_as_float(lo);
}

// One 128-key block of one row: S (TMEM columns of tS) -> P written back in
// place as 8 groups of (8 hi, 8 lo) bf16 pairs, p = 2^pexp x exp2(s x sl2 -
// m_ref); l_sum gains sum(p) / 2^pexp. FULL: every key of every row of the
// warp is valid (no mask). o_live: O already holds earlier blocks. Branches
// around TMEM accesses are warp-uniform.
// Multiplies this row's O (when o_live) and its first n_groups P groups of
// the current block by f (warp-collective: the whole warp calls it; rare).
__device__ __forceinline__ void rescale_row(uint32_t tS, uint32_t tO, float f, bool o_live,
					 int n_groups)
{
	tmem_wait_st();
	if (o_live) {
#pragma unroll 1
		for (int c = 0; c < 8; ++c) {
			float o[16];
			tmem_ld16(tO + 16 * c, o);
#pragma unroll
			for (int i = 0; i < 16; ++i)
				o[i] *= f;
			tmem_st16(tO + 16 * c, o);
		}
	}
#pragma unroll 1
	for (int gg = 0; gg < n_groups; ++gg) {
		float w[16];
		tmem_ld16(tS + 16 * gg, w);
#pragma unroll
		for (int i = 0; i < 8; ++i) {
			const uint32_t hi = __float_as_uint(w[i]), lo = __float_as_uint(w[8 + i]);
			const float q0 = (__uint_as_float(hi << 16) + __uint_as_float(lo << 16)) * f;
			const float q1 = (__uint_as_float(hi & 0xFFFF0000u) +
					  __uint_as_float(lo & 0xFFFF0000u)) * f;
			pack_p_pair(q0, q1, w[i], w[8 + i]);
		}
		tmem_st16(tS + 16 * gg, w);
	}
}

// Waits for this thread's outstanding TMEM loads; all 128 destination
// registers are in/out operands, so their uses follow the wait.
__device__ __forceinline__ void tmem_wait_ld_row(uint32_t (&r)[8][16])
{
#pragma unroll
	for (int q = 0; q < 4; ++q)
		asm volatile("tcgen05.wait::ld.sync.aligned;"
			     : "+r"(r[2 * q][0]), "+r"(r[2 * q][1]), "+r"(r[2 * q][2]), "+r"(r[2 * q][3]),
			       "+r"(r[2 * q][4]), "+r"(r[2 * q][5]), "+r"(r[2 * q][6]), "+r"(r[2 * q][7]),
			       "+r"(r[2 * q][8]), "+r"(r[2 * q][9]), "+r"(r[2 * q][10]), "+r"(r[2 * q][11]),
			       "+r"(r[2 * q][12]), "+r"(r[2 * q][13]), "+r"(r[2 * q][14]), "+r"(r[2 * q][15]),
			       "+r"(r[2 * q + 1][0]), "+r"(r[2 * q + 1][1]), "+r"(r[2 * q + 1][2]),
			       "+r"(r[2 * q + 1][3]), "+r"(r[2 * q + 1][4]), "+r"(r[2 * q + 1][5]),
			       "+r"(r[2 * q + 1][6]), "+r"(r[2 * q + 1][7]), "+r"(r[2 * q + 1][8]),
			       "+r"(r[2 * q + 1][9]), "+r"(r[2 * q + 1][10]), "+r"(r[2 * q + 1][11]),
			       "+r"(r[2 * q + 1][12]), "+r"(r[2 * q + 1][13]), "+r"(r[2 * q + 1][14]),
			       "+r"(r[2 * q + 1][15])
			     :: "memory");
}

// One 128-key block of one row, held in registers: S (TMEM columns of tS)
// -> P written back in place as 8 groups of (8 hi, 8 lo) bf16 pairs,
// p = 2^pexp x exp2(s x sl2 - m_ref); l_sum gains sum(p) / 2^pexp. Invalid
// keys are set to -inf first (p = 0). The row's block max is known before
// any P is written, so raising the reference max rescales only O and l.
// o_live: O already holds earlier blocks. Once keys 0-63 are written the
// thread arrives on p_half, so that half of the PV product can start.
// Branches around TMEM accesses are warp-uniform.
__device__ __forceinline__ void softmax_block(uint32_t tS, uint32_t tO, const uint32_t (&vmask)[4],
					      bool masked, float sl2, float pexp, bool o_live,
					      float &m_ref, float &l_sum, uint64_t *p_half)
{
	uint32_t r[8][16];
#pragma unroll
	for (int g = 0; g < 8; ++g)
		tmem_ld16_nowait(tS + 16 * g, r[g]);
	tmem_wait_ld_row(r);
	if (masked) {
#pragma unroll
		for (int k = 0; k < 128; ++k)
			if (!((vmask[k >> 5] >> (k & 31)) & 1u))
				r[k >> 4][k & 15] = 0xFF800000u;   // -inf
	}
	float mv[8];                           // 8 independent chains of 16, then a tree
#pragma unroll
	for (int i = 0; i < 8; ++i)
		mv[i] = __uint_as_float(r[0][i]);
#pragma unroll
	for (int k = 8; k < 128; ++k)
		mv[k & 7] = fmaxf(mv[k & 7], __uint_as_float(r[k >> 4][k & 15]));
#pragma unroll
	for (int w = 4; w >= 1; w >>= 1)      // tree max
#pragma unroll
		for (int i = 0; i < w; ++i)
			mv[i] = fmaxf(mv[i], mv[i + w]);
	const float gl = mv[0] * sl2;
	const bool raise = gl > m_ref + kRaiseLog2;
	if (__any_sync(0xffffffffu, raise)) {
		const float f = raise ? exp2f(m_ref - gl) : 1.f;
		if (o_live)
			rescale_row(tS, tO, f, true, 0);
		l_sum *= f;
		if (raise)
			m_ref = gl;
	}
	// no valid key yet (m_ref = -inf): every p is 0, not exp2(-inf + inf)
	const float moff = m_ref == -CUDART_INF_F ? -CUDART_INF_F : pexp - m_ref;
	float bsum = 0.f;
#pragma unroll
	for (int g = 0; g < 8; ++g) {
		float w[16];
#pragma unroll
		for (int i = 0; i < 8; ++i) {
			const float q0 = ex2_approx(fmaf(__uint_as_float(r[g][2 * i]), sl2, moff));
			const float q1 = ex2_approx(fmaf(__uint_as_float(r[g][2 * i + 1]), sl2, moff));
			bsum += q0 + q1;
			pack_p_pair(q0, q1, w[i], w[8 + i]);
		}
		tmem_st16_nowait(tS + 16 * g, w);
		if (g == 3) {
			tmem_wait_st();
			tc_fence_before();
			mbar_arrive(p_half);
		}
	}
	tmem_wait_st();
	l_sum += bsum * exp2f(-pexp);
}

template <int G>
__global__ void __maxnreg__(168)
prefill_kernel(const kllm_prefill_args a, const __grid_constant__ CUtensorMap tm_q,
	       const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v)
{
	constexpr int BQ = kRows / G;  // chunk positions per tile
	extern __shared__ __align__(1024) uint8_t smem_raw[];
	PrefillSmem &sm = *reinterpret_cast<PrefillSmem *>(
	    (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);

	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	// the CTAs with the most key blocks (latest positions) start first
	const int cb = gridDim.x - 1 - blockIdx.x, kvh = blockIdx.y, seq = blockIdx.z;
	const int t0 = a.cu_seqlens[seq];
	const int clen = a.cu_seqlens[seq + 1] - t0;        // chunk length
	const int ctx = max(a.ctx_lens[seq], 0);             // cached tokens before it
	const int pos0 = cb * 2 * BQ;                        // first position, tile A
	if (pos0 >= clen)
		return;
	if (a.err && (*reinterpret_cast<volatile uint32_t *>(a.err) & KLLM_ERR_TIMEOUT_BIT))
		return;  // an earlier CTA timed out: the launch is already failed
	const int ctx_cap = min(ctx, a.max_blocks * a.block_size);
	const int n_prior = (ctx_cap + kKeys - 1) / kKeys;
	const int nb_t[2] = {tile_blocks(n_prior, min(pos0 + BQ, clen) - 1),
			     tile_blocks(n_prior, pos0 + BQ < clen ? min(pos0 + 2 * BQ, clen) - 1
								   : -1)};
	const int nb = max(nb_t[0], nb_t[1]);

	// ---- setup ----------------------------------------------------------------
	if (tid == 0) {
		mbar_init(&sm.q_full, 1);
		for (int i = 0; i < kStages; ++i) {
			mbar_init(&sm.k_full[i], 1);
			mbar_init(&sm.k_empty[i], 1);
			mbar_init(&sm.v_full[i], 1);
			mbar_init(&sm.v_empty[i], 1);
		}
		for (int t = 0; t < 2; ++t) {
			mbar_init(&sm.s_full[t], 1);
			mbar_init(&sm.p_half[t], 128);
			mbar_init(&sm.p_full[t], 128);
			mbar_init(&sm.o_full[t], 1);
		}
		mbar_init(&sm.drain, 1);
		sm.abort = 0;
		fence_mbar_init();
	}
	for (int i = tid; i < 256; i += kThreads)
		sm.lut[i] = mx_scale_lut_entry((uint32_t)i);
	if (tid == 0) {
		sm.lut[256] = 16u;
		sm.lut[257] = 1u << 28;
	}
	if (warp == kWarpMma) {
		asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
			     :: "r"(smem_u32(&sm.tmem_base)), "r"(512u));
		asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = sm.tmem_base;
	// TMEM columns: S_A 0, S_B 128, O_A 256, O_B 384
	auto col_s = [](int t) { return (uint32_t)(t * 128); };
	auto col_o = [](int t) { return (uint32_t)(256 + t * 128); };

	if (warp < kWarpsSoftmax) {
		// ================= softmax of tile t, row r ==============================
		const int t = warp >> 2, r = (warp & 3) * 32 + lane;
		const int h = r % G, p = r / G;
		const int qpos = pos0 + t * BQ + p;               // position in the chunk
		const bool row_live = qpos < clen;
		const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
		const uint32_t tS = lane_base + col_s(t), tO = lane_base + col_o(t);
		float m_ref = -CUDART_INF_F, l_sum = 0.f;
		bool ok = true;
		for (int j = 0; j < nb_t[t] && ok; ++j) {
			// warp-uniform outcome: the TMEM accesses below are warp-collective
			if (!__all_sync(0xffffffffu,
					wait_or_abort(sm, &sm.s_full[t], (uint32_t)(j & 1), a))) {
				ok = false;
				break;
			}
			tc_fence_after();
			const bool prior = j < n_prior;
			const int kbase = prior ? j * kKeys : (j - n_prior) * kKeys;
			const float sl2 = a.scale_log2 * (prior && a.kv_dtype == 1 ? 256.f : 1.f);
			// valid keys of this row in the block, 32 per word: cached keys
			// with a page, or chunk keys at or before the row's position
			uint32_t vmask[4];
			{
				const int lim = min(clen, qpos + 1) - kbase;   // chunk keys < lim
#pragma unroll
				for (int c = 0; c < 4; ++c) {
					uint32_t mk;
					if (prior)
						mk = sm.key_ok[j % kStages][c];
					else
						mk = lim >= 32 * (c + 1) ? 0xFFFFFFFFu :
						     (lim <= 32 * c ? 0u : (1u << (lim - 32 * c)) - 1u);
					vmask[c] = row_live ? mk : 0u;
				}
			}
			// cached MX keys/values carry a 2^-8 factor: S is scaled back
			// through sl2 and P is built 2^8 larger for the PV product
			const float pexp = prior && a.kv_dtype == 1 ? 8.f : 0.f;
			const bool full = __all_sync(0xffffffffu, (vmask[0] & vmask[1] & vmask[2] &
								   vmask[3]) == 0xFFFFFFFFu);
			softmax_block(tS, tO, vmask, !full, sl2, pexp, j > 0, m_ref, l_sum, &sm.p_half[t]);
			tc_fence_before();
			mbar_arrive(&sm.p_full[t]);
		}
		// ---- epilogue: O / l -> bf16 (every lane loads: warp-collective) ------
		if (ok && nb_t[t] > 0 &&
		    __all_sync(0xffffffffu, wait_or_abort(sm, &sm.o_full[t], 0u, a))) {
			tc_fence_after();
			const float inv = l_sum > 0.f ? 1.f / l_sum : 0.f;
			uint4 *dst = reinterpret_cast<uint4 *>(
			    reinterpret_cast<uint8_t *>(a.out) +
			    (((size_t)(t0 + (row_live ? qpos : 0)) * a.num_heads + (size_t)kvh * G + h) *
			     kD) * 2);
#pragma unroll
			for (int c = 0; c < 8; ++c) {
				float v[16];
				tmem_ld16(tO + 16 * c, v);
				if (!row_live)
					continue;
#pragma unroll
				for (int i = 0; i < 2; ++i)
					dst[2 * c + i] = make_uint4(
					    pack_bf16x2(v[8 * i] * inv, v[8 * i + 1] * inv),
					    pack_bf16x2(v[8 * i + 2] * inv, v[8 * i + 3] * inv),
					    pack_bf16x2(v[8 * i + 4] * inv, v[8 * i + 5] * inv),
					    pack_bf16x2(v[8 * i + 6] * inv, v[8 * i + 7] * inv));
			}
		}
	} else if (warp >= kWarpProducer0) {
		// ================= producer ==============================================
		const int pt = tid - kWarpProducer0 * 32;          // 0..95
		if (pt == 0) {
			// both query tiles by TMA: box {64 dims, G heads, BQ tokens} per half
			mbar_arrive_expect_tx(&sm.q_full, 4 * kHalfBytes);
			for (int t = 0; t < 2; ++t)
				for (int half = 0; half < 2; ++half)
					tma_load_3d(sm.q[t] + half * kHalfBytes, &tm_q, half * kHalf, kvh * G,
						    t0 + pos0 + t * BQ, &sm.q_full);
		}
		int issued_k[kStages] = {-1, -1}, issued_v[kStages] = {-1, -1};  // TMA fills armed
		bool alive = true;   // thread 0: no wait of its own has failed
		for (int j = 0; j < nb; ++j) {
			const int st = j % kStages, fill = j / kStages;
			const uint32_t par = (uint32_t)((fill - 1) & 1);
			const bool prior = j < n_prior;
			// one thread waits for the stage; the group leaves together
			if (pt == 0) {
				bool okw = alive && (fill == 0 || wait_or_abort(sm, &sm.k_empty[st], par, a));
				if (okw && prior)   // the dequant writes K and V (and the key mask) at once
					okw = fill == 0 || wait_or_abort(sm, &sm.v_empty[st], par, a);
				sm.prod_ok[j & 1] = okw;
			}
			asm volatile("bar.sync 1, 96;" ::: "memory");
			if (!*reinterpret_cast<volatile int *>(&sm.prod_ok[j & 1]))
				break;
			if (prior) {
#pragma unroll 1
			for (int row = pt; row < kKeys; row += kProducerThreads) {   // warp-uniform
				const int kpos = j * kKeys + row;
				int slot = 0;
				const uint8_t *ks = nullptr, *vs = nullptr;
				if (kpos < ctx_cap) {
					ks = cached_section(a, seq, kvh, kpos, 0, slot);
					vs = cached_section(a, seq, kvh, kpos, 1, slot);
				}
				const bool okk = ks != nullptr;
				if (a.kv_dtype == 1) {
					// K and V rows (payload + scales) all in flight, then convert
					uint4 kpay[8], vpay[8], ksc, vsc;
					if (okk) {
						const uint4 *kq = reinterpret_cast<const uint4 *>(ks + (size_t)slot * kD);
						const uint4 *vq = reinterpret_cast<const uint4 *>(vs + (size_t)slot * kD);
#pragma unroll
						for (int i = 0; i < 8; ++i) {
							kpay[i] = kq[i];
							vpay[i] = vq[i];
						}
						const size_t so = (size_t)a.block_size * kD + (size_t)slot * (kD / 8);
						ksc = *reinterpret_cast<const uint4 *>(ks + so);
						vsc = *reinterpret_cast<const uint4 *>(vs + so);
					} else {
#pragma unroll
						for (int i = 0; i < 8; ++i)
							kpay[i] = vpay[i] = make_uint4(0u, 0u, 0u, 0u);
						ksc = vsc = make_uint4(0u, 0u, 0u, 0u);
					}
#pragma unroll
					for (int part = 0; part < 4; ++part) {   // K lo, K hi, V lo, V hi
						const int half = part & 1;
						const uint4 *pay = part < 2 ? kpay : vpay;
						const uint4 sc = part < 2 ? ksc : vsc;
						uint32_t w[32];
						mx_dequant_half(sm.lut, pay + 4 * half,
								half ? make_uint2(sc.z, sc.w) : make_uint2(sc.x, sc.y), w);
						store_half_row(part < 2 ? sm.k[st] : sm.v[st], row, half, w);
					}
				} else {
#pragma unroll 1
					for (int part = 0; part < 4; ++part) {   // K lo, K hi, V lo, V hi
						uint32_t w[32];
						const int half = part & 1;
						if (okk) {
							load_cached_half(a, sm.lut, part < 2 ? ks : vs, slot, half, w);
						} else {
#pragma unroll
							for (int i = 0; i < 32; ++i)
								w[i] = 0u;
						}
						store_half_row(part < 2 ? sm.k[st] : sm.v[st], row, half, w);
					}
				}
				const uint32_t ball = __ballot_sync(0xffffffffu, okk);
				if (lane == 0)
					sm.key_ok[st][row >> 5] = ball;
			}
				fence_async_smem();
				asm volatile("bar.sync 1, 96;" ::: "memory");
				if (pt == 0) {
					mbar_arrive(&sm.k_full[st]);
					mbar_arrive(&sm.v_full[st]);
				}
			} else if (pt == 0) {
				const int y = t0 + (j - n_prior) * kKeys;
				mbar_arrive_expect_tx(&sm.k_full[st], 2 * kHalfBytes);
				for (int half = 0; half < 2; ++half)
					tma_load_2d(sm.k[st] + half * kHalfBytes, &tm_k, kvh * kD + half * kHalf, y,
						    &sm.k_full[st]);
				issued_k[st] = fill;
				alive = fill == 0 || wait_or_abort(sm, &sm.v_empty[st], par, a);
				if (alive) {
					mbar_arrive_expect_tx(&sm.v_full[st], 2 * kHalfBytes);
					for (int half = 0; half < 2; ++half)
						tma_load_2d(sm.v[st] + half * kHalfBytes, &tm_v, kvh * kD + half * kHalf,
							    y, &sm.v_full[st]);
					issued_v[st] = fill;
				}
			}
		}
		// after an abort, wait (bounded) for this CTA's own tensor copies
		if (pt == 0 && *reinterpret_cast<volatile int *>(&sm.abort)) {
			mbar_wait_ns(&sm.q_full, 0u, kWaitNs);
			for (int st = 0; st < kStages; ++st) {
				if (issued_k[st] >= 0)
					mbar_wait_ns(&sm.k_full[st], (uint32_t)(issued_k[st] & 1), kWaitNs);
				if (issued_v[st] >= 0)
					mbar_wait_ns(&sm.v_full[st], (uint32_t)(issued_v[st] & 1), kWaitNs);
			}
		}
	} else {
		// ================= MMA issue =============================================
		// The whole warp runs this role, so the descriptors and addresses are
		// warp-uniform values; one elected lane issues the MMAs and commits.
		const bool leader = elect_one();
		const uint32_t id_s = umma_idesc(false), id_pv = umma_idesc(true);
		const uint32_t sq[2] = {smem_u32(sm.q[0]), smem_u32(sm.q[1])};
		// Operand descriptors are built once: a k-step adds (byte offset >> 4)
		// to the start-address field (bits 0-13), which cannot carry out since
		// shared-memory addresses stay below 2^18. Issue is the single thread's
		// critical path (it shares its scheduler with two softmax warps), so
		// each MMA costs one 64-bit add here.
		const uint64_t dq0 = umma_desc(sq[0], 16u, 1024u), dq1 = umma_desc(sq[1], 16u, 1024u);
		const uint64_t dk0 = umma_desc(smem_u32(sm.k[0]), 16u, 1024u);
		const uint64_t dk1 = umma_desc(smem_u32(sm.k[1]), 16u, 1024u);
		const uint64_t dv0 = umma_desc(smem_u32(sm.v[0]), (uint32_t)kHalfBytes, 1024u);
		const uint64_t dv1 = umma_desc(smem_u32(sm.v[1]), (uint32_t)kHalfBytes, 1024u);
		static_assert(kStages == 2, "descriptor selection assumes two stages");
		auto issue_s = [&](int t, int st) {
			const uint64_t dq = t ? dq1 : dq0, dk = st ? dk1 : dk0;
			const uint32_t d = tmem + col_s(t);
#pragma unroll
			for (int kk = 0; kk < kD / 16; ++kk) {
				const uint64_t off = ((uint64_t)(kk >> 2) * kHalfBytes + (uint64_t)(kk & 3) * 32u) >> 4;
				if (leader)
					umma_f16(d, dq + off, dk + off, id_s, kk > 0);
			}
			__syncwarp();
		};
		// half 0: keys 0-63 (P groups 0-3), half 1: keys 64-127
		auto issue_pv = [&](int t, int st, bool first, int half) {
			const uint64_t dv = st ? dv1 : dv0;
			const uint32_t d = tmem + col_o(t), pa = tmem + col_s(t);
#pragma unroll
			for (int kk = half * kKeys / 16; kk < (half + 1) * kKeys / 16; ++kk) {
				const int g = kk >> 1;     // 16-key group; kk odd: the lo half of P
				if (leader)
					umma_f16_ts(d, pa + 16u * g + 8u * (kk & 1), dv + (uint64_t)((g * 2048) >> 4),
						    id_pv, (first && kk == 0) ? 0u : 1u);
			}
			__syncwarp();
		};
		auto commit = [&](uint64_t *bar) {
			if (leader)
				umma_commit(bar);
			__syncwarp();
		};
		// every lane waits; the outcome is made warp-uniform
		auto wait_all = [&](uint64_t *bar, uint32_t parity) {
			return __all_sync(0xffffffffu, wait_or_abort(sm, bar, parity, a));
		};
		bool ok = wait_all(&sm.q_full, 0u);
		ok = ok && wait_all(&sm.k_full[0], 0u);
		if (ok) {
			tc_fence_after();
			for (int t = 0; t < 2; ++t)
				if (nb_t[t] > 0) {
					issue_s(t, 0);
					commit(&sm.s_full[t]);
				}
			commit(&sm.k_empty[0]);
		}
		for (int j = 0; j < nb && ok; ++j) {
			const int st = j % kStages, ns = (j + 1) % kStages;
			ok = wait_all(&sm.v_full[st], (uint32_t)((j / kStages) & 1));
			for (int t = 0; t < 2 && ok; ++t) {
				if (j < nb_t[t]) {
					if (!wait_all(&sm.p_half[t], (uint32_t)(j & 1))) {
						ok = false;
						break;
					}
					tc_fence_after();
					issue_pv(t, st, j == 0, 0);
					if (!wait_all(&sm.p_full[t], (uint32_t)(j & 1))) {
						ok = false;
						break;
					}
					tc_fence_after();
					issue_pv(t, st, j == 0, 1);
				}
				if (t == 1)
					commit(&sm.v_empty[st]);   // both PV(j) issued: V(j) free when done
				if (t == 0 && j + 1 < nb) {
					// K of block j + 1, for both tiles' next S
					if (!wait_all(&sm.k_full[ns], (uint32_t)(((j + 1) / kStages) & 1))) {
						ok = false;
						break;
					}
					tc_fence_after();
				}
				if (j + 1 < nb_t[t]) {
					issue_s(t, ns);
					commit(&sm.s_full[t]);
				} else if (j + 1 == nb_t[t]) {
					commit(&sm.o_full[t]);
				}
			}
			if (ok && j + 1 < nb)
				commit(&sm.k_empty[ns]);       // both S(j + 1) issued
		}
		// drain: every MMA issued by the leader completes before TMEM is freed
		commit(&sm.drain);
		mbar_wait_ns(&sm.drain, 0u, kWaitNs);
	}

	tc_fence_before();
	__syncthreads();
	if (warp == kWarpMma) {
		__syncwarp();
		tc_fence_after();
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
			     :: "r"(tmem), "r"(512u));
	}
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

// [num_tokens][num_heads][128] bf16 as {dims, heads, tokens}, box 64 dims x
// G heads x 128/G tokens (one 128-row half tile), 128-byte swizzle
bool make_q_map(CUtensorMap *m, const void *base, int num_tokens, int hq, int g)
{
	auto enc = get_encode();
	if (!enc)
		return false;
	cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)hq, (cuuint64_t)num_tokens};
	cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)hq * kD * 2};
	cuuint32_t box[3] = {(cuuint32_t)kHalf, (cuuint32_t)g, (cuuint32_t)(kRows / g)};
	cuuint32_t estr[3] = {1, 1, 1};
	return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims,
		   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
		   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
		   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int G>
int launch_g(const kllm_prefill_args &a, const CUtensorMap &mq, const CUtensorMap &mk,
	     const CUtensorMap &mv,
	     cudaStream_t st)
{
	const size_t smem = sizeof(PrefillSmem) + 1024;
	cudaError_t e = cudaFuncSetAttribute(prefill_kernel<G>,
					     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
	if (e != cudaSuccess)
		return (int)e;
	cudaFuncAttributes fa;
	e = cudaFuncGetAttributes(&fa, prefill_kernel<G>);
	if (e != cudaSuccess)
		return (int)e;
	constexpr int BQ = kRows / G;
	dim3 grid((a.max_chunk + 2 * BQ - 1) / (2 * BQ), a.num_kv_heads, a.num_seqs);
	cudaError_t le = cudaSuccess;
	if (fa.maxThreadsPerBlock < kThreads) {
		le = cudaErrorLaunchOutOfResources;
	} else {
		prefill_kernel<G><<<grid, kThreads, smem, st>>>(a, mq, mk, mv);
		le = cudaGetLastError();
	}
	if (le != cudaSuccess && getenv("KLLM_GPU_DEBUG"))
		fprintf(stderr,
			"prefill_kernel<%d>: %s; regs %d, max threads %d, static smem %zu, "
			"dynamic smem %zu (max %d), local %zu, grid %u x %u x %u x %d\n",
			G, cudaGetErrorString(le), fa.numRegs, fa.maxThreadsPerBlock,
			fa.sharedSizeBytes, smem, fa.maxDynamicSharedSizeBytes, fa.localSizeBytes,
			grid.x, grid.y, grid.z, kThreads);
	return (int)le;
}

}  // namespace
}  // namespace kllm

using namespace kllm;

extern "C" int kllm_prefill_launch(const struct kllm_prefill_args *a, void *stream)
{
	if (a->head_dim != kD)
		return (int)cudaErrorInvalidValue;
	const int g = a->num_heads / a->num_kv_heads;
	CUtensorMap mq, mk, mv;
	if (!make_map(&mk, a->k, a->num_tokens, a->num_kv_heads) ||
	    !make_map(&mv, a->v, a->num_tokens, a->num_kv_heads) ||
	    !make_q_map(&mq, a->q, a->num_tokens, a->num_heads, g))
		return (int)cudaErrorInvalidValue;
	cudaStream_t st = static_cast<cudaStream_t>(stream);
	switch (g) {
	case 1: return launch_g<1>(*a, mq, mk, mv, st);
	case 2: return launch_g<2>(*a, mq, mk, mv, st);
	case 4: return launch_g<4>(*a, mq, mk, mv, st);
	case 8: return launch_g<8>(*a, mq, mk, mv, st);
	default: return (int)cudaErrorInvalidValue;
	}
}
