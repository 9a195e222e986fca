// SPDX-License-Identifier: Apache-2.0
//
// paged_decode.cu - GQA paged-attention decode for sm_100a.
//
// Replaces paged_attention_kernel_cuda (userspace/gpu/paged_attention.cu:24-119):
// the same block-table gather (entries {k_ptr, v_ptr, valid}, invalid entries
// skipped, last page cut at seq_len: paged_attention.cu:55-68), the same GQA
// map (kv_head = q_head / (Hq/Hkv): paged_attention.cu:45), online softmax
// (paged_attention.cu:86-98, with every output lane rescaled) and a BF16 RNE
// store (paged_attention.cu:109-118). Empty contexts give zeros
// (paged_attention.cu:110 with exp_sum == 0).
//
// Work decomposition. A "segment" is one (seq, kv_head) pair; its context is
// cut into tiles of 16 tokens. All tiles of a launch are laid end to end
// (seq-major, then kv head, then tile) and every warp of a persistent grid
// takes an equal contiguous range of that list, so the HBM stream is
// balanced to within one tile no matter how ragged the context lengths are.
// A segment covered by several warps produces fp32 partials (m, l, o) in the
// workspace; the last warp to finish it (arrival counter) merges them with
// the log-sum-exp rule. Without a workspace, warps take whole segments.
//
// Per warp, per tile: lane 0 streams the tile's K and V (and, for MX, their
// scale bytes) from the page into a private shared-memory ring with
// cp.async.bulk (TMA engine, mbarrier completion, L2 evict-first), several
// tiles ahead; block-table entries are prefetched 32 tiles ahead by the whole
// warp. The G query heads of the segment share every K/V byte:
//   S^T[16 tok x 8 heads] = K_tile[16 x D] . Q^T   (mma.m16n8k16, bf16)
//   P^T -> bf16 hi + bf16 lo, transposed in registers (movmatrix)
//   O^T[D x 8 heads] += V_tile^T[D x 16] . (P_hi^T + P_lo^T)  (2 x mma.m16n8k16)
// MX-FP8 tiles are dequantised in registers to f16 (hardware e4m3x2 -> f16x2
// conversion, then one f16x2 multiply by the block's scale / 4) and the MX
// contractions run as f16 MMAs; the query is scaled by a power of two into
// f16 range per segment, and both factors are undone in the softmax scale
// and the final normalisation. Dimensions are permuted consistently inside each
// contraction so that every lane reads contiguous 16-byte runs of shared
// memory; the output permutation is undone at the store.

#include "kllm_device.cuh"
#include "kllm_internal.h"

#include <math_constants.h>

namespace kllm {
namespace {

#ifndef KLLM_DEC_STAGES
#define KLLM_DEC_STAGES 2       // bulk-copy ring depth per warp
#endif
#ifndef KLLM_MERGE_FLY
#define KLLM_MERGE_FLY 16       // wide merge: pieces in flight per warp
#endif
#ifndef KLLM_DEC_MIN_CTAS_MX
#define KLLM_DEC_MIN_CTAS_MX 4  // resident MX decode CTAs per SM (register cap)
#endif

constexpr int kTile = 16;
constexpr int kWarps = KLLM_DEC_WARPS;
constexpr int kSlotO = 0;                       // o[8][128]
constexpr int kSlotM = KLLM_MAX_GROUP * 128;    // m[8]
constexpr int kSlotL = kSlotM + KLLM_MAX_GROUP; // l[8]
constexpr float kLazyLog2 = 8.f;                // reference max slack (p <= 256)

template <int D, int KVT>
struct Geom {
	static constexpr bool MX = (KVT == 1);
	static constexpr int PAY = MX ? kTile * D : kTile * D * 2;  // payload / tile
	static constexpr int SCL = MX ? kTile * D / 8 : 0;          // scales / tile
	static constexpr int KV = PAY + SCL;                        // one of K, V
	static constexpr int STAGE = 2 * KV;
	static constexpr int NST = KLLM_DEC_STAGES;                 // ring depth
	static constexpr int MIN_CTAS = MX ? KLLM_DEC_MIN_CTAS_MX : 2;  // per SM
};

struct DevEntry {  // userspace/gpu/paged_attention.cu:18-22 (24 bytes)
	unsigned long long k, v;
	int valid;
	int pad;
};

struct Seg {
	int s, h, j, ts;  // seq, kv head, tile in segment, tiles in segment
};

// Merge work list (KLLM_MERGE_LIST_BYTES): header, then items.
struct ListHeader {
	unsigned count, done;
	long long T, W;
	long long pad;
};
struct ListItem {
	int s, h, ts, pad;
	long long seg_x0;
};
static_assert(sizeof(ListHeader) == 32 && sizeof(ListItem) == 24, "list layout");

__host__ __device__ inline size_t align_up(size_t x, size_t a)
{
	return (x + a - 1) / a * a;
}

struct SmemLayout {
	size_t stage, bar, meta, lut, prefix, slen, total;
	__host__ __device__ SmemLayout(int stage_bytes, int nst, int S)
	{
		stage = 0;
		bar = align_up((size_t)stage_bytes * nst * kWarps, 128);
		meta = bar + sizeof(uint64_t) * nst * kWarps;
		lut = align_up(meta + sizeof(int) * nst * kWarps, 16);
		prefix = lut + 260 * sizeof(uint32_t);  // 256 scale entries + 4 constants
		slen = prefix + sizeof(int) * (S + 1);
		total = slen + sizeof(int) * S;
	}
};

// Largest s in [0,S) with prefix[s]*H <= x (x < prefix[S]*H): the segment
// holding flattened tile x. Sequences without tiles are never returned.
__device__ __forceinline__ Seg locate(const int *prefix, int S, int H,
				       long long x)
{
	int lo = 0, hi = S - 1;
	while (lo < hi) {
		int mid = (lo + hi + 1) >> 1;
		if ((long long)prefix[mid] * H <= x)
			lo = mid;
		else
			hi = mid - 1;
	}
	Seg c;
	c.s = lo;
	c.ts = prefix[lo + 1] - prefix[lo];
	long long rel = x - (long long)prefix[lo] * H;
	c.h = (int)(rel / c.ts);
	c.j = (int)(rel - (long long)c.h * c.ts);
	return c;
}

__device__ __forceinline__ long long seg_start_at_or_after(
    const int *prefix, int S, int H, long long T, long long y)
{
	if (y >= T)
		return T;
	Seg c = locate(prefix, S, H, y);
	return c.j == 0 ? y : y - c.j + c.ts;
}

// Owner warp of flattened tile x in the balanced split: warp w covers
// [floor(w*T/W), floor((w+1)*T/W)).
__device__ __forceinline__ long long owner_warp(long long x, long long T,
						long long W)
{
	return ((x + 1) * W - 1) / T;
}

template <int N>
__device__ __forceinline__ void lds_words(uint32_t (&w)[N], const uint8_t *p)
{
	if constexpr (N % 4 == 0) {
#pragma unroll
		for (int i = 0; i < N / 4; ++i) {
			uint4 v = reinterpret_cast<const uint4 *>(p)[i];
			w[4 * i] = v.x;
			w[4 * i + 1] = v.y;
			w[4 * i + 2] = v.z;
			w[4 * i + 3] = v.w;
		}
	} else if constexpr (N == 2) {
		uint2 v = *reinterpret_cast<const uint2 *>(p);
		w[0] = v.x;
		w[1] = v.y;
	} else {
		w[0] = *reinterpret_cast<const uint32_t *>(p);
	}
}

// Block-table entries for 32 consecutive tiles of the warp's stream, one per
// lane. load_batch issues the entry loads; finalize_batch (called 32 tiles
// later, when the loads have long landed) turns them into the K/V head
// section addresses of the tile, so issuing a copy costs only shuffles.
struct Batch {
	unsigned long long k, v;  // raw entry, then section base addresses
	int valid;
	int pack;  // ntok | sub << 8 | h << 16; after finalize: ntok | sub << 8
};

__device__ __forceinline__ void load_batch(Batch &b, const kllm_decode_args &a,
					   const int *prefix, const int *slen,
					   long long xa, int n, int base,
					   int lane, int tpp)
{
	int pos = base + lane;
	b.k = 0;
	b.v = 0;
	b.valid = 0;
	b.pack = 0;
	if (pos < n) {
		Seg c = locate(prefix, a.num_seqs, a.num_kv_heads, xa + pos);
		int ntok = slen[c.s] - c.j * kTile;
		ntok = ntok < kTile ? ntok : kTile;
		int page = c.j / tpp, sub = c.j - page * tpp;
		const DevEntry *e = reinterpret_cast<const DevEntry *>(a.table) +
				    (size_t)c.s * a.max_blocks + page;
		b.k = __ldg(&e->k);
		b.v = __ldg(&e->v);
		b.valid = __ldg(&e->valid);
		b.pack = ntok | (sub << 8) | (c.h << 16);
	}
}

// Raw entry -> section addresses; pack keeps ntok (0: nothing to copy) and sub.
__device__ __forceinline__ void finalize_batch(Batch &b, const kllm_decode_args &a,
					       size_t sec)
{
	const int ntok = b.pack & 0xFF, sub = (b.pack >> 8) & 0xFF, h = b.pack >> 16;
	const bool present = b.valid && b.k != 0ull;
	const bool aligned = ((b.k | b.v) & 15ull) == 0ull;
	if (present && !aligned && a.err)
		atomicOr(a.err, 0x2u);
	bool ok = present && aligned && ntok > 0;
	const unsigned long long off = a.layer_off + (unsigned long long)h * sec;
	// registered arenas: a section outside them is skipped, never read
	if (ok && !(in_arenas(a.arenas, b.k + off, sec) && in_arenas(a.arenas, b.v + off, sec))) {
		ok = false;
		if (a.err)
			atomicOr(a.err, KLLM_ERR_PAGE_RANGE_BIT);
	}
	b.k += off;
	b.v += off;
	b.pack = (ok ? ntok : 0) | (sub << 8);
}

template <int D>
__device__ __forceinline__ void load_q(uint32_t (&q)[D / 8],
				       const kllm_decode_args &a, int s, int h,
				       int lane)
{
	const int g = lane >> 2, c = lane & 3;
	if (g < a.group) {
		const uint8_t *p = reinterpret_cast<const uint8_t *>(a.q) +
			(((size_t)s * a.num_heads + (size_t)h * a.group + g) * D +
			 (size_t)c * (D / 4)) * 2;
#pragma unroll
		for (int i = 0; i < D / 32; ++i) {
			uint4 v = __ldg(reinterpret_cast<const uint4 *>(p) + i);
			q[4 * i] = v.x;
			q[4 * i + 1] = v.y;
			q[4 * i + 2] = v.z;
			q[4 * i + 3] = v.w;
		}
	} else {
#pragma unroll
		for (int i = 0; i < D / 8; ++i)
			q[i] = 0u;
	}
}

// MX path: the segment's query rows (bf16, as load_q leaves them) -> f16,
// multiplied by 2^e so that the largest |q| lies in [2^14, 2^15): no
// overflow, and every bf16 value of at least 2^-28 of that maximum converts
// exactly. Returns 2^-e, which multiplies the softmax scale.
template <int D>
__device__ __forceinline__ float q_to_f16(uint32_t (&q)[D / 8])
{
	float mx = 0.f;
#pragma unroll
	for (int i = 0; i < D / 8; ++i)
		mx = fmaxf(mx, fmaxf(fabsf(__uint_as_float(q[i] << 16)),
				     fabsf(__uint_as_float(q[i] & 0xFFFF0000u))));
#pragma unroll
	for (int off = 1; off < 32; off <<= 1)
		mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
	const int E = mx > 0.f ? (int)((__float_as_uint(mx) >> 23) & 0xFFu) - 127 : 0;
	int e = 14 - E;
	e = e < -100 ? -100 : (e > 100 ? 100 : e);
	const float f = __uint_as_float((uint32_t)(e + 127) << 23);
#pragma unroll
	for (int i = 0; i < D / 8; ++i)
		q[i] = pack_f16x2(__uint_as_float(q[i] << 16) * f,
				  __uint_as_float(q[i] & 0xFFFF0000u) * f);
	return __uint_as_float((uint32_t)(127 - e) << 23);
}

// One 16-token tile: scores, online-softmax update and PV accumulation.
template <int D, int KVT>
__device__ __forceinline__ void tile_compute(
    const uint8_t *sK, const uint8_t *sV, const uint32_t *lut, int ntok,
    const uint32_t (&q)[D / 8], float (&o)[D / 16][4], float &m0, float &m1,
    float &l0, float &l1, float &mx0, float &mx1, float scale_log2, int lane)
{
	using Gm = Geom<D, KVT>;
	const int g = lane >> 2, c = lane & 3;

	// ---- S^T[tok][head] = K . Q^T ------------------------------------------
	float s[4] = {0.f, 0.f, 0.f, 0.f};
	float s2[4] = {0.f, 0.f, 0.f, 0.f};  // odd k-steps: halves the MMA chain
	if constexpr (Gm::MX) {
		constexpr int KW = D / 16;
		uint32_t k0[KW], k1[KW];
		lds_words<KW>(k0, sK + g * D + c * (D / 4));
		lds_words<KW>(k1, sK + (g + 8) * D + c * (D / 4));
		uint32_t sw0, sw1;
		if constexpr (D == 128) {
			sw0 = *reinterpret_cast<const uint32_t *>(sK + kTile * D + g * 16 + c * 4);
			sw1 = *reinterpret_cast<const uint32_t *>(sK + kTile * D + (g + 8) * 16 + c * 4);
		} else {
			sw0 = *reinterpret_cast<const uint16_t *>(sK + kTile * D + g * 8 + c * 2);
			sw1 = *reinterpret_cast<const uint16_t *>(sK + kTile * D + (g + 8) * 8 + c * 2);
		}
		uint32_t sc0[D / 32], sc1[D / 32];
#pragma unroll
		for (int b = 0; b < D / 32; ++b) {
			sc0[b] = lut[__byte_perm(sw0, 0u, 0x4440u | b)];
			sc1[b] = lut[__byte_perm(sw1, 0u, 0x4440u | b)];
		}
#pragma unroll
		for (int j = 0; j < D / 16; ++j) {
			// word j = dims 4j..4j+3 of this lane's chunk: (0,1) -> a0/a1, (2,3) -> a2/a3
			const uint32_t a0 = f16x2_mul(e4m3x2_lo_to_f16x2(k0[j]), sc0[j >> 1]);
			const uint32_t a2 = f16x2_mul(e4m3x2_hi_to_f16x2(k0[j]), sc0[j >> 1]);
			const uint32_t a1 = f16x2_mul(e4m3x2_lo_to_f16x2(k1[j]), sc1[j >> 1]);
			const uint32_t a3 = f16x2_mul(e4m3x2_hi_to_f16x2(k1[j]), sc1[j >> 1]);
			if (j & 1)
				mma_f16(s2, a0, a1, a2, a3, q[2 * j], q[2 * j + 1]);
			else
				mma_f16(s, a0, a1, a2, a3, q[2 * j], q[2 * j + 1]);
		}
	} else {
		constexpr int KW = D / 8;
		uint32_t k0[KW], k1[KW];
		lds_words<KW>(k0, sK + (g * D + c * (D / 4)) * 2);
		lds_words<KW>(k1, sK + ((g + 8) * D + c * (D / 4)) * 2);
#pragma unroll
		for (int j = 0; j < D / 16; ++j) {
			if (j & 1)
				mma_bf16(s2, k0[2 * j], k1[2 * j], k0[2 * j + 1],
					 k1[2 * j + 1], q[2 * j], q[2 * j + 1]);
			else
				mma_bf16(s, k0[2 * j], k1[2 * j], k0[2 * j + 1],
					 k1[2 * j + 1], q[2 * j], q[2 * j + 1]);
		}
	}
#pragma unroll
	for (int i = 0; i < 4; ++i)
		s[i] += s2[i];

	// ---- online softmax (log2 domain, lazy reference max) ---------------------
	// m0/m1 are warp-uniform reference maxima per head. They are raised only
	// when some lane's score exceeds them by more than kLazyLog2, so most tiles
	// skip the cross-lane max and the O rescale; p then stays <= 2^kLazyLog2.
	// mx0/mx1 track each lane's exact running maximum for the final triple.
	const bool v0 = g < ntok, v1 = g + 8 < ntok;
	const float x0 = v0 ? s[0] * scale_log2 : -CUDART_INF_F;  // tok g,   head 2c
	const float x1 = v0 ? s[1] * scale_log2 : -CUDART_INF_F;  // tok g,   head 2c+1
	const float x2 = v1 ? s[2] * scale_log2 : -CUDART_INF_F;  // tok g+8, head 2c
	const float x3 = v1 ? s[3] * scale_log2 : -CUDART_INF_F;  // tok g+8, head 2c+1
	float t0 = fmaxf(x0, x2), t1 = fmaxf(x1, x3);
	mx0 = fmaxf(mx0, t0);
	mx1 = fmaxf(mx1, t1);
	if (__any_sync(0xffffffffu, t0 > m0 + kLazyLog2 || t1 > m1 + kLazyLog2)) {
#pragma unroll
		for (int off = 4; off < 32; off <<= 1) {
			t0 = fmaxf(t0, __shfl_xor_sync(0xffffffffu, t0, off));
			t1 = fmaxf(t1, __shfl_xor_sync(0xffffffffu, t1, off));
		}
		const float mn0 = fmaxf(m0, t0), mn1 = fmaxf(m1, t1);  // finite: ntok >= 1
		const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
		l0 *= al0;
		l1 *= al1;
		m0 = mn0;
		m1 = mn1;
#pragma unroll
		for (int mt = 0; mt < D / 16; ++mt) {
			o[mt][0] *= al0;
			o[mt][1] *= al1;
			o[mt][2] *= al0;
			o[mt][3] *= al1;
		}
	}
	const float p0 = exp2f(x0 - m0), p2 = exp2f(x2 - m0);
	const float p1 = exp2f(x1 - m1), p3 = exp2f(x3 - m1);
	l0 += p0 + p2;
	l1 += p1 + p3;
	// P as a hi + lo pair of the V operand's type (bf16: 16 significant bits,
	// f16: 22): one rounded P misses the 1e-3 absolute bound on outputs built
	// from a few large, cancelling V values.
	uint32_t h01, h23, l01, l23;
	if constexpr (Gm::MX) {
		h01 = pack_f16x2(p0, p1);
		h23 = pack_f16x2(p2, p3);
		const float2 f01 = __half22float2(*reinterpret_cast<const __half2 *>(&h01));
		const float2 f23 = __half22float2(*reinterpret_cast<const __half2 *>(&h23));
		l01 = pack_f16x2(p0 - f01.x, p1 - f01.y);
		l23 = pack_f16x2(p2 - f23.x, p3 - f23.y);
	} else {
		h01 = pack_bf16x2(p0, p1);
		h23 = pack_bf16x2(p2, p3);
		l01 = pack_bf16x2(p0 - __uint_as_float(h01 << 16),
				  p1 - __uint_as_float(h01 & 0xFFFF0000u));
		l23 = pack_bf16x2(p2 - __uint_as_float(h23 << 16),
				  p3 - __uint_as_float(h23 & 0xFFFF0000u));
	}
	const uint32_t b0 = movmatrix_trans(h01);   // tok 2c,2c+1;   head g
	const uint32_t b1 = movmatrix_trans(h23);   // tok 2c+8,2c+9; head g
	const uint32_t c0 = movmatrix_trans(l01);
	const uint32_t c1 = movmatrix_trans(l23);

	// ---- O^T[dim][head] += V^T . P^T -----------------------------------------
	const int r0 = 2 * c, r1 = 2 * c + 1, r2 = 2 * c + 8, r3 = 2 * c + 9;
	if constexpr (Gm::MX) {
		constexpr int VW = D / 32;
		uint32_t w0[VW], w1[VW], w2[VW], w3[VW];
		lds_words<VW>(w0, sV + r0 * D + g * (D / 8));
		lds_words<VW>(w1, sV + r1 * D + g * (D / 8));
		lds_words<VW>(w2, sV + r2 * D + g * (D / 8));
		lds_words<VW>(w3, sV + r3 * D + g * (D / 8));
		if (ntok < kTile) {  // zero rows past the context (payload 0 == 0.0)
#pragma unroll
			for (int i = 0; i < VW; ++i) {
				if (r0 >= ntok) w0[i] = 0u;
				if (r1 >= ntok) w1[i] = 0u;
				if (r2 >= ntok) w2[i] = 0u;
				if (r3 >= ntok) w3[i] = 0u;
			}
		}
		constexpr int NB = D / 64;  // scale blocks per lane chunk
		uint32_t s01[NB], s23[NB];
		const uint8_t *sS = sV + kTile * D;
#pragma unroll
		for (int bb = 0; bb < NB; ++bb) {
			const int col = g * NB + bb;
			s01[bb] = __byte_perm(lut[sS[r0 * (D / 8) + col]],
					      lut[sS[r1 * (D / 8) + col]], 0x5410u);
			s23[bb] = __byte_perm(lut[sS[r2 * (D / 8) + col]],
					      lut[sS[r3 * (D / 8) + col]], 0x5410u);
		}
#pragma unroll
		for (int i = 0; i < VW; ++i) {
			const int bb = i >> 1;  // m-tiles 2i, 2i+1 -> dims 4i..4i+3 -> block (4i)/8
			const uint32_t c01a = __byte_perm(w0[i], w1[i], 0x5140u);
			const uint32_t c01b = __byte_perm(w0[i], w1[i], 0x7362u);
			const uint32_t c23a = __byte_perm(w2[i], w3[i], 0x5140u);
			const uint32_t c23b = __byte_perm(w2[i], w3[i], 0x7362u);
			// (R0,R1) / (R2,R3) token pairs of dims 4i, 4i+1 (x) and 4i+2, 4i+3 (y)
			const uint32_t e0 = f16x2_mul(e4m3x2_lo_to_f16x2(c01a), s01[bb]);
			const uint32_t e1 = f16x2_mul(e4m3x2_hi_to_f16x2(c01a), s01[bb]);
			const uint32_t e2 = f16x2_mul(e4m3x2_lo_to_f16x2(c23a), s23[bb]);
			const uint32_t e3 = f16x2_mul(e4m3x2_hi_to_f16x2(c23a), s23[bb]);
			mma_f16(o[2 * i], e0, e1, e2, e3, b0, b1);
			mma_f16(o[2 * i], e0, e1, e2, e3, c0, c1);
			const uint32_t f0 = f16x2_mul(e4m3x2_lo_to_f16x2(c01b), s01[bb]);
			const uint32_t f1 = f16x2_mul(e4m3x2_hi_to_f16x2(c01b), s01[bb]);
			const uint32_t f2 = f16x2_mul(e4m3x2_lo_to_f16x2(c23b), s23[bb]);
			const uint32_t f3 = f16x2_mul(e4m3x2_hi_to_f16x2(c23b), s23[bb]);
			mma_f16(o[2 * i + 1], f0, f1, f2, f3, b0, b1);
			mma_f16(o[2 * i + 1], f0, f1, f2, f3, c0, c1);
		}
	} else {
		constexpr int VW = D / 16;
		uint32_t w0[VW], w1[VW], w2[VW], w3[VW];
		lds_words<VW>(w0, sV + (r0 * D + g * (D / 8)) * 2);
		lds_words<VW>(w1, sV + (r1 * D + g * (D / 8)) * 2);
		lds_words<VW>(w2, sV + (r2 * D + g * (D / 8)) * 2);
		lds_words<VW>(w3, sV + (r3 * D + g * (D / 8)) * 2);
		if (ntok < kTile) {  // rows past the context may hold any bits
#pragma unroll
			for (int i = 0; i < VW; ++i) {
				if (r0 >= ntok) w0[i] = 0u;
				if (r1 >= ntok) w1[i] = 0u;
				if (r2 >= ntok) w2[i] = 0u;
				if (r3 >= ntok) w3[i] = 0u;
			}
		}
#pragma unroll
		for (int mt = 0; mt < D / 16; ++mt) {
			const uint32_t e0 = __byte_perm(w0[mt], w1[mt], 0x5410u);
			const uint32_t e1 = __byte_perm(w0[mt], w1[mt], 0x7632u);
			const uint32_t e2 = __byte_perm(w2[mt], w3[mt], 0x5410u);
			const uint32_t e3 = __byte_perm(w2[mt], w3[mt], 0x7632u);
			mma_bf16(o[mt], e0, e1, e2, e3, b0, b1);
			mma_bf16(o[mt], e0, e1, e2, e3, c0, c1);
		}
	}
}

// Writes one query head's normalised row: bf16 output or fp32 triple.
// vals[k] = dim (D/8)*g + k.
template <int D>
__device__ __forceinline__ void store_head_row(const kllm_decode_args &a,
					       size_t row, int g,
					       const float (&vals)[D / 8],
					       float m_log2, float lsum,
					       float unbias)
{
	const float inv = lsum > 0.f ? unbias / lsum : 0.f;
	if (a.pm) {
		float *po = a.po + row * D + (size_t)g * (D / 8);
#pragma unroll
		for (int k = 0; k < D / 8; k += 4)
			*reinterpret_cast<float4 *>(po + k) = make_float4(
			    vals[k] * inv, vals[k + 1] * inv, vals[k + 2] * inv,
			    vals[k + 3] * inv);
		if (g == 0) {
			a.pm[row] = lsum > 0.f ? m_log2 * 0.69314718055994531f
					       : -CUDART_INF_F;
			a.pl[row] = lsum;
		}
	} else {
		uint32_t packed[D / 16];
#pragma unroll
		for (int k = 0; k < D / 16; ++k)
			packed[k] = pack_bf16x2(vals[2 * k] * inv, vals[2 * k + 1] * inv);
		uint8_t *po = reinterpret_cast<uint8_t *>(a.out) +
			      (row * D + (size_t)g * (D / 8)) * 2;
#pragma unroll
		for (int k = 0; k < D / 16; k += 4)
			*reinterpret_cast<uint4 *>(po + k * 4) =
			    make_uint4(packed[k], packed[k + 1], packed[k + 2], packed[k + 3]);
	}
}

template <int D>
__device__ void write_empty_seq(const kllm_decode_args &a, int s, int lane)
{
	const size_t rows = (size_t)a.num_heads;
	const size_t row0 = (size_t)s * a.num_heads;
	if (a.pm) {
		for (size_t r = lane; r < rows; r += 32) {
			a.pm[row0 + r] = -CUDART_INF_F;
			a.pl[row0 + r] = 0.f;
		}
		float4 *po = reinterpret_cast<float4 *>(a.po + row0 * D);
		for (size_t i = lane; i < rows * D / 4; i += 32)
			po[i] = make_float4(0.f, 0.f, 0.f, 0.f);
	} else if (a.out) {
		uint4 *po = reinterpret_cast<uint4 *>(
		    reinterpret_cast<uint8_t *>(a.out) + row0 * D * 2);
		for (size_t i = lane; i < rows * D / 8; i += 32)
			po[i] = make_uint4(0u, 0u, 0u, 0u);
	}
}

// NL consecutive floats from 8- or 16-byte aligned global memory (L2 only).
template <int NL>
__device__ __forceinline__ void ldcg_vec(float (&v)[NL], const float *src)
{
	if constexpr (NL % 4 == 0) {
#pragma unroll
		for (int i = 0; i < NL / 4; ++i) {
			const float4 x = __ldcg(reinterpret_cast<const float4 *>(src) + i);
			v[4 * i] = x.x;
			v[4 * i + 1] = x.y;
			v[4 * i + 2] = x.z;
			v[4 * i + 3] = x.w;
		}
	} else {
		static_assert(NL == 2, "two or a multiple of four floats");
		const float2 x = __ldcg(reinterpret_cast<const float2 *>(src));
		v[0] = x.x;
		v[1] = x.y;
	}
}

// Log-sum-exp merge of the pieces of one segment, run by the warp that
// finished last; it sits on that warp's critical path (the last arriver of a
// segment is usually the warp whose range ends inside it), so every load is
// issued without waiting on another. GP = the segment's query heads rounded
// up to a power of two; lane -> (head lane / (32/GP), NL dims from
// (lane % (32/GP)) * NL), so all 32 lanes work at every group size.
// Pass 1: each head's maximum over the pieces with mass (the 32/GP lanes of
// a head take every (32/GP)-th piece, four pieces per load batch). Pass 2:
// the pieces' o and l summed against that maximum, KB pieces in flight.
template <int D, int GP>
__device__ __forceinline__ void merge_segment_gp(const kllm_decode_args &a, const Seg &sg,
					      long long seg_x0, long long T, long long W,
					      float unbias, int lane)
{
	constexpr int LPH = 32 / GP;            // lanes per head
	constexpr int NL = D / LPH;             // dims per lane
	constexpr int KB = NL >= 32 ? 1 : 32 / NL;  // pieces in flight in pass 2
	const long long w0 = owner_warp(seg_x0, T, W);
	const int np = (int)(owner_warp(seg_x0 + sg.ts - 1, T, W) - w0 + 1);
	const int hh = lane / LPH, part = lane % LPH;
	const bool active = hh < a.group;
	auto slot_of = [&](int r) -> const float * {
		const long long wr = w0 + r;
		const int which = (r == 0 && wr * T / W != seg_x0) ? 1 : 0;
		return a.ws_part + ((size_t)wr * 2 + which) * KLLM_SLOT_FLOATS;
	};

	// ---- pass 1: the head's maximum (log2 domain) over pieces with mass ----
	float M = -CUDART_INF_F;
	for (int r0 = 0; r0 < np; r0 += 4 * LPH) {
		float mr[4], lr[4];
#pragma unroll
		for (int u = 0; u < 4; ++u) {
			const int r = r0 + part + u * LPH;
			mr[u] = -CUDART_INF_F;
			lr[u] = 0.f;
			if (active && r < np) {
				const float *sl = slot_of(r);
				mr[u] = __ldcg(sl + kSlotM + hh);
				lr[u] = __ldcg(sl + kSlotL + hh);
			}
		}
#pragma unroll
		for (int u = 0; u < 4; ++u)
			if (lr[u] > 0.f)
				M = fmaxf(M, mr[u]);
	}
#pragma unroll
	for (int off = 1; off < LPH; off <<= 1)
		M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));

	// ---- pass 2: weighted sums of o and l against M -------------------------
	float acc[NL];
#pragma unroll
	for (int i = 0; i < NL; ++i)
		acc[i] = 0.f;
	float L = 0.f;
	for (int r0 = 0; r0 < np; r0 += KB) {
		float mr[KB], lr[KB], ov[KB][NL];
#pragma unroll
		for (int u = 0; u < KB; ++u) {
			const int r = r0 + u;
			mr[u] = 0.f;
			lr[u] = 0.f;
			if (active && r < np) {
				const float *sl = slot_of(r);
				mr[u] = __ldcg(sl + kSlotM + hh);
				lr[u] = __ldcg(sl + kSlotL + hh);
				// slots are 4,160-byte strided from a 256-byte aligned base
				ldcg_vec<NL>(ov[u], sl + kSlotO + hh * D + part * NL);
			} else {
#pragma unroll
				for (int i = 0; i < NL; ++i)
					ov[u][i] = 0.f;
			}
		}
#pragma unroll
		for (int u = 0; u < KB; ++u) {
			// a piece's o is relative to its own maximum m: it weighs exp2(m - M)
			const float e = lr[u] > 0.f ? exp2f(mr[u] - M) : 0.f;
			L = fmaf(lr[u], e, L);
#pragma unroll
			for (int i = 0; i < NL; ++i)
				acc[i] = fmaf(ov[u][i], e, acc[i]);
		}
	}
	if (!active)
		return;
	const size_t row = (size_t)sg.s * a.num_heads + (size_t)sg.h * a.group + hh;
	const float inv = L > 0.f ? unbias / L : 0.f;
	if (a.pm) {
		float *po = a.po + row * D + part * NL;
		if constexpr (NL % 4 == 0) {
#pragma unroll
			for (int i = 0; i < NL; i += 4)
				*reinterpret_cast<float4 *>(po + i) = make_float4(
				    acc[i] * inv, acc[i + 1] * inv, acc[i + 2] * inv,
				    acc[i + 3] * inv);
		} else {
			*reinterpret_cast<float2 *>(po) = make_float2(acc[0] * inv, acc[1] * inv);
		}
		if (part == 0) {
			a.pm[row] = L > 0.f ? M * 0.69314718055994531f : -CUDART_INF_F;
			a.pl[row] = L;
		}
	} else {
		uint8_t *po = reinterpret_cast<uint8_t *>(a.out) + (row * D + part * NL) * 2;
		if constexpr (NL % 8 == 0) {
#pragma unroll
			for (int i = 0; i < NL; i += 8)
				*reinterpret_cast<uint4 *>(po + i * 2) = make_uint4(
				    pack_bf16x2(acc[i] * inv, acc[i + 1] * inv),
				    pack_bf16x2(acc[i + 2] * inv, acc[i + 3] * inv),
				    pack_bf16x2(acc[i + 4] * inv, acc[i + 5] * inv),
				    pack_bf16x2(acc[i + 6] * inv, acc[i + 7] * inv));
		} else if constexpr (NL == 4) {
			*reinterpret_cast<uint2 *>(po) = make_uint2(
			    pack_bf16x2(acc[0] * inv, acc[1] * inv),
			    pack_bf16x2(acc[2] * inv, acc[3] * inv));
		} else {
			*reinterpret_cast<uint32_t *>(po) = pack_bf16x2(acc[0] * inv, acc[1] * inv);
		}
	}
}

template <int D>
__device__ __forceinline__ void merge_segment(const kllm_decode_args &a, const Seg &sg,
					      long long seg_x0, long long T, long long W,
					      float unbias, int lane)
{
	if (a.group > 4)
		merge_segment_gp<D, 8>(a, sg, seg_x0, T, W, unbias, lane);
	else if (a.group > 2)
		merge_segment_gp<D, 4>(a, sg, seg_x0, T, W, unbias, lane);
	else if (a.group > 1)
		merge_segment_gp<D, 2>(a, sg, seg_x0, T, W, unbias, lane);
	else
		merge_segment_gp<D, 1>(a, sg, seg_x0, T, W, unbias, lane);
}

// Queues segment (s, h) for the wide merge: its partials merged by a whole
// CTA (exact = 0), or the segment recomputed there from its pages with the
// reference's E4M3 decoding (exact = 1: a piece came out of the tile loop
// non-finite). False when the queue is full.
__device__ __forceinline__ bool queue_segment(const kllm_decode_args &a, int s, int h, int ts,
					      long long seg_x0, long long T, long long W,
					      int exact, int lane)
{
	ListHeader *lh = static_cast<ListHeader *>(a.ws_list);
	ListItem *li = reinterpret_cast<ListItem *>(lh + 1);
	unsigned idx = 0;
	if (lane == 0) {
		idx = atomicAdd(&lh->count, 1u);
		if (idx < KLLM_MERGE_LIST_CAP) {
			li[idx].s = s;
			li[idx].h = h;
			li[idx].ts = ts;
			li[idx].pad = exact;
			li[idx].seg_x0 = seg_x0;
			if (!exact) {
				lh->T = T;
				lh->W = W;
			}
		}
	}
	return __shfl_sync(0xffffffffu, idx, 0) < KLLM_MERGE_LIST_CAP;
}

template <int D, int KVT>
__global__ void __launch_bounds__(kWarps * 32, Geom<D, KVT>::MIN_CTAS)
decode_kernel(const kllm_decode_args a)
{
	using Gm = Geom<D, KVT>;
	extern __shared__ __align__(128) uint8_t smem[];
	const int S = a.num_seqs, H = a.num_kv_heads;
	const SmemLayout lay(Gm::STAGE, Gm::NST, S);
	uint64_t *bars = reinterpret_cast<uint64_t *>(smem + lay.bar);
	int *meta = reinterpret_cast<int *>(smem + lay.meta);
	uint32_t *lut = reinterpret_cast<uint32_t *>(smem + lay.lut);
	int *prefix = reinterpret_cast<int *>(smem + lay.prefix);
	int *slen = reinterpret_cast<int *>(smem + lay.slen);

	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	const int tpp = a.block_size / kTile;

	// ---- per-CTA setup: scale LUT, clamped lengths, tile prefix sums -------
	if constexpr (Gm::MX)
		for (int i = tid; i < 256; i += blockDim.x)
			lut[i] = mx_scale_lut_entry_f16((uint32_t)i);
	bool clamped = false;  // reported after the grid dependency wait
	{
		bool too_long = false;
		const int cap = a.max_blocks * a.block_size;
		for (int s = tid; s < S; s += blockDim.x) {
			int L = a.seq_lens[s];
			L = L < 0 ? 0 : L;
			if (L > cap) {
				L = cap;
				too_long = true;
			}
			slen[s] = L;
		}
		if (too_long && blockIdx.x == 0)
			clamped = true;
	}
	if (lane == 0)
		for (int i = 0; i < Gm::NST; ++i)
			mbar_init(&bars[warp * Gm::NST + i], 1);
	__syncthreads();
	if (warp == 0) {
		int run = 0;
		for (int base = 0; base < S; base += 32) {
			const int s = base + lane;
			const int t = s < S ? (slen[s] + kTile - 1) / kTile : 0;
			int v = t;
#pragma unroll
			for (int off = 1; off < 32; off <<= 1) {
				const int n = __shfl_up_sync(0xffffffffu, v, off);
				if (lane >= off)
					v += n;
			}
			if (s < S)
				prefix[s] = run + v - t;
			run += __shfl_sync(0xffffffffu, v, 31);
		}
		if (lane == 0)
			prefix[S] = run;
	}
	if (lane == 0)
		fence_mbar_init();
	__syncthreads();

	const long long T = (long long)prefix[S] * H;
	const int w = blockIdx.x * kWarps + warp;

	if (T == 0) {
		grid_dependency_wait();
		if (clamped && a.err)
			atomicOr(a.err, KLLM_ERR_SEQ_TOO_LONG_BIT);
		for (int s = w; s < S; s += a.total_warps)
			write_empty_seq<D>(a, s, lane);
		return;
	}

	const long long W = a.split ? (T < a.total_warps ? T : a.total_warps)
				    : a.total_warps;
	if (w >= W) {
		grid_dependency_wait();
		if (clamped && a.err)
			atomicOr(a.err, KLLM_ERR_SEQ_TOO_LONG_BIT);
		for (int s = w; s < S; s += a.total_warps)
			if (prefix[s + 1] == prefix[s])
				write_empty_seq<D>(a, s, lane);
		return;
	}
	long long xa, xb;
	if (a.split) {
		xa = (long long)w * T / W;
		xb = (long long)(w + 1) * T / W;
	} else {
		xa = seg_start_at_or_after(prefix, S, H, T, (long long)w * T / W);
		xb = seg_start_at_or_after(prefix, S, H, T, (long long)(w + 1) * T / W);
	}
	if (xa >= xb) {
		grid_dependency_wait();
		if (clamped && a.err)
			atomicOr(a.err, KLLM_ERR_SEQ_TOO_LONG_BIT);
		for (int s = w; s < S; s += a.total_warps)
			if (prefix[s + 1] == prefix[s])
				write_empty_seq<D>(a, s, lane);
		return;
	}
	const int n = (int)(xb - xa);

	uint8_t *wst = smem + lay.stage + (size_t)warp * Gm::NST * Gm::STAGE;
	uint64_t *wbar = bars + warp * Gm::NST;
	int *wmeta = meta + warp * Gm::NST;
	const uint64_t policy = l2_evict_first_policy();
	const size_t sec = Gm::MX ? (size_t)a.block_size * D * 9 / 8
				  : (size_t)a.block_size * D * 2;
	const float unbias = Gm::MX ? KLLM_MX_DEC_UNBIAS : 1.f;

	// ---- producer: block-table batches and the bulk-copy ring --------------
	Batch cur, nxt;
	load_batch(cur, a, prefix, slen, xa, n, 0, lane, tpp);
	load_batch(nxt, a, prefix, slen, xa, n, 32, lane, tpp);

	// Everything above reads only seq_lens and the block table (and writes
	// shared memory). Launched as a programmatic dependent (overlap), this
	// CTA got here while the previous kernel on the stream was finishing;
	// the query, the pages and every output are touched only after it has
	// completed. The decode itself never signals its dependents early: the
	// next kernel's CTAs, parked on the SMs its warps leave, slowed the
	// decode's last warps (measured), so the wide merge launches when the
	// decode completes, and signals the next decode at once.
	grid_dependency_wait();
	if (clamped && a.err)
		atomicOr(a.err, KLLM_ERR_SEQ_TOO_LONG_BIT);
	for (int s = w; s < S; s += a.total_warps)
		if (prefix[s + 1] == prefix[s])
			write_empty_seq<D>(a, s, lane);

	finalize_batch(cur, a, sec);
	int pb = 0;

	auto issue = [&](int pos) {
		int bi = pos - pb;
		if (bi >= 32) {
			cur = nxt;
			finalize_batch(cur, a, sec);
			pb += 32;
			bi -= 32;
			load_batch(nxt, a, prefix, slen, xa, n, pb + 32, lane, tpp);
		}
		const unsigned long long ek = __shfl_sync(0xffffffffu, cur.k, bi);
		const unsigned long long ev = __shfl_sync(0xffffffffu, cur.v, bi);
		const int pack = __shfl_sync(0xffffffffu, cur.pack, bi);
		if (lane == 0) {
			const int st = pos % Gm::NST;
			const int ntok = pack & 0xFF, sub = pack >> 8;
			wmeta[st] = ntok;
			uint64_t *bar = &wbar[st];
			if (ntok) {
				mbar_arrive_expect_tx(bar, Gm::STAGE);
				uint8_t *dK = wst + (size_t)st * Gm::STAGE;
				uint8_t *dV = dK + Gm::KV;
				const uint8_t *sK = reinterpret_cast<const uint8_t *>(ek);
				const uint8_t *sV = reinterpret_cast<const uint8_t *>(ev);
				if (Gm::MX && tpp == 1) {  // payload + scales contiguous
					bulk_g2s_stream(dK, sK, Gm::KV, bar, policy);
					bulk_g2s_stream(dV, sV, Gm::KV, bar, policy);
				} else {
					bulk_g2s_stream(dK, sK + (size_t)sub * Gm::PAY, Gm::PAY, bar, policy);
					bulk_g2s_stream(dV, sV + (size_t)sub * Gm::PAY, Gm::PAY, bar, policy);
					if (Gm::MX) {
						const size_t so = (size_t)a.block_size * D + (size_t)sub * Gm::SCL;
						bulk_g2s_stream(dK + Gm::PAY, sK + so, Gm::SCL, bar, policy);
						bulk_g2s_stream(dV + Gm::PAY, sV + so, Gm::SCL, bar, policy);
					}
				}
			} else {
				mbar_arrive(bar);
			}
		}
	};

	int p = 0;
	for (; p < n && p < Gm::NST - 1; ++p)
		issue(p);

	// ---- consumer ------------------------------------------------------------
	Seg cc = locate(prefix, S, H, xa);
	long long piece_x0 = xa;
	int piece_j0 = cc.j;
	uint32_t q[D / 8];
	load_q<D>(q, a, cc.s, cc.h, lane);
	float sl2 = a.scale_log2;
	if constexpr (Gm::MX)
		sl2 = a.scale_log2 * q_to_f16<D>(q);
	float o[D / 16][4];
#pragma unroll
	for (int mt = 0; mt < D / 16; ++mt)
		o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
	float m0 = -CUDART_INF_F, m1 = -CUDART_INF_F, l0 = 0.f, l1 = 0.f;
	float mx0 = -CUDART_INF_F, mx1 = -CUDART_INF_F;
	const int g = lane >> 2, c = lane & 3;

	for (int i = 0; i < n; ++i) {
		if (p < n) {
			issue(p);
			++p;
		}
		const int st = i % Gm::NST;
		if (!mbar_wait(&wbar[st], (uint32_t)((i / Gm::NST) & 1))) {
			if (lane == 0 && a.err)
				atomicOr(a.err, KLLM_ERR_TIMEOUT_BIT);
			return;
		}
		const int ntok = *reinterpret_cast<volatile int *>(&wmeta[st]);
		if (ntok > 0) {
			const uint8_t *sK = wst + (size_t)st * Gm::STAGE;
			tile_compute<D, KVT>(sK, sK + Gm::KV, lut, ntok, q, o, m0,
					     m1, l0, l1, mx0, mx1, sl2, lane);
		}
		__syncwarp();

		const bool seg_end = cc.j + 1 == cc.ts;
		const bool last = i + 1 == n;
		if (!(seg_end || last)) {
			++cc.j;
			continue;
		}

		// ---- piece finished: normalise, or publish a partial -------------
		// Re-reference l and O from the lazy maximum to the exact one.
#pragma unroll
		for (int off = 4; off < 32; off <<= 1) {
			mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
			mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
		}
		{
			const float f0 = mx0 > m0 ? exp2f(m0 - mx0) : 1.f;
			const float f1 = mx1 > m1 ? exp2f(m1 - mx1) : 1.f;
			if (mx0 > m0) m0 = mx0;
			if (mx1 > m1) m1 = mx1;
			l0 *= f0;
			l1 *= f1;
#pragma unroll
			for (int mt = 0; mt < D / 16; ++mt) {
				o[mt][0] *= f0;
				o[mt][1] *= f1;
				o[mt][2] *= f0;
				o[mt][3] *= f1;
			}
		}
		float L0 = l0, L1 = l1;
#pragma unroll
		for (int off = 4; off < 32; off <<= 1) {
			L0 += __shfl_xor_sync(0xffffffffu, L0, off);
			L1 += __shfl_xor_sync(0xffffffffu, L1, off);
		}
		const bool full = piece_j0 == 0 && seg_end;
		const size_t row0 = (size_t)cc.s * a.num_heads + (size_t)cc.h * a.group;
		// MX: a non-finite piece means payload codes 0x7F / 0xFF (the
		// hardware conversion's NaN, the reference's +-480); its segment is
		// recomputed exactly by the wide-merge kernel, which runs after this
		// one and overwrites what this one wrote for it
		bool redo = false;
		if constexpr (Gm::MX) {
			bool bad = !isfinite(L0) || !isfinite(L1);
#pragma unroll
			for (int mt = 0; mt < D / 16; ++mt)
				bad |= !isfinite(o[mt][0] + o[mt][1] + o[mt][2] + o[mt][3]);
			redo = __any_sync(0xffffffffu, bad);
		}
		if (full) {
#pragma unroll
			for (int hp = 0; hp < 2; ++hp) {
				const int hh = 2 * c + hp;
				if (hh < a.group) {
					float vals[D / 8];
#pragma unroll
					for (int mt = 0; mt < D / 16; ++mt) {
						vals[2 * mt] = o[mt][hp];
						vals[2 * mt + 1] = o[mt][2 + hp];
					}
					store_head_row<D>(a, row0 + hh, g, vals,
							  hp ? m1 : m0, hp ? L1 : L0, unbias);
				}
			}
			if (redo && !(a.ws_list && queue_segment(a, cc.s, cc.h, cc.ts, 0, T, W, 1,
								  lane)) && lane == 0 && a.err)
				atomicOr(a.err, KLLM_ERR_NONFINITE_BIT);
		} else {
			const int which = piece_x0 == xa ? 0 : 1;
			float *slot = a.ws_part + ((size_t)w * 2 + which) * KLLM_SLOT_FLOATS;
#pragma unroll
			for (int hp = 0; hp < 2; ++hp) {
				const int hh = 2 * c + hp;
				if (hh < a.group) {
					float *dst = slot + kSlotO + hh * D + g * (D / 8);
#pragma unroll
					for (int mt = 0; mt < D / 16; mt += 2)
						*reinterpret_cast<float4 *>(dst + 2 * mt) =
						    make_float4(o[mt][hp], o[mt][2 + hp],
								o[mt + 1][hp], o[mt + 1][2 + hp]);
					if (g == 0) {
						slot[kSlotM + hh] = hp ? m1 : m0;
						slot[kSlotL + hh] = hp ? L1 : L0;
					}
				}
			}
			__threadfence();
			__syncwarp();
			const long long seg_x0 = piece_x0 - piece_j0;
			const long long npieces = owner_warp(seg_x0 + cc.ts - 1, T, W) -
						  owner_warp(seg_x0, T, W) + 1;
			// a segment of few pieces is merged in this kernel; one of many is
			// queued by its last piece, and the wide merge checks its result
			if (redo && npieces <= KLLM_FUSED_MERGE_MAX &&
			    !(a.ws_list && queue_segment(a, cc.s, cc.h, cc.ts, seg_x0, T, W, 1, lane)) &&
			    lane == 0 && a.err)
				atomicOr(a.err, KLLM_ERR_NONFINITE_BIT);
			unsigned old = 0;
			unsigned *cnt = a.ws_cnt + (size_t)cc.s * H + cc.h;
			if (lane == 0)
				old = atomicAdd(cnt, 1u);
			old = __shfl_sync(0xffffffffu, old, 0);
			if ((long long)old == npieces - 1) {
				__threadfence();
				bool fused = npieces <= KLLM_FUSED_MERGE_MAX || !a.ws_list;
				if (!fused)    // long segment: queue it for the wide merge
					fused = !queue_segment(a, cc.s, cc.h, cc.ts, seg_x0, T, W, 0, lane);
				if (fused)
					merge_segment<D>(a, cc, seg_x0, T, W, unbias, lane);
				if (lane == 0)
					*cnt = 0u;  // ready for the next launch
			}
		}

		if (last)
			break;
		// next segment
		cc.j = 0;
		if (++cc.h == H) {
			cc.h = 0;
			do {
				++cc.s;
			} while (prefix[cc.s + 1] == prefix[cc.s]);
			cc.ts = prefix[cc.s + 1] - prefix[cc.s];
		}
		piece_j0 = 0;
		piece_x0 = xa + i + 1;
		load_q<D>(q, a, cc.s, cc.h, lane);
		if constexpr (Gm::MX)
			sl2 = a.scale_log2 * q_to_f16<D>(q);
#pragma unroll
		for (int mt = 0; mt < D / 16; ++mt)
			o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
		m0 = m1 = -CUDART_INF_F;
		mx0 = mx1 = -CUDART_INF_F;
		l0 = l1 = 0.f;
	}
}

// Exact recompute of one (segment, query head) of an MX-FP8 decode by a CTA
// of 8 warps, for segments whose tile-loop result was not finite: payload
// codes 0x7F / 0xFF, which the hardware E4M3 conversion reads as NaN and the
// reference decodes as +-480 (userspace/compute/mx_dequant.h:30-55). No
// writer of either code base emits them, but pages that arrive from a store
// are raw bytes. Warp w takes tiles w, w+8, ... of the segment, reads them
// with plain loads and decodes every value exactly in fp32 (payload x
// scale), lane -> D/32 dims; the warps' (m, l, o) are merged in shared
// memory and the row is written over what the decode wrote for it.
template <int D>
__device__ void exact_pair(const kllm_decode_args &a, int s, int h, int hh, int ts,
			   float (*sm_o)[D], float *sm_m, float *sm_l)
{
	constexpr int NV = D / 32;
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int tpp = a.block_size / kTile;
	const size_t sec = (size_t)a.block_size * D * 9 / 8;
	// the decode's scale carries the 2^2 that undoes its V / 4
	const float sl2 = a.scale_log2 * (1.f / KLLM_MX_DEC_UNBIAS);
	const int cap = a.max_blocks * a.block_size;
	int L = a.seq_lens[s];
	L = L < 0 ? 0 : (L > cap ? cap : L);
	const size_t row = (size_t)s * a.num_heads + (size_t)h * a.group + hh;
	const uint16_t *qp = reinterpret_cast<const uint16_t *>(a.q) + row * D + lane * NV;
	float q[NV], o[NV];
#pragma unroll
	for (int i = 0; i < NV; ++i) {
		q[i] = __uint_as_float((uint32_t)qp[i] << 16);
		o[i] = 0.f;
	}
	float m = -CUDART_INF_F, l = 0.f;
	for (int j = warp; j < ts; j += 8) {
		const int page = j / tpp, sub = j - page * tpp;
		const DevEntry *e = reinterpret_cast<const DevEntry *>(a.table) +
				    (size_t)s * a.max_blocks + page;
		const unsigned long long kp = e->k, vp = e->v;
		if (!e->valid || !kp || ((kp | vp) & 15ull))
			continue;   // skipped by the decode as well
		const int ntok = min(L - j * kTile, kTile);
		const uint8_t *kb = reinterpret_cast<const uint8_t *>(kp) + a.layer_off + (size_t)h * sec;
		const uint8_t *vb = reinterpret_cast<const uint8_t *>(vp) + a.layer_off + (size_t)h * sec;
		for (int t = 0; t < ntok; ++t) {
			const size_t r = (size_t)sub * kTile + t;
			const size_t so = (size_t)a.block_size * D + r * (D / 8) + lane * NV / 8;
			const float ksc = e4m3_ref_to_f32(kb[so]), vsc = e4m3_ref_to_f32(vb[so]);
			float dot = 0.f;
#pragma unroll
			for (int i = 0; i < NV; ++i)
				dot = fmaf(q[i], e4m3_ref_to_f32(kb[r * D + lane * NV + i]) * ksc, dot);
#pragma unroll
			for (int off = 16; off > 0; off >>= 1)
				dot += __shfl_xor_sync(0xffffffffu, dot, off);
			const float x = dot * sl2;
			const float mn = fmaxf(m, x);
			const float f = exp2f(m - mn), pw = exp2f(x - mn);
			l = fmaf(l, f, pw);
#pragma unroll
			for (int i = 0; i < NV; ++i)
				o[i] = fmaf(o[i], f, pw * e4m3_ref_to_f32(vb[r * D + lane * NV + i]) * vsc);
			m = mn;
		}
	}
	if (lane == 0) {
		sm_m[warp] = m;
		sm_l[warp] = l;
	}
#pragma unroll
	for (int i = 0; i < NV; ++i)
		sm_o[warp][lane * NV + i] = o[i];
	__syncthreads();
	if (threadIdx.x < D) {
		const int d = threadIdx.x;
		float M = -CUDART_INF_F;
#pragma unroll
		for (int w = 0; w < 8; ++w)
			if (sm_l[w] > 0.f)
				M = fmaxf(M, sm_m[w]);
		float Lt = 0.f, od = 0.f;
#pragma unroll
		for (int w = 0; w < 8; ++w) {
			const float ew = sm_l[w] > 0.f ? exp2f(sm_m[w] - M) : 0.f;
			Lt = fmaf(sm_l[w], ew, Lt);
			od = fmaf(sm_o[w][d], ew, od);
		}
		const float inv = Lt > 0.f ? 1.f / Lt : 0.f;
		if (a.pm) {
			a.po[row * D + d] = od * inv;
			if (d == 0) {
				a.pm[row] = Lt > 0.f ? M * 0.69314718055994531f : -CUDART_INF_F;
				a.pl[row] = Lt;
			}
		} else {
			reinterpret_cast<__nv_bfloat16 *>(a.out)[row * D + d] = __float2bfloat16_rn(od * inv);
		}
	}
	__syncthreads();
}

// Wide merge of the queued long segments: one CTA of 8 warps per
// (segment, query head). Pass 1: the segment's maximum over all its pieces
// (independent loads by all threads, block reduction). Pass 2: warp w sums
// pieces w, w+8, ... in that order (o and l, each piece relative to its own
// maximum m, weighted by exp2(m - maximum)) eight pieces in flight, so
// the loads do not wait on one another; the warps' sums are added in shared
// memory. The last CTA to finish clears the list header for the next launch.
template <int D>
__global__ void __launch_bounds__(256)
merge_big_kernel(const kllm_decode_args a, float unbias)
{
	__shared__ float sm_red[8];
	__shared__ float sm_l[8];
	__shared__ float sm_o[8][D];
	__shared__ int last;
	grid_dependency_wait();     // the decode that filled the queue has completed
	grid_launch_dependents();
	ListHeader *lh = static_cast<ListHeader *>(a.ws_list);
	const ListItem *li = reinterpret_cast<const ListItem *>(lh + 1);
	const unsigned count = min(*reinterpret_cast<volatile unsigned *>(&lh->count),
				   (unsigned)KLLM_MERGE_LIST_CAP);
	// Nothing queued (every segment was merged inside the decode): the
	// header is already clear, no CTA needs to count itself done.
	if (count == 0)
		return;
	const long long T = lh->T, W = lh->W;
	const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	constexpr int NV = D / 32;
	constexpr int kFly = KLLM_MERGE_FLY;   // pieces in flight per warp
	const long long pairs = (long long)count * a.group;

	for (long long pr = blockIdx.x; pr < pairs; pr += gridDim.x) {
		const ListItem it = li[pr / a.group];
		const int hh = (int)(pr % a.group);
		if (it.pad) {   // queued for an exact recompute (MX payload 0x7F / 0xFF)
			exact_pair<D>(a, it.s, it.h, hh, it.ts, sm_o, sm_red, sm_l);
			continue;
		}
		const long long w0 = owner_warp(it.seg_x0, T, W);
		const long long np = owner_warp(it.seg_x0 + it.ts - 1, T, W) - w0 + 1;
		auto slot_of = [&](long long r) -> const float * {
			const long long wr = w0 + r;
			const int which = (r == 0 && wr * T / W != it.seg_x0) ? 1 : 0;
			return a.ws_part + ((size_t)wr * 2 + which) * KLLM_SLOT_FLOATS;
		};
		// ---- one pass: each warp folds its pieces (eight in flight) into a
		// running (max, sum, o) triple in the log2 domain, rescaled whenever
		// a batch raises its maximum; the CTA then combines the warps' triples
		float Mw = -CUDART_INF_F, L = 0.f, acc[NV];
#pragma unroll
		for (int i = 0; i < NV; ++i)
			acc[i] = 0.f;
		for (long long r0 = warp; r0 < np; r0 += 8 * kFly) {
			float lr[kFly], mr[kFly], ov[kFly][NV];
#pragma unroll
			for (int u = 0; u < kFly; ++u) {
				const long long r = r0 + 8 * u;
				lr[u] = 0.f;
				mr[u] = -CUDART_INF_F;
#pragma unroll
				for (int i = 0; i < NV; ++i)
					ov[u][i] = 0.f;
				if (r < np) {
					const float *sl = slot_of(r);
					lr[u] = __ldcg(sl + kSlotL + hh);
					mr[u] = __ldcg(sl + kSlotM + hh);
					// 16 (D = 128) or 8 (D = 64) bytes per lane, aligned:
					// slots are 4,160-byte strided from an aligned base
					const float *src = sl + kSlotO + hh * D + lane * NV;
					if constexpr (NV == 4) {
						const float4 v = __ldcg(reinterpret_cast<const float4 *>(src));
						ov[u][0] = v.x;
						ov[u][1] = v.y;
						ov[u][2] = v.z;
						ov[u][3] = v.w;
					} else {
						const float2 v = __ldcg(reinterpret_cast<const float2 *>(src));
						ov[u][0] = v.x;
						ov[u][1] = v.y;
					}
				}
			}
			// the batch's maximum over pieces with mass (the same in every
			// lane: all lanes read the same m and l of a piece)
			float mb = -CUDART_INF_F;
#pragma unroll
			for (int u = 0; u < kFly; ++u)
				if (lr[u] > 0.f)
					mb = fmaxf(mb, mr[u]);
			if (mb > Mw) {
				const float f = exp2f(Mw - mb);   // 0 while Mw is -inf
				L *= f;
#pragma unroll
				for (int i = 0; i < NV; ++i)
					acc[i] *= f;
				Mw = mb;
			}
#pragma unroll
			for (int u = 0; u < kFly; ++u) {
				// a piece's o is unnormalised (relative to its own max m): it
				// weighs exp2(m - Mw); its l weighs the same into L
				const float e = lr[u] > 0.f ? exp2f(mr[u] - Mw) : 0.f;
				L = fmaf(lr[u], e, L);
#pragma unroll
				for (int i = 0; i < NV; ++i)
					acc[i] = fmaf(ov[u][i], e, acc[i]);
			}
		}
		if (lane == 0) {
			sm_red[warp] = Mw;
			sm_l[warp] = L;
		}
#pragma unroll
		for (int i = 0; i < NV; ++i)
			sm_o[warp][lane * NV + i] = acc[i];
		__syncthreads();
		float Mt = sm_red[0];
#pragma unroll
		for (int w = 1; w < 8; ++w)
			Mt = fmaxf(Mt, sm_red[w]);
		float Lt = 0.f, o = 0.f;
		if (threadIdx.x < D) {
			const int d = threadIdx.x;
#pragma unroll
			for (int w = 0; w < 8; ++w) {
				const float f = sm_red[w] > -CUDART_INF_F ? exp2f(sm_red[w] - Mt) : 0.f;
				Lt = fmaf(sm_l[w], f, Lt);
				o = fmaf(sm_o[w][d], f, o);
			}
		}
		// MX pieces that came out of the decode non-finite (payload 0x7F /
		// 0xFF): recompute the segment exactly instead of writing them
		const bool bad = threadIdx.x < D && !(isfinite(Lt) && isfinite(o));
		if (__syncthreads_or(bad) && a.kv_dtype == 1) {   // 1: MX-FP8 pages
			exact_pair<D>(a, it.s, it.h, hh, it.ts, sm_o, sm_red, sm_l);
			continue;
		}
		if (threadIdx.x < D) {
			const int d = threadIdx.x;
			const size_t row = (size_t)it.s * a.num_heads + (size_t)it.h * a.group + hh;
			const float inv = Lt > 0.f ? unbias / Lt : 0.f;
			if (a.pm) {
				a.po[row * D + d] = o * inv;
				if (d == 0) {
					a.pm[row] = Lt > 0.f ? Mt * 0.69314718055994531f : -CUDART_INF_F;
					a.pl[row] = Lt;
				}
			} else {
				__nv_bfloat16 b = __float2bfloat16_rn(o * inv);
				reinterpret_cast<__nv_bfloat16 *>(a.out)[row * D + d] = b;
			}
		}
		__syncthreads();
	}
	if (threadIdx.x == 0) {
		__threadfence();
		last = atomicAdd(&lh->done, 1u) == gridDim.x - 1;
	}
	__syncthreads();
	if (last && threadIdx.x == 0) {
		lh->count = 0u;
		lh->done = 0u;
	}
}

// Launches `kernel`, as a programmatic dependent of the previous kernel on
// the stream when `dependent` is set (it may then start while that kernel
// finishes; its griddepcontrol.wait orders everything after it).
template <typename... KArgs, typename... Args>
cudaError_t launch_maybe_dependent(void (*kernel)(KArgs...), int grid, int block,
				   size_t smem, cudaStream_t st, int dependent,
				   Args... args)
{
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3((unsigned)grid);
	cfg.blockDim = dim3((unsigned)block);
	cfg.dynamicSmemBytes = smem;
	cfg.stream = st;
	cudaLaunchAttribute at[1];
	at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	at[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = at;
	cfg.numAttrs = dependent ? 1 : 0;
	return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int D, int KVT>
struct Launcher {
	static size_t smem(int S)
	{
		using Gm = Geom<D, KVT>;
		return SmemLayout(Gm::STAGE, Gm::NST, S).total;
	}
	static cudaError_t prepare(int S)
	{
		return cudaFuncSetAttribute(decode_kernel<D, KVT>,
					    cudaFuncAttributeMaxDynamicSharedMemorySize,
					    (int)smem(S));
	}
	static int occupancy(int S)
	{
		if (prepare(S) != cudaSuccess)
			return 0;
		int n = 0;
		if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(
			&n, decode_kernel<D, KVT>, kWarps * 32, smem(S)) != cudaSuccess)
			return 0;
		return n;
	}
	static cudaError_t launch(const kllm_decode_args &a, int grid,
				  cudaStream_t st)
	{
		cudaError_t e = prepare(a.num_seqs);
		if (e != cudaSuccess)
			return e;
		return launch_maybe_dependent(decode_kernel<D, KVT>, grid, kWarps * 32,
					      smem(a.num_seqs), st, a.overlap, a);
	}
};

}  // namespace
}  // namespace kllm

using namespace kllm;

extern "C" size_t kllm_decode_smem_bytes(int head_dim, int kv_dtype, int num_seqs)
{
	if (head_dim == 128)
		return kv_dtype ? Launcher<128, 1>::smem(num_seqs) : Launcher<128, 0>::smem(num_seqs);
	if (head_dim == 64)
		return kv_dtype ? Launcher<64, 1>::smem(num_seqs) : Launcher<64, 0>::smem(num_seqs);
	return 0;
}

extern "C" int kllm_decode_ctas_per_sm(int head_dim, int kv_dtype, int num_seqs)
{
	if (head_dim == 128)
		return kv_dtype ? Launcher<128, 1>::occupancy(num_seqs)
				: Launcher<128, 0>::occupancy(num_seqs);
	if (head_dim == 64)
		return kv_dtype ? Launcher<64, 1>::occupancy(num_seqs)
				: Launcher<64, 0>::occupancy(num_seqs);
	return 0;
}

extern "C" int kllm_decode_preload(void)
{
	// Querying a kernel's attributes makes the runtime load it now (CUDA
	// loads modules lazily by default), so later launches need no memory
	// for code.
	cudaFuncAttributes fa;
	cudaError_t e = cudaSuccess;
	if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, decode_kernel<128, 0>);
	if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, decode_kernel<128, 1>);
	if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, decode_kernel<64, 0>);
	if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, decode_kernel<64, 1>);
	if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, merge_big_kernel<128>);
	if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, merge_big_kernel<64>);
	return (int)e;
}

extern "C" int kllm_decode_merge_launch(const struct kllm_decode_args *a,
					int num_sms, void *stream)
{
	if (!a->ws_list)
		return 0;
	cudaStream_t st = static_cast<cudaStream_t>(stream);
	const float unbias = a->kv_dtype ? KLLM_MX_DEC_UNBIAS : 1.f;
	// CTAs take (segment, query head) pairs grid-stride; two per SM cover the
	// queue of a decode split over many warps in one wave, and an empty queue
	// costs only the launch
	const int grid = 2 * (num_sms > 0 ? num_sms : 148);
	if (a->head_dim == 128)
		return (int)launch_maybe_dependent(merge_big_kernel<128>, grid, 256, 0, st,
						   a->overlap, *a, unbias);
	if (a->head_dim == 64)
		return (int)launch_maybe_dependent(merge_big_kernel<64>, grid, 256, 0, st,
						   a->overlap, *a, unbias);
	return (int)cudaErrorInvalidValue;
}

extern "C" int kllm_decode_launch(const struct kllm_decode_args *a, int grid,
				  void *stream)
{
	cudaStream_t st = static_cast<cudaStream_t>(stream);
	cudaError_t e;
	if (a->head_dim == 128)
		e = a->kv_dtype ? Launcher<128, 1>::launch(*a, grid, st)
				: Launcher<128, 0>::launch(*a, grid, st);
	else if (a->head_dim == 64)
		e = a->kv_dtype ? Launcher<64, 1>::launch(*a, grid, st)
				: Launcher<64, 0>::launch(*a, grid, st);
	else
		e = cudaErrorInvalidValue;
	return (int)e;
}
