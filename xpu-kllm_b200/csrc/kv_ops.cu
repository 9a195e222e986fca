// SPDX-License-Identifier: Apache-2.0
//
// kv_ops.cu - the paged-cache side of the hot path on sm_100a:
//   * KV append with quantize-on-write (MX-FP8, the reference's BF16-payload
//     MX layout, or plain BF16);
//   * the bit-exact gather used by tests to read the cache back;
//   * the log-sum-exp merge of split-KV partial triples (cross-GPU split).

#include "kllm_device.cuh"
#include "kllm_internal.h"

#include <math_constants.h>

namespace kllm {
namespace {

struct DevEntry {  // userspace/gpu/paged_attention.cu:18-22
	unsigned long long k, v;
	int valid;
	int pad;
};

__device__ __forceinline__ size_t section_bytes(int kv_dtype, int bs, int d)
{
	if (kv_dtype == 1)
		return (size_t)bs * d + (size_t)bs * (d / 8);
	if (kv_dtype == 2)
		return (size_t)bs * d * 2 + (size_t)bs * (d / 8);
	return (size_t)bs * d * 2;
}

// Two floats -> two E4M3 codes, round to nearest even, saturate to +-448.
// Returns lo in byte 0 and hi in byte 1.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi)
{
	uint16_t r;
	asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
	return r;
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Micro-block b (8 elements) of kv head h of row i of K (kv == 0) or V.
__device__ __forceinline__ uint4 append_load(const kllm_append_args &a, int i, int h, int kv,
					     int b)
{
	return *reinterpret_cast<const uint4 *>(
	    reinterpret_cast<const uint8_t *>(kv ? a.v : a.k) +
	    (((size_t)i * a.num_kv_heads + h) * a.head_dim + (size_t)b * 8) * 2);
}

// Tables for the MX quantizer, built at compile time: v[c] = value of E4M3
// code c (the reference decoder's values), v[256 + c] = its reciprocal
// rounded to nearest (compile-time float division is correctly rounded).
struct E4m3Tables {
	float v[512];
};

constexpr float e4m3_value_host(int code)
{
	const int e = (code >> 3) & 0xF, m = code & 7;
	float scale = 1.0f;   // 2^(e - 10) for e > 0, 2^-9 for e == 0
	const int ex = e ? e - 10 : -9;
	for (int i = 0; i < (ex < 0 ? -ex : ex); ++i)
		scale = ex < 0 ? scale * 0.5f : scale * 2.0f;
	const float v = e ? (float)(8 + m) * scale : (float)m * scale;
	return (code & 0x80) ? -v : v;
}

constexpr E4m3Tables make_e4m3_tables()
{
	E4m3Tables t{};
	for (int i = 0; i < 256; ++i) {
		t.v[i] = e4m3_value_host(i);
		t.v[256 + i] = t.v[i] != 0.0f ? 1.0f / t.v[i] : 0.0f;
	}
	return t;
}

__device__ const E4m3Tables g_e4m3 = make_e4m3_tables();

// The same values as {value, reciprocal} pairs, one 8-byte load per code.
struct E4m3Pairs {
	float2 p[256];
};

constexpr E4m3Pairs make_e4m3_pairs()
{
	E4m3Pairs t{};
	for (int i = 0; i < 256; ++i) {
		const float v = e4m3_value_host(i);
		t.p[i] = float2{v, v != 0.0f ? 1.0f / v : 0.0f};
	}
	return t;
}

__device__ const E4m3Pairs g_e4m3_pairs = make_e4m3_pairs();

// Scale rows by the bits of a block's bf16 abs-max. Row i stands for amax =
// bf16 bits kScaleRowLo + i (0.875 .. 200704): the smallest E4M3 code whose
// value v satisfies 448 v >= amax (mx_dequant.h:119-120's scale, rounded up
// to an E4M3 value), with v and -RN(1 / v). Every amax below 0.875 takes
// code 1 (2^-9) and every one above 200704 saturates at 0x7E (448), so a
// clamped index covers each positive finite amax.
constexpr int kScaleRowLo = 0x3F60, kScaleRowHi = 0x4844;
constexpr int kScaleRows = kScaleRowHi - kScaleRowLo + 1;

struct ScaleRow {
	float s, neg_y;
	uint32_t code, pad;
};
struct ScaleRows {
	ScaleRow r[kScaleRows];
};

constexpr double bf16_value_host(int bits)
{
	const int e = (bits >> 7) & 0xFF, m = bits & 0x7F;
	double v = e ? 128 + m : m;
	const int ex = e ? e - 134 : -133;
	for (int i = 0; i < (ex < 0 ? -ex : ex); ++i)
		v = ex < 0 ? v * 0.5 : v * 2.0;
	return v;
}

constexpr ScaleRows make_scale_rows()
{
	ScaleRows t{};
	int c = 1;
	for (int i = 0; i < kScaleRows; ++i) {
		const double amax = bf16_value_host(kScaleRowLo + i);
		while (448.0 * (double)e4m3_value_host(c) < amax)   // both exact in double
			++c;
		const float v = e4m3_value_host(c);
		t.r[i] = ScaleRow{v, -(1.0f / v), (uint32_t)c, 0u};
	}
	return t;
}

__device__ const ScaleRows g_scale_rows = make_scale_rows();

// Packed fp32 pairs (sm_100 f32x2 arithmetic: per lane the same IEEE
// round-to-nearest operation as the scalar instruction).
__device__ __forceinline__ unsigned long long f2_from_bf16x2(uint32_t w)
{
	unsigned long long r;
	asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(w << 16), "r"(w & 0xFFFF0000u));
	return r;
}

__device__ __forceinline__ unsigned long long f2_splat(float x)
{
	unsigned long long r;
	asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(x));
	return r;
}

__device__ __forceinline__ unsigned long long f2_mul(unsigned long long a, unsigned long long b)
{
	unsigned long long r;
	asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
	return r;
}

__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
						     unsigned long long c)
{
	unsigned long long r;
	asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
	return r;
}

// Two bf16 f (one word) over the E4M3 value s, with ny = -RN(1 / s): the
// exact quotient of append_store (reciprocal + one residual step), two lanes
// at a time, computed negated so that a zero keeps its sign: m = -RN(f y),
// r = RN(f + s m) (the residual), w = RN(m - r y) = -q. Encoded as the two
// E4M3 codes of q (byte 0: the low element), the sign bits flipped back.
__device__ __forceinline__ uint32_t quot_e4m3x2(uint32_t w, unsigned long long s,
						unsigned long long ny)
{
	const unsigned long long f = f2_from_bf16x2(w);
	const unsigned long long m = f2_mul(f, ny);
	const unsigned long long nq = f2_fma(f2_fma(s, m, f), ny, m);
	float lo, hi;
	asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(nq));
	return cvt_e4m3x2(lo, hi) ^ 0x8080u;
}

// max |x| of eight bf16 values as a float, NaN when any of them is NaN.
__device__ __forceinline__ float bf16x8_absmax_nan(uint4 x)
{
	uint32_t m01, m23, m;
	asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(m01) : "r"(x.x & 0x7FFF7FFFu), "r"(x.y & 0x7FFF7FFFu));
	asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(m23) : "r"(x.z & 0x7FFF7FFFu), "r"(x.w & 0x7FFF7FFFu));
	asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(m) : "r"(m01), "r"(m23));
	float r;
	asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(__uint_as_float(m << 16)),
	    "f"(__uint_as_float(m & 0xFFFF0000u)));
	return r;
}

// Scale row of a positive finite abs-max (a bf16 value).
__device__ __forceinline__ uint4 scale_row(float amax)
{
	int idx = (int)(__float_as_uint(amax) >> 16) - kScaleRowLo;
	idx = min(max(idx, 0), kScaleRows - 1);
	return __ldg(reinterpret_cast<const uint4 *>(&g_scale_rows.r[idx]));
}

// A micro-block with an infinite or NaN element, quantized as the oracle's
// restatement of the format does it: NaN elements are left out of the
// abs-max; an infinite abs-max saturates the scale code at 0x7E (448); a
// NaN element encodes as S.1111.111 and an infinite one as S.1111.110
// (+-448), S its sign; a block whose abs-max is 0 is all zero. Returns the
// scale code; lo / hi get the payload bytes (byte 0: element 0).
__device__ __forceinline__ uint32_t mx_quantize_nonfinite(uint4 x, uint32_t &lo, uint32_t &hi)
{
	const uint32_t w[4] = {x.x, x.y, x.z, x.w};
	float amax = 0.f;
#pragma unroll
	for (int k = 0; k < 8; ++k) {
		const float a = fabsf(k & 1 ? bf16hi(w[k >> 1]) : bf16lo(w[k >> 1]));
		if (a > amax)   // false for NaN
			amax = a;
	}
	lo = hi = 0u;
	if (!(amax > 0.f))
		return 0u;
	float sv, ny;
	uint32_t code;
	if (amax <= 3.40282347e38f) {
		const uint4 r = scale_row(amax);
		sv = __uint_as_float(r.x);
		ny = __uint_as_float(r.y);
		code = r.z;
	} else {
		const float2 sy = __ldg(&g_e4m3_pairs.p[0x7E]);
		sv = sy.x;
		ny = -sy.y;
		code = 0x7Eu;
	}
	uint32_t b[8];
#pragma unroll
	for (int k = 0; k < 8; ++k) {
		const float f = k & 1 ? bf16hi(w[k >> 1]) : bf16lo(w[k >> 1]);
		const uint32_t sign = (__float_as_uint(f) >> 31) << 7;
		if (isnan(f)) {
			b[k] = sign | 0x7Fu;
		} else if (isinf(f)) {
			b[k] = sign | 0x7Eu;
		} else {   // the negated quotient of quot_e4m3x2
			const float m = f * ny;
			b[k] = (cvt_e4m3x2(fmaf(fmaf(sv, m, f), ny, m), 0.f) & 0xFFu) ^ 0x80u;
		}
	}
	lo = b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24);
	hi = b[4] | (b[5] << 8) | (b[6] << 16) | (b[7] << 24);
	return code;
}

// Smallest E4M3 code >= amax / 448 (the reference quantizer's scale rule,
// mx_dequant.h:119-120, with a real E4M3 encoding in place of its stub).
// t = amax / 448 through the correctly rounded
// reciprocal and one residual step, which is exact whenever the quotient is
// representable; an E4M3 value can only equal RN(amax / 448) when amax / 448
// is exactly that value (a bf16 and 448 x an E4M3 value differ by at least
// 2^-8 relative otherwise), so the code is the one of exact division.
__device__ __forceinline__ uint32_t mx_scale_code_tab(float amax, const float *tab)
{
	if (!(amax > 0.f))
		return 0u;
	constexpr float r448 = 1.0f / 448.0f;
	const float q0 = amax * r448;
	const float t = fmaf(fmaf(-448.0f, q0, amax), r448, q0);
	if (t > 448.0f)
		return 0x7Eu;
	uint32_t c = cvt_e4m3x2(t, 0.f) & 0xFFu;
	if (__ldg(&tab[c]) < t)
		++c;
	return c == 0u ? 1u : c;
}

// Writes micro-block x (b of its kv head, K or V) at `slot` of the kv
// head's section `sec`: bf16 copy, MX-FP8 quantization, or the reference's
// BF16-payload form.
__device__ __forceinline__ void append_store(const kllm_append_args &a, const float *tab,
					     uint4 x, uint8_t *sec, int slot, int b)
{
	const int bs = a.block_size;
	const int d = a.head_dim;
	if (a.kv_dtype == 0) {
		*reinterpret_cast<uint4 *>(sec + ((size_t)slot * d + b * 8) * 2) = x;
		return;
	}
	float f[8] = {bf16lo(x.x), bf16hi(x.x), bf16lo(x.y), bf16hi(x.y),
		      bf16lo(x.z), bf16hi(x.z), bf16lo(x.w), bf16hi(x.w)};
	float amax = 0.f;
#pragma unroll
	for (int k = 0; k < 8; ++k)
		amax = fmaxf(amax, fabsf(f[k]));

	if (a.kv_dtype == 1) {
		uint32_t code = 0u, lo = 0u, hi = 0u;
		const bool finite = bf16x8_absmax_nan(x) <= 3.40282347e38f;   // false for inf / NaN
		if (!finite)
			code = mx_quantize_nonfinite(x, lo, hi);
		else
			code = mx_scale_code_tab(amax, tab);
		if (code != 0u && finite) {
			// x / s through the correctly rounded reciprocal plus one residual
			// step (Markstein): exact whenever the quotient is representable,
			// within one fp32 ulp otherwise. A bf16 x over an E4M3 s is either
			// such an exact quotient or at least 2^-9 (relative) away from every
			// E4M3 rounding midpoint, so the E4M3 rounding below equals that of
			// the correctly rounded quotient.
			// (computed negated, as quot_e4m3x2, so that a zero keeps its sign)
			const float s = __ldg(&tab[code]);
			const float ny = -__ldg(&tab[256 + code]);
			float nq[8];
#pragma unroll
			for (int k = 0; k < 8; ++k) {
				const float m = f[k] * ny;
				nq[k] = fmaf(fmaf(s, m, f[k]), ny, m);
			}
			uint32_t p[4];
#pragma unroll
			for (int k = 0; k < 4; ++k)
				p[k] = cvt_e4m3x2(nq[2 * k], nq[2 * k + 1]) ^ 0x8080u;
			lo = p[0] | (p[1] << 16);
			hi = p[2] | (p[3] << 16);
		}
		*reinterpret_cast<uint2 *>(sec + (size_t)slot * d + b * 8) = make_uint2(lo, hi);
		sec[(size_t)bs * d + (size_t)slot * (d / 8) + b] = (uint8_t)code;
		return;
	}

	// kv_dtype 2: mx_quant_to_bf16 (userspace/compute/mx_dequant.h:105-136)
	const float scale = amax > 0.f ? __fdiv_rn(amax, 448.0f) : 1.0f;
	const float inv = __fdiv_rn(1.0f, scale);
	uint32_t outw[4];
#pragma unroll
	for (int k = 0; k < 4; ++k) {
		uint32_t pr = 0;
#pragma unroll
		for (int hlf = 0; hlf < 2; ++hlf) {
			uint32_t bits = __float_as_uint(__fmul_rn(f[2 * k + hlf], inv));
			bits += 0x7FFFu + ((bits >> 16) & 1u);
			pr |= (bits >> 16) << (16 * hlf);
		}
		outw[k] = pr;
	}
	*reinterpret_cast<uint4 *>(sec + ((size_t)slot * d + b * 8) * 2) =
	    make_uint4(outw[0], outw[1], outw[2], outw[3]);
	sec[(size_t)bs * d * 2 + (size_t)slot * (d / 8) + b] = amax > 0.f ? 64 : 0;
}

// Grid x = groups of kTokensPerCta tokens, y = 256-thread slices of a
// token's 2 x num_kv_heads x head_dim/8 micro-blocks (K first, then V); one
// thread per micro-block and token. The first threads resolve each token's
// page once for the CTA (block-table entry -> K and V section base, slot);
// every thread issues the data loads of all its tokens before it writes, so
// several independent loads are in flight per thread and a warp reads 512
// contiguous bytes per token.
constexpr int kTokensPerCta = 4;

// Page of token t (sequence seq, position pos) for K (kv 0) or V: the
// address of kv head 0's section in the page, or 0 when the token has no
// page (flagged in err, as every write of that token is dropped).
__device__ __forceinline__ unsigned long long append_page(const kllm_append_args &a, int seq,
							  int pos, int kv, int &slot)
{
	const int bs = a.block_size;
	const bool pow2 = (bs & (bs - 1)) == 0;
	const int lg = __ffs(bs) - 1;
	const int blk = pos >= 0 ? (pow2 ? pos >> lg : pos / bs) : -1;
	slot = 0;
	if (seq < 0 || seq >= a.num_seqs || blk < 0 || blk >= a.max_blocks)
		return 0ull;
	const DevEntry *e = reinterpret_cast<const DevEntry *>(a.table) +
			    (size_t)seq * a.max_blocks + blk;
	const unsigned long long base = kv ? e->v : e->k;
	if (!e->valid || !e->k || !base)
		return 0ull;
	if (!in_arenas(a.arenas, base + a.layer_off,
		       (unsigned long long)a.num_kv_heads * section_bytes(a.kv_dtype, bs, a.head_dim))) {
		if (a.err)   // outside the registered arenas: never written
			atomicOr(a.err, KLLM_ERR_PAGE_RANGE_BIT);
		return 0ull;
	}
	slot = pos - blk * bs;
	return base + a.layer_off;
}

// seqs/poss: the CTA's tokens (shared memory, filled before the call).
__device__ __forceinline__ void append_tokens(const kllm_append_args &a, const float *tab, int i0,
					      const int *seqs, const int *poss)
{
	__shared__ unsigned long long s_page[kTokensPerCta][2];
	__shared__ int s_slot[kTokensPerCta][2];
	if (threadIdx.x < 2 * kTokensPerCta) {
		const int t = threadIdx.x >> 1, kv = threadIdx.x & 1;
		int slot = 0;
		unsigned long long page = 0ull;
		if (i0 + t < a.num_tokens) {
			page = append_page(a, seqs[t], poss[t], kv, slot);
			if (!page && a.err)
				atomicOr(a.err, 0x4u);
		}
		s_page[t][kv] = page;
		s_slot[t][kv] = slot;
	}
	__syncthreads();
	const int nb = a.head_dim >> 3;
	const int per_kv = a.num_kv_heads * nb;
	const int u = blockIdx.y * blockDim.x + threadIdx.x;
	if (u >= 2 * per_kv)
		return;
	const int kv = u >= per_kv ? 1 : 0;
	const int rem = u - kv * per_kv;
	const int h = rem / nb, b = rem - h * nb;
	const size_t hoff = (size_t)h * section_bytes(a.kv_dtype, a.block_size, a.head_dim);
	uint4 x[kTokensPerCta];
#pragma unroll
	for (int t = 0; t < kTokensPerCta; ++t)
		if (i0 + t < a.num_tokens)
			x[t] = append_load(a, i0 + t, h, kv, b);
#pragma unroll
	for (int t = 0; t < kTokensPerCta; ++t) {
		const unsigned long long page = s_page[t][kv];
		if (i0 + t < a.num_tokens && page)
			append_store(a, tab, x[t], reinterpret_cast<uint8_t *>(page) + hoff,
				     s_slot[t][kv], b);
	}
}

__global__ void __launch_bounds__(256) append_kernel(const kllm_append_args a)
{
	__shared__ int s_seq[kTokensPerCta], s_pos[kTokensPerCta];
	const float *tab = g_e4m3.v;
	const int i0 = blockIdx.x * kTokensPerCta;
	if (threadIdx.x < kTokensPerCta) {
		const int i = i0 + threadIdx.x;
		const bool in = i < a.num_tokens;
		s_seq[threadIdx.x] = in ? a.token_seq[i] : -1;
		s_pos[threadIdx.x] = in ? a.token_pos[i] : -1;
	}
	__syncthreads();
	append_tokens(a, tab, i0, s_seq, s_pos);
}

// Same, with the (sequence, position) of row i derived from chunk offsets.
__global__ void __launch_bounds__(256) append_chunk_kernel(const kllm_append_args a,
							   const int *cu, const int *ctx)
{
	__shared__ int s_seq[kTokensPerCta], s_pos[kTokensPerCta];
	const float *tab = g_e4m3.v;
	const int i0 = blockIdx.x * kTokensPerCta;
	if (threadIdx.x < kTokensPerCta) {
		const int i = i0 + threadIdx.x;
		int lo = 0, hi = a.num_seqs - 1;   // last s with cu[s] <= i
		while (lo < hi) {
			const int mid = (lo + hi + 1) >> 1;
			if (cu[mid] <= i)
				lo = mid;
			else
				hi = mid - 1;
		}
		const bool in = i < a.num_tokens && i < cu[lo + 1];
		s_seq[threadIdx.x] = in ? lo : -1;   // beyond the last chunk: flagged
		s_pos[threadIdx.x] = in ? ctx[lo] + (i - cu[lo]) : -1;
	}
	__syncthreads();
	append_tokens(a, tab, i0, s_seq, s_pos);
}

// The MX micro-blocks of token i that hold an infinite or NaN element, at
// `slot` of the pages kp / vp (the rest of the token is already stored).
template <int D>
__device__ __noinline__ void append_token_nonfinite(const void *k, const void *v, int i,
						    int num_kv_heads, int block_size,
						    unsigned long long kp, unsigned long long vp,
						    int slot, int lane)
{
	constexpr int NB = D / 8;
	const int per_row = num_kv_heads * NB;
	const size_t sec = (size_t)block_size * D * 9 / 8;
	for (int kv = 0; kv < 2; ++kv) {
		const uint4 *src = reinterpret_cast<const uint4 *>(kv ? v : k) + (size_t)i * per_row;
		for (int mb = lane; mb < per_row; mb += 32) {
			const uint4 x = __ldg(src + mb);
			if (bf16x8_absmax_nan(x) <= 3.40282347e38f)
				continue;
			uint8_t *secp = reinterpret_cast<uint8_t *>(kv ? vp : kp) + (size_t)(mb / NB) * sec;
			const int b = mb % NB;
			uint32_t lo, hi;
			const uint32_t code = mx_quantize_nonfinite(x, lo, hi);
			*reinterpret_cast<uint2 *>(secp + (size_t)slot * D + b * 8) = make_uint2(lo, hi);
			secp[(size_t)block_size * D + (size_t)slot * NB + b] = (uint8_t)code;
		}
	}
}

// Quantize-on-write, one warp per token (head_dim 64 or 128; MX-FP8 or
// BF16 pages). The token's K and V rows (num_kv_heads x D bf16 each, one
// contiguous run) are loaded first, 16 bytes per lane and micro-block, so
// the sequence and page lookup that follows runs while they are in flight;
// lane l then owns micro-blocks l, l+32, ... (head = index / (D/8), at
// compile-time shifts). MX: each lane writes its 8 payload bytes (16 lanes
// cover one head's 128-byte row) and its scale byte.
// `cu` == nullptr: token i goes to (token_seq[i], token_pos[i]); otherwise
// token i of the chunk goes to sequence s (cu[s] <= i < cu[s+1]) at
// position ctx[s] + i - cu[s].
template <int D>
__global__ void __launch_bounds__(256, 4) append_warp_kernel(const kllm_append_args a,
							  const int *cu, const int *ctx)
{
	constexpr int NB = D / 8;      // micro-blocks per head row
	constexpr int HPL = 32 / NB;   // head rows covered by one pass of the warp
	constexpr int kU = 4;          // micro-blocks per lane held per pass
	const int lane = threadIdx.x & 31;
	const int i = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
	if (i >= a.num_tokens)
		return;
	const int H = a.num_kv_heads;
	const int per_row = H * NB;
	const uint4 *ksrc = reinterpret_cast<const uint4 *>(a.k) + (size_t)i * per_row;
	const uint4 *vsrc = reinterpret_cast<const uint4 *>(a.v) + (size_t)i * per_row;

	uint4 xk[kU], xv[kU];
#pragma unroll
	for (int u = 0; u < kU; ++u) {
		const int mb = lane + 32 * u;
		if (mb < per_row) {
			xk[u] = __ldcs(ksrc + mb);
			xv[u] = __ldcs(vsrc + mb);
		}
	}

	// ---- token -> (sequence, position) -> page ------------------------------
	int seq = -1, pos = -1;
	if (!cu) {
		seq = a.token_seq[i];
		pos = a.token_pos[i];
	} else {
		// lane l looks at sequence b0 + l: its chunk start, end and cached
		// length in one round of loads; the sequence holding row i is the
		// lane whose chunk contains it (chunks are ordered and disjoint)
		for (int b0 = 0; b0 < a.num_seqs; b0 += 32) {
			const int s = b0 + lane;
			int c0 = 0, c1 = 0, cx = 0;
			if (s < a.num_seqs) {
				c0 = __ldg(cu + s);
				c1 = __ldg(cu + s + 1);
				cx = __ldg(ctx + s);
			}
			const bool mine = s < a.num_seqs && c0 <= i && i < c1;
			const unsigned hit = __ballot_sync(0xffffffffu, mine);
			if (hit) {
				const int src = __ffs(hit) - 1;
				seq = b0 + src;
				pos = __shfl_sync(0xffffffffu, cx + (i - c0), src);
				break;
			}
			if (__shfl_sync(0xffffffffu, c0, 31) > i)
				break;   // every later chunk starts after row i
		}
	}
	const int bs = a.block_size;
	const int blk = pos >= 0 ? pos / bs : -1;
	unsigned long long kp = 0ull, vp = 0ull;
	if (seq >= 0 && seq < a.num_seqs && blk >= 0 && blk < a.max_blocks) {
		const DevEntry *e = reinterpret_cast<const DevEntry *>(a.table) +
				    (size_t)seq * a.max_blocks + blk;
		kp = e->k;
		vp = e->v;
		if (!e->valid || !kp || !vp)
			kp = vp = 0ull;
	}
	if (!kp) {
		if (lane == 0 && a.err)
			atomicOr(a.err, 0x4u);
		return;
	}
	kp += a.layer_off;
	vp += a.layer_off;
	const bool mx = a.kv_dtype == 1;
	{
		// registered arenas: a page outside them is never written
		const unsigned long long pb = (unsigned long long)H *
					      (mx ? (size_t)a.block_size * D * 9 / 8
						  : (size_t)a.block_size * D * 2);
		if (!(in_arenas(a.arenas, kp, pb) && in_arenas(a.arenas, vp, pb))) {
			if (lane == 0 && a.err)
				atomicOr(a.err, KLLM_ERR_PAGE_RANGE_BIT);
			return;
		}
	}
	// payload stores are 8 (MX) or 16 (BF16) bytes wide
	const unsigned long long need = mx ? 7ull : 15ull;
	if ((kp | vp) & need) {
		if (lane == 0 && a.err)
			atomicOr(a.err, 0x2u);
		return;
	}
	const int slot = pos - blk * bs;
	const size_t sec = mx ? (size_t)bs * D * 9 / 8 : (size_t)bs * D * 2;
	// lane -> micro-block b of head row (lane / NB) + HPL * u of each pass
	const int b = lane % NB;
	const size_t lane_off = (size_t)(lane / NB) * sec;
	const size_t pay_off = mx ? (size_t)slot * D + b * 8 : ((size_t)slot * D + b * 8) * 2;
	const size_t scl_off = (size_t)bs * D + (size_t)slot * NB;
	bool nonfinite = false;

	for (int c0 = 0; c0 < per_row; c0 += 32 * kU) {
		if (c0) {   // more than 4 x 32 micro-blocks per row (many kv heads)
#pragma unroll
			for (int u = 0; u < kU; ++u) {
				const int mb = c0 + lane + 32 * u;
				if (mb < per_row) {
					xk[u] = __ldcs(ksrc + mb);
					xv[u] = __ldcs(vsrc + mb);
				}
			}
		}
		const size_t pass_off = (size_t)(c0 / NB) * sec + lane_off;
#pragma unroll
		for (int kv = 0; kv < 2; ++kv) {
			uint8_t *page = reinterpret_cast<uint8_t *>(kv ? vp : kp) + pass_off;
#pragma unroll
			for (int u = 0; u < kU; ++u) {
				const bool in = c0 + lane + 32 * u < per_row;
				uint8_t *secp = page + (size_t)(HPL * u) * sec;
				const uint4 x = kv ? xv[u] : xk[u];
				if (!mx) {
					if (in)
						*reinterpret_cast<uint4 *>(secp + pay_off) = x;
					continue;
				}
				const float amax = bf16x8_absmax_nan(x);
				uint32_t code = 0u, lo = 0u, hi = 0u;
				if (in && amax > 0.f && amax <= 3.40282347e38f) {
					// every element finite (a NaN fails both compares)
					const uint4 r = scale_row(amax);
					code = r.z;
					// the exact quotient of append_store (reciprocal + residual)
					const unsigned long long sv = f2_splat(__uint_as_float(r.x));
					const unsigned long long ny = f2_splat(__uint_as_float(r.y));
					lo = quot_e4m3x2(x.x, sv, ny) | (quot_e4m3x2(x.y, sv, ny) << 16);
					hi = quot_e4m3x2(x.z, sv, ny) | (quot_e4m3x2(x.w, sv, ny) << 16);
				} else if (in && !(amax <= 3.40282347e38f)) {
					nonfinite = true;
					continue;
				}
				if (in)
					*reinterpret_cast<uint2 *>(secp + pay_off) = make_uint2(lo, hi);
				// one byte per lane: the NB lanes of a head row write its NB
				// scale bytes in one store instruction
				if (in)
					secp[scl_off + b] = (uint8_t)code;
			}
		}
	}
	// rare: micro-blocks holding an infinite or NaN element were skipped
	// above and are quantized out of line, so the loop keeps no extra state
	if (__any_sync(0xffffffffu, nonfinite))
		append_token_nonfinite<D>(a.k, a.v, i, H, bs, kp, vp, slot, lane);
}

// One warp per (seq, kv head): walk the pages in order, skip invalid
// entries, dequantise every valid token row exactly to bf16.
__global__ void gather_kernel(const kllm_gather_args a)
{
	__shared__ uint32_t lut[256];
	for (int i = threadIdx.x; i < 256; i += blockDim.x)
		lut[i] = mx_scale_lut_entry((uint32_t)i);
	__syncthreads();

	const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	const int lane = threadIdx.x & 31;
	if (warp >= a.num_seqs * a.num_kv_heads)
		return;
	const int s = warp / a.num_kv_heads, h = warp % a.num_kv_heads;
	const int d = a.head_dim, bs = a.block_size;
	const size_t cap = (size_t)a.max_blocks * bs;
	uint16_t *ko = reinterpret_cast<uint16_t *>(a.k_out) +
		       ((size_t)s * a.num_kv_heads + h) * cap * d;
	uint16_t *vo = reinterpret_cast<uint16_t *>(a.v_out) +
		       ((size_t)s * a.num_kv_heads + h) * cap * d;
	int len = a.seq_lens[s];
	len = len < 0 ? 0 : len;
	if (len > (int)cap)
		len = (int)cap;
	const int nblocks = (len + bs - 1) / bs;
	const size_t sec = section_bytes(a.kv_dtype, bs, d);
	size_t n = 0;
	for (int blk = 0; blk < nblocks; ++blk) {
		const DevEntry *e = reinterpret_cast<const DevEntry *>(a.table) +
				    (size_t)s * a.max_blocks + blk;
		if (!e->valid || !e->k)
			continue;
		const int ntok = min(bs, len - blk * bs);
		for (int kv = 0; kv < 2; ++kv) {
			const uint8_t *secp = reinterpret_cast<const uint8_t *>(kv ? e->v : e->k) +
					      a.layer_off + (size_t)h * sec;
			uint16_t *dst = (kv ? vo : ko) + n * d;
			for (int idx = lane; idx < ntok * d; idx += 32) {
				const int t = idx / d, col = idx - t * d;
				uint16_t val;
				if (a.kv_dtype == 1) {
					const uint32_t pbyte = secp[(size_t)t * d + col];
					const uint32_t sbyte = secp[(size_t)bs * d + (size_t)t * (d / 8) + col / 8];
					uint32_t x = bf16x2_mul(e4m3x2_to_bf16x2_raw(pbyte, false), lut[sbyte]);
					x = bf16x2_mul(x, 0x43804380u);  // * 256, exact
					val = (uint16_t)(x & 0xFFFFu);
				} else {
					val = reinterpret_cast<const uint16_t *>(secp)[(size_t)t * d + col];
				}
				dst[(size_t)t * d + col] = val;
			}
		}
		n += ntok;
	}
	for (size_t idx = n * d + lane; idx < cap * d; idx += 32) {
		ko[idx] = 0;
		vo[idx] = 0;
	}
	if (lane == 0)
		a.counts[(size_t)s * a.num_kv_heads + h] = (int)n;
}

// One warp per row: M = max m_p, w_p = l_p exp(m_p - M), out = sum w_p o_p / sum w_p.
__global__ void merge_kernel(const float *m, const float *l, const float *o,
			     int parts, int rows, int d, uint16_t *out)
{
	const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
	const int lane = threadIdx.x & 31;
	if (row >= rows)
		return;
	float M = -CUDART_INF_F;
	for (int p = 0; p < parts; ++p) {
		const float lp = l[(size_t)p * rows + row];
		if (lp > 0.f)
			M = fmaxf(M, m[(size_t)p * rows + row]);
	}
	float wsum = 0.f;
	for (int p = 0; p < parts; ++p) {
		const float lp = l[(size_t)p * rows + row];
		if (lp > 0.f)
			wsum += lp * expf(m[(size_t)p * rows + row] - M);
	}
	const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
	for (int col = lane; col < d; col += 32) {
		float acc = 0.f;
		for (int p = 0; p < parts; ++p) {
			const float lp = l[(size_t)p * rows + row];
			if (lp > 0.f)
				acc += lp * expf(m[(size_t)p * rows + row] - M) *
				       o[((size_t)p * rows + row) * d + col];
		}
		__nv_bfloat16 b = __float2bfloat16_rn(acc * inv);
		out[(size_t)row * d + col] = *reinterpret_cast<uint16_t *>(&b);
	}
}

}  // namespace
}  // namespace kllm

using namespace kllm;

static dim3 append_grid(const struct kllm_append_args *a, int threads)
{
	const int per_token = 2 * a->num_kv_heads * (a->head_dim / 8);
	return dim3((unsigned)((a->num_tokens + kTokensPerCta - 1) / kTokensPerCta),
		    (unsigned)((per_token + threads - 1) / threads));
}

// Head dims 64 and 128 with MX-FP8 or BF16 pages take the warp-per-token
// kernel; other shapes and the reference's BF16-payload layout the general one.
static bool append_by_warp(const struct kllm_append_args *a)
{
	return (a->head_dim == 128 || a->head_dim == 64) && (a->kv_dtype == 0 || a->kv_dtype == 1);
}

static int append_warp_launch(const struct kllm_append_args *a, const int *cu,
			      const int *ctx, cudaStream_t st)
{
	const unsigned blocks = (unsigned)((a->num_tokens + 7) / 8);
	if (a->head_dim == 128)
		append_warp_kernel<128><<<blocks, 256, 0, st>>>(*a, cu, ctx);
	else
		append_warp_kernel<64><<<blocks, 256, 0, st>>>(*a, cu, ctx);
	return (int)cudaGetLastError();
}

extern "C" int kllm_append_launch(const struct kllm_append_args *a, void *stream)
{
	if (a->num_tokens <= 0)
		return 0;
	if (append_by_warp(a))
		return append_warp_launch(a, nullptr, nullptr, static_cast<cudaStream_t>(stream));
	append_kernel<<<append_grid(a, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(*a);
	return (int)cudaGetLastError();
}

extern "C" int kllm_append_chunk_launch(const struct kllm_append_args *a,
					const int *cu_seqlens, const int *ctx_lens,
					void *stream)
{
	if (a->num_tokens <= 0)
		return 0;
	if (append_by_warp(a))
		return append_warp_launch(a, cu_seqlens, ctx_lens, static_cast<cudaStream_t>(stream));
	append_chunk_kernel<<<append_grid(a, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
	    *a, cu_seqlens, ctx_lens);
	return (int)cudaGetLastError();
}

extern "C" int kllm_gather_launch(const struct kllm_gather_args *a, void *stream)
{
	const int warps = a->num_seqs * a->num_kv_heads;
	if (warps <= 0)
		return 0;
	const int threads = 128;
	const int blocks = (warps * 32 + threads - 1) / threads;
	gather_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(*a);
	return (int)cudaGetLastError();
}

extern "C" int kllm_merge_launch(const float *m, const float *l, const float *o,
				 int num_parts, int num_rows, int head_dim,
				 void *out, void *stream)
{
	if (num_rows <= 0)
		return 0;
	const int threads = 128;
	const int blocks = (num_rows * 32 + threads - 1) / threads;
	merge_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
	    m, l, o, num_parts, num_rows, head_dim, static_cast<uint16_t *>(out));
	return (int)cudaGetLastError();
}
