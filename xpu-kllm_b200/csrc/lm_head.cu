// SPDX-License-Identifier: Apache-2.0
//
// lm_head.cu - the step after attention: vocabulary projection and token
// sampling on the GPU. The reference has neither on any device: its GPU
// inference returns an all-zero logit vector and takes its argmax
// (userspace/compute/infer_gpu.c:212-229); its samplers are host loops over
// the logits (userspace/decode/decode_loop.c:58-185).
//
// lm_head_kernel<MH>: logits[b][v] = sum_k hidden[b][k] * W[v][k], bf16 in,
// fp32 accumulate, on tcgen05. One CTA per 256 vocabulary rows (MMA N = 256)
// holds all batch rows as MH accumulators of 128 rows (M = 128) in TMEM, so
// every weight byte crosses HBM once. A K-step is 64 hidden elements (one
// 128-byte swizzle row); hidden and weight tiles arrive by TMA through an
// S-stage ring. Warps: 0 producer (one elected lane), 1 TMEM allocation and
// MMA issue (one elected lane), 2-5 epilogue (warp w reads TMEM lanes
// 32 (w % 4) ..). The epilogue writes the fp32 logits and, per (row, tile),
// the tile's max logit, its first argmax and sum(exp((l - max) / T)). Waits
// are bounded in wall time; a timeout sets KLLM_ERR_TIMEOUT and the CTA
// drains its own copies and MMAs before freeing TMEM.
//
// sample_kernel: one CTA per row, the reference's dispatch
// (decode_loop.c:165-183): greedy = first maximum; temperature = first index
// whose running sum of exp((l - max) / T) reaches r x total (tiles in order
// from the partials, then the chosen tile's columns); top-k = the k largest
// logits ordered by (value desc, index asc) as the reference's insertion
// selection orders them: the k-th largest tile maximum bounds them from
// below, so a pass over the tiles whose maximum reaches it collects the
// candidates and a bitonic sort orders them (a radix select over the row
// covers k above the tile count or a candidate overflow), then the
// reference's temperature draw over that list, its running sums in the
// reference's order; top-p = temperature (the reference's nucleus is a TODO).

#include "kllm_device.cuh"
#include "kllm_internal.h"
#include "kllm_umma.cuh"

#include <math_constants.h>

namespace kllm {
namespace {

constexpr int kVN = 256;                  // vocabulary rows per CTA (MMA N)
constexpr int kKt = 64;                   // hidden elements per stage
constexpr int kMR = 128;                  // batch rows per accumulator (MMA M)
constexpr int kABytes = kMR * kKt * 2;    // 16 KB
constexpr int kBBytes = kVN * kKt * 2;    // 32 KB
constexpr int kLmThreads = 192;
constexpr uint64_t kLmWaitNs = 200000000ull;

template <int MH>
struct LmSmem {
	static constexpr int S = MH == 1 ? 4 : 3;
	uint8_t a[S][MH][kABytes];
	uint8_t b[S][kBBytes];
	uint64_t full[S], empty[S];
	uint64_t acc_full, drain;
	uint32_t tmem_base;
	int abort;
};

template <int MH>
__device__ bool lm_wait(LmSmem<MH> &sm, uint64_t *bar, uint32_t parity, uint32_t *err)
{
	if (mbar_try_wait(bar, parity))
		return true;
	const uint64_t t0 = global_ns();
	for (;;) {
		if (mbar_try_wait_sleep(bar, parity, 2000))
			return true;
		if (*reinterpret_cast<volatile int *>(&sm.abort))
			return false;
		if (global_ns() - t0 > kLmWaitNs) {
			*reinterpret_cast<volatile int *>(&sm.abort) = 1;
			if (err)
				atomicOr(err, KLLM_ERR_TIMEOUT_BIT);
			return false;
		}
	}
}

template <int MH>
__global__ void __launch_bounds__(kLmThreads, 1)
lm_head_kernel(const kllm_lm_head_args a, const __grid_constant__ CUtensorMap tm_h,
	       const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_w2)
{
	using Sm = LmSmem<MH>;
	constexpr int S = Sm::S;
	constexpr uint32_t kCols = MH * kVN;
	extern __shared__ __align__(1024) uint8_t smem_raw[];
	Sm &sm = *reinterpret_cast<Sm *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
					 ~(uintptr_t)1023);
	const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
	// CTAs 0..n_full-1 take a whole 256-row vocabulary tile; the rest take
	// one 128-row half of one of the last n_split tiles each, so that the
	// grid's last wave holds twice as many CTAs of half the work. The
	// second half's partial goes to slot NT + i; the sampler folds it in.
	const int NT = a.n_full + a.n_split;
	const int b = blockIdx.x;
	const bool whole = b < a.n_full;
	const int part = whole ? 0 : (b - a.n_full) & 1;
	const int tile = whole ? b : a.n_full + ((b - a.n_full) >> 1);
	const int nn = whole ? kVN : kVN / 2;                   // vocabulary rows (MMA N)
	const int n0 = tile * kVN + part * (kVN / 2);
	const int slot = part ? NT + (tile - a.n_full) : tile;
	const size_t stride = (size_t)NT + a.n_split;           // partial slots per row
	const int KT = a.hidden_dim / kKt;

	if (tid == 0) {
		for (int s = 0; s < S; ++s) {
			mbar_init(&sm.full[s], 1);
			mbar_init(&sm.empty[s], 1);
		}
		mbar_init(&sm.acc_full, 1);
		mbar_init(&sm.drain, 1);
		sm.abort = 0;
		fence_mbar_init();
	}
	if (warp == 1) {
		asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
			     :: "r"(smem_u32(&sm.tmem_base)), "r"(kCols));
		asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
	}
	tc_fence_before();
	__syncthreads();
	tc_fence_after();
	const uint32_t tmem = sm.tmem_base;

	if (warp == 0) {
		// ================= producer ==================================================
		if (elect_one()) {
			int issued[S];
#pragma unroll
			for (int s = 0; s < S; ++s)
				issued[s] = -1;
			for (int kt = 0; kt < KT; ++kt) {
				const int st = kt % S, fill = kt / S;
				if (fill > 0 && !lm_wait(sm, &sm.empty[st], (uint32_t)((fill - 1) & 1), a.err))
					break;
				mbar_arrive_expect_tx(&sm.full[st], MH * kABytes + nn * kKt * 2);
#pragma unroll
				for (int h = 0; h < MH; ++h)
					tma_load_2d(sm.a[st][h], &tm_h, kt * kKt, h * kMR, &sm.full[st]);
				tma_load_2d(sm.b[st], whole ? &tm_w : &tm_w2, kt * kKt, n0, &sm.full[st]);
				issued[st] = fill;
			}
			// after an abort, wait (bounded) for this CTA's own tensor copies
			if (*reinterpret_cast<volatile int *>(&sm.abort))
				for (int s = 0; s < S; ++s)
					if (issued[s] >= 0)
						mbar_wait_ns(&sm.full[s], (uint32_t)(issued[s] & 1), kLmWaitNs);
		}
		__syncwarp();
	} else if (warp == 1) {
		// ================= MMA issue ================================================
		const bool leader = elect_one();
		const uint32_t idesc = umma_idesc_bf16(kMR, nn, false);
		bool ok = true;
		for (int kt = 0; kt < KT; ++kt) {
			const int st = kt % S;
			ok = __all_sync(0xffffffffu, lm_wait(sm, &sm.full[st], (uint32_t)((kt / S) & 1),
							     a.err));
			if (!ok)
				break;
			tc_fence_after();
			const uint64_t db = umma_desc(smem_u32(sm.b[st]), 16u, 1024u);
#pragma unroll
			for (int h = 0; h < MH; ++h) {
				const uint64_t da = umma_desc(smem_u32(sm.a[st][h]), 16u, 1024u);
#pragma unroll
				for (int kk = 0; kk < kKt / 16; ++kk) {
					const uint64_t off = (uint64_t)(kk * 32) >> 4;
					if (leader)
						umma_f16(tmem + (uint32_t)(h * kVN), da + off, db + off, idesc,
							 (kt > 0 || kk > 0) ? 1u : 0u);
				}
			}
			__syncwarp();
			if (leader)
				umma_commit(&sm.empty[st]);   // the stage is free once these MMAs finish
			__syncwarp();
		}
		if (ok) {
			if (leader)
				umma_commit(&sm.acc_full);
			__syncwarp();
		}
		// every MMA issued by the leader completes before TMEM is freed
		if (leader)
			umma_commit(&sm.drain);
		__syncwarp();
		mbar_wait_ns(&sm.drain, 0u, kLmWaitNs);
	} else {
		// ================= epilogue: logits and tile partials ========================
		const int q = warp & 3;
		const bool ok = __all_sync(0xffffffffu, lm_wait(sm, &sm.acc_full, 0u, a.err));
		if (ok) {
			tc_fence_after();
			const bool vec = (a.vocab & 3) == 0;
#pragma unroll 1
			for (int h = 0; h < MH; ++h) {
				const int row = h * kMR + q * 32 + lane;
				const bool live = row < a.num_rows;
				const float T = (live && a.temperature) ? a.temperature[row] : 0.f;
				const bool want_sum = T > 0.f;
				const float inv_t = want_sum ? 1.f / T : 0.f;
				float m = -CUDART_INF_F, ssum = 0.f;
				int am = -1;
#pragma unroll 1
				for (int c = 0; c < nn / 32; ++c) {
					float v[32];
					tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(h * kVN + c * 32), v);
					const int nb = n0 + c * 32;
					if (live && a.logits) {
						float *dst = a.logits + (size_t)row * a.vocab + nb;
						if (vec && nb + 32 <= a.vocab) {
#pragma unroll
							for (int i = 0; i < 32; i += 4)
								*reinterpret_cast<float4 *>(dst + i) =
								    make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
						} else {
#pragma unroll
							for (int i = 0; i < 32; ++i)
								if (nb + i < a.vocab)
									dst[i] = v[i];
						}
					}
					float cm = -CUDART_INF_F;
					int ca = -1;
#pragma unroll
					for (int i = 0; i < 32; ++i)
						if (nb + i < a.vocab && v[i] > cm) {
							cm = v[i];
							ca = nb + i;
						}
					if (cm > m) {
						if (want_sum)
							ssum *= expf((m - cm) * inv_t);
						m = cm;
						am = ca;
					}
					if (want_sum) {
#pragma unroll
						for (int i = 0; i < 32; ++i)
							if (nb + i < a.vocab)
								ssum += expf((v[i] - m) * inv_t);
					}
				}
				if (live) {
					const size_t p = (size_t)row * stride + slot;
					a.part_m[p] = m;
					a.part_s[p] = ssum;
					a.part_a[p] = am;
				}
			}
		}
	}

	tc_fence_before();
	__syncthreads();
	if (warp == 1) {
		__syncwarp();
		tc_fence_after();
		asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
			     :: "r"(tmem), "r"(kCols));
	}
}

// ---- sampling ------------------------------------------------------------------

constexpr int kSampThreads = 256;
constexpr int kTopKMax = 1024;
constexpr int kCand = 2048;               // candidate buffer of the top-k search
constexpr int kTileKeys = 4096;           // tile maxima sortable in shared memory
static_assert(kSampThreads == kVN, "the in-tile scan gives one column to each thread");

// The float order as unsigned integers (larger key = larger value).
__device__ __forceinline__ uint32_t order_key(float f)
{
	const uint32_t u = __float_as_uint(f);
	return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Inclusive block scan of one float per thread (thread order), and the total.
__device__ float block_scan_f(float x, float *sh, float &total)
{
	const int t = threadIdx.x, lane = t & 31, w = t >> 5;
#pragma unroll
	for (int o = 1; o < 32; o <<= 1) {
		const float y = __shfl_up_sync(0xffffffffu, x, o);
		if (lane >= o)
			x += y;
	}
	if (lane == 31)
		sh[w] = x;
	__syncthreads();
	if (w == 0) {
		float s = lane < kSampThreads / 32 ? sh[lane] : 0.f;
#pragma unroll
		for (int o = 1; o < 32; o <<= 1) {
			const float y = __shfl_up_sync(0xffffffffu, s, o);
			if (lane >= o)
				s += y;
		}
		if (lane < kSampThreads / 32)
			sh[lane] = s;
	}
	__syncthreads();
	const float before = w ? sh[w - 1] : 0.f;
	total = sh[kSampThreads / 32 - 1];
	__syncthreads();
	return before + x;
}

struct SampleSmem {
	float fsh[32];
	int ish[32];
	uint32_t hist[256];
	float cand_v[kCand];
	int cand_i[kCand];
	uint32_t tkeys[kTileKeys];
	int found;
	int count;
	uint32_t prefix;
	int remain;
};

// Bitonic sort of n (a power of two) keys in shared memory, descending.
__device__ void sort_keys_desc(uint32_t *key, int n)
{
	for (int size = 2; size <= n; size <<= 1)
		for (int stride = size >> 1; stride > 0; stride >>= 1) {
			for (int j = threadIdx.x; j < n; j += kSampThreads) {
				const int o = j ^ stride;
				if (o > j) {
					const bool desc = (j & size) == 0;
					const uint32_t a = key[j], b = key[o];
					if ((a < b) == desc) {
						key[j] = b;
						key[o] = a;
					}
				}
			}
			__syncthreads();
		}
}

// Candidates for the k largest of a row, when the tile maxima bound them:
// the k-th largest tile maximum tau is an element, so at least k elements
// are >= tau and every one of the k largest is. Only tiles whose maximum
// reaches tau can hold such elements (about k of the row's tiles), so one
// pass over those tiles (16-byte loads, eight in flight per thread)
// collects the elements >= tau; returns their number, or -1 when it
// exceeds the buffer or k exceeds the tiles (the caller then runs the full
// radix select).
__device__ int tile_bound_candidates(const float *lg, int V, const float *pm, int NT, int k,
				     SampleSmem &sm)
{
	if (k > NT || NT > kTileKeys)
		return -1;
	int P = 1;
	while (P < NT)
		P <<= 1;
	for (int t = threadIdx.x; t < P; t += kSampThreads)
		sm.tkeys[t] = t < NT ? order_key(pm[t]) : 0u;
	if (threadIdx.x == 0) {
		sm.count = 0;
		sm.remain = 0;                  // tiles listed below
	}
	__syncthreads();
	sort_keys_desc(sm.tkeys, P);
	const uint32_t tau = sm.tkeys[k - 1];
	__syncthreads();
	// the tiles to scan, listed over the sorted keys (no longer needed)
	uint32_t *tiles = sm.tkeys;
	for (int t = threadIdx.x; t < NT; t += kSampThreads)
		if (order_key(pm[t]) >= tau)
			tiles[atomicAdd(&sm.remain, 1)] = (uint32_t)t;
	__syncthreads();
	const int nt = sm.remain;
	auto take = [&](float v, int i) {
		if (order_key(v) >= tau) {
			const int pos = atomicAdd(&sm.count, 1);
			if (pos < kCand) {
				sm.cand_v[pos] = v;
				sm.cand_i[pos] = i;
			}
		}
	};
	if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(lg) & 15u) == 0) {
		// 64 threads per tile (one float4 each), four tiles side by side
		constexpr int kVec = kVN / 4, kSide = kSampThreads / kVec, kFly = 8;
		const float4 *l4 = reinterpret_cast<const float4 *>(lg);
		const int n4 = V >> 2;
		const int sub = threadIdx.x % kVec, side = threadIdx.x / kVec;
		for (int base = 0; base < nt; base += kSide * kFly) {
			float4 x[kFly];
			int j4[kFly];
#pragma unroll
			for (int u = 0; u < kFly; ++u) {
				const int idx = base + u * kSide + side;
				j4[u] = idx < nt ? (int)tiles[idx] * kVec + sub : n4;
				x[u] = j4[u] < n4 ? l4[j4[u]] : make_float4(0.f, 0.f, 0.f, 0.f);
			}
#pragma unroll
			for (int u = 0; u < kFly; ++u) {
				if (j4[u] < n4) {
					take(x[u].x, 4 * j4[u]);
					take(x[u].y, 4 * j4[u] + 1);
					take(x[u].z, 4 * j4[u] + 2);
					take(x[u].w, 4 * j4[u] + 3);
				}
			}
		}
	} else {
		for (int idx = 0; idx < nt; ++idx) {
			const int i = (int)tiles[idx] * kVN + threadIdx.x;
			if (i < V)
				take(lg[i], i);
		}
	}
	__syncthreads();
	const int n = sm.count;
	__syncthreads();
	return n <= kCand ? n : -1;
}

// Greedy over the tile partials: the largest max, the smallest index on ties.
__device__ int greedy_token(const float *pm, const int *pa, int NT, SampleSmem &sm)
{
	float best = -CUDART_INF_F;
	int bi = 0x7fffffff;
	for (int t = threadIdx.x; t < NT; t += kSampThreads)
		if (pm[t] > best || (pm[t] == best && pa[t] >= 0 && pa[t] < bi)) {
			best = pm[t];
			bi = pa[t];
		}
#pragma unroll
	for (int o = 16; o; o >>= 1) {
		const float ob = __shfl_xor_sync(0xffffffffu, best, o);
		const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
		if (ob > best || (ob == best && oi < bi)) {
			best = ob;
			bi = oi;
		}
	}
	const int w = threadIdx.x >> 5;
	if ((threadIdx.x & 31) == 0) {
		sm.fsh[w] = best;
		sm.ish[w] = bi;
	}
	__syncthreads();
	if (threadIdx.x == 0) {
		for (int i = 1; i < kSampThreads / 32; ++i)
			if (sm.fsh[i] > best || (sm.fsh[i] == best && sm.ish[i] < bi)) {
				best = sm.fsh[i];
				bi = sm.ish[i];
			}
		sm.found = bi == 0x7fffffff ? 0 : bi;
	}
	__syncthreads();
	const int tok = sm.found;
	__syncthreads();
	return tok;
}

// Temperature draw over the whole vocabulary (decode_loop.c:71-113 with the
// probabilities left unnormalised): the first index whose running sum of
// exp((l - M) / T) reaches r x total; the last index when rounding leaves
// none (the reference's default).
__device__ int temperature_token(const kllm_lm_head_args &a, int row, const float *pm,
				 const float *ps, int NT, float T, float r, SampleSmem &sm)
{
	const float inv_t = 1.f / T;
	// the row maximum
	float M = -CUDART_INF_F;
	for (int t = threadIdx.x; t < NT; t += kSampThreads)
		M = fmaxf(M, pm[t]);
#pragma unroll
	for (int o = 16; o; o >>= 1)
		M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
	if ((threadIdx.x & 31) == 0)
		sm.fsh[threadIdx.x >> 5] = M;
	__syncthreads();
	if (threadIdx.x == 0) {
		for (int i = 1; i < kSampThreads / 32; ++i)
			M = fmaxf(M, sm.fsh[i]);
		sm.fsh[0] = M;
	}
	__syncthreads();
	M = sm.fsh[0];
	__syncthreads();
	// tiles in order: thread j owns tiles [j*per, (j+1)*per)
	const int per = (NT + kSampThreads - 1) / kSampThreads;
	const int t0 = threadIdx.x * per;
	float mine = 0.f;
	for (int t = t0; t < min(t0 + per, NT); ++t)
		if (pm[t] > -CUDART_INF_F)
			mine += ps[t] * expf((pm[t] - M) * inv_t);
	float total;
	const float incl = block_scan_f(mine, sm.fsh, total);
	const float thr = r * total;
	if (threadIdx.x == 0)
		sm.found = 0x7fffffff;
	__syncthreads();
	float run = incl - mine;
	for (int t = t0; t < min(t0 + per, NT); ++t) {
		const float e = pm[t] > -CUDART_INF_F ? ps[t] * expf((pm[t] - M) * inv_t) : 0.f;
		if (run + e >= thr && e > 0.f) {
			atomicMin(&sm.found, t);
			break;
		}
		run += e;
	}
	__syncthreads();
	const int tt = sm.found;
	__syncthreads();
	if (tt == 0x7fffffff)
		return a.vocab - 1;
	// the running sum before tile tt, then that tile's columns in order
	float before = 0.f;
	{
		float own = 0.f;
		for (int t = t0; t < min(t0 + per, tt); ++t)
			if (pm[t] > -CUDART_INF_F)
				own += ps[t] * expf((pm[t] - M) * inv_t);
		float tot2;
		block_scan_f(own, sm.fsh, tot2);
		before = tot2;
	}
	const int n = tt * kVN + threadIdx.x;
	const float e = n < a.vocab ? expf((a.logits[(size_t)row * a.vocab + n] - M) * inv_t) : 0.f;
	float tile_sum;
	const float cum = before + block_scan_f(e, sm.fsh, tile_sum);
	if (threadIdx.x == 0)
		sm.found = 0x7fffffff;
	__syncthreads();
	if (n < a.vocab && e > 0.f && cum >= thr)
		atomicMin(&sm.found, n);
	__syncthreads();
	int tok = sm.found;
	if (tok == 0x7fffffff)      // rounding: the tile's last valid column
		tok = min(tt * kVN + kVN, a.vocab) - 1;
	__syncthreads();
	return tok;
}

// Bitonic sort of the first n (a power of two) candidates, descending by
// value, ascending by index on equal values.
__device__ void sort_candidates(SampleSmem &sm, int n)
{
	for (int size = 2; size <= n; size <<= 1)
		for (int stride = size >> 1; stride > 0; stride >>= 1) {
			for (int j = threadIdx.x; j < n; j += kSampThreads) {
				const int o = j ^ stride;
				if (o > j) {
					const bool desc = (j & size) == 0;
					const float vj = sm.cand_v[j], vo = sm.cand_v[o];
					const int ij = sm.cand_i[j], io = sm.cand_i[o];
					const bool j_first = vj > vo || (vj == vo && ij < io);
					if (desc != j_first) {
						sm.cand_v[j] = vo;
						sm.cand_v[o] = vj;
						sm.cand_i[j] = io;
						sm.cand_i[o] = ij;
					}
				}
			}
			__syncthreads();
		}
}

// The reference's temperature draw over the first k sorted candidates
// (decode_loop.c:71-113 on the top-k list). The max, each p = exp((v - max)
// / T) and each p / sum do not depend on the order and run on every thread;
// the two running sums stay sequential, in the reference's order, on one.
__device__ int draw_sorted(SampleSmem &sm, int k, float T, float r)
{
	if (T > 0.f) {
		float mx = -CUDART_INF_F;
		for (int j = threadIdx.x; j < k; j += kSampThreads)
			mx = fmaxf(mx, sm.cand_v[j]);
#pragma unroll
		for (int o = 16; o; o >>= 1)
			mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
		if ((threadIdx.x & 31) == 0)
			sm.fsh[threadIdx.x >> 5] = mx;
		__syncthreads();
		mx = sm.fsh[0];
		for (int i = 1; i < kSampThreads / 32; ++i)
			mx = fmaxf(mx, sm.fsh[i]);
		for (int j = threadIdx.x; j < k; j += kSampThreads)
			sm.cand_v[j] = expf((sm.cand_v[j] - mx) / T);
		__syncthreads();
		if (threadIdx.x == 0) {
			float sum = 0.f;
			for (int j = 0; j < k; ++j)
				sum += sm.cand_v[j];
			sm.fsh[0] = sum;
		}
		__syncthreads();
		const float sum = sm.fsh[0];
		for (int j = threadIdx.x; j < k; j += kSampThreads)
			sm.cand_v[j] = sm.cand_v[j] / sum;
		__syncthreads();
	}
	if (threadIdx.x == 0) {
		int res = 0;
		if (T > 0.f) {
			float cum = 0.f;
			res = k - 1;
			for (int j = 0; j < k; ++j) {
				cum += sm.cand_v[j];
				if (r <= cum) {
					res = j;
					break;
				}
			}
		}
		sm.found = sm.cand_i[res];
	}
	__syncthreads();
	const int tok = sm.found;
	__syncthreads();
	return tok;
}

// decode_loop.c:118-158: the k largest logits, ordered by (value desc,
// index asc), then the reference's temperature draw over them.
__device__ int top_k_token(const kllm_lm_head_args &a, int row, int k, float T, float r,
			   SampleSmem &sm)
{
	const float *lg = a.logits + (size_t)row * a.vocab;
	const int V = a.vocab;
	const int NT = (V + kVN - 1) / kVN;
	const int nc = tile_bound_candidates(lg, V, a.part_m + (size_t)row * (NT + a.n_split), NT,
					     k, sm);
	if (nc >= 0) {
		// the candidates hold the k largest: sort them all, keep the first k
		int P = 1;
		while (P < nc)
			P <<= 1;
		for (int j = nc + threadIdx.x; j < P; j += kSampThreads) {
			sm.cand_v[j] = -CUDART_INF_F;
			sm.cand_i[j] = 0x7fffffff;
		}
		__syncthreads();
		sort_candidates(sm, P);
		return draw_sorted(sm, k, T, r);
	}
	// radix select: the key of the k-th largest logit, 8 bits per pass; every
	// loop is warp-uniform (ballots), histogram adds aggregated per bin
	const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
	if (threadIdx.x == 0) {
		sm.prefix = 0u;
		sm.remain = k;
	}
	__syncthreads();
	for (int pass = 0; pass < 4; ++pass) {
		const int shift = 24 - 8 * pass;
		const uint32_t hi_mask = pass ? (0xFFFFFFFFu << (32 - 8 * pass)) : 0u;
		for (int i = threadIdx.x; i < 256; i += kSampThreads)
			sm.hist[i] = 0u;
		__syncthreads();
		const uint32_t prefix = sm.prefix;
		for (int base = 0; base < V; base += 4 * kSampThreads) {
			uint32_t key4[4];                 // four loads in flight per thread
#pragma unroll
			for (int u = 0; u < 4; ++u) {
				const int i = base + u * kSampThreads + threadIdx.x;
				key4[u] = i < V ? order_key(lg[i]) : 0u;
			}
#pragma unroll
			for (int u = 0; u < 4; ++u) {
				const int i = base + u * kSampThreads + threadIdx.x;
				const bool hit = i < V && (key4[u] & hi_mask) == prefix;
				const unsigned act = __ballot_sync(0xffffffffu, hit);
				if (hit) {
					const uint32_t bin = (key4[u] >> shift) & 0xFFu;
					const unsigned peers = __match_any_sync(act, bin);
					if ((int)(__ffs(peers) - 1) == lane)
						atomicAdd(&sm.hist[bin], (uint32_t)__popc(peers));
				}
			}
		}
		__syncthreads();
		if (threadIdx.x == 0) {
			int rem = sm.remain;
			int bin = 255;
			for (; bin > 0; --bin) {
				if ((int)sm.hist[bin] >= rem)
					break;
				rem -= (int)sm.hist[bin];
			}
			sm.prefix = prefix | ((uint32_t)bin << shift);
			sm.remain = rem;            // how many of the k-th key's equals to take
		}
		__syncthreads();
	}
	const uint32_t kth = sm.prefix;
	const int need_eq = sm.remain;
	// ordered selection, every key above kth and the first need_eq equal to
	// it: warp w scans its contiguous segment twice (count, then place by
	// ballot rank), one prefix over the warps in between
	constexpr int kW = kSampThreads / 32;
	const int seg = ((V + kW - 1) / kW + 31) & ~31;
	const int s0 = min(V, w * seg), s1 = min(V, s0 + seg);
	int cg = 0, ce = 0;
	for (int base = s0; base < s1; base += 128) {
		uint32_t key4[4];
#pragma unroll
		for (int u = 0; u < 4; ++u) {
			const int i = base + 32 * u + lane;
			key4[u] = i < s1 ? order_key(lg[i]) : 0u;
		}
#pragma unroll
		for (int u = 0; u < 4; ++u) {
			const int i = base + 32 * u + lane;
			cg += __popc(__ballot_sync(0xffffffffu, i < s1 && key4[u] > kth));
			ce += __popc(__ballot_sync(0xffffffffu, i < s1 && key4[u] == kth));
		}
	}
	if (lane == 0) {
		sm.ish[w] = cg;
		sm.ish[kW + w] = ce;
	}
	__syncthreads();
	int rg = 0, re = 0;
	for (int j = 0; j < w; ++j) {
		rg += sm.ish[j];
		re += sm.ish[kW + j];
	}
	const unsigned lt = (1u << lane) - 1u;
	int *eq_idx = reinterpret_cast<int *>(sm.cand_v);    // parked equal-key indices
	for (int base = s0; base < s1; base += 128) {
		uint32_t key4[4];
#pragma unroll
		for (int u = 0; u < 4; ++u) {
			const int i = base + 32 * u + lane;
			key4[u] = i < s1 ? order_key(lg[i]) : 0u;
		}
#pragma unroll
		for (int u = 0; u < 4; ++u) {                   // index order: u, then lane
			const int i = base + 32 * u + lane;
			const bool gt = i < s1 && key4[u] > kth, eq = i < s1 && key4[u] == kth;
			const unsigned bg = __ballot_sync(0xffffffffu, gt);
			const unsigned bq = __ballot_sync(0xffffffffu, eq);
			if (gt)
				sm.cand_i[rg + __popc(bg & lt)] = i;
			if (eq) {
				const int pos = re + __popc(bq & lt);
				if (pos < need_eq)
					eq_idx[pos] = i;
			}
			rg += __popc(bg);
			re += __popc(bq);
		}
	}
	__syncthreads();
	// candidates: [0, k - need_eq) above kth (index order), then need_eq equals
	const int n_gt_sel = k - need_eq;
	for (int j = threadIdx.x; j < need_eq; j += kSampThreads)
		sm.cand_i[n_gt_sel + j] = eq_idx[j];
	__syncthreads();
	int P = 1;
	while (P < k)
		P <<= 1;
	for (int j = threadIdx.x; j < P; j += kSampThreads) {
		if (j < k) {
			sm.cand_v[j] = lg[sm.cand_i[j]];
		} else {
			sm.cand_v[j] = -CUDART_INF_F;
			sm.cand_i[j] = 0x7fffffff;
		}
	}
	__syncthreads();
	sort_candidates(sm, P);
	return draw_sorted(sm, k, T, r);
}

__global__ void __launch_bounds__(kSampThreads) sample_kernel(const kllm_lm_head_args a)
{
	__shared__ SampleSmem sm;
	const int row = blockIdx.x;
	const int NT = (a.vocab + kVN - 1) / kVN;
	const size_t stride = (size_t)NT + a.n_split;   // partial slots per row
	float *pm = a.part_m + (size_t)row * stride;
	float *ps = a.part_s + (size_t)row * stride;
	int *pa = a.part_a + (size_t)row * stride;
	const int method = a.method ? a.method[row] : KLLM_SAMPLE_GREEDY_I;
	const float T = a.temperature ? a.temperature[row] : 0.f;
	// tiles computed as two halves: fold the second half (slot NT + i) into
	// the tile's partial, as one pass over the whole tile would have left
	// it (the larger maximum, the first half's index on equal maxima, the
	// sums rescaled to the common maximum)
	{
		const float inv_t = T > 0.f ? 1.f / T : 0.f;
		for (int i = threadIdx.x; i < a.n_split; i += kSampThreads) {
			const int t = a.n_full + i;
			const float m0 = pm[t], m1 = pm[NT + i];
			const float M = fmaxf(m0, m1);
			float sum = 0.f;
			if (M > -CUDART_INF_F) {
				if (m0 > -CUDART_INF_F)
					sum += ps[t] * expf((m0 - M) * inv_t);
				if (m1 > -CUDART_INF_F)
					sum += ps[NT + i] * expf((m1 - M) * inv_t);
			}
			if (m1 > m0)
				pa[t] = pa[NT + i];
			pm[t] = M;
			ps[t] = sum;
		}
		__syncthreads();
	}
	const int k = a.top_k ? a.top_k[row] : 0;
	const float r = a.uniform ? a.uniform[row] : 0.f;
	int tok;
	if (method == KLLM_SAMPLE_TOP_K_I && k > kTopKMax && k < a.vocab) {
		tok = -1;                       // beyond the candidate buffer: refused
		if (threadIdx.x == 0 && a.err)
			atomicOr(a.err, KLLM_ERR_TOPK_RANGE_BIT);
	} else if (method == KLLM_SAMPLE_TOP_K_I && k > 0 && k < a.vocab)
		tok = top_k_token(a, row, k, T, r, sm);
	else if ((method == KLLM_SAMPLE_TEMPERATURE_I || method == KLLM_SAMPLE_TOP_P_I ||
		  method == KLLM_SAMPLE_TOP_K_I) && T > 0.f)
		tok = temperature_token(a, row, pm, ps, NT, T, r, sm);
	else
		tok = greedy_token(pm, pa, NT, sm);
	if (threadIdx.x == 0)
		a.tokens[row] = tok;
}

template <int MH>
int launch_mh(const kllm_lm_head_args &a, const CUtensorMap &mh, const CUtensorMap &mw,
	      const CUtensorMap &mw2, cudaStream_t st)
{
	const size_t smem = sizeof(LmSmem<MH>) + 1024;
	cudaError_t e = cudaFuncSetAttribute(lm_head_kernel<MH>,
					     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
	if (e != cudaSuccess)
		return (int)e;
	lm_head_kernel<MH><<<a.n_full + 2 * a.n_split, kLmThreads, smem, st>>>(a, mh, mw, mw2);
	return (int)cudaGetLastError();
}

// SMs of the current device, queried once per device (0 on error).
int device_sms()
{
	static int cache[16];
	int dev = 0;
	if (cudaGetDevice(&dev) != cudaSuccess || dev < 0)
		return 0;
	if (dev < 16 && cache[dev] > 0)
		return cache[dev];
	int n = 0;
	if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
		return 0;
	if (dev < 16)
		cache[dev] = n;
	return n;
}

// [rows][hidden] bf16, box 64 x box_rows, 128-byte swizzle, zero fill past rows
bool make_rows_map(CUtensorMap *m, const void *base, int rows, int hidden, int box_rows)
{
	auto enc = get_encode();
	if (!enc)
		return false;
	cuuint64_t dims[2] = {(cuuint64_t)hidden, (cuuint64_t)rows};
	cuuint64_t strides[1] = {(cuuint64_t)hidden * 2};
	cuuint32_t box[2] = {(cuuint32_t)kKt, (cuuint32_t)box_rows};
	cuuint32_t estr[2] = {1, 1};
	return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
		   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
		   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
		   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace kllm

using namespace kllm;

extern "C" int kllm_lm_head_tiles(int vocab)
{
	return (vocab + kVN - 1) / kVN;
}

extern "C" int kllm_lm_head_launch(const struct kllm_lm_head_args *a, void *stream)
{
	if (a->num_rows < 1 || a->num_rows > 2 * kMR || a->hidden_dim % kKt || a->vocab < 1)
		return (int)cudaErrorInvalidValue;
	CUtensorMap mh, mw, mw2;
	if (!make_rows_map(&mh, a->hidden, a->num_rows, a->hidden_dim, kMR) ||
	    !make_rows_map(&mw, a->weight, a->vocab, a->hidden_dim, kVN) ||
	    !make_rows_map(&mw2, a->weight, a->vocab, a->hidden_dim, kVN / 2))
		return (int)cudaErrorInvalidValue;
	// One CTA per SM (all of TMEM, ~197 KB of shared memory), each tile the
	// same work: a last wave of r < SMs tiles leaves SMs idle for a whole
	// tile. When 2r CTAs still fit in one wave, those r tiles are computed
	// as 2r halves, so the last wave takes half as long.
	kllm_lm_head_args b = *a;
	const int NT = (a->vocab + kVN - 1) / kVN, sms = device_sms();
	const int r = sms > 0 ? NT % sms : 0;
	b.n_split = (r > 0 && 2 * r <= sms) ? r : 0;
	b.n_full = NT - b.n_split;
	cudaStream_t st = static_cast<cudaStream_t>(stream);
	int rc = a->num_rows > kMR ? launch_mh<2>(b, mh, mw, mw2, st)
				   : launch_mh<1>(b, mh, mw, mw2, st);
	if (rc)
		return rc;
	sample_kernel<<<a->num_rows, kSampThreads, 0, st>>>(b);
	return (int)cudaGetLastError();
}
