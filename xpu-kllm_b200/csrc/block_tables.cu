// SPDX-License-Identifier: Apache-2.0
//
// block_tables.cu - builds the paged-attention block tables on the GPU from
// the token ids and a device mirror of the content-addressed cache index.
//
// The reference does this on the host, one block at a time:
//   key(b)  = SHA-256 of token_ids[0, min((b + 1) * block_size, seq_len)) as
//             little-endian uint32 (userspace/compute/infer_gpu.c:110-118,
//             OpenSSL SHA256(), every prefix hashed from scratch);
//   slot    = kllm_index_lookup(key) (userspace/kvcache/cache_index.c:87-108:
//             bucket = first four key bytes, little-endian, masked; linear
//             probe that stops at the first empty entry; full 32-byte match);
//   page    = arena base + slot * slot_size (userspace/kvcache/arena_alloc.c:
//             196-201, NULL past the last slot).
//
// Here the same keys come from one pass over each sequence: a prefix of 16
// tokens is one 64-byte SHA-256 message block, so the running hash state
// after j message blocks (a "midstate") serves every table block whose
// prefix ends in message block j. Two kernels:
//   chain_kernel     32 sequences per CTA, two warps. The message schedule
//                    depends only on the tokens, so warp 1 expands each
//                    message block into W[t] + K[t] (t = 0..63) in a
//                    shared-memory ring four blocks deep, and warp 0 runs
//                    only the 64 dependent rounds per block (a funnel-shift
//                    rotate, a three-way xor and a three-way add per
//                    critical step) and stores every midstate (32 B) in the
//                    workspace. The chain is latency-bound: the longest
//                    sequence's compressions run one after another;
//   finalize_kernel  one thread per (sequence, table block): the tail tokens
//                    and the FIPS 180-4 padding on top of the right midstate
//                    (one or two compressions), the index probe, the LRU
//                    stamp on a hit, the 24-byte table entry, the key, the
//                    hit/miss counts and the miss list.
// Incremental use: blocks below first_block[s] are neither hashed nor
// written, and the chain restarts from the midstate the workspace kept from
// the previous call for the same sequence row.

#include "kllm_device.cuh"
#include "kllm_internal.h"

namespace kllm {
namespace {

// FIPS 180-4 4.2.2 and 5.3.3 (recomputed from their definition by the tests).
__constant__ uint32_t kShaK[64] = {
	0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u,
	0x923f82a4u, 0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u,
	0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u,
	0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
	0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u,
	0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u,
	0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
	0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
	0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au,
	0x5b9cca4fu, 0x682e6ff3u, 0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u,
	0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u,
};

__device__ __forceinline__ void sha_iv(uint32_t (&h)[8])
{
	h[0] = 0x6a09e667u; h[1] = 0xbb67ae85u; h[2] = 0x3c6ef372u; h[3] = 0xa54ff53au;
	h[4] = 0x510e527fu; h[5] = 0x9b05688cu; h[6] = 0x1f83d9abu; h[7] = 0x5be0cd19u;
}

__device__ __forceinline__ uint32_t rotr(uint32_t x, int n)
{
	return __funnelshift_r(x, x, n);
}

// Token id (little-endian bytes in memory) -> big-endian message word.
__device__ __forceinline__ uint32_t msg_word(uint32_t token)
{
	return __byte_perm(token, 0, 0x0123);
}

// FIPS 180-4 6.2.2 steps 1-4 for one message block; w is consumed (it holds
// the rolling 16-word schedule window).
__device__ __forceinline__ void sha_compress(uint32_t (&h)[8], uint32_t (&w)[16])
{
	uint32_t a = h[0], b = h[1], c = h[2], d = h[3];
	uint32_t e = h[4], f = h[5], g = h[6], hh = h[7];
#pragma unroll
	for (int t = 0; t < 64; ++t) {
		uint32_t wt;
		if (t < 16) {
			wt = w[t];
		} else {
			const uint32_t x15 = w[(t - 15) & 15], x2 = w[(t - 2) & 15];
			const uint32_t s0 = rotr(x15, 7) ^ rotr(x15, 18) ^ (x15 >> 3);
			const uint32_t s1 = rotr(x2, 17) ^ rotr(x2, 19) ^ (x2 >> 10);
			wt = w[t & 15] + s0 + w[(t - 7) & 15] + s1;
			w[t & 15] = wt;
		}
		const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) +
				    ((e & f) ^ (~e & g)) + kShaK[t] + wt;
		const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) +
				    ((a & b) ^ (a & c) ^ (b & c));
		hh = g;
		g = f;
		f = e;
		e = d + t1;
		d = c;
		c = b;
		b = a;
		a = t1 + t2;
	}
	h[0] += a; h[1] += b; h[2] += c; h[3] += d;
	h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

// Tokens of sequence s actually tabled (seq_len clamped to the table).
__device__ __forceinline__ int tabled_len(const kllm_table_args &a, int s)
{
	const int len = a.seq_lens[s];
	const long long cap = (long long)a.max_blocks * a.block_size;
	return len < 0 ? 0 : (len > cap ? (int)cap : len);
}

__device__ __forceinline__ uint32_t *midstate(const kllm_table_args &a, int s, int j)
{
	return a.midstates + ((size_t)s * a.ms_stride + j) * 8;
}

// a + b + c, kept as written: the sums below are grouped so that each
// round's critical path is one rotate, one xor and one three-way add.
__device__ __forceinline__ uint32_t add3(uint32_t a, uint32_t b, uint32_t c)
{
	uint32_t r;
	asm("add.u32 %0, %1, %2;\n\tadd.u32 %0, %0, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
	return r;
}

// FIPS 180-4 6.2.2 step 4 alone: the 64 rounds over a precomputed schedule,
// wk[t * stride] = W[t] + K[t]. Per round, x = h + W + K and y = d + x do
// not depend on the previous round (h and d are e and a of three rounds
// back), so e' = y + S1(e) + Ch and T1 = x + S1(e) + Ch are one add each
// after S1, and a' = T1 + S0(a) + Maj one more.
__device__ __forceinline__ void sha_rounds(uint32_t (&h)[8], const uint32_t *wk, int stride)
{
	uint32_t a = h[0], b = h[1], c = h[2], d = h[3];
	uint32_t e = h[4], f = h[5], g = h[6], hh = h[7];
#pragma unroll
	for (int t = 0; t < 64; ++t) {
		const uint32_t x = hh + wk[t * stride];
		const uint32_t y = d + x;
		const uint32_t s1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
		const uint32_t ch = (e & f) ^ (~e & g);
		const uint32_t s0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
		const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
		const uint32_t t1 = add3(s1, ch, x);
		hh = g;
		g = f;
		f = e;
		e = add3(s1, ch, y);
		d = c;
		c = b;
		b = a;
		a = add3(t1, s0, mj);
	}
	h[0] += a; h[1] += b; h[2] += c; h[3] += d;
	h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

constexpr int kChainLanes = 32;     // sequences per CTA: warp 0 chains, warp 1 schedules
constexpr int kSlots = 4;           // message blocks in flight between the two warps
// Named barriers (64 threads: both warps), ids 1..kSlots: slot written by
// warp 1; ids kSlots+1..2*kSlots: slot read by warp 0. Both warps run the
// same warp-uniform number of iterations, so every barrier instance gets
// its 64 arrivals.
__device__ __forceinline__ void bar_sync64(int id)
{
	asm volatile("bar.sync %0, 64;" :: "r"(id) : "memory");
}
__device__ __forceinline__ void bar_arrive64(int id)
{
	asm volatile("bar.arrive %0, 64;" :: "r"(id) : "memory");
}

__global__ void __launch_bounds__(2 * kChainLanes) chain_kernel(const kllm_table_args a)
{
	__shared__ uint32_t wk[kSlots][64][kChainLanes];    // lane-minor: conflict-free
	const int lane = threadIdx.x & 31, role = threadIdx.x >> 5;
	const int s = blockIdx.x * kChainLanes + lane;
	if (blockIdx.x == 0 && threadIdx.x == 0 && a.miss_count)
		*a.miss_count = 0;
	int full = 0, j0 = 0;
	const uint32_t *tok = a.tokens;
	if (s < a.num_seqs) {
		const int raw = a.seq_lens[s];
		if (role == 0 && (long long)raw > (long long)a.max_blocks * a.block_size && a.err)
			atomicOr(a.err, KLLM_ERR_SEQ_TOO_LONG_BIT);
		const int len = tabled_len(a, s);
		const int b0 = a.first_block ? max(a.first_block[s], 0) : 0;
		full = len >> 4;
		j0 = (int)(((long long)b0 * a.block_size) >> 4);
		tok = a.tokens + a.starts[s];
	}
	// this lane's message blocks j0 .. full - 1; the warp runs the longest
	const int mine = max(full - j0, 0);
	const int n = __reduce_max_sync(0xffffffffu, mine);
	if (n == 0)
		return;                     // the other warp sees the same n
	if (role == 1) {
		// ---- schedule: tokens -> W[t] + K[t], one block ahead in registers
		uint32_t nxt[16];
#pragma unroll
		for (int k = 0; k < 16; ++k)
			nxt[k] = mine > 0 ? tok[(size_t)j0 * 16 + k] : 0u;
		for (int i = 0; i < n; ++i) {
			const int slot = i % kSlots;
			uint32_t w[16];
#pragma unroll
			for (int k = 0; k < 16; ++k)
				w[k] = msg_word(nxt[k]);
			if (i + 1 < mine) {
#pragma unroll
				for (int k = 0; k < 16; ++k)
					nxt[k] = tok[(size_t)(j0 + i + 1) * 16 + k];
			}
			if (i >= kSlots)
				bar_sync64(1 + kSlots + slot);     // warp 0 is done with block i - kSlots
			if (i < mine) {
#pragma unroll
				for (int t = 0; t < 64; ++t) {
					uint32_t wt;
					if (t < 16) {
						wt = w[t];
					} else {
						const uint32_t x15 = w[(t - 15) & 15], x2 = w[(t - 2) & 15];
						const uint32_t s0 = rotr(x15, 7) ^ rotr(x15, 18) ^ (x15 >> 3);
						const uint32_t s1 = rotr(x2, 17) ^ rotr(x2, 19) ^ (x2 >> 10);
						wt = w[t & 15] + s0 + w[(t - 7) & 15] + s1;
						w[t & 15] = wt;
					}
					wk[slot][t][lane] = wt + kShaK[t];
				}
			}
			__threadfence_block();
			bar_arrive64(1 + slot);
		}
		return;
	}
	// ---- chain: 64 rounds per block over the ring, midstate after each
	uint32_t h[8];
	if (j0 == 0 || mine == 0) {
		sha_iv(h);
	} else {
		const uint4 *m = reinterpret_cast<const uint4 *>(midstate(a, s, j0));
		const uint4 lo = m[0], hi = m[1];
		h[0] = lo.x; h[1] = lo.y; h[2] = lo.z; h[3] = lo.w;
		h[4] = hi.x; h[5] = hi.y; h[6] = hi.z; h[7] = hi.w;
	}
	for (int i = 0; i < n; ++i) {
		const int slot = i % kSlots;
		bar_sync64(1 + slot);
		if (i < mine) {
			sha_rounds(h, &wk[slot][0][lane], kChainLanes);
			uint4 *m = reinterpret_cast<uint4 *>(midstate(a, s, j0 + i + 1));
			m[0] = make_uint4(h[0], h[1], h[2], h[3]);
			m[1] = make_uint4(h[4], h[5], h[6], h[7]);
		}
		if (i + kSlots < n)
			bar_arrive64(1 + kSlots + slot);   // warp 1 refills this slot next
	}
}

__global__ void __launch_bounds__(256) finalize_kernel(const kllm_table_args a)
{
	const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
	const int s = (int)(gid / a.max_blocks), b = (int)(gid % a.max_blocks);
	bool hit = false, miss = false;
	if (s < a.num_seqs && b >= (a.first_block ? a.first_block[s] : 0)) {
		const int len = tabled_len(a, s);
		const int nb = (len + a.block_size - 1) / a.block_size;
		const size_t cell = (size_t)s * a.max_blocks + b;
		unsigned long long *te = reinterpret_cast<unsigned long long *>(
		    static_cast<uint8_t *>(a.table) + cell * 24);
		uint4 *hk = a.hashes ? reinterpret_cast<uint4 *>(a.hashes + cell * 32) : nullptr;
		if (b >= nb) {
			te[0] = 0ull;
			te[1] = 0ull;
			te[2] = 0ull;
			if (hk) {
				hk[0] = make_uint4(0, 0, 0, 0);
				hk[1] = make_uint4(0, 0, 0, 0);
			}
		} else {
			const long long pe = (long long)(b + 1) * a.block_size;
			const int prefix = pe < len ? (int)pe : len;
			const int f = prefix >> 4, t = prefix & 15;
			uint32_t h[8];
			if (f == 0) {
				sha_iv(h);
			} else {
				const uint4 *m = reinterpret_cast<const uint4 *>(midstate(a, s, f));
				const uint4 lo = m[0], hi = m[1];
				h[0] = lo.x; h[1] = lo.y; h[2] = lo.z; h[3] = lo.w;
				h[4] = hi.x; h[5] = hi.y; h[6] = hi.z; h[7] = hi.w;
			}
			// FIPS 180-4 5.1.1: tail tokens, the 0x80 byte, zeros, and the
			// 64-bit big-endian bit length (two blocks when t > 13).
			const uint32_t *tail = a.tokens + a.starts[s] + (size_t)f * 16;
			const unsigned long long bits = (unsigned long long)prefix * 32ull;
			const int nfinal = t <= 13 ? 1 : 2;
#pragma unroll 1
			for (int r = 0; r < nfinal; ++r) {
				uint32_t w[16];
#pragma unroll
				for (int k = 0; k < 16; ++k)
					w[k] = r == 0 ? (k < t ? msg_word(__ldg(tail + k))
							       : (k == t ? 0x80000000u : 0u))
						      : 0u;
				if (r == nfinal - 1) {
					w[14] = (uint32_t)(bits >> 32);
					w[15] = (uint32_t)bits;
				}
				sha_compress(h, w);
			}
			// Key bytes are the big-endian state words; as little-endian
			// words (the probe's view of the bytes) they are byte-swapped.
			uint32_t kw[8];
#pragma unroll
			for (int k = 0; k < 8; ++k)
				kw[k] = __byte_perm(h[k], 0, 0x0123);
			if (hk) {
				hk[0] = make_uint4(kw[0], kw[1], kw[2], kw[3]);
				hk[1] = make_uint4(kw[4], kw[5], kw[6], kw[7]);
			}
			const uint32_t mask = a.capacity - 1;
			const uint32_t bucket = kw[0] & mask;
			bool found = false;
			uint32_t fpos = 0, fslot = 0;
			for (uint32_t i = 0; i < a.capacity; ++i) {
				const uint32_t pos = (bucket + i) & mask;
				const uint4 *e = reinterpret_cast<const uint4 *>(a.index + (size_t)pos * 48);
				const uint4 tailw = e[2];
				if (tailw.x == 0xFFFFFFFFu)
					break;
				const uint4 e0 = e[0], e1 = e[1];
				if (e0.x == kw[0] && e0.y == kw[1] && e0.z == kw[2] && e0.w == kw[3] &&
				    e1.x == kw[4] && e1.y == kw[5] && e1.z == kw[6] && e1.w == kw[7]) {
					found = true;
					fpos = pos;
					fslot = tailw.x;
					break;
				}
			}
			unsigned long long kp = 0ull, vp = 0ull, valid = 0ull;
			if (found) {
				hit = true;
				if (a.now_ns)
					*reinterpret_cast<unsigned long long *>(a.index + (size_t)fpos * 48 + 40) =
					    a.now_ns;
				if ((unsigned long long)fslot < a.total_slots) {
					const unsigned long long page = a.arena_base +
									(unsigned long long)fslot * a.slot_bytes;
					kp = page + a.k_offset;
					vp = page + a.v_offset;
					valid = 1ull;
				}
			} else {
				miss = true;
			}
			te[0] = kp;
			te[1] = vp;
			te[2] = valid;
		}
	}
	// Warp-aggregated counters and miss list (every lane of the warp is here).
	const unsigned hm = __ballot_sync(0xffffffffu, hit), mm = __ballot_sync(0xffffffffu, miss);
	const int lane = threadIdx.x & 31;
	if (a.hit_miss && lane == 0) {
		if (hm)
			atomicAdd(a.hit_miss, (unsigned long long)__popc(hm));
		if (mm)
			atomicAdd(a.hit_miss + 1, (unsigned long long)__popc(mm));
	}
	if (a.miss_count && mm) {
		int base = 0;
		if (lane == 0)
			base = atomicAdd(a.miss_count, __popc(mm));
		base = __shfl_sync(0xffffffffu, base, 0);
		if (miss && a.miss_list) {
			const int at = base + __popc(mm & ((1u << lane) - 1u));
			if (at < a.miss_capacity) {
				a.miss_list[2 * at] = s;
				a.miss_list[2 * at + 1] = b;
			}
		}
	}
}

}  // namespace
}  // namespace kllm

using namespace kllm;

extern "C" uint64_t kllm_table_midstate_stride(int max_blocks, int block_size)
{
	return (uint64_t)(((long long)max_blocks * block_size) >> 4) + 1;
}

extern "C" int kllm_table_build_launch(const struct kllm_table_args *a, void *stream)
{
	cudaStream_t st = static_cast<cudaStream_t>(stream);
	chain_kernel<<<(a->num_seqs + kChainLanes - 1) / kChainLanes, 2 * kChainLanes, 0, st>>>(*a);
	cudaError_t e = cudaGetLastError();
	if (e != cudaSuccess)
		return (int)e;
	const long long cells = (long long)a->num_seqs * a->max_blocks;
	const long long grid = (cells + 255) / 256;
	if (grid > 0x7fffffffLL)
		return (int)cudaErrorInvalidValue;
	finalize_kernel<<<(unsigned)grid, 256, 0, st>>>(*a);
	return (int)cudaGetLastError();
}
