// SPDX-License-Identifier: Apache-2.0
//
// p2p_merge.cu - the cross-GPU split-KV exchange and merge as one kernel over
// peer memory (NVLink), for ranks that each hold a contiguous part of one
// long context and produced fp32 partial triples (m, l, o) for the same rows.
//
// Every rank owns an exchange buffer (cudaMalloc'd, opened by its peers
// through CUDA IPC):
//   header: flag[2][KLLM_P2P_MAX_RANKS][KLLM_P2P_MAX_CTAS]  (epoch written by
//           rank q's CTA b after its rows of slot [parity][q] landed here)
//           done[KLLM_P2P_MAX_RANKS][KLLM_P2P_MAX_CTAS]     (epoch rank q's CTA b
//           finished merging, i.e. read its own slots)
//   slots:  [2 parities][KLLM_P2P_MAX_RANKS] x { m[max_rows], l[max_rows],
//           o[max_rows][head_dim] }
// CTA b of every rank handles the same rows (b, b + grid, ...), so it only
// waits for the peers' CTA b: it stores its rows' triples into slot
// [epoch & 1][rank] of every rank (itself included), fences at system scope,
// raises flag[epoch & 1][rank][b] = epoch there, waits until all ranks'
// flags for b carry the epoch, merges its rows, and reports done. Before
// writing epoch e it waits until every peer's CTA b has finished epoch e - 2
// (the last one that used the same slot parity). Every wait is bounded; on
// expiry the kernel ORs KLLM_ERR_TIMEOUT into the error word and returns.
// Plain 16-byte stores and loads only (no TMA, no multicast).

#include "kllm_device.cuh"
#include "kllm_internal.h"

#include <math_constants.h>

namespace kllm {
namespace {

constexpr int kWarpsPerCta = 4;

struct P2PHeader {
	unsigned flag[2][KLLM_P2P_MAX_RANKS][KLLM_P2P_MAX_CTAS];
	unsigned done[KLLM_P2P_MAX_RANKS][KLLM_P2P_MAX_CTAS];
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p)
{
	unsigned v;
	asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
	return v;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v)
{
	asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}

// Spin (bounded by wall time) until *p reaches at least `want` (wrap-safe
// comparison on the 32-bit epoch).
__device__ __forceinline__ bool wait_at_least(const unsigned *p, unsigned want, uint64_t limit_ns)
{
	if ((int)(ld_acquire_sys(p) - want) >= 0)
		return true;
	const uint64_t t0 = global_ns();
	for (;;) {
		__nanosleep(64);
		if ((int)(ld_acquire_sys(p) - want) >= 0)
			return true;
		if (global_ns() - t0 > limit_ns)
			return false;
	}
}

__device__ __forceinline__ float *slot_base(uint8_t *buf, int parity, int rank,
					    const kllm_p2p_args &a)
{
	const size_t per_rank = (size_t)a.max_rows * (2 + a.head_dim);
	return reinterpret_cast<float *>(buf + sizeof(P2PHeader)) +
	       ((size_t)parity * KLLM_P2P_MAX_RANKS + rank) * per_rank;
}

template <int D>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
p2p_merge_kernel(const kllm_p2p_args a)
{
	constexpr int nv = D / 32;                // floats per lane of one o row
	const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
	const int par = (int)(a.epoch & 1u);
	uint8_t *const *peers = a.peers;
	P2PHeader *own = reinterpret_cast<P2PHeader *>(peers[a.rank]);
	__shared__ int s_ok;

	// ---- wait until every peer's CTA b finished the epoch that last used
	//      this slot parity -------------------------------------------------------
	if (threadIdx.x == 0) {
		int ok = 1;
		if (a.epoch > 2u)
			for (int q = 0; q < a.nranks && ok; ++q)
				ok = wait_at_least(&own->done[q][b], a.epoch - 2u, a.timeout_ns);
		s_ok = ok;
	}
	__syncthreads();
	// launched as a programmatic dependent of the kernel that wrote the
	// triples: everything above ran while it finished; from here on its
	// writes are complete and visible
	grid_dependency_wait();
	if (!s_ok) {
		if (threadIdx.x == 0 && a.err)
			atomicOr(a.err, KLLM_ERR_TIMEOUT_BIT);
		return;
	}

	// ---- this rank's rows of the triples into slot [par][rank] everywhere ----
	for (int q = 0; q < a.nranks; ++q) {
		float *dst = slot_base(peers[q], par, a.rank, a);
		float *dm = dst, *dl = dst + a.max_rows, *dov = dst + 2 * a.max_rows;
		for (int row = b * kWarpsPerCta + warp; row < a.num_rows;
		     row += gridDim.x * kWarpsPerCta) {
			if (lane == 0) {
				dm[row] = a.m[row];
				dl[row] = a.l[row];
			}
			const float *src = a.o + (size_t)row * D;
#pragma unroll
			for (int i = lane * 4; i < D; i += 128)
				*reinterpret_cast<float4 *>(dov + (size_t)row * D + i) =
				    *reinterpret_cast<const float4 *>(src + i);
		}
	}
	__threadfence_system();
	__syncthreads();
	if (threadIdx.x < a.nranks) {
		P2PHeader *h = reinterpret_cast<P2PHeader *>(peers[threadIdx.x]);
		st_release_sys(&h->flag[par][a.rank][b], a.epoch);
	}

	// ---- every rank's rows for this CTA have landed ----------------------------
	if (threadIdx.x == 0) {
		int ok = 1;
		for (int q = 0; q < a.nranks && ok; ++q)
			ok = wait_at_least(&own->flag[par][q][b], a.epoch, a.timeout_ns);
		s_ok = ok;
	}
	__syncthreads();
	if (!s_ok) {
		if (threadIdx.x == 0 && a.err)
			atomicOr(a.err, KLLM_ERR_TIMEOUT_BIT);
		return;
	}

	// ---- log-sum-exp merge of the CTA's rows (one warp per row) ----------------
	for (int row = b * kWarpsPerCta + warp; row < a.num_rows; row += gridDim.x * kWarpsPerCta) {
		float M = -CUDART_INF_F;
		for (int q = 0; q < a.nranks; ++q) {
			const float *sq = slot_base(peers[a.rank], par, q, a);
			const float lq = __ldcv(sq + a.max_rows + row);
			if (lq > 0.f)
				M = fmaxf(M, __ldcv(sq + row));
		}
		float L = 0.f, acc[nv];
#pragma unroll
		for (int i = 0; i < nv; ++i)
			acc[i] = 0.f;
		for (int q = 0; q < a.nranks; ++q) {
			const float *sq = slot_base(peers[a.rank], par, q, a);
			const float lq = __ldcv(sq + a.max_rows + row);
			if (!(lq > 0.f))
				continue;
			const float w = lq * __expf(__ldcv(sq + row) - M);
			L += w;
			const float *ov = sq + 2 * a.max_rows + (size_t)row * D;
#pragma unroll
			for (int i = 0; i < nv; ++i)
				acc[i] = fmaf(w, __ldcv(ov + lane + 32 * i), acc[i]);
		}
		const float inv = L > 0.f ? 1.f / L : 0.f;
		__nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(a.out) + (size_t)row * D;
#pragma unroll
		for (int i = 0; i < nv; ++i)
			dst[lane + 32 * i] = __float2bfloat16_rn(acc[i] * inv);
	}

	// ---- this CTA finished reading its slots of the epoch ------------------------
	__syncthreads();
	if (threadIdx.x < a.nranks) {
		P2PHeader *h = reinterpret_cast<P2PHeader *>(peers[threadIdx.x]);
		st_release_sys(&h->done[a.rank][b], a.epoch);
	}
}

}  // namespace
}  // namespace kllm

using namespace kllm;

extern "C" size_t kllm_p2p_buffer_bytes(int max_rows, int head_dim)
{
	return sizeof(P2PHeader) +
	       (size_t)2 * KLLM_P2P_MAX_RANKS * (size_t)max_rows * (2 + (size_t)head_dim) * 4;
}

extern "C" int kllm_p2p_grid(int num_rows)
{
	const int g = (num_rows + kWarpsPerCta - 1) / kWarpsPerCta;
	return g < 1 ? 1 : (g > KLLM_P2P_MAX_CTAS ? KLLM_P2P_MAX_CTAS : g);
}

extern "C" int kllm_p2p_merge_launch(const struct kllm_p2p_args *a, void *stream)
{
	cudaLaunchConfig_t cfg = {};
	cfg.gridDim = dim3((unsigned)kllm_p2p_grid(a->num_rows));
	cfg.blockDim = dim3(kWarpsPerCta * 32);
	cfg.stream = static_cast<cudaStream_t>(stream);
	// programmatic dependent of the previous kernel on the stream (the one
	// that wrote m, l, o): the slot-reuse wait overlaps its end, and
	// griddepcontrol.wait orders every read of the triples after it
	cudaLaunchAttribute at[1];
	at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
	at[0].val.programmaticStreamSerializationAllowed = 1;
	cfg.attrs = at;
	cfg.numAttrs = 1;
	if (a->head_dim == 128)
		return (int)cudaLaunchKernelEx(&cfg, p2p_merge_kernel<128>, *a);
	if (a->head_dim == 64)
		return (int)cudaLaunchKernelEx(&cfg, p2p_merge_kernel<64>, *a);
	return (int)cudaErrorInvalidValue;
}
