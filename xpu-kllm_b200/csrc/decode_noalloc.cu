// SPDX-License-Identifier: Apache-2.0
//
// decode_noalloc.cu - split-KV paged decode for callers that cannot allocate.
//
// Who needs this: the decode step of xpu-kllm runs on an SPDK reactor thread
// that polls without blocking and allocates nothing once it is running. A
// cudaMalloc there can stall the poll loop (the driver may synchronise the
// device to satisfy it) and can simply fail once the KV arena has claimed
// the GPU's memory. Such a caller cannot create a context either, because
// kllm_gpu_create allocates the context's split-KV workspace. This entry
// point takes only the inputs and outputs from the caller and keeps its
// scratch in a fixed array that the library image carries on every GPU that
// loads it, so nothing is allocated when it is called.
//
// Scratch: kScratchBytes (16 MiB) of file-scope device memory per device,
// held until the process exits: arrival counters for up to kMaxSegments
// (seq, kv head) pairs, split-KV partial slots, and the queue of long
// segments for the wide merge. The grid is cut to the number of partial
// slots that fit. Every call reuses the same array, so
// calls whose kernels overlap on the GPU (different streams, or different
// host threads) race on it and must be serialised by the caller.
//
// Set-up: CUDA loads a library's device code lazily, so the array (and the
// decode kernels) reach a GPU only when first used there. The first call on
// a device therefore loads them and looks up the array's address; it may
// need device memory and issues runtime queries. A call with num_seqs == 0
// does only this set-up: make one per device at start-up, before the KV
// arena claims the GPU's memory and before any stream capture.
//
// The caller's current device (its current CUDA context) is the same after
// a call as before it, whichever device the stream belongs to.

#include "kllm_device.cuh"
#include "kllm_gpu.h"
#include "kllm_internal.h"

#include <cuda.h>

#include <cstring>
#include <mutex>

namespace {

constexpr size_t kScratchBytes = 16u << 20;          // 16 MiB per device
constexpr int kMaxSegments = 65536;                  // num_seqs * num_kv_heads
constexpr size_t kCounterBytes = sizeof(unsigned) * kMaxSegments;  // 256 KiB
constexpr size_t kSlotBytes = 2ull * KLLM_SLOT_FLOATS * sizeof(float);  // per warp
constexpr size_t kListOffset = kScratchBytes - KLLM_MERGE_LIST_BYTES;  // merge queue
constexpr int kMaxWarps = (int)((kListOffset - kCounterBytes) / kSlotBytes);
constexpr int kMaxDevices = 64;

// The scratch itself. Host code must not use this name as an address: on
// the host it is only a stand-in symbol, so its device address is looked up
// once per device below and that address is what the kernel receives.
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

std::mutex g_setup_mu;
unsigned char *g_scratch_ptr[kMaxDevices];  // device address per ordinal

// The calling thread's current context, saved on entry and put back on
// every return, so a call on another GPU's stream leaves the caller's
// current device as it was (also when the caller had none yet).
using ctx_get_fn = CUresult (*)(CUcontext *);
using ctx_set_fn = CUresult (*)(CUcontext);
ctx_get_fn g_ctx_get;
ctx_set_fn g_ctx_set;
std::once_flag g_ctx_once;

void resolve_ctx_calls()
{
	void *fg = nullptr, *fs = nullptr;
	cudaDriverEntryPointQueryResult qg, qs;
	if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fg, cudaEnableDefault, &qg) ==
		cudaSuccess && qg == cudaDriverEntryPointSuccess &&
	    cudaGetDriverEntryPoint("cuCtxSetCurrent", &fs, cudaEnableDefault, &qs) ==
		cudaSuccess && qs == cudaDriverEntryPointSuccess && fg && fs) {
		g_ctx_get = reinterpret_cast<ctx_get_fn>(fg);
		g_ctx_set = reinterpret_cast<ctx_set_fn>(fs);
	}
	(void)cudaGetLastError();
}

struct CurrentContextGuard {
	CUcontext saved = nullptr;
	bool held = false;
	CurrentContextGuard()
	{
		std::call_once(g_ctx_once, resolve_ctx_calls);
		held = g_ctx_get && g_ctx_get(&saved) == CUDA_SUCCESS;
	}
	~CurrentContextGuard()
	{
		if (held)
			(void)g_ctx_set(saved);
	}
};

// Per-device set-up, done once per device with that device current: loads
// the decode kernels (CUDA loads modules lazily, and with them this
// module's scratch array) and looks up the scratch's device address. Both
// may need device memory and are runtime calls, so the first call on a
// device (a call with num_seqs == 0 does only this) belongs before the KV
// arena claims the GPU's memory and before any stream capture.
cudaError_t setup_for(int dev, unsigned char **out)
{
	std::lock_guard<std::mutex> lk(g_setup_mu);
	if (!g_scratch_ptr[dev]) {
		cudaError_t e = static_cast<cudaError_t>(kllm_decode_preload());
		if (e != cudaSuccess)
			return e;
		void *p = nullptr;
		e = cudaGetSymbolAddress(&p, g_decode_scratch);
		if (e != cudaSuccess)
			return e;
		g_scratch_ptr[dev] = static_cast<unsigned char *>(p);
	}
	*out = g_scratch_ptr[dev];
	return cudaSuccess;
}

}  // namespace

extern "C" int kllm_gpu_paged_attention_v2_noalloc(
    const struct kllm_gpu_attention_params_v2 *p)
{
	if (!p || p->struct_size < sizeof(*p))
		return KLLM_EINVAL;
	if (p->num_seqs < 0 || p->num_heads <= 0 || p->num_kv_heads <= 0 ||
	    p->max_blocks_per_seq <= 0 || p->num_heads % p->num_kv_heads)
		return KLLM_EINVAL;
	if (p->num_heads / p->num_kv_heads > KLLM_MAX_GROUP ||
	    (p->head_dim != 64 && p->head_dim != 128) || p->block_size < 16 ||
	    p->block_size > 128 || p->block_size % 16 ||
	    (p->kv_dtype != KLLM_KV_BF16 && p->kv_dtype != KLLM_KV_MX_FP8_E4M3))
		return KLLM_ENOSYS;
	// the kernels index a sequence's tokens with 32-bit integers
	if ((uint64_t)p->max_blocks_per_seq * (uint64_t)p->block_size > (1ull << 30))
		return KLLM_EINVAL;
	// the counters hold one word per (seq, kv head) of the call
	if ((long long)p->num_seqs * p->num_kv_heads > kMaxSegments)
		return KLLM_ENOSPC;
	const int partial = p->partial_m || p->partial_l || p->partial_o;
	if (p->num_seqs > 0) {
		if (partial && !(p->partial_m && p->partial_l && p->partial_o))
			return KLLM_EINVAL;
		if (!p->query || !p->block_tables || !p->seq_lens ||
		    (!p->output && !partial))
			return KLLM_EINVAL;
		if ((p->layer_stride & 15u) || p->layer < 0 ||
		    (((uintptr_t)p->query | (uintptr_t)p->output |
		      (uintptr_t)p->partial_o) & 15u))
			return KLLM_EINVAL;
	}

	cudaStream_t st = static_cast<cudaStream_t>(p->stream);
	CurrentContextGuard guard;
	int dev = 0;
	cudaError_t e = st ? cudaStreamGetDevice(st, &dev) : cudaGetDevice(&dev);
	if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
		(void)cudaGetLastError();
		return KLLM_ENODEV;
	}
	int cur = -1;
	if (cudaGetDevice(&cur) != cudaSuccess ||
	    (cur != dev && cudaSetDevice(dev) != cudaSuccess)) {
		(void)cudaGetLastError();
		return KLLM_ENODEV;
	}
	int major = 0, sms = 0;
	cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
	cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
	if (major != 10) {
		(void)cudaGetLastError();
		return KLLM_ENODEV;
	}
	unsigned char *scratch = nullptr;
	if (setup_for(dev, &scratch) != cudaSuccess) {
		(void)cudaGetLastError();
		return KLLM_EIO;
	}
	if (p->num_seqs == 0)
		return KLLM_OK;
	unsigned *cnt = reinterpret_cast<unsigned *>(scratch);
	float *part = reinterpret_cast<float *>(scratch + kCounterBytes);
	void *list = scratch + kListOffset;

	// split < 0: one warp per (seq, kv head), no partial slots (as in v2);
	// the queue is still used to recompute MX segments exactly.
	const int split = p->split >= 0;
	// The counters and the queue header must start at zero; the array keeps
	// whatever the last call left, so clear the words this call uses (no
	// allocation involved).
	const size_t segs = (size_t)p->num_seqs * p->num_kv_heads;
	if ((split && cudaMemsetAsync(cnt, 0, segs * sizeof(unsigned), st) != cudaSuccess) ||
	    cudaMemsetAsync(list, 0, 32, st) != cudaSuccess) {
		(void)cudaGetLastError();
		return KLLM_EIO;
	}

	struct kllm_decode_args a;
	memset(&a, 0, sizeof(a));
	a.out = partial ? nullptr : p->output;
	a.q = p->query;
	a.table = p->block_tables;
	a.seq_lens = p->seq_lens;
	a.num_heads = p->num_heads;
	a.num_kv_heads = p->num_kv_heads;
	a.group = p->num_heads / p->num_kv_heads;
	a.head_dim = p->head_dim;
	a.max_blocks = p->max_blocks_per_seq;
	a.block_size = p->block_size;
	a.kv_dtype = p->kv_dtype;
	a.layer_off = (uint64_t)p->layer * p->layer_stride;
	a.scale_log2 = p->scale * 1.4426950408889634f *
		       (p->kv_dtype == KLLM_KV_MX_FP8_E4M3 ? KLLM_MX_DEC_UNBIAS : 1.0f);
	a.pm = p->partial_m;
	a.pl = p->partial_l;
	a.po = p->partial_o;
	a.err = p->err_word;
	a.split = split;
	a.ws_part = split ? part : nullptr;
	a.ws_cnt = split ? cnt : nullptr;
	a.ws_list = list;

	const size_t row = (size_t)p->num_heads * p->head_dim;
	for (int s0 = 0; s0 < p->num_seqs; s0 += KLLM_MAX_SEQS_LAUNCH) {
		const int ns = p->num_seqs - s0 < KLLM_MAX_SEQS_LAUNCH ?
			       p->num_seqs - s0 : KLLM_MAX_SEQS_LAUNCH;
		struct kllm_decode_args c = a;
		c.num_seqs = ns;
		c.q = static_cast<const uint8_t *>(p->query) + (size_t)s0 * row * 2;
		if (c.out)
			c.out = static_cast<uint8_t *>(p->output) + (size_t)s0 * row * 2;
		c.table = static_cast<const uint8_t *>(p->block_tables) +
			  (size_t)s0 * p->max_blocks_per_seq * sizeof(struct kllm_block_table_entry);
		c.seq_lens = p->seq_lens + s0;
		if (split)
			c.ws_cnt = cnt + (size_t)s0 * p->num_kv_heads;
		if (partial) {
			c.pm = p->partial_m + (size_t)s0 * p->num_heads;
			c.pl = p->partial_l + (size_t)s0 * p->num_heads;
			c.po = p->partial_o + (size_t)s0 * row;
		}
		const int ctas = kllm_decode_ctas_per_sm(p->head_dim, p->kv_dtype, ns);
		if (ctas <= 0)
			return KLLM_EIO;
		int grid = sms * ctas;
		if (split && grid * KLLM_DEC_WARPS > kMaxWarps)
			grid = kMaxWarps / KLLM_DEC_WARPS;
		c.total_warps = grid * KLLM_DEC_WARPS;
		if (kllm_decode_launch(&c, grid, st) != 0 ||
		    kllm_decode_merge_launch(&c, sms, st) != 0) {
			(void)cudaGetLastError();
			return KLLM_EIO;
		}
	}
	return KLLM_OK;
}
