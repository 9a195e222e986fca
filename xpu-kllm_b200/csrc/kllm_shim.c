/* SPDX-License-Identifier: Apache-2.0 */
/*
 * kllm_shim.c - host side of the B200 paged-attention backend: a thin C
 * shim over the CUDA runtime that implements the reference backend ABI
 * (userspace/gpu/gpu_attention.h) for real - stream, allocation, copies -
 * and validates every call before launching the sm_100a kernels.
 *
 * Replaces userspace/gpu/gpu_attention.c (dlopen vendor probe + switch
 * dispatch, :20-107) and its TODO stubs (:56-63, :109-133). There is one
 * backend (CUDA sm_100a), no multi-vendor dispatch and no CPU fallback: a
 * context without a usable device reports KLLM_GPU_NONE and every compute
 * call returns KLLM_ENODEV.
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <sched.h>
#include <errno.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <cuda_runtime_api.h>
#include <nccl.h>

#include "kllm_gpu.h"
#include "kllm_internal.h"

#define KLLM_CNT_CAP       (1u << 18)  /* split-KV arrival counters per launch */
#define KLLM_COMM_ROWS_CAP 8192        /* rows per kllm_gpu_comm_merge call */
#define KLLM_COMM_DIM_CAP  128

/* NCCL entry points, resolved at kllm_gpu_comm_init time so that the library
 * loads without NCCL. */
struct nccl_api {
	void *handle;
	ncclResult_t (*get_unique_id)(ncclUniqueId *);
	ncclResult_t (*init_rank_config)(ncclComm_t *, int, ncclUniqueId, int,
					 ncclConfig_t *);
	ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t *);
	ncclResult_t (*abort_)(ncclComm_t);
	ncclResult_t (*destroy)(ncclComm_t);
	ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t,
				   ncclComm_t, cudaStream_t);
	ncclResult_t (*group_start)(void);
	ncclResult_t (*group_end)(void);
};

struct kllm_gpu_ctx {
	enum kllm_gpu_backend backend;
	int device;
	int num_sms;
	cudaStream_t stream;
	/* split-KV workspace */
	float *ws_part;
	unsigned *ws_cnt;
	uint64_t ws_part_bytes;
	int ws_max_warps;
	/* occupancy memo */
	int occ_key_d, occ_key_kv, occ_key_s, occ_val;
	struct kllm_gpu_stats stats;
	/* NCCL split-KV exchange */
	struct nccl_api nccl;
	ncclComm_t comm;
	int nranks, rank;
	float *comm_recv;   /* m [nranks][rows], l [nranks][rows], o [nranks][rows][D] */
	/* peer-memory exchange */
	uint8_t *p2p_buf;                        /* this rank's exchange buffer */
	uint8_t *p2p_peer[KLLM_P2P_MAX_RANKS];   /* every rank's, as mapped here */
	uint8_t **p2p_peers_dev;                 /* the same table in device memory */
	int p2p_max_rows, p2p_head_dim, p2p_nranks, p2p_rank;
	unsigned p2p_epoch;
	/* registered KV arenas (page range checks) */
	struct kllm_arenas arenas;
	/* per-call GPU timing: a ring of event pairs created when enabled */
	struct trace_slot *trace;
	int trace_cap;
	uint64_t trace_head, trace_tail, trace_dropped, trace_tag;
};

struct trace_slot {
	cudaEvent_t ev0, ev1;
	uint64_t submit_ns, tag;
	uint32_t op;
};

static uint64_t mono_ns(void)
{
	struct timespec ts;
	clock_gettime(CLOCK_MONOTONIC, &ts);
	return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

/* Opens a traced call on `st`: returns its ring slot, or -1 (tracing off, or
 * the ring is full because records were not read: the call is counted as
 * dropped). */
static int trace_begin(struct kllm_gpu_ctx *ctx, cudaStream_t st, uint32_t op)
{
	if (!ctx || !ctx->trace)
		return -1;
	if (ctx->trace_head - ctx->trace_tail >= (uint64_t)ctx->trace_cap) {
		ctx->trace_dropped++;
		return -1;
	}
	int i = (int)(ctx->trace_head % (uint64_t)ctx->trace_cap);
	struct trace_slot *t = &ctx->trace[i];
	t->submit_ns = mono_ns();
	t->tag = ctx->trace_tag;
	t->op = op;
	if (cudaEventRecord(t->ev0, st) != cudaSuccess) {
		(void)cudaGetLastError();
		return -1;
	}
	return i;
}

static void trace_end(struct kllm_gpu_ctx *ctx, cudaStream_t st, int i)
{
	if (i < 0)
		return;
	if (cudaEventRecord(ctx->trace[i].ev1, st) != cudaSuccess) {
		(void)cudaGetLastError();
		return;
	}
	ctx->trace_head++;
}

static void trace_free(struct kllm_gpu_ctx *ctx)
{
	if (!ctx->trace)
		return;
	for (int i = 0; i < ctx->trace_cap; i++) {
		cudaEventDestroy(ctx->trace[i].ev0);
		cudaEventDestroy(ctx->trace[i].ev1);
	}
	free(ctx->trace);
	ctx->trace = NULL;
	ctx->trace_cap = 0;
	ctx->trace_head = ctx->trace_tail = 0;
}

static int fail(struct kllm_gpu_ctx *ctx, int code)
{
	if (ctx) {
		ctx->stats.errors++;
		ctx->stats.last_error = code;
	}
	return code;
}

static int cuda_fail(struct kllm_gpu_ctx *ctx, cudaError_t e)
{
	cudaError_t last = cudaGetLastError();  /* clears a non-sticky error */
	if (ctx)
		ctx->stats.last_cuda_error = (int)(e != cudaSuccess ? e : last);
	return fail(ctx, KLLM_EIO);
}

static int ready(struct kllm_gpu_ctx *ctx)
{
	if (!ctx || ctx->backend != KLLM_GPU_CUDA)
		return 0;
	return cudaSetDevice(ctx->device) == cudaSuccess;
}

static cudaStream_t pick_stream(struct kllm_gpu_ctx *ctx, void *s)
{
	return s ? (cudaStream_t)s : ctx->stream;
}

/* ---- device probing ------------------------------------------------------ */

static int usable_device(int dev)
{
	int major = 0;
	if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) !=
	    cudaSuccess)
		return 0;
	return major == 10;  /* kernels are built for sm_100a only */
}

static int max_decode_ctas(void)
{
	int best = 0;
	const int dims[2] = {64, 128};
	for (int i = 0; i < 2; i++)
		for (int kv = 0; kv < 2; kv++) {
			int n = kllm_decode_ctas_per_sm(dims[i], kv, 1);
			if (n > best)
				best = n;
		}
	return best;
}

struct kllm_gpu_ctx *kllm_gpu_create(void)
{
	struct kllm_gpu_ctx *ctx = calloc(1, sizeof(*ctx));
	if (!ctx)
		return NULL;
	ctx->backend = KLLM_GPU_NONE;
	ctx->device = -1;
	ctx->stats.device = -1;

	int ndev = 0;
	if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) {
		(void)cudaGetLastError();
		return ctx;
	}
	int dev = -1;
	const char *env = getenv("KLLM_GPU_DEVICE");
	if (env && *env)
		dev = atoi(env);
	else if (cudaGetDevice(&dev) != cudaSuccess)
		dev = 0;
	if (dev < 0 || dev >= ndev || !usable_device(dev))
		return ctx;
	if (cudaSetDevice(dev) != cudaSuccess)
		return ctx;
	ctx->device = dev;
	cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, dev);
	if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess)
		goto fail_dev;

	int ctas = max_decode_ctas();
	if (ctas <= 0)
		goto fail_stream;
	ctx->ws_max_warps = ctx->num_sms * ctas * KLLM_DEC_WARPS;
	ctx->ws_part_bytes = (uint64_t)ctx->ws_max_warps * 2 * KLLM_SLOT_FLOATS * sizeof(float) +
			     KLLM_MERGE_LIST_BYTES;
	if (cudaMalloc((void **)&ctx->ws_part, ctx->ws_part_bytes) != cudaSuccess)
		goto fail_stream;
	if (cudaMalloc((void **)&ctx->ws_cnt, sizeof(unsigned) * KLLM_CNT_CAP) != cudaSuccess)
		goto fail_ws;
	if (cudaMemset(ctx->ws_cnt, 0, sizeof(unsigned) * KLLM_CNT_CAP) != cudaSuccess)
		goto fail_cnt;
	/* the merge list lives at the end of the partial region; its header
	 * must start at zero (the kernels leave it at zero after each call) */
	if (cudaMemset((uint8_t *)ctx->ws_part + ctx->ws_part_bytes - KLLM_MERGE_LIST_BYTES,
		       0, KLLM_MERGE_LIST_BYTES) != cudaSuccess)
		goto fail_cnt;
	if (cudaDeviceSynchronize() != cudaSuccess)
		goto fail_cnt;

	ctx->backend = KLLM_GPU_CUDA;
	ctx->stats.device = dev;
	ctx->stats.num_sms = ctx->num_sms;
	{
		const char *tr = getenv("KLLM_GPU_TRACE");
		if (tr && atoi(tr) > 0)
			(void)kllm_gpu_trace_enable(ctx, atoi(tr));
	}
	return ctx;

fail_cnt:
	cudaFree(ctx->ws_cnt);
	ctx->ws_cnt = NULL;
fail_ws:
	cudaFree(ctx->ws_part);
	ctx->ws_part = NULL;
fail_stream:
	cudaStreamDestroy(ctx->stream);
	ctx->stream = NULL;
fail_dev:
	(void)cudaGetLastError();
	ctx->device = -1;
	return ctx;
}

void kllm_gpu_destroy(struct kllm_gpu_ctx *ctx)
{
	if (!ctx)
		return;
	if (ctx->backend == KLLM_GPU_CUDA) {
		cudaSetDevice(ctx->device);
		cudaStreamSynchronize(ctx->stream);
		kllm_gpu_comm_destroy(ctx);
		kllm_gpu_p2p_destroy(ctx);
		trace_free(ctx);
		cudaFree(ctx->ws_part);
		cudaFree(ctx->ws_cnt);
		cudaStreamDestroy(ctx->stream);
	}
	free(ctx);
}

enum kllm_gpu_backend kllm_gpu_get_backend(struct kllm_gpu_ctx *ctx)
{
	return ctx ? ctx->backend : KLLM_GPU_NONE;
}

void *kllm_gpu_get_stream(struct kllm_gpu_ctx *ctx)
{
	return ctx ? (void *)ctx->stream : NULL;
}

/* ---- memory ---------------------------------------------------------------- */

void *kllm_gpu_malloc(struct kllm_gpu_ctx *ctx, uint64_t size)
{
	void *p = NULL;
	if (!ready(ctx) || size == 0)
		return NULL;
	if (cudaMalloc(&p, size) != cudaSuccess) {
		cuda_fail(ctx, cudaErrorMemoryAllocation);
		return NULL;
	}
	return p;
}

void kllm_gpu_free(struct kllm_gpu_ctx *ctx, void *ptr)
{
	if (!ptr || !ready(ctx))
		return;
	cudaFree(ptr);
}

void *kllm_gpu_host_alloc(struct kllm_gpu_ctx *ctx, uint64_t size)
{
	void *p = NULL;
	if (!ready(ctx) || size == 0)
		return NULL;
	if (cudaMallocHost(&p, size) != cudaSuccess) {
		cuda_fail(ctx, cudaErrorMemoryAllocation);
		return NULL;
	}
	return p;
}

void kllm_gpu_host_free(struct kllm_gpu_ctx *ctx, void *ptr)
{
	if (!ptr || !ready(ctx))
		return;
	cudaFreeHost(ptr);
}

static int copy_async(struct kllm_gpu_ctx *ctx, void *dst, const void *src,
		      uint64_t size, enum cudaMemcpyKind kind, cudaStream_t st)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (size == 0)
		return KLLM_OK;
	if (!dst || !src)
		return fail(ctx, KLLM_EINVAL);
	cudaError_t e = cudaMemcpyAsync(dst, src, size, kind, st);
	return e == cudaSuccess ? KLLM_OK : cuda_fail(ctx, e);
}

int kllm_gpu_memcpy_h2d(struct kllm_gpu_ctx *ctx, void *dst, const void *src,
			uint64_t size)
{
	int rc = copy_async(ctx, dst, src, size, cudaMemcpyHostToDevice, ctx ? ctx->stream : NULL);
	if (rc)
		return rc;
	cudaError_t e = cudaStreamSynchronize(ctx->stream);
	return e == cudaSuccess ? KLLM_OK : cuda_fail(ctx, e);
}

int kllm_gpu_memcpy_d2h(struct kllm_gpu_ctx *ctx, void *dst, const void *src,
			uint64_t size)
{
	int rc = copy_async(ctx, dst, src, size, cudaMemcpyDeviceToHost, ctx ? ctx->stream : NULL);
	if (rc)
		return rc;
	cudaError_t e = cudaStreamSynchronize(ctx->stream);
	return e == cudaSuccess ? KLLM_OK : cuda_fail(ctx, e);
}

int kllm_gpu_memcpy_h2d_async(struct kllm_gpu_ctx *ctx, void *dst,
			      const void *src, uint64_t size, void *stream)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	return copy_async(ctx, dst, src, size, cudaMemcpyHostToDevice, pick_stream(ctx, stream));
}

int kllm_gpu_memcpy_d2h_async(struct kllm_gpu_ctx *ctx, void *dst,
			      const void *src, uint64_t size, void *stream)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	return copy_async(ctx, dst, src, size, cudaMemcpyDeviceToHost, pick_stream(ctx, stream));
}

static double now_ms(void)
{
	struct timespec ts;
	clock_gettime(CLOCK_MONOTONIC, &ts);
	return (double)ts.tv_sec * 1e3 + (double)ts.tv_nsec * 1e-6;
}

static void nap_us(long us)
{
	struct timespec ts = {0, us * 1000L};
	nanosleep(&ts, NULL);
}

static int wait_stream(struct kllm_gpu_ctx *ctx, cudaStream_t st, int timeout_ms)
{
	if (timeout_ms <= 0) {
		cudaError_t e = cudaStreamSynchronize(st);
		return e == cudaSuccess ? KLLM_OK : cuda_fail(ctx, e);
	}
	double deadline = now_ms() + timeout_ms;
	for (;;) {
		cudaError_t e = cudaStreamQuery(st);
		if (e == cudaSuccess)
			return KLLM_OK;
		if (e != cudaErrorNotReady)
			return cuda_fail(ctx, e);
		if (now_ms() > deadline)
			return fail(ctx, KLLM_ETIMEDOUT);
		nap_us(50);
	}
}

int kllm_gpu_synchronize(struct kllm_gpu_ctx *ctx, int timeout_ms)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	return wait_stream(ctx, ctx->stream, timeout_ms);
}

int kllm_gpu_get_stats(struct kllm_gpu_ctx *ctx, struct kllm_gpu_stats *out)
{
	if (!ctx || !out)
		return KLLM_EINVAL;
	*out = ctx->stats;
	return KLLM_OK;
}

/* ---- decode ------------------------------------------------------------------ */

static int decode_ctas(struct kllm_gpu_ctx *ctx, int d, int kv, int s)
{
	if (ctx && ctx->occ_key_d == d && ctx->occ_key_kv == kv && ctx->occ_key_s == s)
		return ctx->occ_val;
	int n = kllm_decode_ctas_per_sm(d, kv, s);
	if (ctx) {
		ctx->occ_key_d = d;
		ctx->occ_key_kv = kv;
		ctx->occ_key_s = s;
		ctx->occ_val = n;
	}
	return n;
}

static int check_decode_shape(int num_seqs, int num_heads, int num_kv_heads,
			      int head_dim, int max_blocks, int block_size,
			      int kv_dtype)
{
	if (num_seqs < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_blocks <= 0)
		return KLLM_EINVAL;
	if (num_heads % num_kv_heads)
		return KLLM_EINVAL;
	if (num_heads / num_kv_heads > KLLM_MAX_GROUP)
		return KLLM_ENOSYS;
	if (head_dim != 64 && head_dim != 128)
		return KLLM_ENOSYS;
	if (block_size < 16 || block_size > 128 || block_size % 16)
		return KLLM_ENOSYS;
	if (kv_dtype != KLLM_KV_BF16 && kv_dtype != KLLM_KV_MX_FP8_E4M3)
		return KLLM_ENOSYS;
	if ((uint64_t)max_blocks * block_size > (1ull << 30))
		return KLLM_EINVAL;
	return KLLM_OK;
}

/* Launches one decode over sequences [s0, s0+ns) of the batch. */
static int decode_chunk(struct kllm_gpu_ctx *ctx, struct kllm_decode_args *a,
			int split, float *ws_part, unsigned *ws_cnt, void *ws_list,
			int max_warps, int num_sms, cudaStream_t st)
{
	int ctas = decode_ctas(ctx, a->head_dim, a->kv_dtype, a->num_seqs);
	if (ctas <= 0)
		return KLLM_EIO;
	int grid = num_sms * ctas;
	if (split && grid * KLLM_DEC_WARPS > max_warps)
		grid = max_warps / KLLM_DEC_WARPS;
	if (grid <= 0)
		return KLLM_ENOSPC;
	a->split = split;
	a->ws_part = ws_part;
	a->ws_cnt = ws_cnt;
	/* the queue also carries MX segments to recompute exactly (payload codes
	 * 0x7F / 0xFF), with or without split-KV */
	a->ws_list = ws_list;
	a->total_warps = grid * KLLM_DEC_WARPS;
	int e = kllm_decode_launch(a, grid, st);
	if (e)
		return KLLM_EIO;
	if (ctx)
		ctx->stats.launches++;
	if (ws_list && (split || a->kv_dtype == KLLM_KV_MX_FP8_E4M3)) {
		if (kllm_decode_merge_launch(a, num_sms, st))
			return KLLM_EIO;
		if (ctx)
			ctx->stats.launches++;
	}
	return KLLM_OK;
}

static int decode_common(struct kllm_gpu_ctx *ctx, struct kllm_decode_args *base,
			 int split, float *ws_part, uint64_t ws_part_bytes,
			 unsigned *ws_cnt, uint64_t cnt_cap, int num_sms,
			 cudaStream_t st)
{
	int S = base->num_seqs, hkv = base->num_kv_heads;
	if (S == 0)
		return KLLM_OK;
	int per = KLLM_MAX_SEQS_LAUNCH;
	if (split) {
		uint64_t by_cnt = cnt_cap / (uint64_t)hkv;
		if (by_cnt == 0)
			return KLLM_ENOSPC;
		if ((uint64_t)per > by_cnt)
			per = (int)by_cnt;
	}
	void *ws_list = NULL;
	if (ws_part && ws_part_bytes >= KLLM_MERGE_LIST_BYTES) {
		ws_part_bytes -= KLLM_MERGE_LIST_BYTES;
		ws_list = (uint8_t *)ws_part + ws_part_bytes;
	} else if (split) {
		return KLLM_ENOSPC;
	}
	int max_warps = (int)(ws_part_bytes / (2ull * KLLM_SLOT_FLOATS * sizeof(float)));
	if (split && max_warps < KLLM_DEC_WARPS)
		return KLLM_ENOSPC;
	size_t row = (size_t)base->num_heads * base->head_dim;
	for (int s0 = 0; s0 < S; s0 += per) {
		struct kllm_decode_args a = *base;
		int ns = S - s0 < per ? S - s0 : per;
		a.num_seqs = ns;
		a.q = (const uint8_t *)base->q + (size_t)s0 * row * 2;
		if (a.out)
			a.out = (uint8_t *)base->out + (size_t)s0 * row * 2;
		a.table = (const uint8_t *)base->table +
			  (size_t)s0 * base->max_blocks * sizeof(struct kllm_block_table_entry);
		a.seq_lens = base->seq_lens + s0;
		if (a.pm) {
			a.pm = base->pm + (size_t)s0 * base->num_heads;
			a.pl = base->pl + (size_t)s0 * base->num_heads;
			a.po = base->po + (size_t)s0 * row;
		}
		int rc = decode_chunk(ctx, &a, split, ws_part, ws_cnt, ws_list, max_warps,
				      num_sms, st);
		if (rc)
			return rc;
	}
	return KLLM_OK;
}

static void fill_args(struct kllm_decode_args *a, void *out, const void *q,
		      const void *table, const int *seq_lens, int S, int hq,
		      int hkv, int d, int max_blocks, int bs, int kv,
		      uint64_t layer_off, float scale)
{
	memset(a, 0, sizeof(*a));
	a->out = out;
	a->q = q;
	a->table = table;
	a->seq_lens = seq_lens;
	a->num_seqs = S;
	a->num_heads = hq;
	a->num_kv_heads = hkv;
	a->group = hq / hkv;
	a->head_dim = d;
	a->max_blocks = max_blocks;
	a->block_size = bs;
	a->kv_dtype = kv;
	a->layer_off = layer_off;
	/* log2 domain; MX tiles are dequantised with an extra 2^-8 */
	a->scale_log2 = scale * 1.4426950408889634f *
			(kv == KLLM_KV_MX_FP8_E4M3 ? KLLM_MX_DEC_UNBIAS : 1.0f);
}

/* userspace/gpu/paged_attention.cu:121-146: v1 semantics, BF16 128-token pages. */
int kllm_gpu_paged_attention_cuda(void *output, const void *query,
				  const void *block_tables, const int *seq_lens,
				  int num_seqs, int num_heads, int num_kv_heads,
				  int head_dim, int max_blocks_per_seq,
				  float scale, void *stream)
{
	int rc = check_decode_shape(num_seqs, num_heads, num_kv_heads, head_dim,
				    max_blocks_per_seq, 128, KLLM_KV_BF16);
	if (rc)
		return rc;
	if (num_seqs == 0)
		return KLLM_OK;
	if (!output || !query || !block_tables || !seq_lens)
		return KLLM_EINVAL;
	int dev = 0, sms = 0;
	if (cudaGetDevice(&dev) != cudaSuccess || !usable_device(dev)) {
		(void)cudaGetLastError();
		return KLLM_ENODEV;
	}
	cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
	struct kllm_decode_args a;
	fill_args(&a, output, query, block_tables, seq_lens, num_seqs, num_heads,
		  num_kv_heads, head_dim, max_blocks_per_seq, 128, KLLM_KV_BF16, 0,
		  scale);
	return decode_common(NULL, &a, 0, NULL, 0, NULL, 0, sms, (cudaStream_t)stream);
}

int kllm_gpu_paged_attention(struct kllm_gpu_ctx *ctx,
			     const struct kllm_gpu_attention_params *p)
{
	if (!p)
		return fail(ctx, KLLM_EINVAL);
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	struct kllm_gpu_attention_params_v2 v2;
	memset(&v2, 0, sizeof(v2));
	v2.struct_size = sizeof(v2);
	v2.output = p->output;
	v2.query = p->query;
	v2.block_tables = p->block_tables;
	v2.seq_lens = p->seq_lens;
	v2.num_seqs = p->num_seqs;
	v2.num_heads = p->num_heads;
	v2.num_kv_heads = p->num_kv_heads;
	v2.head_dim = p->head_dim;
	v2.max_blocks_per_seq = p->max_blocks_per_seq;
	v2.block_size = 128;
	v2.kv_dtype = KLLM_KV_BF16;
	v2.scale = p->scale;
	v2.split = 1;
	v2.stream = p->stream;
	return kllm_gpu_paged_attention_v2(ctx, &v2);
}

uint64_t kllm_gpu_decode_workspace_size(struct kllm_gpu_ctx *ctx, int num_seqs,
					int num_kv_heads)
{
	(void)num_seqs;
	(void)num_kv_heads;
	if (!ctx || ctx->backend != KLLM_GPU_CUDA)
		return 0;
	return ctx->ws_part_bytes;
}

int kllm_gpu_paged_attention_v2(struct kllm_gpu_ctx *ctx,
				const struct kllm_gpu_attention_params_v2 *p)
{
	if (!p || p->struct_size < sizeof(*p) || (p->flags & ~KLLM_DECODE_OVERLAP_PREV))
		return fail(ctx, KLLM_EINVAL);
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	int rc = check_decode_shape(p->num_seqs, p->num_heads, p->num_kv_heads,
				    p->head_dim, p->max_blocks_per_seq,
				    p->block_size, p->kv_dtype);
	if (rc)
		return fail(ctx, rc);
	if (p->num_seqs == 0)
		return KLLM_OK;
	int partial = p->partial_m || p->partial_l || p->partial_o;
	if (partial && !(p->partial_m && p->partial_l && p->partial_o))
		return fail(ctx, KLLM_EINVAL);
	if (!p->query || !p->block_tables || !p->seq_lens || (!p->output && !partial))
		return fail(ctx, KLLM_EINVAL);
	if ((p->layer_stride & 15u) || p->layer < 0)
		return fail(ctx, KLLM_EINVAL);
	if (((uintptr_t)p->query | (uintptr_t)p->output) & 15u)
		return fail(ctx, KLLM_EINVAL);
	if (partial && (((uintptr_t)p->partial_o) & 15u))
		return fail(ctx, KLLM_EINVAL);

	int split = p->split >= 0;
	float *wsp = ctx->ws_part;
	uint64_t wsp_bytes = ctx->ws_part_bytes;
	unsigned *cnt = ctx->ws_cnt;
	uint64_t cnt_cap = KLLM_CNT_CAP;
	if (split && p->workspace) {
		/* caller workspace: counters first, then the partial slots and
		 * the merge list; the caller zeroes it once, the kernels leave it
		 * ready for the next call */
		uint64_t cnt_bytes = sizeof(unsigned) * (uint64_t)p->num_seqs * p->num_kv_heads;
		cnt_bytes = (cnt_bytes + 255) & ~255ull;
		if (p->workspace_size <= cnt_bytes)
			return fail(ctx, KLLM_ENOSPC);
		cnt = (unsigned *)p->workspace;
		cnt_cap = (uint64_t)p->num_seqs * p->num_kv_heads;
		wsp = (float *)((uint8_t *)p->workspace + cnt_bytes);
		wsp_bytes = p->workspace_size - cnt_bytes;
	}

	struct kllm_decode_args a;
	fill_args(&a, p->output, p->query, p->block_tables, p->seq_lens,
		  p->num_seqs, p->num_heads, p->num_kv_heads, p->head_dim,
		  p->max_blocks_per_seq, p->block_size, p->kv_dtype,
		  (uint64_t)p->layer * p->layer_stride, p->scale);
	a.pm = p->partial_m;
	a.pl = p->partial_l;
	a.po = p->partial_o;
	a.err = p->err_word;
	a.overlap = (p->flags & KLLM_DECODE_OVERLAP_PREV) != 0;
	a.arenas = ctx->arenas;
	if (partial)
		a.out = NULL;
	cudaStream_t st = pick_stream(ctx, p->stream);
	int tr = trace_begin(ctx, st, KLLM_TRACE_DECODE);
	rc = decode_common(ctx, &a, split, wsp, wsp_bytes, cnt, cnt_cap, ctx->num_sms, st);
	trace_end(ctx, st, tr);
	if (rc)
		return rc == KLLM_EIO ? cuda_fail(ctx, cudaErrorLaunchFailure) : fail(ctx, rc);
	return KLLM_OK;
}

/* ---- append / gather / merge ---------------------------------------------- */

int kllm_gpu_kv_append_v2(struct kllm_gpu_ctx *ctx,
			  const struct kllm_gpu_kv_append_params *p)
{
	if (!p || p->struct_size < sizeof(*p))
		return fail(ctx, KLLM_EINVAL);
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (p->num_tokens < 0 || p->num_seqs <= 0 || p->num_kv_heads <= 0 ||
	    p->max_blocks_per_seq <= 0)
		return fail(ctx, KLLM_EINVAL);
	if (p->head_dim <= 0 || p->head_dim % 8 || p->head_dim > 1024)
		return fail(ctx, KLLM_ENOSYS);
	if (p->block_size <= 0 || p->block_size > 1024)
		return fail(ctx, KLLM_ENOSYS);
	if (p->kv_dtype < KLLM_KV_BF16 || p->kv_dtype > KLLM_KV_MX_BF16_COMPAT)
		return fail(ctx, KLLM_ENOSYS);
	if (p->num_tokens == 0)
		return KLLM_OK;
	if (!p->k || !p->v || !p->token_seq || !p->token_pos || !p->block_tables)
		return fail(ctx, KLLM_EINVAL);
	if ((((uintptr_t)p->k | (uintptr_t)p->v) & 15u) || (p->layer_stride & 15u) || p->layer < 0)
		return fail(ctx, KLLM_EINVAL);
	struct kllm_append_args a;
	memset(&a, 0, sizeof(a));
	a.k = p->k;
	a.v = p->v;
	a.token_seq = p->token_seq;
	a.token_pos = p->token_pos;
	a.num_tokens = p->num_tokens;
	a.num_seqs = p->num_seqs;
	a.table = p->block_tables;
	a.max_blocks = p->max_blocks_per_seq;
	a.num_kv_heads = p->num_kv_heads;
	a.head_dim = p->head_dim;
	a.block_size = p->block_size;
	a.kv_dtype = p->kv_dtype;
	a.layer_off = (uint64_t)p->layer * p->layer_stride;
	a.err = p->err_word;
	a.arenas = ctx->arenas;
	cudaStream_t st = pick_stream(ctx, p->stream);
	int tr = trace_begin(ctx, st, KLLM_TRACE_APPEND);
	int le = kllm_append_launch(&a, st);
	trace_end(ctx, st, tr);
	if (le)
		return cuda_fail(ctx, cudaErrorLaunchFailure);
	ctx->stats.launches++;
	return KLLM_OK;
}

int kllm_gpu_prefill_v2(struct kllm_gpu_ctx *ctx,
			const struct kllm_gpu_prefill_params *p)
{
	if (!p || p->struct_size < sizeof(*p))
		return fail(ctx, KLLM_EINVAL);
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (p->num_seqs < 0 || p->num_tokens < 0 || p->max_chunk < 0 || p->num_heads <= 0 ||
	    p->num_kv_heads <= 0 || p->num_heads % p->num_kv_heads || p->max_blocks_per_seq <= 0)
		return fail(ctx, KLLM_EINVAL);
	int g = p->num_heads / p->num_kv_heads;
	if (p->head_dim != 128 || (g != 1 && g != 2 && g != 4 && g != 8))
		return fail(ctx, KLLM_ENOSYS);
	if (p->block_size < 1 || p->block_size > 1024 ||
	    (p->kv_dtype != KLLM_KV_BF16 && p->kv_dtype != KLLM_KV_MX_FP8_E4M3))
		return fail(ctx, KLLM_ENOSYS);
	if (p->num_seqs == 0 || p->num_tokens == 0)
		return KLLM_OK;
	if (!p->output || !p->q || !p->k || !p->v || !p->cu_seqlens || !p->ctx_lens ||
	    !p->block_tables)
		return fail(ctx, KLLM_EINVAL);
	if ((((uintptr_t)p->q | (uintptr_t)p->k | (uintptr_t)p->v | (uintptr_t)p->output) & 15u) ||
	    (p->layer_stride & 15u) || p->layer < 0)
		return fail(ctx, KLLM_EINVAL);
	cudaStream_t st = pick_stream(ctx, p->stream);
	struct kllm_prefill_args a;
	memset(&a, 0, sizeof(a));
	a.out = p->output;
	a.q = p->q;
	a.k = p->k;
	a.v = p->v;
	a.cu_seqlens = p->cu_seqlens;
	a.ctx_lens = p->ctx_lens;
	a.table = p->block_tables;
	a.max_blocks = p->max_blocks_per_seq;
	a.num_seqs = p->num_seqs;
	a.num_tokens = p->num_tokens;
	a.max_chunk = p->max_chunk;
	a.num_heads = p->num_heads;
	a.num_kv_heads = p->num_kv_heads;
	a.head_dim = p->head_dim;
	a.block_size = p->block_size;
	a.kv_dtype = p->kv_dtype;
	a.layer_off = (uint64_t)p->layer * p->layer_stride;
	a.scale_log2 = p->scale * 1.4426950408889634f;
	a.err = p->err_word;
	a.arenas = ctx->arenas;
	int tr = trace_begin(ctx, st, KLLM_TRACE_PREFILL);
	int le = kllm_prefill_launch(&a, st);
	if (le) {
		trace_end(ctx, st, tr);
		return cuda_fail(ctx, (cudaError_t)le);
	}
	ctx->stats.launches++;
	if (p->append) {
		struct kllm_append_args b;
		memset(&b, 0, sizeof(b));
		b.k = p->k;
		b.v = p->v;
		b.num_tokens = p->num_tokens;
		b.num_seqs = p->num_seqs;
		b.table = p->block_tables;
		b.max_blocks = p->max_blocks_per_seq;
		b.num_kv_heads = p->num_kv_heads;
		b.head_dim = p->head_dim;
		b.block_size = p->block_size;
		b.kv_dtype = p->kv_dtype;
		b.layer_off = a.layer_off;
		b.err = p->err_word;
		b.arenas = ctx->arenas;
		if (kllm_append_chunk_launch(&b, p->cu_seqlens, p->ctx_lens, st)) {
			trace_end(ctx, st, tr);
			return cuda_fail(ctx, cudaErrorLaunchFailure);
		}
		ctx->stats.launches++;
	}
	trace_end(ctx, st, tr);
	return KLLM_OK;
}

int kllm_gpu_gather_debug(struct kllm_gpu_ctx *ctx,
			  const struct kllm_gpu_gather_params *p)
{
	if (!p || p->struct_size < sizeof(*p))
		return fail(ctx, KLLM_EINVAL);
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (p->num_seqs < 0 || p->num_kv_heads <= 0 || p->max_blocks_per_seq <= 0 ||
	    p->head_dim <= 0 || p->head_dim % 8 || p->block_size <= 0)
		return fail(ctx, KLLM_EINVAL);
	if (p->kv_dtype != KLLM_KV_BF16 && p->kv_dtype != KLLM_KV_MX_FP8_E4M3)
		return fail(ctx, KLLM_ENOSYS);
	if (p->num_seqs == 0)
		return KLLM_OK;
	if (!p->k_out || !p->v_out || !p->counts_out || !p->block_tables || !p->seq_lens)
		return fail(ctx, KLLM_EINVAL);
	struct kllm_gather_args a;
	memset(&a, 0, sizeof(a));
	a.k_out = p->k_out;
	a.v_out = p->v_out;
	a.counts = p->counts_out;
	a.table = p->block_tables;
	a.seq_lens = p->seq_lens;
	a.num_seqs = p->num_seqs;
	a.num_kv_heads = p->num_kv_heads;
	a.head_dim = p->head_dim;
	a.max_blocks = p->max_blocks_per_seq;
	a.block_size = p->block_size;
	a.kv_dtype = p->kv_dtype;
	a.layer_off = (uint64_t)p->layer * p->layer_stride;
	if (kllm_gather_launch(&a, pick_stream(ctx, p->stream)))
		return cuda_fail(ctx, cudaErrorLaunchFailure);
	ctx->stats.launches++;
	return KLLM_OK;
}

uint64_t kllm_gpu_table_workspace_size(int num_seqs, int max_blocks_per_seq,
				       int block_size)
{
	if (num_seqs < 0 || max_blocks_per_seq <= 0 || block_size <= 0)
		return 0;
	return (uint64_t)num_seqs *
	       kllm_table_midstate_stride(max_blocks_per_seq, block_size) * 32u;
}

int kllm_gpu_build_block_tables(struct kllm_gpu_ctx *ctx,
				const struct kllm_gpu_table_build_params *p)
{
	if (!p || p->struct_size < sizeof(*p))
		return fail(ctx, KLLM_EINVAL);
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (p->num_seqs < 0 || p->max_blocks_per_seq <= 0 || p->block_size <= 0 ||
	    p->miss_capacity < 0 || p->index_capacity == 0 ||
	    (p->index_capacity & (p->index_capacity - 1)) ||
	    (int64_t)p->max_blocks_per_seq * p->block_size > INT32_MAX)
		return fail(ctx, KLLM_EINVAL);
	if (p->num_seqs == 0)
		return KLLM_OK;
	if (!p->token_ids || !p->token_starts || !p->seq_lens || !p->index ||
	    !p->block_tables || !p->workspace || (p->miss_capacity > 0 && !p->miss_list))
		return fail(ctx, KLLM_EINVAL);
	if (((uintptr_t)p->index | (uintptr_t)p->hashes | (uintptr_t)p->workspace) & 15u ||
	    ((uintptr_t)p->block_tables & 7u) || ((uintptr_t)p->token_ids & 3u))
		return fail(ctx, KLLM_EINVAL);
	if (p->workspace_bytes < kllm_gpu_table_workspace_size(p->num_seqs, p->max_blocks_per_seq,
							       p->block_size))
		return fail(ctx, KLLM_ENOSPC);
	struct kllm_table_args a;
	memset(&a, 0, sizeof(a));
	a.tokens = p->token_ids;
	a.starts = p->token_starts;
	a.seq_lens = p->seq_lens;
	a.first_block = p->first_block;
	a.num_seqs = p->num_seqs;
	a.max_blocks = p->max_blocks_per_seq;
	a.block_size = p->block_size;
	a.index = (uint8_t *)p->index;
	a.capacity = p->index_capacity;
	a.now_ns = p->now_ns;
	a.arena_base = p->arena_base;
	a.slot_bytes = p->slot_bytes;
	a.total_slots = p->total_slots;
	a.k_offset = p->k_offset;
	a.v_offset = p->v_offset;
	a.table = p->block_tables;
	a.hashes = p->hashes;
	a.midstates = (uint32_t *)p->workspace;
	a.ms_stride = kllm_table_midstate_stride(p->max_blocks_per_seq, p->block_size);
	a.miss_list = p->miss_list;
	a.miss_capacity = p->miss_list ? p->miss_capacity : 0;
	a.miss_count = p->miss_count;
	a.hit_miss = (unsigned long long *)p->hit_miss;
	a.err = p->err_word;
	int rc = kllm_table_build_launch(&a, pick_stream(ctx, p->stream));
	if (rc)
		return cuda_fail(ctx, rc);
	ctx->stats.launches += 2;
	return KLLM_OK;
}

uint64_t kllm_gpu_lm_head_workspace_size(int num_rows, int vocab)
{
	if (num_rows <= 0 || vocab <= 0)
		return 0;
	return (uint64_t)num_rows * (uint64_t)kllm_lm_head_tiles(vocab) * 24u + 32u;
}

int kllm_gpu_lm_head_sample(struct kllm_gpu_ctx *ctx, const struct kllm_gpu_lm_head_params *p)
{
	if (!p || p->struct_size < sizeof(*p))
		return fail(ctx, KLLM_EINVAL);
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (p->num_rows <= 0 || p->hidden_dim <= 0 || p->vocab <= 0 || !p->hidden || !p->weight ||
	    !p->tokens || !p->workspace || (p->method && !p->logits))
		return fail(ctx, KLLM_EINVAL);
	if (p->num_rows > 256 || p->hidden_dim % 64)
		return fail(ctx, KLLM_ENOSYS);
	if (((uintptr_t)p->hidden | (uintptr_t)p->weight | (uintptr_t)p->workspace) & 15u)
		return fail(ctx, KLLM_EINVAL);
	if (p->workspace_bytes < kllm_gpu_lm_head_workspace_size(p->num_rows, p->vocab))
		return fail(ctx, KLLM_ENOSPC);
	/* per row: a partial (max, sum, argmax) for every 256-row vocabulary
	 * tile, plus room for the second halves of tiles split in two */
	const uint64_t tiles = 2u * (uint64_t)kllm_lm_head_tiles(p->vocab) * (uint64_t)p->num_rows;
	struct kllm_lm_head_args a;
	memset(&a, 0, sizeof(a));
	a.hidden = p->hidden;
	a.weight = p->weight;
	a.num_rows = p->num_rows;
	a.hidden_dim = p->hidden_dim;
	a.vocab = p->vocab;
	a.logits = p->logits;
	a.method = p->method;
	a.temperature = p->temperature;
	a.top_k = p->top_k;
	a.uniform = p->uniform;
	a.tokens = p->tokens;
	a.part_m = (float *)p->workspace;
	a.part_s = a.part_m + tiles;
	a.part_a = (int *)(a.part_s + tiles);
	a.err = p->err_word;
	int rc = kllm_lm_head_launch(&a, pick_stream(ctx, p->stream));
	if (rc)
		return cuda_fail(ctx, rc);
	ctx->stats.launches += 2;
	return KLLM_OK;
}

int kllm_gpu_merge_partials(struct kllm_gpu_ctx *ctx, const float *m,
			    const float *l, const float *o, int num_parts,
			    int num_rows, int head_dim, void *out, void *stream)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (num_parts <= 0 || num_rows < 0 || head_dim <= 0)
		return fail(ctx, KLLM_EINVAL);
	if (num_rows == 0)
		return KLLM_OK;
	if (!m || !l || !o || !out)
		return fail(ctx, KLLM_EINVAL);
	if (kllm_merge_launch(m, l, o, num_parts, num_rows, head_dim, out,
			      pick_stream(ctx, stream)))
		return cuda_fail(ctx, cudaErrorLaunchFailure);
	ctx->stats.launches++;
	return KLLM_OK;
}

/* ---- NCCL split-KV exchange ------------------------------------------------- */

static int nccl_load(struct nccl_api *api)
{
	if (api->handle)
		return 0;
	void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
	if (!h)
		return -1;
#define NCCL_SYM(field, name) \
	do { *(void **)(&api->field) = dlsym(h, name); if (!api->field) goto bad; } while (0)
	NCCL_SYM(get_unique_id, "ncclGetUniqueId");
	NCCL_SYM(init_rank_config, "ncclCommInitRankConfig");
	NCCL_SYM(get_async_error, "ncclCommGetAsyncError");
	NCCL_SYM(abort_, "ncclCommAbort");
	NCCL_SYM(destroy, "ncclCommDestroy");
	NCCL_SYM(all_gather, "ncclAllGather");
	NCCL_SYM(group_start, "ncclGroupStart");
	NCCL_SYM(group_end, "ncclGroupEnd");
#undef NCCL_SYM
	api->handle = h;
	return 0;
bad:
	dlclose(h);
	memset(api, 0, sizeof(*api));
	return -1;
}

int kllm_gpu_comm_get_unique_id(uint8_t id[128])
{
	struct nccl_api api;
	memset(&api, 0, sizeof(api));
	if (!id)
		return KLLM_EINVAL;
	if (nccl_load(&api))
		return KLLM_ENOSYS;
	ncclUniqueId uid;
	if (api.get_unique_id(&uid) != ncclSuccess)
		return KLLM_EIO;
	memcpy(id, uid.internal, 128);
	return KLLM_OK;
}

/* Polls the communicator until it leaves ncclInProgress or the deadline
 * passes; aborts it on expiry or error. An enqueue finishes in microseconds,
 * so the first 2 ms only yield the CPU between polls; after that the poll
 * sleeps 100 us at a time. */
static int comm_wait(struct kllm_gpu_ctx *ctx, int timeout_ms)
{
	double t0 = now_ms();
	double deadline = t0 + (timeout_ms > 0 ? timeout_ms : 60000);
	for (;;) {
		ncclResult_t st = ncclInProgress;
		if (ctx->nccl.get_async_error(ctx->comm, &st) != ncclSuccess)
			st = ncclSystemError;
		if (st == ncclSuccess)
			return KLLM_OK;
		if (st != ncclInProgress || now_ms() > deadline) {
			ctx->nccl.abort_(ctx->comm);
			ctx->comm = NULL;
			return st == ncclInProgress ? KLLM_ETIMEDOUT : KLLM_EIO;
		}
		if (now_ms() - t0 < 2.0)
			sched_yield();
		else
			nap_us(100);
	}
}

int kllm_gpu_comm_init(struct kllm_gpu_ctx *ctx, int nranks, int rank,
		       const uint8_t id[128], int timeout_ms)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (!id || nranks <= 0 || rank < 0 || rank >= nranks || ctx->comm)
		return fail(ctx, KLLM_EINVAL);
	if (nccl_load(&ctx->nccl))
		return fail(ctx, KLLM_ENOSYS);
	size_t recv_floats = (size_t)nranks * KLLM_COMM_ROWS_CAP * (KLLM_COMM_DIM_CAP + 2);
	if (cudaMalloc((void **)&ctx->comm_recv, recv_floats * sizeof(float)) != cudaSuccess)
		return cuda_fail(ctx, cudaErrorMemoryAllocation);

	ncclUniqueId uid;
	memcpy(uid.internal, id, 128);
	ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
	cfg.blocking = 0;
	ncclResult_t r = ctx->nccl.init_rank_config(&ctx->comm, nranks, uid, rank, &cfg);
	if (r != ncclSuccess && r != ncclInProgress) {
		cudaFree(ctx->comm_recv);
		ctx->comm_recv = NULL;
		ctx->comm = NULL;
		return fail(ctx, KLLM_EIO);
	}
	int rc = comm_wait(ctx, timeout_ms);
	if (rc) {
		cudaFree(ctx->comm_recv);
		ctx->comm_recv = NULL;
		return fail(ctx, rc);
	}
	ctx->nranks = nranks;
	ctx->rank = rank;
	return KLLM_OK;
}

int kllm_gpu_comm_merge(struct kllm_gpu_ctx *ctx, const float *m,
			const float *l, const float *o, int num_rows,
			int head_dim, void *out, void *stream, int timeout_ms)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (!ctx->comm)
		return fail(ctx, KLLM_EINVAL);
	if (num_rows <= 0 || num_rows > KLLM_COMM_ROWS_CAP || head_dim <= 0 ||
	    head_dim > KLLM_COMM_DIM_CAP || !m || !l || !o || !out)
		return fail(ctx, KLLM_EINVAL);
	cudaStream_t st = pick_stream(ctx, stream);
	int n = ctx->nranks;
	float *rm = ctx->comm_recv;
	float *rl = rm + (size_t)n * num_rows;
	float *ro = rl + (size_t)n * num_rows;

	ncclResult_t r = ctx->nccl.group_start();
	if (r == ncclSuccess) {
		ctx->nccl.all_gather(m, rm, (size_t)num_rows, ncclFloat32, ctx->comm, st);
		ctx->nccl.all_gather(l, rl, (size_t)num_rows, ncclFloat32, ctx->comm, st);
		ctx->nccl.all_gather(o, ro, (size_t)num_rows * head_dim, ncclFloat32, ctx->comm, st);
		r = ctx->nccl.group_end();
	}
	if (r != ncclSuccess && r != ncclInProgress)
		return fail(ctx, KLLM_EIO);
	if (r == ncclInProgress) {
		int rc = comm_wait(ctx, timeout_ms);
		if (rc)
			return fail(ctx, rc);
	}
	if (kllm_merge_launch(rm, rl, ro, n, num_rows, head_dim, out, st))
		return cuda_fail(ctx, cudaErrorLaunchFailure);
	ctx->stats.launches++;
	if (timeout_ms > 0) {
		double deadline = now_ms() + timeout_ms;
		for (;;) {
			cudaError_t e = cudaStreamQuery(st);
			if (e == cudaSuccess)
				break;
			if (e != cudaErrorNotReady)
				return cuda_fail(ctx, e);
			ncclResult_t as = ncclSuccess;
			ctx->nccl.get_async_error(ctx->comm, &as);
			if ((as != ncclSuccess && as != ncclInProgress) || now_ms() > deadline) {
				ctx->nccl.abort_(ctx->comm);
				ctx->comm = NULL;
				return fail(ctx, as == ncclSuccess || as == ncclInProgress ?
						     KLLM_ETIMEDOUT : KLLM_EIO);
			}
			sched_yield();
		}
	}
	return KLLM_OK;
}

void kllm_gpu_comm_destroy(struct kllm_gpu_ctx *ctx)
{
	if (!ctx)
		return;
	if (ctx->comm && ctx->nccl.destroy)
		ctx->nccl.destroy(ctx->comm);
	ctx->comm = NULL;
	if (ctx->comm_recv)
		cudaFree(ctx->comm_recv);
	ctx->comm_recv = NULL;
}

/* ---- peer-memory split-KV exchange ---------------------------------------- */

int kllm_gpu_p2p_export(struct kllm_gpu_ctx *ctx, int max_rows, int head_dim,
			uint8_t handle[KLLM_P2P_HANDLE_BYTES])
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (!handle || max_rows <= 0 || max_rows > 65536 || (head_dim != 64 && head_dim != 128) ||
	    ctx->p2p_buf)
		return fail(ctx, KLLM_EINVAL);
	const int rows = (max_rows + 3) & ~3;   /* 16-byte aligned rows of the slots */
	const size_t bytes = kllm_p2p_buffer_bytes(rows, head_dim);
	cudaError_t e = cudaMalloc((void **)&ctx->p2p_buf, bytes);
	if (e != cudaSuccess) {
		ctx->p2p_buf = NULL;
		return cuda_fail(ctx, e);
	}
	e = cudaMemset(ctx->p2p_buf, 0, bytes);
	cudaIpcMemHandle_t h;
	if (e == cudaSuccess)
		e = cudaIpcGetMemHandle(&h, ctx->p2p_buf);
	if (e != cudaSuccess) {
		cudaFree(ctx->p2p_buf);
		ctx->p2p_buf = NULL;
		return cuda_fail(ctx, e);
	}
	memcpy(handle, &h, KLLM_P2P_HANDLE_BYTES);
	ctx->p2p_max_rows = rows;
	ctx->p2p_head_dim = head_dim;
	ctx->p2p_epoch = 0;
	return KLLM_OK;
}

int kllm_gpu_p2p_import(struct kllm_gpu_ctx *ctx, int nranks, int rank,
			const uint8_t *handles)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (!ctx->p2p_buf || !handles || nranks < 1 || nranks > KLLM_P2P_MAX_RANKS || rank < 0 ||
	    rank >= nranks || ctx->p2p_peers_dev)
		return fail(ctx, KLLM_EINVAL);
	memset(ctx->p2p_peer, 0, sizeof(ctx->p2p_peer));
	for (int q = 0; q < nranks; ++q) {
		if (q == rank) {
			ctx->p2p_peer[q] = ctx->p2p_buf;
			continue;
		}
		cudaIpcMemHandle_t h;
		memcpy(&h, handles + (size_t)q * KLLM_P2P_HANDLE_BYTES, KLLM_P2P_HANDLE_BYTES);
		void *p = NULL;
		cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
		if (e != cudaSuccess) {
			for (int k = 0; k < q; ++k)
				if (k != rank && ctx->p2p_peer[k])
					cudaIpcCloseMemHandle(ctx->p2p_peer[k]);
			memset(ctx->p2p_peer, 0, sizeof(ctx->p2p_peer));
			return cuda_fail(ctx, e);
		}
		ctx->p2p_peer[q] = (uint8_t *)p;
	}
	cudaError_t e = cudaMalloc((void **)&ctx->p2p_peers_dev, sizeof(uint8_t *) * nranks);
	if (e == cudaSuccess)
		e = cudaMemcpy(ctx->p2p_peers_dev, ctx->p2p_peer, sizeof(uint8_t *) * nranks,
			       cudaMemcpyHostToDevice);
	if (e != cudaSuccess)
		return cuda_fail(ctx, e);
	ctx->p2p_nranks = nranks;
	ctx->p2p_rank = rank;
	return KLLM_OK;
}

int kllm_gpu_p2p_merge(struct kllm_gpu_ctx *ctx, const float *m, const float *l,
		       const float *o, int num_rows, int head_dim, void *out,
		       uint32_t *err_word, int timeout_ms, void *stream)
{
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (!ctx->p2p_peers_dev || !m || !l || !o || !out || num_rows <= 0 ||
	    num_rows > ctx->p2p_max_rows || head_dim != ctx->p2p_head_dim ||
	    ((uintptr_t)o & 15u))
		return fail(ctx, KLLM_EINVAL);
	struct kllm_p2p_args a;
	memset(&a, 0, sizeof(a));
	a.peers = ctx->p2p_peers_dev;
	a.rank = ctx->p2p_rank;
	a.nranks = ctx->p2p_nranks;
	a.epoch = ++ctx->p2p_epoch;
	a.num_rows = num_rows;
	a.max_rows = ctx->p2p_max_rows;
	a.head_dim = head_dim;
	a.m = m;
	a.l = l;
	a.o = o;
	a.out = out;
	a.err = err_word;
	a.timeout_ns = (uint64_t)(timeout_ms > 0 ? timeout_ms : 2000) * 1000000ull;
	if (kllm_p2p_merge_launch(&a, pick_stream(ctx, stream)))
		return cuda_fail(ctx, cudaErrorLaunchFailure);
	ctx->stats.launches++;
	return KLLM_OK;
}

void kllm_gpu_p2p_destroy(struct kllm_gpu_ctx *ctx)
{
	if (!ctx)
		return;
	for (int q = 0; q < KLLM_P2P_MAX_RANKS; ++q)
		if (ctx->p2p_peer[q] && ctx->p2p_peer[q] != ctx->p2p_buf)
			cudaIpcCloseMemHandle(ctx->p2p_peer[q]);
	memset(ctx->p2p_peer, 0, sizeof(ctx->p2p_peer));
	if (ctx->p2p_peers_dev)
		cudaFree(ctx->p2p_peers_dev);
	if (ctx->p2p_buf)
		cudaFree(ctx->p2p_buf);
	ctx->p2p_peers_dev = NULL;
	ctx->p2p_buf = NULL;
	ctx->p2p_nranks = 0;
}

/* ---- registered arenas ------------------------------------------------------ */

int kllm_gpu_register_arena(struct kllm_gpu_ctx *ctx, const void *base, uint64_t bytes)
{
	if (!ctx)
		return KLLM_EINVAL;
	if (!base || !bytes || (uint64_t)(uintptr_t)base + bytes < (uint64_t)(uintptr_t)base)
		return fail(ctx, KLLM_EINVAL);
	if (ctx->arenas.count >= KLLM_MAX_ARENAS)
		return fail(ctx, KLLM_ENOSPC);
	int n = ctx->arenas.count;
	ctx->arenas.lo[n] = (unsigned long long)(uintptr_t)base;
	ctx->arenas.hi[n] = (unsigned long long)(uintptr_t)base + bytes;
	ctx->arenas.count = n + 1;
	return KLLM_OK;
}

void kllm_gpu_clear_arenas(struct kllm_gpu_ctx *ctx)
{
	if (ctx)
		memset(&ctx->arenas, 0, sizeof(ctx->arenas));
}

/* ---- per-call GPU timing ----------------------------------------------------- */

int kllm_gpu_trace_enable(struct kllm_gpu_ctx *ctx, int capacity)
{
	if (!ctx || capacity < 0 || capacity > KLLM_TRACE_MAX)
		return fail(ctx, KLLM_EINVAL);
	if (!ready(ctx))
		return fail(ctx, KLLM_ENODEV);
	if (cudaSetDevice(ctx->device) != cudaSuccess)
		return cuda_fail(ctx, cudaGetLastError());
	/* records still queued are dropped with the old ring */
	if (ctx->trace) {
		cudaStreamSynchronize(ctx->stream);
		trace_free(ctx);
	}
	if (capacity == 0)
		return KLLM_OK;
	struct trace_slot *t = calloc((size_t)capacity, sizeof(*t));
	if (!t)
		return fail(ctx, KLLM_ENOMEM);
	for (int i = 0; i < capacity; i++) {
		if (cudaEventCreate(&t[i].ev0) != cudaSuccess ||
		    cudaEventCreate(&t[i].ev1) != cudaSuccess) {
			(void)cudaGetLastError();
			for (int k = 0; k <= i; k++) {
				if (t[k].ev0)
					cudaEventDestroy(t[k].ev0);
				if (t[k].ev1)
					cudaEventDestroy(t[k].ev1);
			}
			free(t);
			return fail(ctx, KLLM_ENOMEM);
		}
	}
	ctx->trace = t;
	ctx->trace_cap = capacity;
	ctx->trace_head = ctx->trace_tail = ctx->trace_dropped = 0;
	return KLLM_OK;
}

void kllm_gpu_trace_tag(struct kllm_gpu_ctx *ctx, uint64_t tag)
{
	if (ctx)
		ctx->trace_tag = tag;
}

int kllm_gpu_trace_read(struct kllm_gpu_ctx *ctx, struct kllm_gpu_trace_record *out,
			int max_records, uint64_t *dropped)
{
	if (!ctx || (!out && max_records > 0) || max_records < 0)
		return KLLM_EINVAL;
	if (dropped)
		*dropped = ctx->trace_dropped;
	if (!ctx->trace)
		return 0;
	int n = 0;
	while (n < max_records && ctx->trace_tail < ctx->trace_head) {
		struct trace_slot *t = &ctx->trace[ctx->trace_tail % (uint64_t)ctx->trace_cap];
		cudaError_t q = cudaEventQuery(t->ev1);
		if (q == cudaErrorNotReady)
			break;                   /* in order: later calls are not done either */
		float ms = 0.f;
		if (q != cudaSuccess || cudaEventElapsedTime(&ms, t->ev0, t->ev1) != cudaSuccess) {
			(void)cudaGetLastError();
			ms = -1.f;
		}
		out[n].seq = ctx->trace_tail;
		out[n].tag = t->tag;
		out[n].submit_ns = t->submit_ns;
		out[n].op = t->op;
		out[n].gpu_us = ms < 0.f ? -1.f : ms * 1000.f;
		n++;
		ctx->trace_tail++;
	}
	return n;
}
