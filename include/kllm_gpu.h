/* SPDX-License-Identifier: Apache-2.0 */
/*
 * kllm_gpu.h - C ABI of the B200 (sm_100a) paged-attention backend.
 *
 * Part 1 is the xpu-kllm GPU backend interface, kept symbol-for-symbol and
 * signature-for-signature so existing callers (compute/infer_gpu.c) link
 * against this library unchanged:
 *     userspace/gpu/gpu_attention.h:19-24   enum kllm_gpu_backend
 *     userspace/gpu/gpu_attention.h:26-38   struct kllm_gpu_attention_params
 *     userspace/gpu/gpu_attention.h:43-62   create/destroy/get_backend/
 *                                           paged_attention/malloc/free/
 *                                           memcpy_h2d/get_stream
 *     userspace/gpu/gpu_attention.h:70-73   kllm_gpu_paged_attention_cuda
 *     userspace/gpu/paged_attention.cu:18-22 struct block_table_entry
 *
 * Part 2 adds versioned entry points the reference lacks: 16-token pages,
 * the MX-FP8 KV format, split-KV partial outputs, KV append with
 * quantize-on-write, the partial merge, chunked prefill, a bit-exact gather
 * for tests and the NCCL split-KV exchange.
 *
 * Conventions (all calls):
 *   - every pointer inside a params struct is a DEVICE pointer unless the
 *     field comment says otherwise;
 *   - `stream` is a cudaStream_t; NULL selects the context's own stream
 *     (userspace/gpu/gpu_attention.c:82);
 *   - launches are asynchronous; 0 means "launched", a negative value is one
 *     of the KLLM_E* codes below and nothing was launched;
 *   - no call allocates device memory except kllm_gpu_create and
 *     kllm_gpu_malloc.
 */
#ifndef KLLM_GPU_H
#define KLLM_GPU_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Part 1: reference interface (userspace/gpu/gpu_attention.h)              */
/* ------------------------------------------------------------------------ */

/* userspace/gpu/gpu_attention.h:19-24. This backend reports KLLM_GPU_CUDA on
 * an sm_100 device and KLLM_GPU_NONE otherwise. */
enum kllm_gpu_backend {
	KLLM_GPU_NONE = 0,
	KLLM_GPU_XE,
	KLLM_GPU_CUDA,
	KLLM_GPU_ROCM,
};

/* userspace/gpu/gpu_attention.h:26-38, unchanged. Semantics of the v1 call:
 * BF16 Q/O [num_seqs][num_heads][head_dim]; BF16 K/V pages of 128 tokens laid
 * out [num_kv_heads][128][head_dim] (userspace/gpu/paged_attention.cu:14,62-65);
 * head_dim must be 64 or 128. */
struct kllm_gpu_attention_params {
	void *output;             /* device ptr: [num_seqs, num_heads, head_dim] bf16 */
	const void *query;        /* device ptr */
	const void *block_tables; /* device ptr: block_table_entry array */
	const int *seq_lens;      /* device ptr */
	int num_seqs;
	int num_heads;
	int num_kv_heads;
	int head_dim;
	int max_blocks_per_seq;
	float scale;
	void *stream;             /* cudaStream_t */
};

/* userspace/gpu/paged_attention.cu:18-22: one page descriptor, 24 bytes.
 * An entry with valid == 0 or k_ptr == NULL is skipped, as in the reference
 * kernel (paged_attention.cu:59-60). Page pointers must be 16-byte aligned. */
struct kllm_block_table_entry {
	void *k_ptr;
	void *v_ptr;
	int valid;
};

struct kllm_gpu_ctx;

/* userspace/gpu/gpu_attention.h:43. Binds the device named by the env var
 * KLLM_GPU_DEVICE (default: the current device), creates a non-blocking
 * stream and a split-KV workspace. Returns a context whose backend is
 * KLLM_GPU_NONE when no sm_100 device is usable; every compute call on such a
 * context returns KLLM_ENODEV. Returns NULL only on host allocation failure. */
struct kllm_gpu_ctx *kllm_gpu_create(void);
/* userspace/gpu/gpu_attention.h:44 */
void kllm_gpu_destroy(struct kllm_gpu_ctx *ctx);
/* userspace/gpu/gpu_attention.h:47 */
enum kllm_gpu_backend kllm_gpu_get_backend(struct kllm_gpu_ctx *ctx);
/* userspace/gpu/gpu_attention.h:50-51. Same semantics as
 * kllm_gpu_paged_attention_cuda, but uses the context's split-KV workspace,
 * so long contexts are spread over every SM. */
int kllm_gpu_paged_attention(struct kllm_gpu_ctx *ctx,
			     const struct kllm_gpu_attention_params *params);
/* userspace/gpu/gpu_attention.h:54-55 (the reference stubs return NULL). */
void *kllm_gpu_malloc(struct kllm_gpu_ctx *ctx, uint64_t size);
void kllm_gpu_free(struct kllm_gpu_ctx *ctx, void *ptr);
/* userspace/gpu/gpu_attention.h:58-59: synchronous host-to-device copy
 * (the reference stub returns -1). */
int kllm_gpu_memcpy_h2d(struct kllm_gpu_ctx *ctx, void *dst,
			const void *src, uint64_t size);
/* userspace/gpu/gpu_attention.h:62: the context's cudaStream_t. */
void *kllm_gpu_get_stream(struct kllm_gpu_ctx *ctx);

/* userspace/gpu/gpu_attention.h:70-73 (defined at paged_attention.cu:121-146).
 * Stateless launcher: needs no context and no workspace; every
 * (seq, kv_head) pair is processed whole by one warp, as in the reference
 * launch shape. Returns 0 when the launch was accepted, negative otherwise. */
int kllm_gpu_paged_attention_cuda(
    void *output, const void *query, const void *block_tables,
    const int *seq_lens, int num_seqs, int num_heads, int num_kv_heads,
    int head_dim, int max_blocks_per_seq, float scale, void *stream);

/* ------------------------------------------------------------------------ */
/* Part 2: additions                                                         */
/* ------------------------------------------------------------------------ */

/* Error codes (negative errno values). */
#define KLLM_OK          0
#define KLLM_EIO        (-5)    /* CUDA runtime / NCCL error */
#define KLLM_ENOMEM     (-12)
#define KLLM_ENODEV     (-19)   /* no usable sm_100 device */
#define KLLM_EINVAL     (-22)   /* bad argument */
#define KLLM_ENOSPC     (-28)   /* workspace too small */
#define KLLM_ENOSYS     (-38)   /* shape not supported by this build */
#define KLLM_ETIMEDOUT  (-110)  /* bounded host wait expired */

/* Bits the kernels OR into *err_word (when given) instead of trapping. */
#define KLLM_ERR_SEQ_TOO_LONG   0x1u  /* seq_len > max_blocks_per_seq * block_size: clamped */
#define KLLM_ERR_MISALIGNED     0x2u  /* page pointer not 16-byte aligned: page skipped */
#define KLLM_ERR_APPEND_NOPAGE  0x4u  /* append target page invalid / position out of table */
#define KLLM_ERR_TIMEOUT        0x8u  /* a bounded device-side wait expired; the warp stopped */
#define KLLM_ERR_TOPK_RANGE     0x10u /* lm_head: top_k in (1024, vocab): token -1 for that row */
#define KLLM_ERR_PAGE_RANGE     0x40u /* a page outside every arena registered with
                                        kllm_gpu_register_arena: skipped, never read
                                        or written */
#define KLLM_ERR_NONFINITE      0x20u /* decode: an MX-FP8 page holds payload 0x7F / 0xFF and the
                                        segment could not be recomputed exactly (split < 0, or
                                        the wide-merge queue was full): its rows are not finite */

/* KV page formats. One page holds `block_size` tokens of one layer.
 *
 * KLLM_KV_BF16: K page = [num_kv_heads][block_size][head_dim] bf16, V alike.
 *
 * KLLM_KV_MX_FP8_E4M3: K page = num_kv_heads head sections; each section is
 *   [block_size][head_dim] E4M3 payload bytes followed by
 *   [block_size][head_dim/8] E4M3 scale bytes (one scale per 8 consecutive
 *   elements along head_dim, userspace/compute/mx_dequant.h:27). Real value =
 *   e4m3(payload) * e4m3(scale), decoded as userspace/compute/mx_dequant.h:30-55
 *   (0x7F/0xFF decode to +-480). The append never writes payload 0x7F/0xFF;
 *   the decode's tile loop converts with the hardware OCP E4M3 conversion,
 *   which reads them as NaN, and a segment where that happened is recomputed
 *   exactly (with split >= 0; see KLLM_ERR_NONFINITE). V page alike.
 *
 * KLLM_KV_MX_BF16_COMPAT: the reference's own MX layout
 *   (userspace/compute/mx_dequant.h:10-16): sections of [block_size][head_dim]
 *   bf16 payload followed by [block_size][head_dim/8] scale bytes, written by
 *   the reference quantizer mx_quant_to_bf16 (mx_dequant.h:105-136). Append
 *   only (the reference never reads it on a GPU). */
enum kllm_kv_dtype {
	KLLM_KV_BF16 = 0,
	KLLM_KV_MX_FP8_E4M3 = 1,
	KLLM_KV_MX_BF16_COMPAT = 2,
};

/* kllm_gpu_attention_params_v2.flags */
/* The decode may begin while the kernel issued just before it on the same
 * stream is still finishing (programmatic dependent launch): it reads
 * block_tables and seq_lens before that kernel has completed, and the query,
 * the pages and every output only after. Set it only when that previous
 * kernel writes neither block_tables nor seq_lens (for example consecutive
 * layers of one step, or a KV append followed by the decode); it hides most
 * of the launch and set-up time of each layer's decode. */
#define KLLM_DECODE_OVERLAP_PREV 0x1u

/* Decode attention, versioned. Zero-initialise, set struct_size, fill in. */
struct kllm_gpu_attention_params_v2 {
	uint32_t struct_size;        /* sizeof(struct kllm_gpu_attention_params_v2) */
	uint32_t flags;              /* 0 or KLLM_DECODE_OVERLAP_PREV */
	void *output;                /* bf16 [num_seqs][num_heads][head_dim]; may be NULL
	                                when partial_m/l/o are given */
	const void *query;           /* bf16 [num_seqs][num_heads][head_dim] */
	const void *block_tables;    /* kllm_block_table_entry [num_seqs][max_blocks_per_seq] */
	const int *seq_lens;         /* int32 [num_seqs]: tokens of context (<= 0: empty) */
	int num_seqs;
	int num_heads;               /* query heads */
	int num_kv_heads;            /* num_heads % num_kv_heads == 0, ratio <= 8 */
	int head_dim;                /* 64 or 128 */
	int max_blocks_per_seq;
	int block_size;              /* tokens per page: 16, 32, 64 or 128 */
	int kv_dtype;                /* KLLM_KV_BF16 or KLLM_KV_MX_FP8_E4M3 */
	int layer;                   /* page offset = layer * layer_stride bytes */
	uint64_t layer_stride;       /* multiple of 16 */
	float scale;                 /* softmax scale (1/sqrt(head_dim) typically) */
	int split;                   /* 1 (default when 0): balance tiles over every SM with
	                                split-KV; -1: one warp per (seq, kv_head), no workspace */
	/* Optional split-KV triples, fp32, one per (seq, query head), for a
	 * cross-GPU merge (kllm_gpu_merge_partials): m = max of scale*q.k (natural
	 * log domain), l = sum exp(scale*q.k - m), o = normalised output
	 * [num_seqs][num_heads][head_dim]. An empty context gives m = -inf, l = 0,
	 * o = 0. All three or none. */
	float *partial_m;
	float *partial_l;
	float *partial_o;
	uint32_t *err_word;          /* optional; KLLM_ERR_* bits are OR-ed in */
	void *workspace;             /* optional; NULL = the context's workspace. A
	                                caller workspace is zero-filled once before
	                                its first use; calls leave it reusable */
	uint64_t workspace_size;
	void *stream;
};

int kllm_gpu_paged_attention_v2(struct kllm_gpu_ctx *ctx,
				const struct kllm_gpu_attention_params_v2 *p);

/* Allocation-free variant of kllm_gpu_paged_attention_v2 (no counterpart in
 * the reference). For callers that must not allocate device memory, such as
 * a polling reactor thread that runs with a zero-allocation rule: cudaMalloc
 * can stall it and can fail once the KV arena owns the GPU's memory, and a
 * context cannot be created there because kllm_gpu_create allocates its
 * workspace. Needs no context; the caller passes inputs and outputs (the
 * device is the one `stream` belongs to, or the current device when stream
 * is NULL). Split-KV scratch lives in a fixed 16 MiB device array inside the
 * library, present on every GPU that loads it until the process exits.
 * Set-up: the first call on a device loads the library's decode code and
 * that array onto the device (CUDA loads device code lazily, which may need
 * device memory) and looks up the array's address (a runtime query). A call
 * with num_seqs == 0 does only this: make one per device at start-up,
 * before the KV arena is allocated and before any stream capture on that
 * device. Every call shares the array, so calls that overlap on the GPU
 * race; serialise them. Limit: num_seqs * num_kv_heads <= 65536, else
 * KLLM_ENOSPC. split < 0 runs one warp per (seq, kv head) and uses no
 * scratch. The caller's current device is unchanged on return. The
 * workspace fields of *p are ignored. */
int kllm_gpu_paged_attention_v2_noalloc(
    const struct kllm_gpu_attention_params_v2 *p);

/* Bytes of workspace a split-KV decode needs on this context's device. */
uint64_t kllm_gpu_decode_workspace_size(struct kllm_gpu_ctx *ctx, int num_seqs,
					int num_kv_heads);

/* KV append with quantize-on-write. Token i (row i of k/v) goes to position
 * token_pos[i] of sequence token_seq[i]: page = block_tables[seq][pos /
 * block_size], slot = pos % block_size. Rows whose sequence or position is out
 * of the table, or whose page entry is invalid, are skipped and flagged with
 * KLLM_ERR_APPEND_NOPAGE.
 *   BF16:            bytes copied.
 *   MX_FP8_E4M3:     per 8 elements: amax; scale = smallest E4M3 >= amax/448
 *                    (0 when amax == 0); payload = RNE-satfinite E4M3 of
 *                    x / scale (0 when amax == 0).
 *   MX_BF16_COMPAT:  mx_quant_to_bf16 (userspace/compute/mx_dequant.h:105-136),
 *                    bit for bit, including its constant scale byte. */
struct kllm_gpu_kv_append_params {
	uint32_t struct_size;
	uint32_t flags;
	const void *k;               /* bf16 [num_tokens][num_kv_heads][head_dim] */
	const void *v;               /* bf16 [num_tokens][num_kv_heads][head_dim] */
	const int *token_seq;        /* int32 [num_tokens] */
	const int *token_pos;        /* int32 [num_tokens] */
	int num_tokens;
	int num_seqs;                /* rows of block_tables; token_seq outside
	                                [0, num_seqs) is skipped and flagged */
	const void *block_tables;    /* kllm_block_table_entry [num_seqs][max_blocks_per_seq] */
	int max_blocks_per_seq;
	int num_kv_heads;
	int head_dim;
	int block_size;
	int kv_dtype;
	int layer;
	uint64_t layer_stride;
	uint32_t *err_word;
	void *stream;
};

int kllm_gpu_kv_append_v2(struct kllm_gpu_ctx *ctx,
			  const struct kllm_gpu_kv_append_params *p);

/* Bit-exact logical view of the paged cache, for tests: for every
 * (seq, kv_head) the valid tokens in order (invalid pages skipped, the last
 * page cut at seq_len), dequantised to bf16 exactly (an E4M3 x E4M3 product
 * is exact in bf16), written to k_out/v_out [num_seqs][num_kv_heads]
 * [max_blocks_per_seq*block_size][head_dim]; counts_out [num_seqs]
 * [num_kv_heads] receives the token counts. Rows past the count are zeroed. */
struct kllm_gpu_gather_params {
	uint32_t struct_size;
	uint32_t flags;
	void *k_out;
	void *v_out;
	int *counts_out;
	const void *block_tables;
	const int *seq_lens;
	int num_seqs;
	int num_kv_heads;
	int head_dim;
	int max_blocks_per_seq;
	int block_size;
	int kv_dtype;                /* KLLM_KV_BF16 or KLLM_KV_MX_FP8_E4M3 */
	int layer;
	uint64_t layer_stride;
	void *stream;
};

int kllm_gpu_gather_debug(struct kllm_gpu_ctx *ctx,
			  const struct kllm_gpu_gather_params *p);

/* Chunked prefill (no counterpart in the reference GPU path, which has no
 * prefill; the math is userspace/compute/ace_attention.c:85-134 per query row
 * with keys [0, position]). The chunks of num_seqs sequences are packed
 * token-major: sequence s owns rows cu_seqlens[s] .. cu_seqlens[s+1]-1 of
 * q/k/v/output. Query j of sequence s sits at position ctx_lens[s] + j and
 * attends to the sequence's first ctx_lens[s] tokens, read from the paged
 * cache through the block table (pages of block_size tokens, kv_dtype BF16
 * or MX-FP8, invalid pages skipped), and to chunk keys 0..j (causal).
 * head_dim 128; num_heads / num_kv_heads in {1, 2, 4, 8}. max_chunk bounds
 * every chunk length (it sizes the grid). append = 1 also writes the chunk's
 * K/V into the cache at positions ctx_lens[s] + j (quantize-on-write, as
 * kllm_gpu_kv_append_v2). Runs on the tcgen05 tensor cores. */
struct kllm_gpu_prefill_params {
	uint32_t struct_size;
	uint32_t flags;
	void *output;                /* bf16 [num_tokens][num_heads][head_dim] */
	const void *q;               /* bf16 [num_tokens][num_heads][head_dim] */
	const void *k;               /* bf16 [num_tokens][num_kv_heads][head_dim] */
	const void *v;               /* bf16 [num_tokens][num_kv_heads][head_dim] */
	const int *cu_seqlens;       /* int32 [num_seqs + 1], cu_seqlens[0] = 0 */
	const int *ctx_lens;         /* int32 [num_seqs] */
	int num_seqs;
	int num_tokens;              /* cu_seqlens[num_seqs] */
	int max_chunk;
	int num_heads;
	int num_kv_heads;
	int head_dim;
	const void *block_tables;    /* kllm_block_table_entry [num_seqs][max_blocks_per_seq] */
	int max_blocks_per_seq;
	int block_size;
	int kv_dtype;
	int layer;
	uint64_t layer_stride;
	float scale;
	int append;
	uint32_t *err_word;
	void *stream;
};

int kllm_gpu_prefill_v2(struct kllm_gpu_ctx *ctx,
			const struct kllm_gpu_prefill_params *p);

/* LSE merge of split-KV triples: for each of num_rows rows (seq x query
 * head), M = max_i m_i, w_i = l_i exp(m_i - M), out = sum_i w_i o_i / sum_i w_i
 * (0 when every l_i is 0). Inputs are stacked by part: m/l [num_parts]
 * [num_rows], o [num_parts][num_rows][head_dim]. out: bf16 [num_rows]
 * [head_dim]. */
int kllm_gpu_merge_partials(struct kllm_gpu_ctx *ctx, const float *m,
			    const float *l, const float *o, int num_parts,
			    int num_rows, int head_dim, void *out, void *stream);

/* Synchronous device-to-host copy (counterpart of kllm_gpu_memcpy_h2d). */
int kllm_gpu_memcpy_d2h(struct kllm_gpu_ctx *ctx, void *dst,
			const void *src, uint64_t size);
/* Asynchronous copies on `stream` (NULL: the context stream). */
int kllm_gpu_memcpy_h2d_async(struct kllm_gpu_ctx *ctx, void *dst,
			      const void *src, uint64_t size, void *stream);
int kllm_gpu_memcpy_d2h_async(struct kllm_gpu_ctx *ctx, void *dst,
			      const void *src, uint64_t size, void *stream);
/* Page-locked host memory for the async copies. */
void *kllm_gpu_host_alloc(struct kllm_gpu_ctx *ctx, uint64_t size);
void kllm_gpu_host_free(struct kllm_gpu_ctx *ctx, void *ptr);
/* Waits for the context stream; returns KLLM_ETIMEDOUT after timeout_ms
 * milliseconds (<= 0: wait without limit). */
int kllm_gpu_synchronize(struct kllm_gpu_ctx *ctx, int timeout_ms);

struct kllm_gpu_stats {
	uint64_t launches;           /* kernels launched through this context */
	uint64_t kv_bytes;           /* algorithmic KV bytes of decode launches
	                                (valid pages x bytes per page, host estimate) */
	uint64_t errors;             /* calls that returned an error */
	int last_error;              /* last negative return code */
	int device;                  /* CUDA ordinal */
	int num_sms;
	int last_cuda_error;         /* cudaError_t behind the last KLLM_EIO (0: none) */
};
int kllm_gpu_get_stats(struct kllm_gpu_ctx *ctx, struct kllm_gpu_stats *out);

/* Page range checks (no counterpart in the reference, whose kernel checks
 * only valid / NULL, userspace/gpu/paged_attention.cu:59-60). Registers
 * [base, base + bytes) as a KV arena of this context (up to 8). While any
 * arena is registered, the decode, append and prefill launched through this
 * context check every page a block-table entry names: a page (the kv head
 * section read, or the whole page written) outside all arenas is skipped
 * and KLLM_ERR_PAGE_RANGE is OR-ed into err_word. Nothing traps. */
int kllm_gpu_register_arena(struct kllm_gpu_ctx *ctx, const void *base, uint64_t bytes);
void kllm_gpu_clear_arenas(struct kllm_gpu_ctx *ctx);

/* Per-call GPU timing for the tracer's GPU_SUBMIT / GPU_COMPLETE stages
 * (bpf/kllm_trace.bpf.c:37-38, which nothing in the reference emits). With
 * tracing enabled (kllm_gpu_trace_enable, or KLLM_GPU_TRACE=<capacity> in the
 * environment at kllm_gpu_create), every decode, append and prefill call
 * through the context records a CUDA event pair around its launches; the
 * events are created when tracing is enabled, none in the call. An event
 * between two decodes keeps the second from overlapping the first
 * (KLLM_DECODE_OVERLAP_PREV), so tracing costs some throughput.
 * kllm_gpu_trace_read returns completed records in call order without
 * blocking; calls made while capacity records are unread are dropped and
 * counted. */
#define KLLM_TRACE_DECODE  1u
#define KLLM_TRACE_APPEND  2u
#define KLLM_TRACE_PREFILL 3u
#define KLLM_TRACE_MAX     65536
struct kllm_gpu_trace_record {
	uint64_t seq;                /* call number since tracing was enabled */
	uint64_t tag;                /* kllm_gpu_trace_tag at the call (e.g. request id) */
	uint64_t submit_ns;          /* CLOCK_MONOTONIC at the call (the tracer's clock) */
	uint32_t op;                 /* KLLM_TRACE_* */
	float gpu_us;                /* device time of the call's kernels (-1: unknown) */
};
int kllm_gpu_trace_enable(struct kllm_gpu_ctx *ctx, int capacity);  /* 0: off */
void kllm_gpu_trace_tag(struct kllm_gpu_ctx *ctx, uint64_t tag);
int kllm_gpu_trace_read(struct kllm_gpu_ctx *ctx, struct kllm_gpu_trace_record *out,
			int max_records, uint64_t *dropped);

/* Cross-GPU split-KV exchange over NCCL (NVLink). One context per rank.
 * kllm_gpu_comm_get_unique_id runs on one rank; its 128 bytes reach the
 * others through the caller's channel. Init is non-blocking and bounded:
 * KLLM_ETIMEDOUT (communicator aborted) when the peers do not join within
 * timeout_ms. */
int kllm_gpu_comm_get_unique_id(uint8_t id[128]);
int kllm_gpu_comm_init(struct kllm_gpu_ctx *ctx, int nranks, int rank,
		       const uint8_t id[128], int timeout_ms);
/* All-gathers this rank's triples (m, l [num_rows], o [num_rows][head_dim],
 * fp32, as produced by kllm_gpu_paged_attention_v2's partial_* outputs) from
 * every rank and merges them into out (bf16 [num_rows][head_dim]) on every
 * rank. Enqueued on `stream`; the exchange is waited for with a bound of
 * timeout_ms when timeout_ms > 0 (KLLM_ETIMEDOUT: communicator aborted). */
int kllm_gpu_comm_merge(struct kllm_gpu_ctx *ctx, const float *m,
			const float *l, const float *o, int num_rows,
			int head_dim, void *out, void *stream, int timeout_ms);
void kllm_gpu_comm_destroy(struct kllm_gpu_ctx *ctx);

/* Content-addressed block-table build on the GPU (the reference does this on
 * the host per block: userspace/compute/infer_gpu.c:110-118 computes the
 * block key, userspace/kvcache/cache_index.c:87-108 looks it up,
 * userspace/kvcache/arena_alloc.c:196-201 maps the slot to its page).
 *
 * Block b of sequence s has the key SHA-256(token_ids[0, min((b+1) *
 * block_size, seq_len)) as little-endian uint32), looked up in a device
 * mirror of the cache index with the reference's probe: bucket = first four
 * key bytes (little-endian) & (capacity - 1), linear probing that stops at
 * the first empty entry (slot_index 0xFFFFFFFF), full 32-byte match. A hit
 * writes the entry {arena_base + slot * slot_bytes + k_offset, ... +
 * v_offset, valid = 1} (valid = 0 when slot >= total_slots) and, when
 * now_ns != 0, stamps the index entry's last_access_ns; a miss writes a zero
 * entry and is counted and listed. Blocks in [ceil(len / block_size),
 * max_blocks_per_seq) get zero entries; a sequence longer than the table is
 * cut at max_blocks_per_seq * block_size tokens and flagged with
 * KLLM_ERR_SEQ_TOO_LONG.
 *
 * Incremental use: with first_block, blocks below first_block[s] are left
 * untouched and the hash chain restarts from the state the workspace kept;
 * first_block[s] * block_size must not exceed the tokens of sequence s that
 * an earlier call with the same workspace (same sequence row) covered, and
 * those tokens must be unchanged. */
struct kllm_gpu_index_entry {           /* userspace/kvcache/cache_index.h:22-27 */
	uint8_t hash[32];
	uint32_t slot_index;                /* 0xFFFFFFFF: empty */
	uint32_t flags;
	uint64_t last_access_ns;
};

struct kllm_gpu_table_build_params {
	uint32_t struct_size;
	uint32_t flags;
	const uint32_t *token_ids;   /* packed token ids of all sequences */
	const int64_t *token_starts; /* [num_seqs]: index of sequence s's first token */
	const int *seq_lens;         /* [num_seqs] */
	const int *first_block;      /* [num_seqs] or NULL (all 0) */
	int num_seqs;
	int max_blocks_per_seq;
	int block_size;              /* tokens per block */
	struct kllm_gpu_index_entry *index; /* [index_capacity], 16-byte aligned */
	uint32_t index_capacity;     /* power of two */
	uint64_t now_ns;             /* LRU stamp for hits; 0 leaves the index unchanged */
	uint64_t arena_base;         /* device address of slot 0 */
	uint64_t slot_bytes;
	uint64_t total_slots;
	uint64_t k_offset;           /* K page offset inside a slot */
	uint64_t v_offset;           /* V page offset inside a slot */
	void *block_tables;          /* out: kllm_block_table_entry [num_seqs][max_blocks_per_seq] */
	uint8_t *hashes;             /* out, optional: [num_seqs][max_blocks_per_seq][32], 16-byte aligned */
	void *workspace;             /* kllm_gpu_table_workspace_size bytes, 16-byte aligned */
	uint64_t workspace_bytes;
	int *miss_list;              /* out, optional: (seq, block) int pairs, unordered */
	int miss_capacity;           /* pairs miss_list holds */
	int *miss_count;             /* out, optional: misses of this call (may exceed miss_capacity) */
	uint64_t *hit_miss;          /* optional: [2] += hits, misses (kllm_index_stats counters) */
	uint32_t *err_word;
	void *stream;
};

uint64_t kllm_gpu_table_workspace_size(int num_seqs, int max_blocks_per_seq,
				       int block_size);
int kllm_gpu_build_block_tables(struct kllm_gpu_ctx *ctx,
				const struct kllm_gpu_table_build_params *p);

/* Vocabulary projection (lm_head) and token sampling on the GPU: the step
 * after attention. The reference's GPU inference returns zero logits and
 * takes their argmax (userspace/compute/infer_gpu.c:212-229); its samplers
 * are host loops (userspace/decode/decode_loop.c:58-185), restated here:
 *   logits[r][v] = sum_k hidden[r][k] * weight[v][k]   (bf16 in, fp32 sums,
 *                                                       tcgen05 tensor cores)
 *   method GREEDY      first maximum logit
 *          TEMPERATURE first index whose running sum of exp((l - max) / T)
 *                      reaches uniform[r] x the total (T <= 0: greedy)
 *          TOP_K       the top_k[r] largest logits in (value desc, index asc)
 *                      order, then the temperature draw over them (top_k 0 or
 *                      >= vocab: TEMPERATURE; at most 1024)
 *          TOP_P       as TEMPERATURE (the reference's nucleus is a TODO)
 * uniform[r] in [0, 1] stands for the reference's rand() / RAND_MAX. The
 * full-vocabulary temperature sum runs in parallel, so where r lands within
 * rounding of a cumulative boundary the token can be the neighbour of the
 * one a sequential sum picks. num_rows <= 256, hidden_dim % 64 == 0,
 * hidden and weight 16-byte aligned. logits is required unless every row
 * is greedy (method NULL). */
enum kllm_sampling {                    /* userspace/decode/decode_loop.h:27-32 */
	KLLM_SAMPLE_GREEDY = 0,
	KLLM_SAMPLE_TOP_K = 1,
	KLLM_SAMPLE_TOP_P = 2,
	KLLM_SAMPLE_TEMPERATURE = 3,
};

struct kllm_gpu_lm_head_params {
	uint32_t struct_size;
	uint32_t flags;
	const void *hidden;          /* bf16 [num_rows][hidden_dim] */
	const void *weight;          /* bf16 [vocab][hidden_dim] */
	int num_rows;
	int hidden_dim;
	int vocab;
	float *logits;               /* out: fp32 [num_rows][vocab], or NULL (greedy only) */
	const int *method;           /* [num_rows] enum kllm_sampling, or NULL (all greedy) */
	const float *temperature;    /* [num_rows], or NULL */
	const int *top_k;            /* [num_rows], or NULL */
	const float *uniform;        /* [num_rows] in [0, 1], or NULL */
	int *tokens;                 /* out: [num_rows] */
	void *workspace;             /* kllm_gpu_lm_head_workspace_size bytes, 16-byte aligned */
	uint64_t workspace_bytes;
	uint32_t *err_word;
	void *stream;
};

uint64_t kllm_gpu_lm_head_workspace_size(int num_rows, int vocab);
int kllm_gpu_lm_head_sample(struct kllm_gpu_ctx *ctx,
			    const struct kllm_gpu_lm_head_params *p);

/* Cross-GPU split-KV exchange over peer memory (no counterpart in the
 * reference): the same result as kllm_gpu_comm_merge, computed by one kernel
 * per rank that stores this rank's triples into every peer's exchange
 * buffer over NVLink (CUDA IPC mappings, plain stores), raises per-block
 * flags there, waits (bounded) for the peers' flags and merges. One process
 * per GPU on one node.
 *   1. kllm_gpu_p2p_export on every rank: allocates the exchange buffer for
 *      up to max_rows rows (<= 65536) of head_dim (64 or 128) and returns its
 *      KLLM_P2P_HANDLE_BYTES-byte IPC handle;
 *   2. the handles reach every rank through the caller's channel;
 *   3. kllm_gpu_p2p_import with all ranks' handles (rank-major, nranks <= 8);
 *   4. kllm_gpu_p2p_merge on every rank, in the same order on all ranks (each
 *      call is one exchange epoch). A wait that expires ORs KLLM_ERR_TIMEOUT
 *      into *err_word (optional) instead of hanging. */
#define KLLM_P2P_HANDLE_BYTES 64
int kllm_gpu_p2p_export(struct kllm_gpu_ctx *ctx, int max_rows, int head_dim,
			uint8_t handle[KLLM_P2P_HANDLE_BYTES]);
int kllm_gpu_p2p_import(struct kllm_gpu_ctx *ctx, int nranks, int rank,
			const uint8_t *handles);
int kllm_gpu_p2p_merge(struct kllm_gpu_ctx *ctx, const float *m, const float *l,
		       const float *o, int num_rows, int head_dim, void *out,
		       uint32_t *err_word, int timeout_ms, void *stream);
void kllm_gpu_p2p_destroy(struct kllm_gpu_ctx *ctx);

#ifdef __cplusplus
}
#endif

#endif /* KLLM_GPU_H */
