/* SPDX-License-Identifier: Apache-2.0 */
/*
 * kllm_internal.h - launch interface between the C host shim (kllm_shim.c)
 * and the CUDA translation units. Plain C, no CUDA types.
 */
#ifndef KLLM_INTERNAL_H
#define KLLM_INTERNAL_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef KLLM_DEC_WARPS
#define KLLM_DEC_WARPS      4     /* warps per decode CTA */
#endif
#define KLLM_MAX_GROUP      8     /* query heads per kv head (mma N) */
#define KLLM_SLOT_FLOATS    1040  /* one split-KV partial: o[8][128], m[8], l[8] */
#define KLLM_MAX_SEQS_LAUNCH 4096 /* sequences per decode launch (smem prefix) */

#define KLLM_ERR_SEQ_TOO_LONG_BIT 0x1u /* seq_len beyond the table: clamped */
#define KLLM_ERR_TIMEOUT_BIT 0x8u /* a bounded device wait expired */
#define KLLM_ERR_TOPK_RANGE_BIT 0x10u /* a row asked for top-k above 1024 */
#define KLLM_ERR_NONFINITE_BIT 0x20u /* MX payload 0x7F/0xFF not recomputed */
#define KLLM_ERR_PAGE_RANGE_BIT 0x40u /* a page outside the registered arenas: skipped */

/* Device memory ranges the caller registered as KV arenas; when count > 0
 * every page a kernel reads or writes must lie inside one of them. */
#define KLLM_MAX_ARENAS 8
struct kllm_arenas {
	int count;
	int pad;
	unsigned long long lo[KLLM_MAX_ARENAS], hi[KLLM_MAX_ARENAS];  /* [lo, hi) */
};
/* MX-FP8 decode computes with K/V values scaled by 2^-2 (payload x scale
 * stays below the f16 maximum); scores and outputs are multiplied back. */
#define KLLM_MX_DEC_UNBIAS   4.0f

struct kllm_decode_args {
	void *out;                /* bf16 [S][Hq][D] or NULL */
	const void *q;            /* bf16 [S][Hq][D] */
	const void *table;        /* 24-byte entries [S][max_blocks] */
	const int *seq_lens;      /* [S] */
	int num_seqs;
	int num_heads;
	int num_kv_heads;
	int group;                /* num_heads / num_kv_heads */
	int head_dim;             /* 64 or 128 */
	int max_blocks;
	int block_size;           /* 16..128, multiple of 16 */
	int kv_dtype;             /* 0 bf16, 1 mx-fp8 */
	uint64_t layer_off;       /* bytes added to k_ptr/v_ptr */
	float scale_log2;         /* softmax scale * log2(e) */
	float *pm, *pl, *po;      /* optional split-KV triples */
	uint32_t *err;            /* optional error word */
	int split;                /* 1: tile-balanced split-KV; 0: one warp per segment */
	float *ws_part;           /* split: partial slots [warps][2][KLLM_SLOT_FLOATS] */
	unsigned *ws_cnt;         /* split: arrival counters [S*Hkv], zero between calls */
	void *ws_list;            /* split: merge work list (KLLM_MERGE_LIST_BYTES, header
	                             zero between calls) or NULL: merge in the decode */
	int total_warps;          /* warps launched (grid * KLLM_DEC_WARPS) */
	int overlap;              /* launch as a programmatic dependent of the previous
	                             kernel on the stream (KLLM_DECODE_OVERLAP_PREV) */
	struct kllm_arenas arenas;
};

/* Segments split over more than KLLM_FUSED_MERGE_MAX warps are not merged by
 * the last warp of the decode but queued for kllm_decode_merge_launch, which
 * merges each (segment, query head) with a whole CTA. */
#ifndef KLLM_FUSED_MERGE_MAX
#define KLLM_FUSED_MERGE_MAX   16
#endif
#define KLLM_MERGE_LIST_CAP    1024
#define KLLM_MERGE_LIST_BYTES  (32 + 24 * KLLM_MERGE_LIST_CAP)

/* Merges the queued segments of the decode launched with `a` (same args). */
int kllm_decode_merge_launch(const struct kllm_decode_args *a, int num_sms,
			     void *stream);

/* Dynamic shared memory of one decode CTA for this shape. */
size_t kllm_decode_smem_bytes(int head_dim, int kv_dtype, int num_seqs);
/* Resident CTAs per SM for this shape (0 on error). */
int kllm_decode_ctas_per_sm(int head_dim, int kv_dtype, int num_seqs);
/* Loads every decode and wide-merge kernel on the current device now
 * instead of at first launch; 0 or a cudaError_t. */
int kllm_decode_preload(void);
/* Launches the decode on `stream` with `grid` CTAs; 0 or a cudaError_t. */
int kllm_decode_launch(const struct kllm_decode_args *a, int grid,
		       void *stream);

struct kllm_append_args {
	const void *k, *v;
	const int *token_seq, *token_pos;
	int num_tokens;
	int num_seqs;
	const void *table;
	int max_blocks, num_kv_heads, head_dim, block_size, kv_dtype;
	uint64_t layer_off;
	uint32_t *err;
	struct kllm_arenas arenas;
};
int kllm_append_launch(const struct kllm_append_args *a, void *stream);

struct kllm_gather_args {
	void *k_out, *v_out;
	int *counts;
	const void *table;
	const int *seq_lens;
	int num_seqs, num_kv_heads, head_dim, max_blocks, block_size, kv_dtype;
	uint64_t layer_off;
};
int kllm_gather_launch(const struct kllm_gather_args *a, void *stream);

struct kllm_prefill_args {
	void *out;                /* bf16 [num_tokens][num_heads][128] */
	const void *q;            /* bf16 [num_tokens][num_heads][128] */
	const void *k, *v;        /* bf16 [num_tokens][num_kv_heads][128] */
	const int *cu_seqlens;    /* [num_seqs+1] */
	const int *ctx_lens;      /* [num_seqs] */
	const void *table;
	int max_blocks;
	int num_seqs, num_tokens, max_chunk;
	int num_heads, num_kv_heads, head_dim;
	int block_size, kv_dtype;
	uint64_t layer_off;
	float scale_log2;
	uint32_t *err;
	struct kllm_arenas arenas;
};
int kllm_prefill_launch(const struct kllm_prefill_args *a, void *stream);

/* Quantize-on-write of a chunk: token i of sequence s (cu_seqlens[s] <= i <
 * cu_seqlens[s+1]) goes to position ctx_lens[s] + i - cu_seqlens[s]. */
int kllm_append_chunk_launch(const struct kllm_append_args *a,
			     const int *cu_seqlens, const int *ctx_lens,
			     void *stream);

int kllm_merge_launch(const float *m, const float *l, const float *o,
		      int num_parts, int num_rows, int head_dim, void *out,
		      void *stream);

/* Peer-memory split-KV exchange + merge (p2p_merge.cu). */
#define KLLM_P2P_MAX_RANKS 8
#define KLLM_P2P_MAX_CTAS  64
struct kllm_p2p_args {
	uint8_t *const *peers;    /* device array [nranks]: every rank's exchange buffer */
	int rank, nranks;
	unsigned epoch;           /* 1, 2, ... per call, identical on every rank */
	int num_rows, max_rows, head_dim;
	const float *m, *l, *o;   /* this rank's triples (m natural-log domain) */
	void *out;                /* bf16 [num_rows][head_dim] */
	uint32_t *err;
	uint64_t timeout_ns;
};
size_t kllm_p2p_buffer_bytes(int max_rows, int head_dim);
int kllm_p2p_grid(int num_rows);
int kllm_p2p_merge_launch(const struct kllm_p2p_args *a, void *stream);

/* Content-addressed block-table build (block_tables.cu). */
struct kllm_table_args {
	const uint32_t *tokens;   /* packed token ids */
	const int64_t *starts;    /* [num_seqs] first token of each sequence */
	const int *seq_lens;      /* [num_seqs] */
	const int *first_block;   /* [num_seqs] or NULL */
	int num_seqs, max_blocks, block_size;
	uint8_t *index;           /* 48-byte entries [capacity], 16-byte aligned */
	uint32_t capacity;        /* power of two */
	unsigned long long now_ns;
	unsigned long long arena_base, slot_bytes, total_slots, k_offset, v_offset;
	void *table;              /* 24-byte entries [num_seqs][max_blocks] */
	uint8_t *hashes;          /* [num_seqs][max_blocks][32] or NULL */
	uint32_t *midstates;      /* [num_seqs][ms_stride][8] */
	uint64_t ms_stride;
	int *miss_list;           /* (seq, block) pairs or NULL */
	int miss_capacity;
	int *miss_count;          /* or NULL */
	unsigned long long *hit_miss; /* [2] or NULL */
	uint32_t *err;
};
uint64_t kllm_table_midstate_stride(int max_blocks, int block_size);
int kllm_table_build_launch(const struct kllm_table_args *a, void *stream);

/* Vocabulary projection + sampling (lm_head.cu). Sampling methods as
 * userspace/decode/decode_loop.h:27-32 numbers them. */
#define KLLM_SAMPLE_GREEDY_I      0
#define KLLM_SAMPLE_TOP_K_I       1
#define KLLM_SAMPLE_TOP_P_I       2
#define KLLM_SAMPLE_TEMPERATURE_I 3
struct kllm_lm_head_args {
	const void *hidden;       /* bf16 [num_rows][hidden_dim] */
	const void *weight;       /* bf16 [vocab][hidden_dim] */
	int num_rows, hidden_dim, vocab;
	float *logits;            /* fp32 [num_rows][vocab] or NULL */
	const int *method;        /* [num_rows] or NULL (greedy) */
	const float *temperature; /* [num_rows] or NULL */
	const int *top_k;         /* [num_rows] or NULL */
	const float *uniform;     /* [num_rows] or NULL */
	int *tokens;              /* [num_rows] */
	float *part_m, *part_s;   /* [num_rows][2 x tiles] */
	int *part_a;              /* [num_rows][2 x tiles] */
	uint32_t *err;
	/* set by kllm_lm_head_launch: tiles 0..n_full-1 are computed whole,
	 * the last n_split as two 128-row halves (the second half's partial
	 * in slot tiles + i until the sampler folds it in) */
	int n_full, n_split;
};
int kllm_lm_head_tiles(int vocab);
int kllm_lm_head_launch(const struct kllm_lm_head_args *a, void *stream);

/* Block arrival: one chunk of records already copied to device memory at
 * src_dev; record i (bytes[i] at src_dev + off[i], off 16-byte aligned) goes
 * to dst[i], a range the host checked lies in device memory of this GPU. */
#define KLLM_WF_SCATTER_MAX 64
struct kllm_wf_scatter {
	uint32_t n;
	uint32_t reserved;
	uint64_t dst[KLLM_WF_SCATTER_MAX];
	uint32_t bytes[KLLM_WF_SCATTER_MAX];
	uint32_t off[KLLM_WF_SCATTER_MAX];
};
int kllm_wf_scatter_launch(const struct kllm_wf_scatter *s, const void *src_dev, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* KLLM_INTERNAL_H */
