/* SPDX-License-Identifier: Apache-2.0 */
/*
 * kllm_oracle.h - CPU restatement of the xpu-kllm paged-attention path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * backend: only tests/, the smoke check and the benchmark's CPU-baseline leg
 * load it. The product library never links, calls or falls back to it.
 *
 * Every function names the reference file:line it restates. Parity pinning:
 * the codec, the compat quantizer and the attention are checked against the
 * reference's own C code compiled from its sources (oracle/Makefile -> _ref),
 * and against golden fixtures produced by that build (tests/golden/).
 */
#ifndef KLLM_ORACLE_H
#define KLLM_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Page descriptor, as the GPU reads it (userspace/gpu/paged_attention.cu:18-22);
 * here the pointers are host pointers into a host copy of the arena. */
struct orc_entry {
	const void *k_ptr;
	const void *v_ptr;
	int32_t valid;
	int32_t _pad;
};

enum { ORC_KV_BF16 = 0, ORC_KV_MX_FP8 = 1, ORC_KV_MX_BF16_COMPAT = 2 };

/* ace_attention.c:67-72 */
float orc_bf16_to_f32(uint16_t v);
/* ace_attention.c:74-80 (round to nearest even by the reference's bit trick) */
uint16_t orc_f32_to_bf16(float v);

/* mx_dequant.h:30-55: E4M3 code -> float, bias 7, subnormals, 0x7F -> 480 */
float orc_e4m3_decode(uint8_t code);
/* float -> E4M3, round to nearest even, saturating to +-448 (0x7E/0xFE);
 * NaN -> 0x7F. The encoder the reference TODO at mx_dequant.h:124 asks for. */
uint8_t orc_e4m3_encode(float v);
/* Smallest positive E4M3 code whose value is >= amax/448 (mx_dequant.h:119-120
 * rule), 0 for amax == 0, 0x7E when amax/448 > 448. */
uint8_t orc_mx_scale_code(float amax);

/* MX-FP8 quantizer for `count` elements (count % 8 == 0): per 8 elements the
 * structure of mx_quant_to_bf16 (mx_dequant.h:108-135) with an E4M3 payload:
 * payload = orc_e4m3_encode(x / decode(scale)). */
void orc_mx_quantize_fp8(const uint16_t *x_bf16, uint8_t *payload,
			 uint8_t *scales, uint32_t count);
/* mx_quant_to_bf16 (mx_dequant.h:105-136) restated bit for bit. */
void orc_mx_quantize_bf16_compat(const float *in, uint16_t *data,
				 uint8_t *scales, uint32_t count);

/* Scaled-dot-product attention, two-pass exact softmax, restating the scalar
 * path of kllm_ace_attention (ace_attention.c:85-134, entry :236-270):
 * q [query_len][num_heads][head_dim], k/v [seq_len][num_heads][head_dim],
 * out likewise for q; returns -1 on the reference's argument errors. */
int orc_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v,
		  uint16_t *out, uint32_t num_heads, uint32_t head_dim,
		  uint32_t seq_len, uint32_t query_len, float scale);

/* Block-table gather (paged_attention.cu:55-68 semantics) for one
 * (seq, kv_head): walks pages 0..ceil(seq_len/block_size)-1, clamped to
 * max_blocks, skips entries with !valid || !k_ptr, cuts the last page at
 * seq_len; K/V become contiguous [n][head_dim] bf16 (MX values dequantised
 * with orc_e4m3_decode, exact). Returns n. */
size_t orc_gather(const struct orc_entry *row, int max_blocks, int seq_len,
		  int kv_head, int num_kv_heads, int head_dim, int block_size,
		  int kv_dtype, uint64_t layer_off, uint16_t *k_out,
		  uint16_t *v_out);

/* Paged GQA decode: per (seq, kv_head) gather, then orc_attention with
 * num_heads = 1, query_len = G over the G query heads sharing the kv head
 * (q_head / G == kv_head, paged_attention.cu:45). Empty contexts give zeros
 * (paged_attention.cu:109-118 with exp_sum == 0). nthreads > 1 spreads
 * (seq, kv_head) units over pthreads. */
int orc_paged_decode(uint16_t *out, const uint16_t *q,
		     const struct orc_entry *table, const int32_t *seq_lens,
		     int num_seqs, int num_heads, int num_kv_heads, int head_dim,
		     int max_blocks, float scale, int block_size, int kv_dtype,
		     uint64_t layer_off, int nthreads);

/* Split-KV triples of the same decode (new: absent in the reference):
 * m = max_t s_t (s_t = scale * q.k_t), l = sum_t exp(s_t - m),
 * o = sum_t exp(s_t - m) v_t / l, fp32, [num_seqs][num_heads](*head_dim).
 * Empty: m = -inf, l = 0, o = 0. */
int orc_paged_decode_partials(float *m, float *l, float *o, const uint16_t *q,
			      const struct orc_entry *table,
			      const int32_t *seq_lens, int num_seqs,
			      int num_heads, int num_kv_heads, int head_dim,
			      int max_blocks, float scale, int block_size,
			      int kv_dtype, uint64_t layer_off);

/* LSE merge of split-KV triples (new): M = max m_i, w_i = l_i exp(m_i - M),
 * out = bf16(sum w_i o_i / sum w_i); 0 when sum w_i == 0. */
void orc_merge_partials(const float *m, const float *l, const float *o,
			int num_parts, int num_rows, int head_dim,
			uint16_t *out);

/* KV append / quantize-on-write into host pages (new on the GPU path):
 * row i goes to page table[seq][pos / block_size], slot pos % block_size.
 * Returns the number of rows skipped for lack of a valid page. */
int orc_kv_append(const uint16_t *k, const uint16_t *v, const int32_t *tok_seq,
		  const int32_t *tok_pos, int num_tokens,
		  const struct orc_entry *table, int max_blocks,
		  int num_kv_heads, int head_dim, int block_size, int kv_dtype,
		  uint64_t layer_off);

/* Causal attention for a chunk of query rows (new: the reference has no
 * mask): query row r of sequence s sits at absolute position pos0 + r and
 * attends keys [0, pos0 + r]; K/V for one kv head come as contiguous
 * [n_keys][head_dim] bf16 (prefix from the paged cache, then the chunk).
 * Built from orc_attention with seq_len = pos0 + r + 1, query_len = G.
 * q/out: [n_rows][G][head_dim]. */
int orc_causal_rows(const uint16_t *q, const uint16_t *k, const uint16_t *v,
		    uint16_t *out, int n_rows, int pos0, int group,
		    int head_dim, float scale);

/* ---- content-addressed block tables (content_index.c) -------------------- */

/* Entry of the reference's cache index, same 48-byte layout
 * (userspace/kvcache/cache_index.h:22-27). */
#define ORC_INDEX_EMPTY 0xFFFFFFFFu  /* cache_index.c:16 EMPTY_SLOT */
struct orc_index_entry {
	uint8_t hash[32];
	uint32_t slot_index;
	uint32_t flags;
	uint64_t last_access_ns;
};

/* SHA-256 (FIPS 180-4), the function the reference calls through OpenSSL. */
void orc_sha256(const void *msg, size_t len, uint8_t out[32]);
/* infer_gpu.c:110-118: SHA-256 of tokens[0, min((b+1)*block_size, seq_len)). */
void orc_block_key(const uint32_t *tokens, int seq_len, int block_size, int b,
		   uint8_t out[32]);
/* cache_index.c:35-41, 87-108: position of the key's entry, or -1. */
int64_t orc_index_probe(const struct orc_index_entry *entries, uint32_t capacity,
			const uint8_t hash[32]);
/* Content-addressed block-table build (key, probe, slot -> page pointers);
 * table entries carry device addresses. Returns 1 if a sequence was cut at
 * max_blocks * block_size tokens, else 0. */
int orc_build_block_tables(const uint32_t *tokens, const int64_t *starts,
			   const int32_t *seq_lens, const int32_t *first_block,
			   int num_seqs, int max_blocks, int block_size,
			   struct orc_index_entry *index, uint32_t capacity,
			   uint64_t now_ns, uint64_t arena_base,
			   uint64_t slot_bytes, uint64_t total_slots,
			   uint64_t k_offset, uint64_t v_offset,
			   struct orc_entry *table, uint8_t *hashes,
			   uint64_t *hits, uint64_t *misses);

/* ---- vocabulary projection and sampling (sampling.c) --------------------- */

/* logits[r][j] = sum_k hidden[r][k] * weight[v_j][k] (fp32, k ascending) for
 * the vocabulary rows v_j = vocab_ids[j] (all rows 0..n_ids-1 when NULL). */
void orc_lm_head_logits(const uint16_t *hidden, const uint16_t *weight, int rows, int hidden_dim,
			int vocab, const int32_t *vocab_ids, int n_ids, float *out);
/* decode_loop.c:58-183 with the uniform draw r given */
uint32_t orc_sample_greedy(const float *logits, uint32_t vocab);
uint32_t orc_sample_temperature(const float *logits, uint32_t vocab, float temperature, float r);
uint32_t orc_sample_top_k(const float *logits, uint32_t vocab, uint32_t k, float temperature,
			  float r);
uint32_t orc_sample_token(const float *logits, uint32_t vocab, int method, float temperature,
			  uint32_t top_k, float r);

#ifdef __cplusplus
}
#endif

#endif /* KLLM_ORACLE_H */
