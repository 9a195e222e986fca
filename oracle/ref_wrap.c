/* SPDX-License-Identifier: Apache-2.0 */
/*
 * ref_wrap.c - exports the reference's header-only MX codec and its CPU
 * attention under stable names, for pinning the oracle. TEST
 * INFRASTRUCTURE ONLY: compiled by oracle/Makefile together with the
 * reference's unmodified userspace/compute/ace_attention.c, including the
 * reference's unmodified userspace/compute/mx_dequant.h, into
 * oracle/_ref/libkllm_ref_*.so. No reference source is copied here.
 */
#include <stddef.h>
#include <stdint.h>

#include "ace_attention.h"
#include "mx_dequant.h"

/* userspace/compute/mx_dequant.h:30 */
float ref_fp8_e4m3_to_f32(uint8_t v)
{
	return fp8_e4m3_to_f32(v);
}

/* userspace/compute/mx_dequant.h:65 */
void ref_mx_dequant_bf16(const uint16_t *data, const uint8_t *scales,
			 float *out, uint32_t count)
{
	mx_dequant_bf16(data, scales, out, count);
}

/* userspace/compute/mx_dequant.h:82 */
float ref_mx_dot_product(const uint16_t *a, const uint16_t *b,
			 const uint8_t *b_scales, uint32_t dim)
{
	return mx_dot_product(a, b, b_scales, dim);
}

/* userspace/compute/mx_dequant.h:105 */
void ref_mx_quant_to_bf16(const float *in, uint16_t *data, uint8_t *scales,
			  uint32_t count)
{
	mx_quant_to_bf16(in, data, scales, count);
}

/* userspace/compute/ace_attention.c:40 */
int ref_ace_probe(void)
{
	return kllm_ace_probe();
}

/* userspace/compute/ace_attention.c:236, with the params struct spelled out
 * so a foreign-function caller needs no struct layout. */
int ref_ace_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v,
		      uint16_t *out, uint32_t num_heads, uint32_t head_dim,
		      uint32_t seq_len, uint32_t query_len, float scale)
{
	struct kllm_attention_params p = {
		.num_heads = num_heads,
		.head_dim = head_dim,
		.seq_len = seq_len,
		.query_len = query_len,
		.scale = scale,
	};
	return kllm_ace_attention(q, k, v, out, NULL, &p);
}
