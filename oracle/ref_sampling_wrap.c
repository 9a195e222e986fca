/* SPDX-License-Identifier: Apache-2.0 */
/*
 * ref_sampling_wrap.c - exposes the reference's own samplers
 * (userspace/decode/decode_loop.c:58-183, static functions) under stable
 * names by compiling that file into this unit from the reference tree
 * (oracle/Makefile passes its directory); pins oracle/sampling.c. TEST
 * INFRASTRUCTURE ONLY. No reference source is copied here.
 *
 * decode_loop.c calls six functions of the rest of the reference (dispatch,
 * CPU/GPU inference, response path) from kllm_decode_run, which is never
 * called here; they are defined below so the unit links.
 */
#include "decode_loop.c"

enum kllm_dispatch_target kllm_dispatch_decide(struct kllm_dispatch_ctx *ctx, uint32_t seq_len,
					       bool cache_hit)
{
	(void)ctx;
	(void)seq_len;
	(void)cache_hit;
	return KLLM_TARGET_CPU;
}

int kllm_infer_cpu(struct kllm_infer_cpu_ctx *ctx, const uint32_t *token_ids, uint32_t seq_len,
		   struct kllm_infer_result *result)
{
	(void)ctx;
	(void)token_ids;
	(void)seq_len;
	(void)result;
	return -1;
}

int kllm_infer_gpu(struct kllm_infer_gpu_ctx *ctx, const uint32_t *token_ids, uint32_t seq_len,
		   struct kllm_infer_result *result)
{
	(void)ctx;
	(void)token_ids;
	(void)seq_len;
	(void)result;
	return -1;
}

int kllm_infer_gpu_escalate(struct kllm_infer_gpu_ctx *ctx, struct kllm_infer_cpu_ctx *cpu_ctx,
			    const uint32_t *token_ids, uint32_t seq_len,
			    struct kllm_infer_result *result)
{
	(void)ctx;
	(void)cpu_ctx;
	(void)token_ids;
	(void)seq_len;
	(void)result;
	return -1;
}

int kllm_response_emit_one(struct kllm_response_ctx *ctx, uint32_t token)
{
	(void)ctx;
	(void)token;
	return 0;
}

int kllm_response_eos(struct kllm_response_ctx *ctx)
{
	(void)ctx;
	return 0;
}

/* decode_loop.c:160 sample_token, the method given as its enum value */
uint32_t ref_sample_token(const float *logits, uint32_t vocab, int method, float temperature,
			  uint32_t top_k, float top_p)
{
	struct kllm_decode_params p = {
		.max_tokens = 1,
		.eos_token_id = 0,
		.sampling = (enum kllm_sampling_method)method,
		.temperature = temperature,
		.top_k = top_k,
		.top_p = top_p,
	};
	return sample_token(logits, vocab, &p);
}

/* the reference draws rand() / RAND_MAX (decode_loop.c:95): a test seeds the
 * generator, reads the draw, seeds again and calls the sampler */
void ref_srand(unsigned int seed)
{
	srand(seed);
}

int ref_rand(void)
{
	return rand();
}
