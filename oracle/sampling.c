/* SPDX-License-Identifier: Apache-2.0 */
/*
 * sampling.c - CPU restatement of the vocabulary projection and the token
 * samplers. TEST INFRASTRUCTURE ONLY (see kllm_oracle.h).
 *
 * The samplers follow userspace/decode/decode_loop.c:58-158 with the
 * uniform draw passed in (the reference draws rand() / RAND_MAX inside
 * sample_temperature, :95); they are pinned against the reference's own
 * functions compiled from that file (oracle/ref_sampling_wrap.c).
 */
#include "kllm_oracle.h"

#include <math.h>
#include <stdlib.h>

/* logits[r][v] = sum_k hidden[r][k] * weight[v][k], fp32, k ascending. */
void orc_lm_head_logits(const uint16_t *hidden, const uint16_t *weight, int rows, int hidden_dim,
			int vocab, const int32_t *vocab_ids, int n_ids, float *out)
{
	for (int r = 0; r < rows; r++)
		for (int j = 0; j < n_ids; j++) {
			const int v = vocab_ids ? vocab_ids[j] : j;
			const uint16_t *h = hidden + (size_t)r * hidden_dim;
			const uint16_t *w = weight + (size_t)v * hidden_dim;
			float s = 0.f;
			for (int k = 0; k < hidden_dim; k++)
				s += orc_bf16_to_f32(h[k]) * orc_bf16_to_f32(w[k]);
			out[(size_t)r * n_ids + j] = s;
		}
	(void)vocab;
}

/* decode_loop.c:58-70 */
uint32_t orc_sample_greedy(const float *logits, uint32_t vocab)
{
	float max_val = -INFINITY;
	uint32_t max_idx = 0;
	for (uint32_t i = 0; i < vocab; i++)
		if (logits[i] > max_val) {
			max_val = logits[i];
			max_idx = i;
		}
	return max_idx;
}

/* decode_loop.c:71-113, with r given */
uint32_t orc_sample_temperature(const float *logits, uint32_t vocab, float temperature, float r)
{
	if (temperature <= 0.0f)
		return orc_sample_greedy(logits, vocab);
	float *probs = malloc(vocab * sizeof(float));
	if (!probs)
		return orc_sample_greedy(logits, vocab);
	float max_logit = -INFINITY;
	for (uint32_t i = 0; i < vocab; i++)
		if (logits[i] > max_logit)
			max_logit = logits[i];
	float sum = 0.0f;
	for (uint32_t i = 0; i < vocab; i++) {
		probs[i] = expf((logits[i] - max_logit) / temperature);
		sum += probs[i];
	}
	for (uint32_t i = 0; i < vocab; i++)
		probs[i] /= sum;
	float cumsum = 0.0f;
	uint32_t token = vocab - 1;
	for (uint32_t i = 0; i < vocab; i++) {
		cumsum += probs[i];
		if (r <= cumsum) {
			token = i;
			break;
		}
	}
	free(probs);
	return token;
}

/* decode_loop.c:115-158: the k largest by insertion (a value enters when it
 * beats the current k-th strictly and bubbles up past strictly smaller
 * ones), then the temperature draw over them. */
uint32_t orc_sample_top_k(const float *logits, uint32_t vocab, uint32_t k, float temperature,
			  float r)
{
	if (k == 0 || k >= vocab)
		return orc_sample_temperature(logits, vocab, temperature, r);
	float *vals = malloc(k * sizeof(float));
	uint32_t *idxs = malloc(k * sizeof(uint32_t));
	if (!vals || !idxs) {
		free(vals);
		free(idxs);
		return orc_sample_greedy(logits, vocab);
	}
	for (uint32_t i = 0; i < k; i++) {
		vals[i] = -INFINITY;
		idxs[i] = 0;
	}
	for (uint32_t i = 0; i < vocab; i++) {
		if (logits[i] > vals[k - 1]) {
			vals[k - 1] = logits[i];
			idxs[k - 1] = i;
			for (int j = (int)k - 2; j >= 0; j--) {
				if (vals[j + 1] > vals[j]) {
					const float tv = vals[j];
					vals[j] = vals[j + 1];
					vals[j + 1] = tv;
					const uint32_t ti = idxs[j];
					idxs[j] = idxs[j + 1];
					idxs[j + 1] = ti;
				}
			}
		}
	}
	const uint32_t res = orc_sample_temperature(vals, k, temperature, r);
	const uint32_t token = idxs[res < k ? res : 0];
	free(vals);
	free(idxs);
	return token;
}

/* decode_loop.c:160-183 */
uint32_t orc_sample_token(const float *logits, uint32_t vocab, int method, float temperature,
			  uint32_t top_k, float r)
{
	switch (method) {
	case 0:
		return orc_sample_greedy(logits, vocab);
	case 3:
		return orc_sample_temperature(logits, vocab, temperature, r);
	case 1:
		return orc_sample_top_k(logits, vocab, top_k, temperature, r);
	case 2:
		return orc_sample_temperature(logits, vocab, temperature, r);
	default:
		return orc_sample_greedy(logits, vocab);
	}
}
