/* SPDX-License-Identifier: Apache-2.0 */
/*
 * kllm_oracle.c - CPU restatement of the xpu-kllm paged-attention path.
 *
 * TEST INFRASTRUCTURE ONLY (see kllm_oracle.h): the parity checker for the
 * CUDA backend, never part of the product path.
 */
#include "kllm_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---- BF16 (ace_attention.c:67-80) ---------------------------------------- */

float orc_bf16_to_f32(uint16_t v)
{
	uint32_t bits = (uint32_t)v << 16;
	float f;
	memcpy(&f, &bits, sizeof(f));
	return f;
}

uint16_t orc_f32_to_bf16(float v)
{
	uint32_t bits;
	memcpy(&bits, &v, sizeof(bits));
	bits += 0x7FFFu + ((bits >> 16) & 1u);
	return (uint16_t)(bits >> 16);
}

/* ---- E4M3 codec ---------------------------------------------------------- */

/* mx_dequant.h:30-55: sign, 4-bit exponent (bias 7), 3-bit mantissa;
 * exponent 0 is subnormal (m/8 * 2^-6); no NaN: 0x7F decodes to 480. */
float orc_e4m3_decode(uint8_t code)
{
	int sign = (code >> 7) & 1;
	int e = (code >> 3) & 0xF;
	int m = code & 0x7;
	float r;

	if (e == 0)
		r = ldexpf((float)m / 8.0f, -6);
	else
		r = ldexpf(1.0f + (float)m / 8.0f, e - 7);
	return sign ? -r : r;
}

/* Round-to-nearest-even of a float to E4M3, saturating at 448. Works on the
 * IEEE bits: the float is m24 * 2^(e-23); E4M3 keeps 3 mantissa bits for
 * e >= -6 and a fixed 2^-9 quantum below. */
uint8_t orc_e4m3_encode(float v)
{
	uint32_t b;
	memcpy(&b, &v, sizeof(b));
	uint8_t sign = (uint8_t)((b >> 31) << 7);
	uint32_t a = b & 0x7FFFFFFFu;

	if (a > 0x7F800000u)
		return sign | 0x7F;            /* NaN */
	if (a >= 0x43E00000u)                  /* |v| >= 448 (and inf) */
		return sign | 0x7E;

	int e = (int)(a >> 23) - 127;
	uint32_t mant = (a & 0x7FFFFFu) | (e > -127 ? 0x800000u : 0u);

	if (e < -6) {
		/* quantum 2^-9: q = mant * 2^(e - 23 + 9) = mant >> (14 - e) */
		int shift = 14 - e;
		if (e == -127)
			shift = 14 + 126;      /* float subnormal: value < 2^-126 */
		if (shift >= 26)
			return sign;           /* < 2^-11: rounds to zero */
		uint32_t q = mant >> shift;
		uint32_t rem = mant & ((1u << shift) - 1u);
		uint32_t half = 1u << (shift - 1);
		if (rem > half || (rem == half && (q & 1u)))
			q++;
		return sign | (uint8_t)q;      /* q == 8 is the smallest normal */
	}

	uint32_t q = (mant >> 20) & 0x7u;      /* 3 mantissa bits */
	uint32_t rem = mant & 0xFFFFFu;
	if (rem > 0x80000u || (rem == 0x80000u && (q & 1u)))
		q++;
	if (q == 8) {
		q = 0;
		e++;
	}
	uint32_t code = ((uint32_t)(e + 7) << 3) | q;
	if (code > 0x7E)
		code = 0x7E;
	return sign | (uint8_t)code;
}

uint8_t orc_mx_scale_code(float amax)
{
	if (!(amax > 0.0f))
		return 0;
	float t = amax / 448.0f;               /* mx_dequant.h:120 */
	if (t > 448.0f)
		return 0x7E;
	uint8_t c = orc_e4m3_encode(t);
	if (orc_e4m3_decode(c) < t)
		c++;
	if (c == 0)
		c = 1;
	return c;
}

void orc_mx_quantize_fp8(const uint16_t *x, uint8_t *payload, uint8_t *scales,
			 uint32_t count)
{
	for (uint32_t blk = 0; blk < count; blk += 8) {
		float amax = 0.0f;
		for (uint32_t i = blk; i < blk + 8; i++) {
			float av = fabsf(orc_bf16_to_f32(x[i]));
			if (av > amax)
				amax = av;
		}
		uint8_t sc = orc_mx_scale_code(amax);
		scales[blk / 8] = sc;
		if (sc == 0) {
			memset(payload + blk, 0, 8);
			continue;
		}
		float s = orc_e4m3_decode(sc);
		for (uint32_t i = blk; i < blk + 8; i++)
			payload[i] = orc_e4m3_encode(orc_bf16_to_f32(x[i]) / s);
	}
}

/* mx_dequant.h:105-136, step for step. */
void orc_mx_quantize_bf16_compat(const float *in, uint16_t *data,
				 uint8_t *scales, uint32_t count)
{
	for (uint32_t blk = 0; blk < count; blk += 8) {
		float amax = 0.0f;
		uint32_t end = blk + 8;
		if (end > count)
			end = count;
		for (uint32_t i = blk; i < end; i++) {
			float av = in[i] < 0 ? -in[i] : in[i];
			if (av > amax)
				amax = av;
		}
		float scale = (amax > 0.0f) ? amax / 448.0f : 1.0f;
		float inv_scale = 1.0f / scale;
		scales[blk / 8] = (uint8_t)(amax > 0 ? 64 : 0);
		for (uint32_t i = blk; i < end; i++) {
			float scaled = in[i] * inv_scale;
			uint32_t bits;
			memcpy(&bits, &scaled, sizeof(bits));
			bits += 0x7FFFu + ((bits >> 16) & 1u);
			data[i] = (uint16_t)(bits >> 16);
		}
	}
}

/* ---- attention (ace_attention.c:85-134) ---------------------------------- */

int orc_attention(const uint16_t *q, const uint16_t *k, const uint16_t *v,
		  uint16_t *out, uint32_t num_heads, uint32_t head_dim,
		  uint32_t seq_len, uint32_t query_len, float scale)
{
	if (!q || !k || !v || !out)
		return -1;
	if (head_dim == 0 || seq_len == 0 || num_heads == 0)
		return -1;

	float *scores = (float *)malloc(sizeof(float) * seq_len);
	if (!scores)
		return -1;

	for (uint32_t h = 0; h < num_heads; h++) {
		for (uint32_t qi = 0; qi < query_len; qi++) {
			const uint16_t *qv = q + ((size_t)qi * num_heads + h) * head_dim;
			float max_score = -INFINITY;

			for (uint32_t si = 0; si < seq_len; si++) {
				const uint16_t *kv = k + ((size_t)si * num_heads + h) * head_dim;
				float dot = 0.0f;
				for (uint32_t d = 0; d < head_dim; d++)
					dot += orc_bf16_to_f32(qv[d]) * orc_bf16_to_f32(kv[d]);
				scores[si] = dot * scale;
				if (scores[si] > max_score)
					max_score = scores[si];
			}

			float sum = 0.0f;
			for (uint32_t si = 0; si < seq_len; si++) {
				scores[si] = expf(scores[si] - max_score);
				sum += scores[si];
			}
			for (uint32_t si = 0; si < seq_len; si++)
				scores[si] /= sum;

			uint16_t *ov = out + ((size_t)qi * num_heads + h) * head_dim;
			for (uint32_t d = 0; d < head_dim; d++) {
				float acc = 0.0f;
				for (uint32_t si = 0; si < seq_len; si++) {
					const uint16_t *vv = v + ((size_t)si * num_heads + h) * head_dim;
					acc += scores[si] * orc_bf16_to_f32(vv[d]);
				}
				ov[d] = orc_f32_to_bf16(acc);
			}
		}
	}
	free(scores);
	return 0;
}

/* ---- page layout ---------------------------------------------------------- */

static uint64_t section_bytes(int kv_dtype, int bs, int d)
{
	switch (kv_dtype) {
	case ORC_KV_MX_FP8:
		return (uint64_t)bs * d + (uint64_t)bs * (d / 8);
	case ORC_KV_MX_BF16_COMPAT:
		return (uint64_t)bs * d * 2 + (uint64_t)bs * (d / 8);
	default:
		return (uint64_t)bs * d * 2;
	}
}

/* One token row of one head section as bf16 (exact for BF16 and MX-FP8). */
static void load_row(const uint8_t *sec, int kv_dtype, int bs, int d, int t,
		     uint16_t *dst)
{
	if (kv_dtype == ORC_KV_BF16) {
		memcpy(dst, sec + (size_t)t * d * 2, (size_t)d * 2);
	} else if (kv_dtype == ORC_KV_MX_FP8) {
		const uint8_t *p = sec + (size_t)t * d;
		const uint8_t *s = sec + (size_t)bs * d + (size_t)t * (d / 8);
		for (int i = 0; i < d; i++)
			dst[i] = orc_f32_to_bf16(orc_e4m3_decode(p[i]) *
						 orc_e4m3_decode(s[i / 8]));
	} else {
		const uint16_t *p = (const uint16_t *)(sec + (size_t)t * d * 2);
		const uint8_t *s = sec + (size_t)bs * d * 2 + (size_t)t * (d / 8);
		for (int i = 0; i < d; i++)
			dst[i] = orc_f32_to_bf16(orc_bf16_to_f32(p[i]) *
						 orc_e4m3_decode(s[i / 8]));
	}
}

size_t orc_gather(const struct orc_entry *row, int max_blocks, int seq_len,
		  int kv_head, int num_kv_heads, int head_dim, int block_size,
		  int kv_dtype, uint64_t layer_off, uint16_t *k_out,
		  uint16_t *v_out)
{
	(void)num_kv_heads;
	if (seq_len <= 0)
		return 0;
	int nblocks = (seq_len + block_size - 1) / block_size;
	if (nblocks > max_blocks)
		nblocks = max_blocks;
	uint64_t sec = section_bytes(kv_dtype, block_size, head_dim);
	size_t n = 0;

	for (int b = 0; b < nblocks; b++) {
		const struct orc_entry *e = &row[b];
		if (!e->valid || !e->k_ptr)       /* paged_attention.cu:59-60 */
			continue;
		const uint8_t *ks = (const uint8_t *)e->k_ptr + layer_off + sec * kv_head;
		const uint8_t *vs = (const uint8_t *)e->v_ptr + layer_off + sec * kv_head;
		int start = b * block_size;
		int ntok = seq_len - start < block_size ? seq_len - start : block_size;
		for (int t = 0; t < ntok; t++) {
			load_row(ks, kv_dtype, block_size, head_dim, t,
				 k_out + n * head_dim);
			load_row(vs, kv_dtype, block_size, head_dim, t,
				 v_out + n * head_dim);
			n++;
		}
	}
	return n;
}

/* ---- paged decode ---------------------------------------------------------- */

struct decode_job {
	uint16_t *out;
	float *pm, *pl, *po;            /* partials mode when non-NULL */
	const uint16_t *q;
	const struct orc_entry *table;
	const int32_t *seq_lens;
	int num_seqs, num_heads, num_kv_heads, head_dim, max_blocks, block_size;
	int kv_dtype;
	float scale;
	uint64_t layer_off;
	int next;                       /* unit counter, guarded by lock */
	pthread_mutex_t lock;
};

static void partial_triple(const uint16_t *qv, const uint16_t *k,
			   const uint16_t *v, size_t n, int d, float scale,
			   float *m, float *l, float *o)
{
	if (n == 0) {
		*m = -INFINITY;
		*l = 0.0f;
		memset(o, 0, sizeof(float) * d);
		return;
	}
	float *sc = (float *)malloc(sizeof(float) * n);
	float mx = -INFINITY;
	for (size_t t = 0; t < n; t++) {
		float dot = 0.0f;
		for (int i = 0; i < d; i++)
			dot += orc_bf16_to_f32(qv[i]) * orc_bf16_to_f32(k[t * d + i]);
		sc[t] = dot * scale;
		if (sc[t] > mx)
			mx = sc[t];
	}
	float sum = 0.0f;
	for (size_t t = 0; t < n; t++) {
		sc[t] = expf(sc[t] - mx);
		sum += sc[t];
	}
	for (int i = 0; i < d; i++) {
		float acc = 0.0f;
		for (size_t t = 0; t < n; t++)
			acc += sc[t] * orc_bf16_to_f32(v[t * d + i]);
		o[i] = acc / sum;
	}
	*m = mx;
	*l = sum;
	free(sc);
}

static void decode_unit(struct decode_job *j, int unit, uint16_t *kbuf,
			uint16_t *vbuf)
{
	int s = unit / j->num_kv_heads, h = unit % j->num_kv_heads;
	int g = j->num_heads / j->num_kv_heads;
	int d = j->head_dim;
	size_t n = orc_gather(j->table + (size_t)s * j->max_blocks, j->max_blocks,
			      j->seq_lens[s], h, j->num_kv_heads, d,
			      j->block_size, j->kv_dtype, j->layer_off, kbuf,
			      vbuf);
	size_t row0 = (size_t)s * j->num_heads + (size_t)h * g;
	const uint16_t *qg = j->q + row0 * d;

	if (j->pm) {
		for (int i = 0; i < g; i++)
			partial_triple(qg + (size_t)i * d, kbuf, vbuf, n, d,
				       j->scale, j->pm + row0 + i,
				       j->pl + row0 + i,
				       j->po + (row0 + i) * d);
		return;
	}
	uint16_t *og = j->out + row0 * d;
	if (n == 0) {
		memset(og, 0, sizeof(uint16_t) * g * d);
		return;
	}
	orc_attention(qg, kbuf, vbuf, og, 1, (uint32_t)d, (uint32_t)n,
		      (uint32_t)g, j->scale);
}

static void *decode_worker(void *arg)
{
	struct decode_job *j = (struct decode_job *)arg;
	size_t cap = (size_t)j->max_blocks * j->block_size * j->head_dim;
	uint16_t *kbuf = (uint16_t *)malloc(cap * sizeof(uint16_t) + 16);
	uint16_t *vbuf = (uint16_t *)malloc(cap * sizeof(uint16_t) + 16);
	int units = j->num_seqs * j->num_kv_heads;

	for (;;) {
		pthread_mutex_lock(&j->lock);
		int u = j->next++;
		pthread_mutex_unlock(&j->lock);
		if (u >= units)
			break;
		decode_unit(j, u, kbuf, vbuf);
	}
	free(kbuf);
	free(vbuf);
	return NULL;
}

static int run_decode(struct decode_job *j, int nthreads)
{
	if (j->num_kv_heads <= 0 || j->num_heads % j->num_kv_heads)
		return -1;
	pthread_mutex_init(&j->lock, NULL);
	j->next = 0;
	if (nthreads <= 1) {
		decode_worker(j);
	} else {
		pthread_t *th = (pthread_t *)calloc(nthreads, sizeof(pthread_t));
		for (int i = 0; i < nthreads; i++)
			pthread_create(&th[i], NULL, decode_worker, j);
		for (int i = 0; i < nthreads; i++)
			pthread_join(th[i], NULL);
		free(th);
	}
	pthread_mutex_destroy(&j->lock);
	return 0;
}

int orc_paged_decode(uint16_t *out, const uint16_t *q,
		     const struct orc_entry *table, const int32_t *seq_lens,
		     int num_seqs, int num_heads, int num_kv_heads, int head_dim,
		     int max_blocks, float scale, int block_size, int kv_dtype,
		     uint64_t layer_off, int nthreads)
{
	struct decode_job j;
	memset(&j, 0, sizeof(j));
	j.out = out;
	j.q = q;
	j.table = table;
	j.seq_lens = seq_lens;
	j.num_seqs = num_seqs;
	j.num_heads = num_heads;
	j.num_kv_heads = num_kv_heads;
	j.head_dim = head_dim;
	j.max_blocks = max_blocks;
	j.block_size = block_size;
	j.kv_dtype = kv_dtype;
	j.scale = scale;
	j.layer_off = layer_off;
	return run_decode(&j, nthreads);
}

int orc_paged_decode_partials(float *m, float *l, float *o, const uint16_t *q,
			      const struct orc_entry *table,
			      const int32_t *seq_lens, int num_seqs,
			      int num_heads, int num_kv_heads, int head_dim,
			      int max_blocks, float scale, int block_size,
			      int kv_dtype, uint64_t layer_off)
{
	struct decode_job j;
	memset(&j, 0, sizeof(j));
	j.pm = m;
	j.pl = l;
	j.po = o;
	j.q = q;
	j.table = table;
	j.seq_lens = seq_lens;
	j.num_seqs = num_seqs;
	j.num_heads = num_heads;
	j.num_kv_heads = num_kv_heads;
	j.head_dim = head_dim;
	j.max_blocks = max_blocks;
	j.block_size = block_size;
	j.kv_dtype = kv_dtype;
	j.scale = scale;
	j.layer_off = layer_off;
	return run_decode(&j, 1);
}

void orc_merge_partials(const float *m, const float *l, const float *o,
			int num_parts, int num_rows, int head_dim,
			uint16_t *out)
{
	for (int r = 0; r < num_rows; r++) {
		float mx = -INFINITY;
		for (int p = 0; p < num_parts; p++)
			if (l[(size_t)p * num_rows + r] > 0.0f &&
			    m[(size_t)p * num_rows + r] > mx)
				mx = m[(size_t)p * num_rows + r];
		float wsum = 0.0f;
		for (int p = 0; p < num_parts; p++) {
			float lp = l[(size_t)p * num_rows + r];
			if (lp > 0.0f)
				wsum += lp * expf(m[(size_t)p * num_rows + r] - mx);
		}
		for (int i = 0; i < head_dim; i++) {
			float acc = 0.0f;
			for (int p = 0; p < num_parts; p++) {
				float lp = l[(size_t)p * num_rows + r];
				if (lp > 0.0f)
					acc += lp * expf(m[(size_t)p * num_rows + r] - mx) *
					       o[((size_t)p * num_rows + r) * head_dim + i];
			}
			out[(size_t)r * head_dim + i] =
				orc_f32_to_bf16(wsum > 0.0f ? acc / wsum : 0.0f);
		}
	}
}

/* ---- KV append ------------------------------------------------------------ */

int orc_kv_append(const uint16_t *k, const uint16_t *v, const int32_t *tok_seq,
		  const int32_t *tok_pos, int num_tokens,
		  const struct orc_entry *table, int max_blocks,
		  int num_kv_heads, int head_dim, int block_size, int kv_dtype,
		  uint64_t layer_off)
{
	uint64_t sec = section_bytes(kv_dtype, block_size, head_dim);
	float *tmp = (float *)malloc(sizeof(float) * head_dim);
	int skipped = 0;

	for (int i = 0; i < num_tokens; i++) {
		int s = tok_seq[i], pos = tok_pos[i];
		int blk = pos >= 0 ? pos / block_size : -1;
		if (s < 0 || blk < 0 || blk >= max_blocks) {
			skipped++;
			continue;
		}
		const struct orc_entry *e = &table[(size_t)s * max_blocks + blk];
		if (!e->valid || !e->k_ptr) {
			skipped++;
			continue;
		}
		int slot = pos % block_size;
		for (int kv = 0; kv < 2; kv++) {
			const uint16_t *src = (kv ? v : k) +
				((size_t)i * num_kv_heads) * head_dim;
			uint8_t *base = (uint8_t *)(kv ? e->v_ptr : e->k_ptr) + layer_off;
			for (int h = 0; h < num_kv_heads; h++) {
				const uint16_t *x = src + (size_t)h * head_dim;
				uint8_t *secp = base + sec * h;
				if (kv_dtype == ORC_KV_BF16) {
					memcpy(secp + (size_t)slot * head_dim * 2, x,
					       (size_t)head_dim * 2);
				} else if (kv_dtype == ORC_KV_MX_FP8) {
					orc_mx_quantize_fp8(
						x, secp + (size_t)slot * head_dim,
						secp + (size_t)block_size * head_dim +
							(size_t)slot * (head_dim / 8),
						(uint32_t)head_dim);
				} else {
					for (int d = 0; d < head_dim; d++)
						tmp[d] = orc_bf16_to_f32(x[d]);
					orc_mx_quantize_bf16_compat(
						tmp,
						(uint16_t *)(secp + (size_t)slot * head_dim * 2),
						secp + (size_t)block_size * head_dim * 2 +
							(size_t)slot * (head_dim / 8),
						(uint32_t)head_dim);
				}
			}
		}
	}
	free(tmp);
	return skipped;
}

/* ---- causal rows (chunked prefill) ---------------------------------------- */

int orc_causal_rows(const uint16_t *q, const uint16_t *k, const uint16_t *v,
		    uint16_t *out, int n_rows, int pos0, int group,
		    int head_dim, float scale)
{
	for (int r = 0; r < n_rows; r++) {
		const uint16_t *qr = q + (size_t)r * group * head_dim;
		uint16_t *orow = out + (size_t)r * group * head_dim;
		if (orc_attention(qr, k, v, orow, 1, (uint32_t)head_dim,
				  (uint32_t)(pos0 + r + 1), (uint32_t)group,
				  scale) < 0)
			return -1;
	}
	return 0;
}
