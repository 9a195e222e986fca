/* SPDX-License-Identifier: Apache-2.0 */
/*
 * abi_consumer.c - a plain C caller of libkllm_gpu, as the reference's
 * reactor calls its GPU backend (userspace/compute/infer_gpu.c:189-203):
 * context, device allocations, host-to-device copies, then
 *   1. the v1 entry point on 128-token BF16 pages (gpu_attention.h:26-51);
 *   2. v2 on 16-token BF16 pages;
 *   3. v2 on MX-FP8 pages written on the device by kllm_gpu_kv_append_v2,
 *      read back through kllm_gpu_gather_debug (the exact dequantised cache)
 * each checked against a double-precision attention over the same cache
 * values: |got - ref| <= 1e-3 + 2e-2 |ref| after bf16 rounding of ref.
 * Exit 0 when all pass, 1 on a mismatch or an error, 77 without an sm_100
 * device.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "kllm_gpu.h"

enum { S = 3, HQ = 32, HKV = 8, D = 128, G = HQ / HKV };
static const int lens[S] = {200, 1, 300};

static uint64_t rng_state = 0x9E3779B97F4A7C15ull;

static double uniform01(void)
{
	rng_state += 0x9E3779B97F4A7C15ull;            /* splitmix64 */
	uint64_t z = rng_state;
	z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
	z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
	z ^= z >> 31;
	return ((double)(z >> 11) + 0.5) / 9007199254740992.0;
}

static float normal(void)
{
	const double u = uniform01(), v = uniform01();
	return (float)(sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v));
}

static uint16_t f2bf(float f)                       /* round to nearest even */
{
	uint32_t u;
	memcpy(&u, &f, 4);
	u += 0x7FFFu + ((u >> 16) & 1u);
	return (uint16_t)(u >> 16);
}

static float bf2f(uint16_t b)
{
	const uint32_t u = (uint32_t)b << 16;
	float f;
	memcpy(&f, &u, 4);
	return f;
}

#define CHECK(x) do { int rc_ = (x); if (rc_ != 0) { \
	fprintf(stderr, "%s:%d: %s = %d\n", __FILE__, __LINE__, #x, rc_); return 1; } } while (0)

/* Double-precision attention of one query head over kv[t][d] (t < n). */
static void attend(const float *q, const float *k, const float *v, int n, double scale,
		   double *out)
{
	double mx = -INFINITY, l = 0.0;
	double *w = malloc(sizeof(double) * (n ? n : 1));
	for (int t = 0; t < n; t++) {
		double s = 0.0;
		for (int d = 0; d < D; d++)
			s += (double)q[d] * k[(size_t)t * D + d];
		w[t] = s * scale;
		if (w[t] > mx)
			mx = w[t];
	}
	for (int d = 0; d < D; d++)
		out[d] = 0.0;
	for (int t = 0; t < n; t++) {
		w[t] = exp(w[t] - mx);
		l += w[t];
		for (int d = 0; d < D; d++)
			out[d] += w[t] * v[(size_t)t * D + d];
	}
	for (int d = 0; d < D; d++)
		out[d] = l > 0 ? out[d] / l : 0.0;
	free(w);
}

/* got [S][HQ][D] bf16 against attention over kf/vf [S][HKV][tokens][D]. */
static int compare(const char *what, const uint16_t *got, const float *qf, const float *kf,
		   const float *vf, int maxlen, double scale)
{
	double out[D], worst = 0.0;
	for (int s = 0; s < S; s++)
		for (int h = 0; h < HQ; h++) {
			const int kv = h / G;
			const float *k = kf + ((size_t)(s * HKV + kv) * maxlen) * D;
			const float *v = vf + ((size_t)(s * HKV + kv) * maxlen) * D;
			attend(qf + ((size_t)s * HQ + h) * D, k, v, lens[s], scale, out);
			for (int d = 0; d < D; d++) {
				const double r = bf2f(f2bf((float)out[d]));
				const double g = bf2f(got[((size_t)s * HQ + h) * D + d]);
				const double ratio = fabs(g - r) / (1e-3 + 2e-2 * fabs(r));
				if (!(ratio <= 1.0)) {
					fprintf(stderr, "%s: seq %d head %d dim %d got %g want %g\n", what, s,
						h, d, g, r);
					return 1;
				}
				if (ratio > worst)
					worst = ratio;
			}
		}
	printf("%s ok (worst error %.3f of the tolerance)\n", what, worst);
	return 0;
}

int main(void)
{
	struct kllm_gpu_ctx *ctx = kllm_gpu_create();
	if (!ctx || kllm_gpu_get_backend(ctx) != KLLM_GPU_CUDA) {
		printf("no sm_100 device: skipped\n");
		kllm_gpu_destroy(ctx);
		return 77;
	}
	int maxlen = 0;
	for (int s = 0; s < S; s++)
		maxlen = lens[s] > maxlen ? lens[s] : maxlen;
	const double scale = 1.0 / sqrt((double)D);
	/* host data: q [S][HQ][D], k/v [S][HKV][maxlen][D] (bf16 values) */
	const size_t nq = (size_t)S * HQ * D, nkv = (size_t)S * HKV * maxlen * D;
	uint16_t *q = malloc(nq * 2), *k = malloc(nkv * 2), *v = malloc(nkv * 2);
	float *qf = malloc(nq * 4), *kf = malloc(nkv * 4), *vf = malloc(nkv * 4);
	for (size_t i = 0; i < nq; i++) {
		q[i] = f2bf(normal());
		qf[i] = bf2f(q[i]);
	}
	for (size_t i = 0; i < nkv; i++) {
		k[i] = f2bf(normal());
		v[i] = f2bf(normal() * 2.0f);
		kf[i] = bf2f(k[i]);
		vf[i] = bf2f(v[i]);
	}
	int *dlens = kllm_gpu_malloc(ctx, sizeof(lens));
	void *dq = kllm_gpu_malloc(ctx, nq * 2), *dout = kllm_gpu_malloc(ctx, nq * 2);
	uint16_t *out = malloc(nq * 2);
	CHECK(kllm_gpu_memcpy_h2d(ctx, dlens, lens, sizeof(lens)));
	CHECK(kllm_gpu_memcpy_h2d(ctx, dq, q, nq * 2));

	/* 1 and 2: BF16 pages of 128 tokens (v1) and 16 tokens (v2), one page per
	 * slot, [HKV][block][D], slots in order */
	for (int pass = 0; pass < 2; pass++) {
		const int block = pass ? 16 : 128;
		const int mb = (maxlen + block - 1) / block;
		const size_t page = (size_t)HKV * block * D * 2;
		uint8_t *arena = kllm_gpu_malloc(ctx, (size_t)S * mb * 2 * page);
		uint16_t *hpage = calloc(1, page);
		struct kllm_block_table_entry *tab = calloc((size_t)S * mb, sizeof(*tab));
		for (int s = 0; s < S; s++)
			for (int b = 0; b < mb; b++) {
				uint8_t *kp = arena + ((size_t)(s * mb + b) * 2) * page;
				uint8_t *vp = kp + page;
				for (int which = 0; which < 2; which++) {
					const uint16_t *src = which ? v : k;
					memset(hpage, 0, page);
					for (int h = 0; h < HKV; h++)
						for (int t = 0; t < block && b * block + t < lens[s]; t++)
							memcpy(hpage + ((size_t)h * block + t) * D,
							       src + (((size_t)(s * HKV + h) * maxlen) + b * block + t) * D,
							       D * 2);
					CHECK(kllm_gpu_memcpy_h2d(ctx, which ? vp : kp, hpage, page));
				}
				tab[s * mb + b].k_ptr = kp;
				tab[s * mb + b].v_ptr = vp;
				tab[s * mb + b].valid = b * block < lens[s];
			}
		void *dtab = kllm_gpu_malloc(ctx, (size_t)S * mb * sizeof(*tab));
		CHECK(kllm_gpu_memcpy_h2d(ctx, dtab, tab, (size_t)S * mb * sizeof(*tab)));
		if (pass == 0) {
			struct kllm_gpu_attention_params p = {
				.output = dout, .query = dq, .block_tables = dtab, .seq_lens = dlens,
				.num_seqs = S, .num_heads = HQ, .num_kv_heads = HKV, .head_dim = D,
				.max_blocks_per_seq = mb, .scale = (float)scale, .stream = NULL,
			};
			CHECK(kllm_gpu_paged_attention(ctx, &p));
		} else {
			struct kllm_gpu_attention_params_v2 p;
			memset(&p, 0, sizeof(p));
			p.struct_size = sizeof(p);
			p.output = dout;
			p.query = dq;
			p.block_tables = dtab;
			p.seq_lens = dlens;
			p.num_seqs = S;
			p.num_heads = HQ;
			p.num_kv_heads = HKV;
			p.head_dim = D;
			p.max_blocks_per_seq = mb;
			p.block_size = block;
			p.kv_dtype = KLLM_KV_BF16;
			p.layer_stride = 2 * page;
			p.scale = (float)scale;
			p.split = 1;
			CHECK(kllm_gpu_paged_attention_v2(ctx, &p));
		}
		CHECK(kllm_gpu_synchronize(ctx, 10000));
		CHECK(kllm_gpu_memcpy_d2h(ctx, out, dout, nq * 2));
		if (compare(pass ? "v2 bf16 16-token pages" : "v1 bf16 128-token pages", out, qf, kf,
			    vf, maxlen, scale))
			return 1;
		kllm_gpu_free(ctx, dtab);
		kllm_gpu_free(ctx, arena);
		free(hpage);
		free(tab);
	}

	/* 3: MX-FP8 pages written by the append kernel, read back exactly */
	{
		const int block = 16, mb = (maxlen + block - 1) / block;
		const size_t sec = (size_t)block * D + (size_t)block * (D / 8);
		const size_t page = HKV * sec;
		uint8_t *arena = kllm_gpu_malloc(ctx, (size_t)S * mb * 2 * page);
		struct kllm_block_table_entry *tab = calloc((size_t)S * mb, sizeof(*tab));
		for (int s = 0; s < S; s++)
			for (int b = 0; b < mb; b++) {
				tab[s * mb + b].k_ptr = arena + ((size_t)(s * mb + b) * 2) * page;
				tab[s * mb + b].v_ptr = (uint8_t *)tab[s * mb + b].k_ptr + page;
				tab[s * mb + b].valid = 1;
			}
		void *dtab = kllm_gpu_malloc(ctx, (size_t)S * mb * sizeof(*tab));
		CHECK(kllm_gpu_memcpy_h2d(ctx, dtab, tab, (size_t)S * mb * sizeof(*tab)));
		/* token rows [n][HKV][D] in (seq, position) order */
		int n = 0;
		for (int s = 0; s < S; s++)
			n += lens[s];
		uint16_t *rk = malloc((size_t)n * HKV * D * 2), *rv = malloc((size_t)n * HKV * D * 2);
		int *tseq = malloc(n * sizeof(int)), *tpos = malloc(n * sizeof(int));
		int i = 0;
		for (int s = 0; s < S; s++)
			for (int t = 0; t < lens[s]; t++, i++) {
				tseq[i] = s;
				tpos[i] = t;
				for (int h = 0; h < HKV; h++) {
					memcpy(rk + ((size_t)i * HKV + h) * D,
					       k + (((size_t)(s * HKV + h) * maxlen) + t) * D, D * 2);
					memcpy(rv + ((size_t)i * HKV + h) * D,
					       v + (((size_t)(s * HKV + h) * maxlen) + t) * D, D * 2);
				}
			}
		void *drk = kllm_gpu_malloc(ctx, (size_t)n * HKV * D * 2);
		void *drv = kllm_gpu_malloc(ctx, (size_t)n * HKV * D * 2);
		int *dseq = kllm_gpu_malloc(ctx, n * sizeof(int)), *dpos = kllm_gpu_malloc(ctx, n * sizeof(int));
		CHECK(kllm_gpu_memcpy_h2d(ctx, drk, rk, (size_t)n * HKV * D * 2));
		CHECK(kllm_gpu_memcpy_h2d(ctx, drv, rv, (size_t)n * HKV * D * 2));
		CHECK(kllm_gpu_memcpy_h2d(ctx, dseq, tseq, n * sizeof(int)));
		CHECK(kllm_gpu_memcpy_h2d(ctx, dpos, tpos, n * sizeof(int)));
		struct kllm_gpu_kv_append_params a;
		memset(&a, 0, sizeof(a));
		a.struct_size = sizeof(a);
		a.k = drk;
		a.v = drv;
		a.token_seq = dseq;
		a.token_pos = dpos;
		a.num_tokens = n;
		a.num_seqs = S;
		a.block_tables = dtab;
		a.max_blocks_per_seq = mb;
		a.num_kv_heads = HKV;
		a.head_dim = D;
		a.block_size = block;
		a.kv_dtype = KLLM_KV_MX_FP8_E4M3;
		a.layer_stride = 2 * page;
		CHECK(kllm_gpu_kv_append_v2(ctx, &a));
		/* the exact dequantised cache, for the double-precision reference */
		const size_t cap = (size_t)mb * block;
		void *gk = kllm_gpu_malloc(ctx, (size_t)S * HKV * cap * D * 2);
		void *gv = kllm_gpu_malloc(ctx, (size_t)S * HKV * cap * D * 2);
		int *gcnt = kllm_gpu_malloc(ctx, (size_t)S * HKV * sizeof(int));
		struct kllm_gpu_gather_params gp;
		memset(&gp, 0, sizeof(gp));
		gp.struct_size = sizeof(gp);
		gp.k_out = gk;
		gp.v_out = gv;
		gp.counts_out = gcnt;
		gp.block_tables = dtab;
		gp.seq_lens = dlens;
		gp.num_seqs = S;
		gp.num_kv_heads = HKV;
		gp.head_dim = D;
		gp.max_blocks_per_seq = mb;
		gp.block_size = block;
		gp.kv_dtype = KLLM_KV_MX_FP8_E4M3;
		gp.layer_stride = 2 * page;
		CHECK(kllm_gpu_gather_debug(ctx, &gp));
		struct kllm_gpu_attention_params_v2 p;
		memset(&p, 0, sizeof(p));
		p.struct_size = sizeof(p);
		p.output = dout;
		p.query = dq;
		p.block_tables = dtab;
		p.seq_lens = dlens;
		p.num_seqs = S;
		p.num_heads = HQ;
		p.num_kv_heads = HKV;
		p.head_dim = D;
		p.max_blocks_per_seq = mb;
		p.block_size = block;
		p.kv_dtype = KLLM_KV_MX_FP8_E4M3;
		p.layer_stride = 2 * page;
		p.scale = (float)scale;
		p.split = 1;
		CHECK(kllm_gpu_paged_attention_v2(ctx, &p));
		CHECK(kllm_gpu_synchronize(ctx, 10000));
		CHECK(kllm_gpu_memcpy_d2h(ctx, out, dout, nq * 2));
		uint16_t *hk = malloc((size_t)S * HKV * cap * D * 2), *hv = malloc((size_t)S * HKV * cap * D * 2);
		CHECK(kllm_gpu_memcpy_d2h(ctx, hk, gk, (size_t)S * HKV * cap * D * 2));
		CHECK(kllm_gpu_memcpy_d2h(ctx, hv, gv, (size_t)S * HKV * cap * D * 2));
		float *mkf = malloc((size_t)S * HKV * cap * D * 4), *mvf = malloc((size_t)S * HKV * cap * D * 4);
		for (size_t j = 0; j < (size_t)S * HKV * cap * D; j++) {
			mkf[j] = bf2f(hk[j]);
			mvf[j] = bf2f(hv[j]);
		}
		if (compare("v2 mx-fp8 pages (appended on the device)", out, qf, mkf, mvf, (int)cap,
			    scale))
			return 1;
	}
	kllm_gpu_destroy(ctx);
	return 0;
}
