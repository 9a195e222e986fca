/* SPDX-License-Identifier: Apache-2.0 */
/*
 * paged_harness.c - multi-threaded CPU paged decode, timed as the CPU
 * baseline. TEST AND CPU-BASELINE INFRASTRUCTURE ONLY.
 *
 * Built twice by oracle/Makefile:
 *   - liboracle.so: attention = orc_attention (the C restatement, "port");
 *   - _ref/libkllm_ref_*.so (-DHARNESS_REF): attention = the reference's own
 *     kllm_ace_attention (userspace/compute/ace_attention.c:236) compiled from
 *     its sources, MX bytes decoded with the reference decoder
 *     fp8_e4m3_to_f32 (userspace/compute/mx_dequant.h:30), "reference".
 *
 * Work units are (seq, kv_head) pairs pulled from a shared counter by
 * nthreads pthreads. Per unit: gather the valid tokens through the block
 * table into contiguous [n][head_dim] bf16 (dequantising MX pages), then one
 * attention call with num_heads = 1 and query_len = G, which is exact GQA
 * (ace_attention.c:97,104 index q/k as (qi*num_heads + h)*head_dim).
 */
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "kllm_oracle.h"

#ifdef HARNESS_REF
#include "ace_attention.h"
#include "mx_dequant.h"
#define HN_NAME(x) ref_##x
#else
#define HN_NAME(x) orc_##x
#endif

static float g_dec[256];
static pthread_once_t g_dec_once = PTHREAD_ONCE_INIT;

static void init_dec(void)
{
	for (int c = 0; c < 256; c++) {
#ifdef HARNESS_REF
		g_dec[c] = fp8_e4m3_to_f32((fp8_e4m3_t)c);
#else
		g_dec[c] = orc_e4m3_decode((uint8_t)c);
#endif
	}
#ifdef HARNESS_REF
	kllm_ace_probe();          /* selects the reference's ISA path */
#endif
}

static double now_s(void)
{
	struct timespec ts;
	clock_gettime(CLOCK_MONOTONIC, &ts);
	return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

static inline uint16_t to_bf16(float f)
{
	uint32_t b;
	memcpy(&b, &f, 4);
	b += 0x7FFFu + ((b >> 16) & 1u);
	return (uint16_t)(b >> 16);
}

struct hn_job {
	uint16_t *out;
	const uint16_t *q;
	const struct orc_entry *table;
	const int32_t *seq_lens;
	int num_seqs, num_heads, num_kv_heads, head_dim, max_blocks, block_size;
	int kv_dtype;
	float scale;
	uint64_t layer_off;
	int next;
	pthread_mutex_t lock;
	double gather_s, attn_s;    /* summed over threads */
};

static size_t hn_gather(const struct hn_job *j, int s, int h, uint16_t *kb,
			uint16_t *vb)
{
	int seq_len = j->seq_lens[s];
	int bs = j->block_size, d = j->head_dim;
	if (seq_len <= 0)
		return 0;
	int nblocks = (seq_len + bs - 1) / bs;
	if (nblocks > j->max_blocks)
		nblocks = j->max_blocks;
	uint64_t sec = j->kv_dtype == ORC_KV_MX_FP8 ?
		(uint64_t)bs * d + (uint64_t)bs * (d / 8) : (uint64_t)bs * d * 2;
	const struct orc_entry *row = j->table + (size_t)s * j->max_blocks;
	size_t n = 0;

	for (int b = 0; b < nblocks; b++) {
		const struct orc_entry *e = &row[b];
		if (!e->valid || !e->k_ptr)
			continue;
		int ntok = seq_len - b * bs < bs ? seq_len - b * bs : bs;
		for (int kv = 0; kv < 2; kv++) {
			const uint8_t *secp = (const uint8_t *)(kv ? e->v_ptr : e->k_ptr) +
				j->layer_off + sec * h;
			uint16_t *dst = (kv ? vb : kb) + n * d;
			if (j->kv_dtype == ORC_KV_BF16) {
				memcpy(dst, secp, (size_t)ntok * d * 2);
				continue;
			}
			for (int t = 0; t < ntok; t++) {
				const uint8_t *p = secp + (size_t)t * d;
				const uint8_t *sc = secp + (size_t)bs * d + (size_t)t * (d / 8);
				for (int i = 0; i < d; i++)
					dst[(size_t)t * d + i] =
						to_bf16(g_dec[p[i]] * g_dec[sc[i >> 3]]);
			}
		}
		n += ntok;
	}
	return n;
}

static void *hn_worker(void *arg)
{
	struct hn_job *j = (struct hn_job *)arg;
	int d = j->head_dim, g = j->num_heads / j->num_kv_heads;
	size_t cap = (size_t)j->max_blocks * j->block_size * d + 16;
	uint16_t *kb = (uint16_t *)malloc(cap * 2);
	uint16_t *vb = (uint16_t *)malloc(cap * 2);
	int units = j->num_seqs * j->num_kv_heads;
	double tg = 0.0, ta = 0.0;

	for (;;) {
		pthread_mutex_lock(&j->lock);
		int u = j->next++;
		pthread_mutex_unlock(&j->lock);
		if (u >= units)
			break;
		int s = u / j->num_kv_heads, h = u % j->num_kv_heads;
		double t0 = now_s();
		size_t n = hn_gather(j, s, h, kb, vb);
		double t1 = now_s();
		size_t row0 = (size_t)s * j->num_heads + (size_t)h * g;
		uint16_t *og = j->out + row0 * d;
		if (n == 0) {
			memset(og, 0, (size_t)g * d * 2);
		} else {
#ifdef HARNESS_REF
			struct kllm_attention_params p = {
				.num_heads = 1,
				.head_dim = (uint32_t)d,
				.seq_len = (uint32_t)n,
				.query_len = (uint32_t)g,
				.scale = j->scale,
			};
			kllm_ace_attention(j->q + row0 * d, kb, vb, og, NULL, &p);
#else
			orc_attention(j->q + row0 * d, kb, vb, og, 1, (uint32_t)d,
				      (uint32_t)n, (uint32_t)g, j->scale);
#endif
		}
		ta += now_s() - t1;
		tg += t1 - t0;
	}
	pthread_mutex_lock(&j->lock);
	j->gather_s += tg;
	j->attn_s += ta;
	pthread_mutex_unlock(&j->lock);
	free(kb);
	free(vb);
	return NULL;
}

/* Runs the decode with nthreads threads; times[0] = wall seconds,
 * times[1] = summed gather+dequant thread-seconds, times[2] = summed
 * attention thread-seconds. Returns 0, or -1 on bad shapes. */
int HN_NAME(harness_paged_decode)(uint16_t *out, const uint16_t *q,
				  const struct orc_entry *table,
				  const int32_t *seq_lens, int num_seqs,
				  int num_heads, int num_kv_heads, int head_dim,
				  int max_blocks, float scale, int block_size,
				  int kv_dtype, uint64_t layer_off, int nthreads,
				  double *times)
{
	if (num_kv_heads <= 0 || num_heads % num_kv_heads)
		return -1;
	if (kv_dtype != ORC_KV_BF16 && kv_dtype != ORC_KV_MX_FP8)
		return -1;
	pthread_once(&g_dec_once, init_dec);

	struct hn_job j;
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
	pthread_mutex_init(&j.lock, NULL);

	double t0 = now_s();
	if (nthreads <= 1) {
		hn_worker(&j);
	} else {
		pthread_t *th = (pthread_t *)calloc(nthreads, sizeof(pthread_t));
		for (int i = 0; i < nthreads; i++)
			pthread_create(&th[i], NULL, hn_worker, &j);
		for (int i = 0; i < nthreads; i++)
			pthread_join(th[i], NULL);
		free(th);
	}
	if (times) {
		times[0] = now_s() - t0;
		times[1] = j.gather_s;
		times[2] = j.attn_s;
	}
	pthread_mutex_destroy(&j.lock);
	return 0;
}
