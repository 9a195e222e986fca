/* SPDX-License-Identifier: Apache-2.0 */
/*
 * ref_index_wrap.c - drives the reference's own content-addressed cache
 * index (userspace/kvcache/cache_index.c, compiled unmodified from its
 * sources by oracle/Makefile) and its block-key computation (OpenSSL
 * SHA256() called as userspace/compute/infer_gpu.c:110-118 calls it), for
 * pinning the oracle and as the reference CPU baseline of the block-table
 * build. TEST INFRASTRUCTURE ONLY. No reference source is copied here.
 *
 * The reference's arena (userspace/kvcache/arena_alloc.c) needs libnuma's
 * <numaif.h>, which this image lacks, so the four arena calls the index
 * makes are provided below with the same slot semantics
 * (arena_alloc.c:135-201: first free slot scanning a bitmap from a hint
 * word, slot pointer = base + index * slot_size, NULL past the end).
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <openssl/sha.h>

#include "cache_index.h"

struct kllm_arena {
	uint8_t *base;
	uint64_t slot_size;
	uint64_t total_slots;
	uint64_t *bitmap;          /* bit set = free */
	uint64_t words;
	uint64_t hint;
};

void *kllm_arena_alloc(struct kllm_arena *a)
{
	for (uint64_t pass = 0; pass < 2; pass++) {
		const uint64_t lo = pass ? 0 : a->hint, hi = pass ? a->hint : a->words;
		for (uint64_t w = lo; w < hi; w++) {
			if (!a->bitmap[w])
				continue;
			const uint64_t slot = w * 64 + (uint64_t)__builtin_ctzll(a->bitmap[w]);
			if (slot >= a->total_slots)
				return NULL;
			a->bitmap[w] &= ~(1ull << (slot % 64));
			a->hint = w;
			return a->base + slot * a->slot_size;
		}
	}
	return NULL;
}

void kllm_arena_free(struct kllm_arena *a, void *block)
{
	const uint64_t slot = (uint64_t)((uint8_t *)block - a->base) / a->slot_size;
	a->bitmap[slot / 64] |= 1ull << (slot % 64);
	if (slot / 64 < a->hint)
		a->hint = slot / 64;
}

uint32_t kllm_arena_slot_index(struct kllm_arena *a, void *block)
{
	return (uint32_t)((uint64_t)((uint8_t *)block - a->base) / a->slot_size);
}

void *kllm_arena_slot_ptr(struct kllm_arena *a, uint32_t index)
{
	if (index >= a->total_slots)
		return NULL;
	return a->base + (uint64_t)index * a->slot_size;
}

struct ref_index {
	struct kllm_arena arena;
	struct kllm_cache_index *idx;
};

/* The first member of the reference's private index struct
 * (cache_index.c:19-26) is the entry array; the tests read it through this
 * view to mirror the index on the device. */
struct ref_index_view {
	struct kllm_cache_entry *entries;
};

void ref_index_free(struct ref_index *r);

struct ref_index *ref_index_new(uint32_t capacity, uint64_t total_slots)
{
	struct ref_index *r = calloc(1, sizeof(*r));
	if (!r)
		return NULL;
	r->arena.slot_size = 1;
	r->arena.total_slots = total_slots;
	r->arena.words = (total_slots + 63) / 64;
	r->arena.base = malloc(total_slots ? total_slots : 1);
	r->arena.bitmap = malloc(r->arena.words * 8 + 8);
	if (!r->arena.base || !r->arena.bitmap) {
		ref_index_free(r);
		return NULL;
	}
	for (uint64_t w = 0; w < r->arena.words; w++)
		r->arena.bitmap[w] = ~0ull;
	if (total_slots % 64)
		r->arena.bitmap[r->arena.words - 1] = (1ull << (total_slots % 64)) - 1;
	struct kllm_index_config cfg = { .capacity = capacity, .arena = &r->arena };
	r->idx = kllm_index_create(&cfg);
	if (!r->idx) {
		ref_index_free(r);
		return NULL;
	}
	return r;
}

void ref_index_free(struct ref_index *r)
{
	if (!r)
		return;
	if (r->idx)
		kllm_index_destroy(r->idx);
	free(r->arena.base);
	free(r->arena.bitmap);
	free(r);
}

/* cache_index.c:117 kllm_index_insert; returns the slot or -1. */
int64_t ref_index_insert(struct ref_index *r, const uint8_t hash[32])
{
	void *p = kllm_index_insert(r->idx, hash);
	return p ? (int64_t)kllm_arena_slot_index(&r->arena, p) : -1;
}

/* cache_index.c:87 kllm_index_lookup; returns the slot or -1. */
int64_t ref_index_lookup(struct ref_index *r, const uint8_t hash[32])
{
	void *p = kllm_index_lookup(r->idx, hash);
	return p ? (int64_t)kllm_arena_slot_index(&r->arena, p) : -1;
}

/* cache_index.c:168 kllm_index_evict */
int ref_index_evict(struct ref_index *r, const uint8_t hash[32])
{
	return kllm_index_evict(r->idx, hash) ? 1 : 0;
}

const void *ref_index_entries(struct ref_index *r)
{
	return ((const struct ref_index_view *)(const void *)r->idx)->entries;
}

/* hits, misses, evictions, insertions, occupied, capacity */
void ref_index_stats(struct ref_index *r, uint64_t out[6])
{
	struct kllm_index_stats s;
	kllm_index_get_stats(r->idx, &s);
	out[0] = s.hits;
	out[1] = s.misses;
	out[2] = s.evictions;
	out[3] = s.insertions;
	out[4] = s.occupied;
	out[5] = s.capacity;
}

/* infer_gpu.c:110-118: the key of every block of one sequence. */
void ref_block_keys(const uint32_t *tokens, uint32_t seq_len, uint32_t block_size,
		    uint32_t n_blocks, uint8_t *out)
{
	for (uint32_t b = 0; b < n_blocks; b++) {
		uint32_t prefix_len = (b + 1) * block_size;
		if (prefix_len > seq_len)
			prefix_len = seq_len;
		SHA256((const unsigned char *)tokens, prefix_len * sizeof(uint32_t),
		       out + (size_t)b * 32);
	}
}

/* The reference's per-block path for a batch (key, then kllm_index_lookup),
 * one sequence after another on the calling thread: slots[s * max_blocks + b]
 * receives the slot or -1. Used as the timed CPU baseline. */
void ref_build_slots(struct ref_index *r, const uint32_t *tokens, const int64_t *starts,
		     const int32_t *seq_lens, int num_seqs, int max_blocks,
		     int block_size, int64_t *slots)
{
	for (int s = 0; s < num_seqs; s++) {
		const uint32_t *tok = tokens + starts[s];
		const uint32_t len = (uint32_t)seq_lens[s];
		const uint32_t nb = (len + (uint32_t)block_size - 1) / (uint32_t)block_size;
		for (int b = 0; b < max_blocks; b++) {
			int64_t v = -1;
			if ((uint32_t)b < nb) {
				uint8_t key[32];
				uint32_t prefix_len = (uint32_t)(b + 1) * (uint32_t)block_size;
				if (prefix_len > len)
					prefix_len = len;
				SHA256((const unsigned char *)tok, prefix_len * sizeof(uint32_t), key);
				v = ref_index_lookup(r, key);
			}
			slots[(size_t)s * max_blocks + b] = v;
		}
	}
}

/* The same path with the keys spread over nthreads host threads (the keys
 * are independent SHA256 calls, as infer_gpu.c:110-118 makes them), then
 * the lookups on the calling thread (the index is lock-free single-threaded
 * by design, userspace/reactor/batch_scheduler.h:30-31). times[0] = keys
 * seconds, times[1] = lookup seconds. keys: [num_seqs][max_blocks][32]. */
struct key_job {
	const uint32_t *tokens;
	const int64_t *starts;
	const int32_t *seq_lens;
	int num_seqs, max_blocks, block_size, nthreads, tid;
	uint8_t *keys;
};

static void *key_worker(void *arg)
{
	struct key_job *j = arg;
	for (int s = j->tid; s < j->num_seqs; s += j->nthreads) {
		const uint32_t len = (uint32_t)j->seq_lens[s];
		const uint32_t nb = (len + (uint32_t)j->block_size - 1) / (uint32_t)j->block_size;
		for (uint32_t b = 0; b < nb && b < (uint32_t)j->max_blocks; b++) {
			uint32_t prefix_len = (b + 1) * (uint32_t)j->block_size;
			if (prefix_len > len)
				prefix_len = len;
			SHA256((const unsigned char *)(j->tokens + j->starts[s]),
			       prefix_len * sizeof(uint32_t),
			       j->keys + ((size_t)s * j->max_blocks + b) * 32);
		}
	}
	return NULL;
}

static double wall_s(void)
{
	struct timespec ts;
	clock_gettime(CLOCK_MONOTONIC, &ts);
	return ts.tv_sec + ts.tv_nsec * 1e-9;
}

int ref_build_slots_mt(struct ref_index *r, const uint32_t *tokens, const int64_t *starts,
		       const int32_t *seq_lens, int num_seqs, int max_blocks, int block_size,
		       int64_t *slots, uint8_t *keys, int nthreads, double times[2])
{
	if (nthreads < 1)
		nthreads = 1;
	if (nthreads > 256)
		nthreads = 256;
	pthread_t th[256];
	struct key_job jobs[256];
	const double t0 = wall_s();
	for (int t = 0; t < nthreads; t++) {
		jobs[t] = (struct key_job){ tokens, starts, seq_lens, num_seqs, max_blocks,
					    block_size, nthreads, t, keys };
		if (pthread_create(&th[t], NULL, key_worker, &jobs[t]))
			return -1;
	}
	for (int t = 0; t < nthreads; t++)
		pthread_join(th[t], NULL);
	const double t1 = wall_s();
	for (int s = 0; s < num_seqs; s++) {
		const uint32_t len = (uint32_t)seq_lens[s];
		const uint32_t nb = (len + (uint32_t)block_size - 1) / (uint32_t)block_size;
		for (int b = 0; b < max_blocks; b++)
			slots[(size_t)s * max_blocks + b] =
			    (uint32_t)b < nb
				? ref_index_lookup(r, keys + ((size_t)s * max_blocks + b) * 32)
				: -1;
	}
	times[0] = t1 - t0;
	times[1] = wall_s() - t1;
	return 0;
}
