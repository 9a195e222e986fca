/* SPDX-License-Identifier: Apache-2.0 */
/*
 * content_index.c - CPU restatement of the content-addressed block-table
 * path: the block key (SHA-256 of the token prefix), the probe of the cache
 * index, and the slot -> page pointer map. TEST INFRASTRUCTURE ONLY (see
 * kllm_oracle.h).
 *
 * The reference computes the key with OpenSSL's SHA256() (OpenSSL 3.0.13 in
 * this image); the function below restates the published algorithm, FIPS
 * 180-4 section 6.2, and is pinned against that library call (and against
 * Python's hashlib) by the tests.
 */
#include "kllm_oracle.h"

#include <string.h>

/* FIPS 180-4 4.2.2: first 32 bits of the fractional parts of the cube roots
 * of the first 64 primes (the tests recompute them from that definition). */
static const uint32_t sha_k[64] = {
	0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u,
	0x923f82a4u, 0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u,
	0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u,
	0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
	0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u,
	0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u,
	0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
	0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
	0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au,
	0x5b9cca4fu, 0x682e6ff3u, 0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u,
	0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u,
};

/* FIPS 180-4 5.3.3: first 32 bits of the fractional parts of the square
 * roots of the first 8 primes. */
static const uint32_t sha_h0[8] = {
	0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
	0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u,
};

static uint32_t rotr(uint32_t x, int n)
{
	return (x >> n) | (x << (32 - n));
}

/* FIPS 180-4 6.2.2: one compression of a 64-byte message block. */
static void sha_compress(uint32_t h[8], const uint8_t blk[64])
{
	uint32_t w[64];
	for (int t = 0; t < 16; t++)
		w[t] = (uint32_t)blk[4 * t] << 24 | (uint32_t)blk[4 * t + 1] << 16 |
		       (uint32_t)blk[4 * t + 2] << 8 | (uint32_t)blk[4 * t + 3];
	for (int t = 16; t < 64; t++) {
		uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
		uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
		w[t] = w[t - 16] + s0 + w[t - 7] + s1;
	}
	uint32_t a = h[0], b = h[1], c = h[2], d = h[3];
	uint32_t e = h[4], f = h[5], g = h[6], hh = h[7];
	for (int t = 0; t < 64; t++) {
		uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) +
			      ((e & f) ^ (~e & g)) + sha_k[t] + w[t];
		uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) +
			      ((a & b) ^ (a & c) ^ (b & c));
		hh = g;
		g = f;
		f = e;
		e = d + t1;
		d = c;
		c = b;
		b = a;
		a = t1 + t2;
	}
	h[0] += a;
	h[1] += b;
	h[2] += c;
	h[3] += d;
	h[4] += e;
	h[5] += f;
	h[6] += g;
	h[7] += hh;
}

void orc_sha256(const void *msg, size_t len, uint8_t out[32])
{
	const uint8_t *p = (const uint8_t *)msg;
	uint32_t h[8];
	uint8_t blk[64];
	size_t full = len / 64, rem = len % 64;

	memcpy(h, sha_h0, sizeof(h));
	for (size_t i = 0; i < full; i++)
		sha_compress(h, p + 64 * i);
	/* FIPS 180-4 5.1.1: 0x80, zeros, 64-bit big-endian bit length. */
	memset(blk, 0, sizeof(blk));
	memcpy(blk, p + 64 * full, rem);
	blk[rem] = 0x80;
	if (rem >= 56) {
		sha_compress(h, blk);
		memset(blk, 0, sizeof(blk));
	}
	const uint64_t bits = (uint64_t)len * 8u;
	for (int i = 0; i < 8; i++)
		blk[56 + i] = (uint8_t)(bits >> (56 - 8 * i));
	sha_compress(h, blk);
	for (int i = 0; i < 8; i++) {
		out[4 * i] = (uint8_t)(h[i] >> 24);
		out[4 * i + 1] = (uint8_t)(h[i] >> 16);
		out[4 * i + 2] = (uint8_t)(h[i] >> 8);
		out[4 * i + 3] = (uint8_t)h[i];
	}
}

/* userspace/compute/infer_gpu.c:110-118: the key of block b hashes the
 * token ids [0, min((b + 1) * block_size, seq_len)) as stored (uint32,
 * little-endian bytes), from scratch for every block as the reference
 * does. */
void orc_block_key(const uint32_t *tokens, int seq_len, int block_size, int b,
		   uint8_t out[32])
{
	int64_t n = (int64_t)(b + 1) * block_size;
	if (n > seq_len)
		n = seq_len;
	orc_sha256(tokens, (size_t)n * sizeof(uint32_t), out);
}

/* userspace/kvcache/cache_index.c:35-41 (bucket = first four key bytes read
 * as a little-endian uint32, masked) and :87-108 (linear probe that stops at
 * the first empty entry; a full-key match is a hit). Returns the entry's
 * position or -1. */
int64_t orc_index_probe(const struct orc_index_entry *entries, uint32_t capacity,
			const uint8_t hash[32])
{
	const uint32_t mask = capacity - 1;
	uint32_t bucket = (uint32_t)hash[0] | (uint32_t)hash[1] << 8 |
			  (uint32_t)hash[2] << 16 | (uint32_t)hash[3] << 24;
	bucket &= mask;
	for (uint32_t i = 0; i < capacity; i++) {
		const uint32_t pos = (bucket + i) & mask;
		const struct orc_index_entry *e = &entries[pos];
		if (e->slot_index == ORC_INDEX_EMPTY)
			return -1;
		if (memcmp(e->hash, hash, 32) == 0)
			return pos;
	}
	return -1;
}

/* The block-table builder, restated from its reference pieces: per block b
 * of sequence s (b >= first_block[s]), key = orc_block_key, position =
 * orc_index_probe; a hit stamps the entry's last_access_ns with now_ns
 * (cache_index.c:101, when now_ns != 0) and maps the slot to the page
 * pointers arena_base + slot * slot_bytes + {k,v}_offset
 * (arena_alloc.c:196-201: NULL for slot >= total_slots, which the table
 * marks invalid). Blocks past the sequence (up to max_blocks) become zero
 * entries; blocks below first_block are left as they are. Returns the
 * KLLM_ERR_SEQ_TOO_LONG bit (1) when a sequence had to be cut at
 * max_blocks * block_size tokens. */
int orc_build_block_tables(const uint32_t *tokens, const int64_t *starts,
			   const int32_t *seq_lens, const int32_t *first_block,
			   int num_seqs, int max_blocks, int block_size,
			   struct orc_index_entry *index, uint32_t capacity,
			   uint64_t now_ns, uint64_t arena_base,
			   uint64_t slot_bytes, uint64_t total_slots,
			   uint64_t k_offset, uint64_t v_offset,
			   struct orc_entry *table, uint8_t *hashes,
			   uint64_t *hits, uint64_t *misses)
{
	int err = 0;
	for (int s = 0; s < num_seqs; s++) {
		int len = seq_lens[s] < 0 ? 0 : seq_lens[s];
		if ((int64_t)len > (int64_t)max_blocks * block_size) {
			len = max_blocks * block_size;
			err |= 1;
		}
		const int nb = (len + block_size - 1) / block_size;
		const int b0 = first_block ? first_block[s] : 0;
		const uint32_t *tok = tokens + starts[s];
		for (int b = b0 < 0 ? 0 : b0; b < max_blocks; b++) {
			struct orc_entry *te = &table[(size_t)s * max_blocks + b];
			uint8_t *hk = hashes ? hashes + ((size_t)s * max_blocks + b) * 32 : NULL;
			memset(te, 0, sizeof(*te));
			if (b >= nb) {
				if (hk)
					memset(hk, 0, 32);
				continue;
			}
			uint8_t key[32];
			orc_block_key(tok, len, block_size, b, key);
			if (hk)
				memcpy(hk, key, 32);
			const int64_t pos = orc_index_probe(index, capacity, key);
			if (pos < 0) {
				(*misses)++;
				continue;
			}
			(*hits)++;
			if (now_ns)
				index[pos].last_access_ns = now_ns;
			const uint64_t slot = index[pos].slot_index;
			if (slot >= total_slots)
				continue;
			const uint64_t page = arena_base + slot * slot_bytes;
			te->k_ptr = (const void *)(uintptr_t)(page + k_offset);
			te->v_ptr = (const void *)(uintptr_t)(page + v_offset);
			te->valid = 1;
		}
	}
	return err;
}
