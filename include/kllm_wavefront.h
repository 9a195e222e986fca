/* SPDX-License-Identifier: Apache-2.0 */
/*
 * kllm_wavefront.h - KV block arrival into VRAM: batched block fetches
 * ("wavefronts") from a content-addressed block store, completed
 * asynchronously and polled without blocking.
 *
 * Part 1 is the reference's interface, same names, struct layouts and
 * return conventions (userspace/gpu/nvme_ep_wavefront.h:28-80), whose
 * reference implementation is a stub: submit returns 0 without reading and
 * poll never reports a completion (userspace/gpu/nvme_ep_wavefront.c:
 * 74-104), so the waiting caller (userspace/compute/infer_gpu.c:147-151)
 * spins forever. Here submit queues real reads and poll reports them.
 *
 * The store: a file (or block device) holding fixed-size block records; a
 * block's obj_key is resolved to its record through an index with the
 * cache index's layout and probe (struct kllm_gpu_index_entry, slot_index =
 * record number), given by kllm_wavefront_set_index. Resolution happens in
 * submit, on the caller's thread, which also checks that every
 * vram_dest_addr range lies in one device allocation on the context's GPU
 * (a block that does not is reported failed). Up to four I/O threads (one
 * per two staging buffers) split each wavefront's blocks, read the records
 * into their own page-locked staging buffers, copy each buffer to the GPU
 * in one piece and place its records with one kernel launch, on their own
 * CUDA streams; completion is one CUDA event per thread that poll queries,
 * and jobs are reported in submit order.
 *
 * Return conventions: submit 0 / -1 (reference), poll the number of
 * completions filled. Extensions return 0 or a negative KLLM_E* code.
 * Threading: submit, poll and wait are called from one thread (the
 * reactor's); the context owns its I/O threads.
 */
#ifndef KLLM_WAVEFRONT_H
#define KLLM_WAVEFRONT_H

#include <stdint.h>

#include "kllm_gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- Part 1: the reference's interface (nvme_ep_wavefront.h:28-80) ---- */

#define KLLM_WAVEFRONT_MAX_BLOCKS	64
#define KLLM_SEQ_HASH_BYTES		32

struct kllm_wf_block_desc {
	uint8_t  obj_key[KLLM_SEQ_HASH_BYTES];  /* content-address key */
	uint64_t vram_dest_addr;                  /* device destination */
	uint32_t block_size;                      /* bytes to transfer */
	uint32_t layer_start;
	uint32_t layer_count;
	uint32_t _pad;
};

struct kllm_wavefront {
	uint32_t num_blocks;
	uint32_t flags;
	uint64_t sequence_id;                     /* echoed in the completion */
	struct kllm_wf_block_desc blocks[KLLM_WAVEFRONT_MAX_BLOCKS];
};

#define KLLM_WF_FLAG_WEIGHT_LOAD	(1 << 0)
#define KLLM_WF_FLAG_KV_FETCH		(1 << 1)
#define KLLM_WF_FLAG_PREFETCH		(1 << 2)

struct kllm_wf_completion {
	uint64_t sequence_id;
	uint32_t blocks_completed;
	uint32_t blocks_failed;                   /* key not in the store, short read */
	uint64_t total_bytes;
	uint64_t latency_ns;                      /* submit -> copies complete */
};

struct kllm_wavefront_ctx;

/* Opens the store (path of a file or block device) on the device named by
 * KLLM_GPU_DEVICE (default 0), with 8 staging buffers of 4 MiB; NULL on
 * failure (no such file, no CUDA device). */
struct kllm_wavefront_ctx *kllm_wavefront_create(const char *nvme_ep_dev);
void kllm_wavefront_destroy(struct kllm_wavefront_ctx *ctx);
/* Queues the wavefront (FIFO, at most 64 in flight); 0, or -1 on a bad
 * argument, a full queue or no index set. Never blocks on I/O. */
int kllm_wavefront_submit(struct kllm_wavefront_ctx *ctx,
			  const struct kllm_wavefront *wf);
/* Fills up to max_completions records of finished wavefronts, in submit
 * order; never blocks. Returns the count, or -1 on a bad argument. */
int kllm_wavefront_poll(struct kllm_wavefront_ctx *ctx,
			struct kllm_wf_completion *completions, int max_completions);

/* ---- Part 2: extensions ------------------------------------------------- */

/* As kllm_wavefront_create with the device, the largest block (at most
 * 1 GiB) and the number of staging buffers (2..64) chosen; the buffers are
 * shared out over min(4, staging_buffers / 2) I/O threads, and each holds
 * max(largest block, 2 MiB) in page-locked host memory plus as much device
 * memory. */
struct kllm_wavefront_ctx *kllm_wavefront_create2(const char *store_path, int device,
						  uint64_t max_block_bytes, int staging_buffers);
/* The key -> record map: entries (host memory, [capacity], capacity a
 * power of two) stay owned by the caller and are read by submit only; a
 * key's record starts at base_offset + slot_index * record_bytes. */
int kllm_wavefront_set_index(struct kllm_wavefront_ctx *ctx,
			     const struct kllm_gpu_index_entry *entries, uint32_t capacity,
			     uint64_t record_bytes, uint64_t base_offset);
/* Bounded wait: polls until at least one completion is filled or
 * timeout_ms passes (then returns 0). Replaces the unbounded spin of
 * infer_gpu.c:147-151. */
int kllm_wavefront_wait(struct kllm_wavefront_ctx *ctx,
			struct kllm_wf_completion *completions, int max_completions,
			int timeout_ms);
/* The I/O thread's first error (a failed CUDA call: KLLM_EIO), else 0. */
int kllm_wavefront_error(struct kllm_wavefront_ctx *ctx);

#ifdef __cplusplus
}
#endif

#endif /* KLLM_WAVEFRONT_H */
