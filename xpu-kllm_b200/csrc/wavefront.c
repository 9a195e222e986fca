/* SPDX-License-Identifier: Apache-2.0 */
/*
 * wavefront.c - KV block arrival into VRAM behind the reference's wavefront
 * interface (userspace/gpu/nvme_ep_wavefront.h), whose reference
 * implementation is a stub (nvme_ep_wavefront.c:74-104).
 *
 * submit (caller's thread): resolves every block's obj_key through the
 * caller's index (the cache index probe: bucket = first four key bytes,
 * little-endian, masked; linear probe to the first empty entry) to a record
 * offset, and queues the job. One I/O thread per context takes jobs in
 * order: pread of each record into the next page-locked staging buffer
 * (after that buffer's previous copy has completed), cudaMemcpyAsync to the
 * destination on the context's stream, an event per buffer and one per job.
 * poll (caller's thread) reports jobs whose event completed, in submit
 * order. Nothing here waits without a bound except the I/O thread on a
 * staging buffer's own earlier copy.
 */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <cuda_runtime_api.h>

#include "kllm_gpu.h"
#include "kllm_wavefront.h"

#define WF_QUEUE 64

enum { JOB_FREE = 0, JOB_QUEUED, JOB_ISSUED };

struct wf_item {
	uint64_t off;
	uint64_t dst;
	uint32_t bytes;
	int ok;
};

struct wf_job {
	int state;
	uint64_t seq;
	uint64_t t0;
	uint32_t n, failed;
	uint64_t bytes;
	cudaEvent_t done;
	struct wf_item items[KLLM_WAVEFRONT_MAX_BLOCKS];
};

struct kllm_wavefront_ctx {
	int fd;
	int device;
	cudaStream_t stream;
	const struct kllm_gpu_index_entry *index;
	uint32_t capacity;
	uint64_t record_bytes, base_offset;
	int n_stage;
	uint64_t stage_bytes;
	uint8_t *stage[64];
	cudaEvent_t stage_ev[64];
	int stage_next;
	struct wf_job jobs[WF_QUEUE];
	uint32_t head;      /* next job to issue (I/O thread) */
	uint32_t tail;      /* next free slot (submit) */
	uint32_t reported;  /* next job to report (poll) */
	pthread_t thr;
	int thr_started;
	pthread_mutex_t mu;
	pthread_cond_t cv;
	int stop;
	int error;
};

static uint64_t mono_ns(void)
{
	struct timespec ts;
	clock_gettime(CLOCK_MONOTONIC, &ts);
	return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

/* userspace/kvcache/cache_index.c:35-41, 87-108 */
static int64_t probe(const struct kllm_gpu_index_entry *e, uint32_t capacity,
		     const uint8_t key[32])
{
	const uint32_t mask = capacity - 1;
	uint32_t bucket = (uint32_t)key[0] | (uint32_t)key[1] << 8 |
			  (uint32_t)key[2] << 16 | (uint32_t)key[3] << 24;
	bucket &= mask;
	for (uint32_t i = 0; i < capacity; i++) {
		const uint32_t pos = (bucket + i) & mask;
		if (e[pos].slot_index == 0xFFFFFFFFu)
			return -1;
		if (memcmp(e[pos].hash, key, 32) == 0)
			return (int64_t)e[pos].slot_index;
	}
	return -1;
}

static int read_full(int fd, uint8_t *dst, uint64_t bytes, uint64_t off)
{
	uint64_t got = 0;
	while (got < bytes) {
		ssize_t r = pread(fd, dst + got, bytes - got, (off_t)(off + got));
		if (r < 0 && errno == EINTR)
			continue;
		if (r <= 0)
			return -1;
		got += (uint64_t)r;
	}
	return 0;
}

static void set_error(struct kllm_wavefront_ctx *c)
{
	pthread_mutex_lock(&c->mu);
	if (!c->error)
		c->error = KLLM_EIO;
	pthread_mutex_unlock(&c->mu);
}

static void issue(struct kllm_wavefront_ctx *c, struct wf_job *j)
{
	for (uint32_t i = 0; i < j->n; i++) {
		struct wf_item *it = &j->items[i];
		if (!it->ok)
			continue;
		const int b = c->stage_next;
		c->stage_next = (b + 1) % c->n_stage;
		/* the buffer's previous copy must have left it */
		if (cudaEventSynchronize(c->stage_ev[b]) != cudaSuccess) {
			set_error(c);
			it->ok = 0;
			j->failed++;
			continue;
		}
		if (read_full(c->fd, c->stage[b], it->bytes, it->off)) {
			it->ok = 0;
			j->failed++;
			continue;
		}
		if (cudaMemcpyAsync((void *)(uintptr_t)it->dst, c->stage[b], it->bytes,
				    cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
		    cudaEventRecord(c->stage_ev[b], c->stream) != cudaSuccess) {
			set_error(c);
			it->ok = 0;
			j->failed++;
			continue;
		}
		j->bytes += it->bytes;
	}
	if (cudaEventRecord(j->done, c->stream) != cudaSuccess)
		set_error(c);
}

static void *io_main(void *arg)
{
	struct kllm_wavefront_ctx *c = arg;
	cudaSetDevice(c->device);
	pthread_mutex_lock(&c->mu);
	for (;;) {
		while (!c->stop && c->head == c->tail)
			pthread_cond_wait(&c->cv, &c->mu);
		if (c->head == c->tail && c->stop)
			break;
		struct wf_job *j = &c->jobs[c->head % WF_QUEUE];
		pthread_mutex_unlock(&c->mu);
		issue(c, j);
		pthread_mutex_lock(&c->mu);
		j->state = JOB_ISSUED;
		c->head++;
	}
	pthread_mutex_unlock(&c->mu);
	return NULL;
}

void kllm_wavefront_destroy(struct kllm_wavefront_ctx *c)
{
	if (!c)
		return;
	if (c->thr_started) {
		pthread_mutex_lock(&c->mu);
		c->stop = 1;
		pthread_cond_signal(&c->cv);
		pthread_mutex_unlock(&c->mu);
		pthread_join(c->thr, NULL);
	}
	if (c->stream)
		cudaStreamSynchronize(c->stream);
	for (int b = 0; b < c->n_stage; b++) {
		if (c->stage[b])
			cudaFreeHost(c->stage[b]);
		if (c->stage_ev[b])
			cudaEventDestroy(c->stage_ev[b]);
	}
	for (int i = 0; i < WF_QUEUE; i++)
		if (c->jobs[i].done)
			cudaEventDestroy(c->jobs[i].done);
	if (c->stream)
		cudaStreamDestroy(c->stream);
	if (c->fd >= 0)
		close(c->fd);
	pthread_cond_destroy(&c->cv);
	pthread_mutex_destroy(&c->mu);
	free(c);
}

struct kllm_wavefront_ctx *kllm_wavefront_create2(const char *store_path, int device,
						  uint64_t max_block_bytes, int staging_buffers)
{
	if (!store_path || device < 0 || max_block_bytes == 0 || staging_buffers < 2 ||
	    staging_buffers > 64)
		return NULL;
	struct kllm_wavefront_ctx *c = calloc(1, sizeof(*c));
	if (!c)
		return NULL;
	c->fd = -1;
	pthread_mutex_init(&c->mu, NULL);
	pthread_cond_init(&c->cv, NULL);
	c->device = device;
	c->n_stage = staging_buffers;
	c->stage_bytes = max_block_bytes;
	c->fd = open(store_path, O_RDONLY | O_CLOEXEC);
	int ndev = 0, prev = -1;
	if (c->fd < 0 || cudaGetDeviceCount(&ndev) != cudaSuccess || device >= ndev ||
	    cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess)
		goto fail;
	/* the caller's current device is put back before returning */
	const cudaError_t se = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
	if (se != cudaSuccess)
		goto fail_dev;
	for (int b = 0; b < c->n_stage; b++)
		if (cudaHostAlloc((void **)&c->stage[b], max_block_bytes, cudaHostAllocDefault) !=
			cudaSuccess ||
		    cudaEventCreateWithFlags(&c->stage_ev[b], cudaEventDisableTiming) != cudaSuccess)
			goto fail_dev;
	for (int i = 0; i < WF_QUEUE; i++)
		if (cudaEventCreateWithFlags(&c->jobs[i].done, cudaEventDisableTiming) != cudaSuccess)
			goto fail_dev;
	if (pthread_create(&c->thr, NULL, io_main, c))
		goto fail_dev;
	c->thr_started = 1;
	cudaSetDevice(prev);
	return c;
fail_dev:
	kllm_wavefront_destroy(c);
	cudaSetDevice(prev);
	cudaGetLastError();
	return NULL;
fail:
	cudaGetLastError();
	kllm_wavefront_destroy(c);
	return NULL;
}

struct kllm_wavefront_ctx *kllm_wavefront_create(const char *nvme_ep_dev)
{
	const char *dv = getenv("KLLM_GPU_DEVICE");
	return kllm_wavefront_create2(nvme_ep_dev, dv ? atoi(dv) : 0, 4ull << 20, 8);
}

int kllm_wavefront_set_index(struct kllm_wavefront_ctx *c,
			     const struct kllm_gpu_index_entry *entries, uint32_t capacity,
			     uint64_t record_bytes, uint64_t base_offset)
{
	if (!c || !entries || !capacity || (capacity & (capacity - 1)) || !record_bytes)
		return KLLM_EINVAL;
	c->index = entries;
	c->capacity = capacity;
	c->record_bytes = record_bytes;
	c->base_offset = base_offset;
	return KLLM_OK;
}

int kllm_wavefront_submit(struct kllm_wavefront_ctx *c, const struct kllm_wavefront *wf)
{
	if (!c || !wf || wf->num_blocks == 0 || wf->num_blocks > KLLM_WAVEFRONT_MAX_BLOCKS ||
	    !c->index)
		return -1;
	if (c->tail - c->reported >= WF_QUEUE)
		return -1;                                /* every job slot is in flight */
	struct wf_job *j = &c->jobs[c->tail % WF_QUEUE];
	j->seq = wf->sequence_id;
	j->t0 = mono_ns();
	j->n = wf->num_blocks;
	j->failed = 0;
	j->bytes = 0;
	for (uint32_t i = 0; i < j->n; i++) {
		const struct kllm_wf_block_desc *d = &wf->blocks[i];
		struct wf_item *it = &j->items[i];
		const int64_t rec = probe(c->index, c->capacity, d->obj_key);
		it->dst = d->vram_dest_addr;
		it->bytes = d->block_size;
		it->off = c->base_offset + (uint64_t)(rec < 0 ? 0 : rec) * c->record_bytes;
		it->ok = rec >= 0 && d->block_size > 0 && d->block_size <= c->stage_bytes &&
			 d->block_size <= c->record_bytes && d->vram_dest_addr;
		if (!it->ok)
			j->failed++;
	}
	pthread_mutex_lock(&c->mu);
	j->state = JOB_QUEUED;
	c->tail++;
	pthread_cond_signal(&c->cv);
	pthread_mutex_unlock(&c->mu);
	return 0;
}

int kllm_wavefront_poll(struct kllm_wavefront_ctx *c, struct kllm_wf_completion *out,
			int max_completions)
{
	if (!c || (!out && max_completions > 0) || max_completions < 0)
		return -1;
	int n = 0;
	while (n < max_completions) {
		pthread_mutex_lock(&c->mu);
		const int issued = c->reported != c->head;
		pthread_mutex_unlock(&c->mu);
		if (!issued)
			break;
		struct wf_job *j = &c->jobs[c->reported % WF_QUEUE];
		const cudaError_t q = cudaEventQuery(j->done);
		if (q == cudaErrorNotReady)
			break;
		if (q != cudaSuccess) {
			cudaGetLastError();
			set_error(c);
		}
		out[n].sequence_id = j->seq;
		out[n].blocks_failed = j->failed;
		out[n].blocks_completed = j->n - j->failed;
		out[n].total_bytes = j->bytes;
		out[n].latency_ns = mono_ns() - j->t0;
		n++;
		pthread_mutex_lock(&c->mu);
		j->state = JOB_FREE;
		c->reported++;
		pthread_mutex_unlock(&c->mu);
	}
	return n;
}

int kllm_wavefront_wait(struct kllm_wavefront_ctx *c, struct kllm_wf_completion *out,
			int max_completions, int timeout_ms)
{
	if (!c || max_completions <= 0 || !out)
		return -1;
	const uint64_t limit = mono_ns() + (uint64_t)(timeout_ms < 0 ? 0 : timeout_ms) * 1000000ull;
	for (;;) {
		const int n = kllm_wavefront_poll(c, out, max_completions);
		if (n != 0 || mono_ns() >= limit)
			return n;
		struct timespec ts = { 0, 20000 };      /* 20 us between polls */
		nanosleep(&ts, NULL);
	}
}

int kllm_wavefront_error(struct kllm_wavefront_ctx *c)
{
	if (!c)
		return KLLM_EINVAL;
	pthread_mutex_lock(&c->mu);
	const int e = c->error;
	pthread_mutex_unlock(&c->mu);
	return e;
}
