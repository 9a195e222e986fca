/* SPDX-License-Identifier: Apache-2.0 */
/*
 * wavefront.c - KV block arrival into VRAM behind the reference's wavefront
 * interface (userspace/gpu/nvme_ep_wavefront.h), whose reference
 * implementation is a stub (nvme_ep_wavefront.c:74-104).
 *
 * submit (caller's thread): resolves every block's obj_key through the
 * caller's index (the cache index probe: bucket = first four key bytes,
 * little-endian, masked; linear probe to the first empty entry) to a record
 * offset, and queues the job. Up to four I/O threads per context take every
 * job in order, thread t the blocks i with i % threads == t. A thread
 * preads its blocks of a job into its next page-locked staging chunk (after
 * that chunk's previous use has completed), copies the chunk to device
 * memory with one cudaMemcpyAsync on its own stream, and launches one
 * scatter kernel that places each record at its destination
 * (wavefront_scatter.cu); an event per chunk and one per (job, thread).
 * Per-block copies were bound by the driver's per-call cost, which one copy
 * and one launch per chunk amortise. Because a kernel (not the copy engine)
 * writes the destinations, submit checks each one: device memory of this
 * context's GPU, inside one allocation; a block that fails is reported as
 * failed. poll (caller's thread) reports a job once every thread has passed
 * it and its events completed, in submit order. Nothing here waits without
 * a bound except an I/O thread on a staging chunk's own earlier use.
 */
#define _GNU_SOURCE
#include <errno.h>
#include <fcntl.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <cuda.h>
#include <cuda_runtime_api.h>

#include "kllm_gpu.h"
#include "kllm_internal.h"
#include "kllm_wavefront.h"

#define WF_QUEUE 64
#define WF_MAX_THREADS 4
#define WF_MAX_STAGE 16                 /* staging chunks per I/O thread */
#define WF_MIN_CHUNK (2u << 20)         /* a chunk holds many small blocks */
#define WF_RANGES 4                     /* allocations remembered within one submit */

struct wf_item {
	uint64_t off;
	uint64_t dst;
	uint32_t bytes;
	int ok;
};

struct wf_job {
	uint64_t seq;
	uint64_t t0;
	uint32_t n;
	uint32_t failed;                /* unresolved at submit, then added by the threads */
	uint64_t bytes;                 /* added by the threads */
	cudaEvent_t done[WF_MAX_THREADS];
	struct wf_item items[KLLM_WAVEFRONT_MAX_BLOCKS];
};

struct kllm_wavefront_ctx;

struct wf_worker {
	struct kllm_wavefront_ctx *c;
	int id;
	pthread_t thr;
	int started;
	cudaStream_t stream;
	int n_stage, next;
	uint8_t *stage[WF_MAX_STAGE];           /* page-locked host chunks */
	uint8_t *dev_stage[WF_MAX_STAGE];       /* their device copies */
	cudaEvent_t stage_ev[WF_MAX_STAGE];     /* the chunk's scatter has finished */
	uint32_t head;                  /* next job this thread issues (under mu) */
};

struct kllm_wavefront_ctx {
	int fd;
	int device;
	const struct kllm_gpu_index_entry *index;
	uint32_t capacity;
	uint64_t record_bytes, base_offset;
	uint64_t stage_bytes;                   /* largest block */
	uint64_t chunk_bytes;                   /* staging chunk */
	CUresult (*get_range)(CUdeviceptr *, size_t *, CUdeviceptr);
	int nthr;
	struct wf_worker w[WF_MAX_THREADS];
	struct wf_job jobs[WF_QUEUE];
	uint32_t tail;                  /* next free slot (submit) */
	uint32_t reported;              /* next job to report (poll) */
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

static uint64_t round16(uint64_t x)
{
	return (x + 15u) & ~(uint64_t)15u;
}

/* Copies chunk b (`used` bytes) to the device and places its records. */
static int flush(struct kllm_wavefront_ctx *c, struct wf_worker *wk, int b,
		 const struct kllm_wf_scatter *s, uint64_t used)
{
	if (cudaMemcpyAsync(wk->dev_stage[b], wk->stage[b], used, cudaMemcpyHostToDevice,
			    wk->stream) != cudaSuccess ||
	    kllm_wf_scatter_launch(s, wk->dev_stage[b], wk->stream) != 0 ||
	    cudaEventRecord(wk->stage_ev[b], wk->stream) != cudaSuccess) {
		cudaGetLastError();
		set_error(c);
		return -1;
	}
	return 0;
}

/* This thread's share of one job: blocks id, id + threads, ... */
static void issue(struct kllm_wavefront_ctx *c, struct wf_worker *wk, struct wf_job *j)
{
	uint32_t failed = 0;
	uint64_t bytes = 0, chunk_sum = 0, used = 0;
	struct kllm_wf_scatter s;
	int b = -1;                             /* chunk being filled */
	s.n = 0;
	s.reserved = 0;
	for (uint32_t i = (uint32_t)wk->id; i < j->n; i += (uint32_t)c->nthr) {
		struct wf_item *it = &j->items[i];
		if (!it->ok)
			continue;
		if (b >= 0 && used + round16(it->bytes) > c->chunk_bytes) {
			if (flush(c, wk, b, &s, used))
				failed += s.n;
			else
				bytes += chunk_sum;
			b = -1;
		}
		if (b < 0) {
			b = wk->next;
			wk->next = (b + 1) % wk->n_stage;
			/* the chunk's previous scatter must have finished with it */
			if (cudaEventSynchronize(wk->stage_ev[b]) != cudaSuccess) {
				cudaGetLastError();
				set_error(c);
				failed++;
				b = -1;
				continue;
			}
			s.n = 0;
			used = chunk_sum = 0;
		}
		if (read_full(c->fd, wk->stage[b] + used, it->bytes, it->off)) {
			failed++;
			continue;
		}
		s.dst[s.n] = it->dst;
		s.bytes[s.n] = it->bytes;
		s.off[s.n] = (uint32_t)used;
		s.n++;
		used += round16(it->bytes);
		chunk_sum += it->bytes;
	}
	if (b >= 0 && s.n) {
		if (flush(c, wk, b, &s, used))
			failed += s.n;
		else
			bytes += chunk_sum;
	}
	__atomic_add_fetch(&j->failed, failed, __ATOMIC_RELAXED);
	__atomic_add_fetch(&j->bytes, bytes, __ATOMIC_RELAXED);
	if (cudaEventRecord(j->done[wk->id], wk->stream) != cudaSuccess)
		set_error(c);
}

static void *io_main(void *arg)
{
	struct wf_worker *wk = arg;
	struct kllm_wavefront_ctx *c = wk->c;
	cudaSetDevice(c->device);
	pthread_mutex_lock(&c->mu);
	for (;;) {
		while (!c->stop && wk->head == c->tail)
			pthread_cond_wait(&c->cv, &c->mu);
		if (wk->head == c->tail && c->stop)
			break;
		struct wf_job *j = &c->jobs[wk->head % WF_QUEUE];
		pthread_mutex_unlock(&c->mu);
		issue(c, wk, j);
		pthread_mutex_lock(&c->mu);
		wk->head++;                     /* the mutex publishes this thread's counts */
	}
	pthread_mutex_unlock(&c->mu);
	return NULL;
}

/* Every thread has issued job `idx` (caller holds mu). */
static int issued_by_all(const struct kllm_wavefront_ctx *c, uint32_t idx)
{
	for (int t = 0; t < c->nthr; t++)
		if ((int32_t)(c->w[t].head - idx) <= 0)
			return 0;
	return 1;
}

void kllm_wavefront_destroy(struct kllm_wavefront_ctx *c)
{
	if (!c)
		return;
	pthread_mutex_lock(&c->mu);
	c->stop = 1;
	pthread_cond_broadcast(&c->cv);
	pthread_mutex_unlock(&c->mu);
	for (int t = 0; t < c->nthr; t++)
		if (c->w[t].started)
			pthread_join(c->w[t].thr, NULL);
	int prev = -1;
	const int switched = c->nthr > 0 && cudaGetDevice(&prev) == cudaSuccess &&
			     cudaSetDevice(c->device) == cudaSuccess;
	for (int t = 0; t < c->nthr; t++) {
		struct wf_worker *wk = &c->w[t];
		if (wk->stream)
			cudaStreamSynchronize(wk->stream);
		for (int b = 0; b < wk->n_stage; b++) {
			if (wk->stage[b])
				cudaFreeHost(wk->stage[b]);
			if (wk->dev_stage[b])
				cudaFree(wk->dev_stage[b]);
			if (wk->stage_ev[b])
				cudaEventDestroy(wk->stage_ev[b]);
		}
		if (wk->stream)
			cudaStreamDestroy(wk->stream);
	}
	for (int i = 0; i < WF_QUEUE; i++)
		for (int t = 0; t < WF_MAX_THREADS; t++)
			if (c->jobs[i].done[t])
				cudaEventDestroy(c->jobs[i].done[t]);
	if (switched)
		cudaSetDevice(prev);
	if (c->fd >= 0)
		close(c->fd);
	pthread_cond_destroy(&c->cv);
	pthread_mutex_destroy(&c->mu);
	free(c);
}

struct kllm_wavefront_ctx *kllm_wavefront_create2(const char *store_path, int device,
						  uint64_t max_block_bytes, int staging_buffers)
{
	if (!store_path || device < 0 || max_block_bytes == 0 ||
	    max_block_bytes > (1ull << 30) || staging_buffers < 2 || staging_buffers > 64)
		return NULL;
	struct kllm_wavefront_ctx *c = calloc(1, sizeof(*c));
	if (!c)
		return NULL;
	c->fd = -1;
	pthread_mutex_init(&c->mu, NULL);
	pthread_cond_init(&c->cv, NULL);
	c->device = device;
	c->stage_bytes = max_block_bytes;
	c->chunk_bytes = round16(max_block_bytes) > WF_MIN_CHUNK ? round16(max_block_bytes)
								 : WF_MIN_CHUNK;
	/* two or more staging chunks per thread, at most four threads */
	c->nthr = staging_buffers / 2 < WF_MAX_THREADS ? staging_buffers / 2 : WF_MAX_THREADS;
	const int per = staging_buffers / c->nthr < WF_MAX_STAGE ? staging_buffers / c->nthr
								 : WF_MAX_STAGE;
	c->fd = open(store_path, O_RDONLY | O_CLOEXEC);
	int ndev = 0, prev = -1;
	if (c->fd < 0 || cudaGetDeviceCount(&ndev) != cudaSuccess || device >= ndev ||
	    cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(device) != cudaSuccess) {
		cudaGetLastError();
		c->nthr = 0;
		kllm_wavefront_destroy(c);
		return NULL;
	}
	/* the caller's current device is put back before returning */
	void *fn = NULL;
	enum cudaDriverEntryPointQueryResult q;
	if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) !=
		cudaSuccess ||
	    q != cudaDriverEntryPointSuccess || !fn)
		goto fail_dev;
	c->get_range = (CUresult(*)(CUdeviceptr *, size_t *, CUdeviceptr))fn;
	for (int t = 0; t < c->nthr; t++) {
		struct wf_worker *wk = &c->w[t];
		wk->c = c;
		wk->id = t;
		wk->n_stage = per;
		if (cudaStreamCreateWithFlags(&wk->stream, cudaStreamNonBlocking) != cudaSuccess)
			goto fail_dev;
		for (int b = 0; b < per; b++)
			if (cudaHostAlloc((void **)&wk->stage[b], c->chunk_bytes,
					  cudaHostAllocDefault) != cudaSuccess ||
			    cudaMalloc((void **)&wk->dev_stage[b], c->chunk_bytes) != cudaSuccess ||
			    cudaEventCreateWithFlags(&wk->stage_ev[b], cudaEventDisableTiming) !=
				cudaSuccess)
				goto fail_dev;
	}
	for (int i = 0; i < WF_QUEUE; i++)
		for (int t = 0; t < c->nthr; t++)
			if (cudaEventCreateWithFlags(&c->jobs[i].done[t], cudaEventDisableTiming) !=
			    cudaSuccess)
				goto fail_dev;
	for (int t = 0; t < c->nthr; t++) {
		if (pthread_create(&c->w[t].thr, NULL, io_main, &c->w[t]))
			goto fail_dev;
		c->w[t].started = 1;
	}
	cudaSetDevice(prev);
	return c;
fail_dev:
	kllm_wavefront_destroy(c);
	cudaSetDevice(prev);
	cudaGetLastError();
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

struct wf_range {
	uint64_t lo, hi;
};

/* [dst, dst + bytes) lies inside one allocation of device memory on this
 * context's GPU. `seen` remembers the allocations found during one submit. */
static int dest_ok(struct kllm_wavefront_ctx *c, uint64_t dst, uint64_t bytes,
		   struct wf_range *seen, int *n_seen)
{
	const uint64_t end = dst + bytes;
	if (!dst || end < dst)
		return 0;
	for (int r = 0; r < *n_seen; r++)
		if (dst >= seen[r].lo && end <= seen[r].hi)
			return 1;
	struct cudaPointerAttributes a;
	memset(&a, 0, sizeof(a));
	if (cudaPointerGetAttributes(&a, (const void *)(uintptr_t)dst) != cudaSuccess) {
		cudaGetLastError();
		return 0;
	}
	if ((a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) ||
	    a.device != c->device)
		return 0;
	int prev = -1;
	CUdeviceptr base = 0;
	size_t size = 0;
	if (cudaGetDevice(&prev) != cudaSuccess || cudaSetDevice(c->device) != cudaSuccess) {
		cudaGetLastError();
		return 0;
	}
	const CUresult r = c->get_range(&base, &size, (CUdeviceptr)dst);
	cudaSetDevice(prev);
	if (r != CUDA_SUCCESS || dst < (uint64_t)base || end > (uint64_t)base + size)
		return 0;
	if (*n_seen < WF_RANGES) {
		seen[*n_seen].lo = (uint64_t)base;
		seen[*n_seen].hi = (uint64_t)base + size;
		(*n_seen)++;
	}
	return 1;
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
	struct wf_range seen[WF_RANGES];
	int n_seen = 0;
	for (uint32_t i = 0; i < j->n; i++) {
		const struct kllm_wf_block_desc *d = &wf->blocks[i];
		struct wf_item *it = &j->items[i];
		const int64_t rec = probe(c->index, c->capacity, d->obj_key);
		it->dst = d->vram_dest_addr;
		it->bytes = d->block_size;
		it->off = c->base_offset + (uint64_t)(rec < 0 ? 0 : rec) * c->record_bytes;
		it->ok = rec >= 0 && d->block_size > 0 && d->block_size <= c->stage_bytes &&
			 d->block_size <= c->record_bytes &&
			 dest_ok(c, d->vram_dest_addr, d->block_size, seen, &n_seen);
		if (!it->ok)
			j->failed++;
	}
	pthread_mutex_lock(&c->mu);
	c->tail++;
	pthread_cond_broadcast(&c->cv);
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
		const int issued = c->reported != c->tail && issued_by_all(c, c->reported);
		pthread_mutex_unlock(&c->mu);
		if (!issued)
			break;
		struct wf_job *j = &c->jobs[c->reported % WF_QUEUE];
		int busy = 0;
		for (int t = 0; t < c->nthr && !busy; t++) {
			const cudaError_t q = cudaEventQuery(j->done[t]);
			if (q == cudaErrorNotReady) {
				busy = 1;
			} else if (q != cudaSuccess) {
				cudaGetLastError();
				set_error(c);
			}
		}
		if (busy)
			break;
		out[n].sequence_id = j->seq;
		out[n].blocks_failed = j->failed;
		out[n].blocks_completed = j->n - j->failed;
		out[n].total_bytes = j->bytes;
		out[n].latency_ns = mono_ns() - j->t0;
		n++;
		pthread_mutex_lock(&c->mu);
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
