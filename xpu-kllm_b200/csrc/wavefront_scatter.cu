// SPDX-License-Identifier: Apache-2.0
//
// wavefront_scatter.cu - the device half of KV block arrival.
//
// An I/O thread of the wavefront reads up to 64 block records into one
// page-locked chunk, copies the chunk to device memory with one
// host-to-device copy, and launches this kernel to place each record at its
// destination. One copy and one launch per chunk replace one copy per block,
// whose per-call cost in the driver bounded the host-staged path. Every
// destination range was checked on the host (device memory of this GPU,
// inside one allocation) before it reaches a descriptor.

#include "kllm_internal.h"

#include <cuda_runtime.h>

namespace {

constexpr int kThreads = 256;

// One CTA per record: 16-byte stores when the destination allows them, the
// ragged tail (and an unaligned destination) byte by byte.
__global__ void __launch_bounds__(kThreads)
wf_scatter_kernel(const __grid_constant__ kllm_wf_scatter s, const uint8_t *__restrict__ src)
{
	const uint32_t b = blockIdx.x;
	uint8_t *dst = reinterpret_cast<uint8_t *>(s.dst[b]);
	const uint8_t *from = src + s.off[b];                   // 16-byte aligned by the host
	const uint32_t bytes = s.bytes[b];
	uint32_t done = 0;
	if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
		const uint32_t n16 = bytes >> 4;
		const uint4 *f4 = reinterpret_cast<const uint4 *>(from);
		uint4 *d4 = reinterpret_cast<uint4 *>(dst);
		for (uint32_t i = threadIdx.x; i < n16; i += kThreads)
			d4[i] = f4[i];
		done = n16 << 4;
	}
	for (uint32_t i = done + threadIdx.x; i < bytes; i += kThreads)
		dst[i] = from[i];
}

}  // namespace

extern "C" int kllm_wf_scatter_launch(const struct kllm_wf_scatter *s, const void *src_dev,
				      void *stream)
{
	if (!s || !src_dev || s->n == 0 || s->n > KLLM_WF_SCATTER_MAX)
		return -1;
	wf_scatter_kernel<<<s->n, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
	    *s, static_cast<const uint8_t *>(src_dev));
	return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
