// Device-to-device copy: the measured ceiling every streaming kernel here is compared with (the
// reference reports its prefill kernels as a fraction of a same-bytes D2D copy,
// benchmarks/copy_baseline.py:38-90). It moves exactly what a prefill moves, each byte read once
// and written once, with the widest accesses sm_100 has (32-byte vectors), so the gap between a
// kernel and this copy is what the kernel's own work costs.
//
// copy_kernel: one tile of kCopyThreads x kCopyUnroll 32-byte chunks per CTA, every thread
// issuing its kCopyUnroll loads before its stores, and as many CTAs as tiles: the hardware runs them
// in waves, so the bytes requested at any moment lie in a narrow window of consecutive tiles.
// Measured on B200 with 512 MiB in and out: 162.2 us with one tile of 2 chunks per thread, against
// 172.0 us for cudaMemcpyAsync and 184-186 us for a single wave of CTAs each walking a long run
// (per-warp runs or a grid-stride loop). A tail that is not a whole chunk is copied byte by byte.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace cc1d {

namespace {

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 2;

__global__ void __launch_bounds__(kCopyThreads)
    copy_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, int64_t chunks,
                int64_t bytes) {
    const int64_t k0 = (int64_t)blockIdx.x * kCopyThreads * kCopyUnroll + threadIdx.x;
    uint4 lo[kCopyUnroll], hi[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t k = k0 + u * kCopyThreads;
        if (k < chunks) ldg32_stream(src + k * 32, lo[u], hi[u]);
    }
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t k = k0 + u * kCopyThreads;
        if (k < chunks) st32_stream(dst + k * 32, lo[u], hi[u]);
    }
    if (blockIdx.x == 0 && threadIdx.x < 32) {
        for (int64_t i = chunks * 32 + threadIdx.x; i < bytes; i += 32) dst[i] = src[i];
    }
}

}  // namespace

cudaError_t launch_copy(void* dst, const void* src, int64_t bytes, cudaStream_t stream) {
    if (bytes <= 0) return cudaSuccess;
    const int64_t chunks = bytes / 32;
    const int64_t blocks =
        std::max<int64_t>(1, ceil_div(chunks, (int64_t)kCopyThreads * kCopyUnroll));
    if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
    copy_kernel<<<(unsigned)blocks, kCopyThreads, 0, stream>>>((uint8_t*)dst, (const uint8_t*)src,
                                                               chunks, bytes);
    return cudaGetLastError();
}

}  // namespace cc1d
