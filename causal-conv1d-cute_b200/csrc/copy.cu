// Device-to-device copy: the measured ceiling every streaming kernel here is compared with (the
// reference reports its prefill kernels as a fraction of a same-bytes D2D copy,
// benchmarks/copy_baseline.py:38-90). It moves exactly what a prefill moves, each byte read once
// and written once, with the widest accesses sm_100 has (32-byte vectors), so the gap between a
// kernel and this copy is what the kernel's own work costs.
//
// copy_kernel: one wave of CTAs; warp w walks a contiguous run of 32-byte chunks, every lane
// keeping U chunks in flight (all U loads issued before the first store), so the loads of a warp
// cover U * 1 KB of consecutive bytes. A tail that is not a whole chunk is copied byte by byte.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace cc1d {

namespace {

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;

__global__ void __launch_bounds__(kCopyThreads)
    copy_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, int64_t chunks,
                int64_t per_warp, int64_t bytes) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * kCopyThreads + threadIdx.x) >> 5;
    const int64_t c0 = warp * per_warp;
    const int64_t c1 = c0 + per_warp < chunks ? c0 + per_warp : chunks;
    for (int64_t c = c0; c < c1; c += 32 * kCopyUnroll) {
        uint4 lo[kCopyUnroll], hi[kCopyUnroll];
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) {
            const int64_t k = c + u * 32 + lane;
            if (k < c1) ldg32_stream(src + k * 32, lo[u], hi[u]);
        }
#pragma unroll
        for (int u = 0; u < kCopyUnroll; ++u) {
            const int64_t k = c + u * 32 + lane;
            if (k < c1) st32_stream(dst + k * 32, lo[u], hi[u]);
        }
    }
    if (warp == 0) {
        for (int64_t i = chunks * 32 + lane; i < bytes; i += 32) dst[i] = src[i];
    }
}

}  // namespace

cudaError_t launch_copy(void* dst, const void* src, int64_t bytes, cudaStream_t stream) {
    if (bytes <= 0) return cudaSuccess;
    const int64_t chunks = bytes / 32;
    static int slot_cache[kSlotCacheDevices] = {};
    const int64_t slots = std::max(1, device_slots((const void*)copy_kernel, kCopyThreads, slot_cache));
    const int64_t warps_wave = slots * (kCopyThreads / 32);
    // Runs a whole number of warp steps (32 lanes x U chunks) long, one wave of warps in total.
    const int64_t step = 32 * kCopyUnroll;
    const int64_t per_warp = std::max<int64_t>(step, ceil_div(ceil_div(chunks, warps_wave), step) * step);
    const int64_t warps = std::max<int64_t>(1, ceil_div(chunks, per_warp));
    const int64_t blocks = ceil_div(warps * 32, (int64_t)kCopyThreads);
    copy_kernel<<<(unsigned)blocks, kCopyThreads, 0, stream>>>((uint8_t*)dst, (const uint8_t*)src,
                                                               chunks, per_warp, bytes);
    return cudaGetLastError();
}

}  // namespace cc1d
