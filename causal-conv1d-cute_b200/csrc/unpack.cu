// Fused Gated DeltaNet decode step (replaces ConvUpdateUnpack, causal_conv1d_cute/unpack.py).
//
// One launch does what the serving engine otherwise does with a conv update and three copies:
// thread j of batch row b convolves channel group j of the leading `dim` columns of the
// [Q|K|V|Z] row (read in place), updates its conv-state block, and copies group j of Z and
// element j of B and A into their own contiguous tensors. Rows whose slot is the pad slot or
// lies outside the cache keep their state and get their conv input copied to the output.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace cc1d {

namespace {

constexpr int kUnpackThreads = 64;

template <typename T, int W>
__global__ void __launch_bounds__(kUnpackThreads) unpack_kernel(const UnpackArgs a, bool bvec) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
    const int64_t j = (int64_t)blockIdx.x * kUnpackThreads + threadIdx.x;
    const int64_t bi = blockIdx.y;
    const int64_t G = a.D / V, GZ = a.zdim / V;
    const T* qrow = (const T*)a.qkvz + bi * a.q_sb;
    // Every load that does not depend on the slot is issued before any store (a store waits for
    // its data, so a copy placed first would hold back everything behind it): the slot, which
    // heads the one dependent chain (slot -> state), then Z, B and A, x and the filter. Measured on
    // B200 at the reference's sglang shape (10240 conv channels, 16384-column rows, 48 heads, bf16,
    // L2 flushed before every call): B = 64 5.35 -> 4.56 us; B = 256 11.35 -> 10.82 us.
    const int32_t slot = j < G ? __ldg(a.idx + bi) : 0;
    uint4 zr;
    if (j < GZ) zr = ldg16(qrow + a.D + j * V);
    uint32_t bv = 0, av = 0;
    const char* brow = (const char*)a.ba + bi * a.ba_sb * a.gsize;
    if (j < a.heads) {
        if (a.gsize == 4) {
            bv = __ldg(reinterpret_cast<const uint32_t*>(brow) + j);
            av = __ldg(reinterpret_cast<const uint32_t*>(brow) + a.heads + j);
        } else {
            bv = __ldg(reinterpret_cast<const uint16_t*>(brow) + j);
            av = __ldg(reinterpret_cast<const uint16_t*>(brow) + a.heads + j);
        }
    }
    const bool conv = j < G;
    const int64_t c0 = j * V;
    uint4 xr, wt[W], bt;
    if (conv) {
        xr = ldg16(qrow + c0);
        load_filter_raw<T, W>((const T*)a.w, W, 1, (const T*)a.bias, 1, c0, true, bvec, wt, bt);
    }
    const bool live = conv && slot != a.pad && slot >= 0 && (int64_t)slot < a.nslots;
    T* sp = (T*)a.state + (int64_t)slot * a.D * K + c0 * K;
    uint4 blk[K];
    if (live) {
#pragma unroll
        for (int q = 0; q < K; ++q) blk[q] = ld16(sp + q * V);
    }
    if (j < GZ) st16((T*)a.z + bi * a.zdim + j * V, zr);
    if (j < a.heads) {
        const int64_t o = bi * a.heads + j;
        if (a.gsize == 4) {
            reinterpret_cast<uint32_t*>(a.b)[o] = bv;
            reinterpret_cast<uint32_t*>(a.a)[o] = av;
        } else {
            reinterpret_cast<uint16_t*>(a.b)[o] = (uint16_t)bv;
            reinterpret_cast<uint16_t*>(a.a)[o] = (uint16_t)av;
        }
    }
    if (!conv) return;
    T* op = (T*)a.out + bi * a.D + c0;
    if (!live) {
        st16(op, xr);
        return;
    }
    uint4 tm[K];
#pragma unroll
    for (int e = 0; e < V; ++e)
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int flat = e * K + k;
            set_lane<T>(tm[k], e, lane_of<T>(blk[flat / V], flat % V));
        }
    float acc[V];
    unpack16<T>(bt, acc);
#pragma unroll
    for (int k = 0; k < K; ++k) {
        float f[V], wk[V];
        unpack16<T>(tm[k], f);
        unpack16<T>(wt[k], wk);
#pragma unroll
        for (int e = 0; e < V; ++e) acc[e] = fmaf(f[e], wk[e], acc[e]);
    }
    {
        float f[V], wk[V];
        unpack16<T>(xr, f);
        unpack16<T>(wt[K], wk);
#pragma unroll
        for (int e = 0; e < V; ++e) acc[e] = activate<T>(fmaf(f[e], wk[e], acc[e]), a.silu != 0);
    }
    // New state: drop the oldest entry, append x.
#pragma unroll
    for (int k = 0; k + 1 < K; ++k) tm[k] = tm[k + 1];
    tm[K - 1] = xr;
#pragma unroll
    for (int q = 0; q < K; ++q)
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int flat = q * V + i;
            set_lane<T>(blk[q], i, lane_of<T>(tm[flat % K], flat / K));
        }
#pragma unroll
    for (int q = 0; q < K; ++q) st16(sp + q * V, blk[q]);
    st16(op, pack16<T>(acc));
}

template <typename T, int W>
cudaError_t run_unpack(const UnpackArgs& a, cudaStream_t stream) {
    constexpr int V = Vec<T>::V;
    const bool bvec = a.bias != nullptr && host_aligned16(a.bias);
    const int64_t lanes = std::max<int64_t>(std::max<int64_t>(a.D / V, a.zdim / V), a.heads);
    dim3 grid((unsigned)ceil_div(lanes, kUnpackThreads), (unsigned)a.B);
    unpack_kernel<T, W><<<grid, kUnpackThreads, 0, stream>>>(a, bvec);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_unpack(const UnpackArgs& a, int width, int dtype, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    CC1D_DISPATCH_DTYPE(dtype, CC1D_DISPATCH_WIDTH(width, err = (run_unpack<T, kW>(a, stream))));
    return err;
}

}  // namespace cc1d
