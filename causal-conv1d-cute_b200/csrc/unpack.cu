// Fused Gated DeltaNet decode step (replaces ConvUpdateUnpack, causal_conv1d_cute/unpack.py).
//
// One launch does what the serving engine otherwise does with a conv update and three copies:
// thread j of a group of batch rows convolves channel group j of the leading `dim` columns of
// each row's [Q|K|V|Z] (read in place), updates the row's conv-state block, and copies group j
// of Z and element j of B and A into their own contiguous tensors. Rows whose slot is the pad slot or
// lies outside the cache keep their state and get their conv input copied to the output.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace cc1d {

namespace {

// R batch rows per thread and NB bytes of channels per thread (the shape of the lean decode in
// update.cu): every load of all R rows is issued before any store (a store waits for its data, so
// a copy placed first would hold back everything behind it): the slots, which head the one
// dependent chain (slot -> state), then Z, B and A, x and the filter, then the state blocks.
template <typename T, int W, int R, int NB, int NT, int MINB>
__global__ void __launch_bounds__(NT, MINB) unpack_kernel(const UnpackArgs a, bool bvec) {
    using RV = typename RawVec<NB>::type;
    constexpr int V = NB / (int)sizeof(T);
    constexpr int K = W - 1;
    const int64_t j = (int64_t)blockIdx.x * NT + threadIdx.x;
    const int64_t b0 = (int64_t)blockIdx.y * R;
    const int64_t G = a.D / V, GZ = a.zdim / V;
    const bool conv = j < G;
    const int64_t c0 = j * V;
    int32_t slot[R];
#pragma unroll
    for (int r = 0; r < R; ++r) slot[r] = conv && b0 + r < a.B ? __ldg(a.idx + b0 + r) : a.pad;
    RV zr[R];
    if (j < GZ) {
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (b0 + r < a.B) zr[r] = ldg_raw<NB>((const T*)a.qkvz + (b0 + r) * a.q_sb + a.D + j * V);
    }
    uint32_t bv[R], av[R];
    if (j < a.heads) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (b0 + r >= a.B) continue;
            const char* brow = (const char*)a.ba + (b0 + r) * a.ba_sb * a.gsize;
            if (a.gsize == 4) {
                bv[r] = __ldg(reinterpret_cast<const uint32_t*>(brow) + j);
                av[r] = __ldg(reinterpret_cast<const uint32_t*>(brow) + a.heads + j);
            } else {
                bv[r] = __ldg(reinterpret_cast<const uint16_t*>(brow) + j);
                av[r] = __ldg(reinterpret_cast<const uint16_t*>(brow) + a.heads + j);
            }
        }
    }
    RV xr[R], wt[W], bt;
    if (conv) {
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (b0 + r < a.B) xr[r] = ldg_raw<NB>((const T*)a.qkvz + (b0 + r) * a.q_sb + c0);
        load_filter_raw<T, W>((const T*)a.w, W, 1, (const T*)a.bias, 1, c0, true, bvec, wt, bt);
    }
    bool live[R];
    RV blk[R][K];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        live[r] = slot[r] != a.pad && slot[r] >= 0 && (int64_t)slot[r] < a.nslots;
        if (live[r]) {
            const T* sp = (const T*)a.state + (int64_t)slot[r] * a.D * K + c0 * K;
#pragma unroll
            for (int q = 0; q < K; ++q) blk[r][q] = ld_raw<NB>(sp + q * V);
        }
    }
    if (j < GZ) {
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (b0 + r < a.B) st_raw<NB>((T*)a.z + (b0 + r) * a.zdim + j * V, zr[r]);
    }
    if (j < a.heads) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (b0 + r >= a.B) continue;
            const int64_t o = (b0 + r) * a.heads + j;
            if (a.gsize == 4) {
                reinterpret_cast<uint32_t*>(a.b)[o] = bv[r];
                reinterpret_cast<uint32_t*>(a.a)[o] = av[r];
            } else {
                reinterpret_cast<uint16_t*>(a.b)[o] = (uint16_t)bv[r];
                reinterpret_cast<uint16_t*>(a.a)[o] = (uint16_t)av[r];
            }
        }
    }
    if (!conv) return;
    const bool use_silu = a.silu != 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (b0 + r >= a.B) continue;
        T* op = (T*)a.out + (b0 + r) * a.D + c0;
        if (!live[r]) {
            st_raw<NB>(op, xr[r]);
            continue;
        }
        RV win[K];
        block_to_time<T, K>(blk[r], win);
        float acc[V];
        unpack_raw<T, NB>(bt, acc);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            float f[V], wk[V];
            unpack_raw<T, NB>(win[k], f);
            unpack_raw<T, NB>(wt[k], wk);
#pragma unroll
            for (int e = 0; e < V; ++e) acc[e] = fmaf(f[e], wk[e], acc[e]);
        }
        {
            float f[V], wk[V];
            unpack_raw<T, NB>(xr[r], f);
            unpack_raw<T, NB>(wt[K], wk);
#pragma unroll
            for (int e = 0; e < V; ++e) acc[e] = activate<T>(fmaf(f[e], wk[e], acc[e]), use_silu);
        }
        // New state: drop the oldest entry, append x.
#pragma unroll
        for (int k = 0; k + 1 < K; ++k) win[k] = win[k + 1];
        win[K - 1] = xr[r];
        RV nb[K];
        time_to_block<T, K>(win, nb);
        T* sp = (T*)a.state + (int64_t)slot[r] * a.D * K + c0 * K;
#pragma unroll
        for (int q = 0; q < K; ++q) st_raw<NB>(sp + q * V, nb[q]);
        st_raw<NB>(op, pack_raw<T, NB>(acc));
    }
}

template <typename T, int W, int R, int NB, int NT, int MINB>
cudaError_t launch_unpack_shape(const UnpackArgs& a, bool bvec, cudaStream_t stream) {
    constexpr int V = NB / (int)sizeof(T);
    const int64_t lanes = std::max<int64_t>(std::max<int64_t>(a.D / V, a.zdim / V), a.heads);
    dim3 grid((unsigned)ceil_div(lanes, NT), (unsigned)ceil_div(a.B, (int64_t)R));
    unpack_kernel<T, W, R, NB, NT, MINB><<<grid, NT, 0, stream>>>(a, bvec);
    return cudaGetLastError();
}

// Launch table. 16-bit types: two rows per thread and 8-byte vectors (4 channels), 64-thread CTAs
// below 128 rows and 128-thread CTAs capped at 56 registers from 128 rows (W <= 4; wider filters
// get a looser cap). fp32: one row of 16-byte vectors. Measured on B200 at the reference's sglang
// shape (10240 conv channels, 16384-column rows, 48 heads, 310 slots, bf16, W = 4, CUDA graphs
// with a 256 MiB L2 flush before every call (cold) or back to back (warm)), us cold / warm, as
// (rows, bytes, threads): B = 64: (1, 16, 64) 4.49 / 3.67, (1, 8, 64) 4.79 / 3.67,
// (2, 8, 64) 4.51 / 2.95, (2, 8, 128) 4.51 / 3.03, (2, 16, 128) 4.83 / 3.59, (4, 8, 128) 6.67 /
// 3.99; B = 256: (1, 16, 64) 10.65 / 9.62, (1, 8, 64) 11.00 / 8.33, (2, 8, 64) 10.80 / 7.48,
// (2, 8, 128) 10.06 / 7.27, (2, 16, 128) 10.26 / 8.20, (4, 8, 128) 12.58 / 7.96. Four rows need
// 89 registers, which halves the resident CTAs; one row leaves too few loads in flight per thread.
template <typename T, int W>
cudaError_t run_unpack(const UnpackArgs& a, cudaStream_t stream) {
    const bool bvec = a.bias != nullptr && host_aligned16(a.bias);
    if constexpr (sizeof(T) == 2) {
        if (a.B >= 128) return launch_unpack_shape<T, W, 2, 8, 128, W <= 4 ? 9 : 6>(a, bvec, stream);
        return launch_unpack_shape<T, W, 2, 8, 64, W <= 4 ? 16 : 12>(a, bvec, stream);
    } else {
        return launch_unpack_shape<T, W, 1, 16, 64, 8>(a, bvec, stream);
    }
}

}  // namespace

cudaError_t launch_unpack(const UnpackArgs& a, int width, int dtype, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    CC1D_DISPATCH_DTYPE(dtype, CC1D_DISPATCH_WIDTH(width, err = (run_unpack<T, kW>(a, stream))));
    return err;
}

}  // namespace cc1d
