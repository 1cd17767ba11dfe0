// Single-token decode on a ring conv state (replaces ConvUpdateRing, causal_conv1d_cute/ring.py).
//
// The ring state (slots, W-1, D) keeps the last W-1 inputs of a sequence unordered: row
// seen % (W-1) holds the oldest. A step reads the W-1 rows and x, writes the output and
// overwrites only the oldest row with x, so it stores one state row instead of W-1. Each thread
// owns a vector of channels (8 bytes for 16-bit types, 16 for fp32) of R batch rows. The rows are already time-major vectors;
// tap k (oldest first) takes row (pos + k) % (W-1), picked from registers by a select chain so
// that the weight loads never wait on the sequence length. The taps are summed oldest first, the
// order of the ordered-state decode, so both layouts give identical outputs.
//
// to_ring / from_ring (ring.py:33-67) run here too: a thread moves one 16-byte channel vector of
// one slot between the channel-major state block (W-1 vectors, transposed in registers) and the
// W-1 ring rows, rotated by the slot's sequence length.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace cc1d {

namespace {

constexpr int kRingThreads = 128;
constexpr int kGenThreads = 256;

__device__ __forceinline__ int ring_pos(int32_t seen, int K) {
    int p = seen % K;
    return p < 0 ? p + K : p;
}

// R batch rows per thread (gridDim.y == ceil(B / R)) and NB bytes of channels per thread; raw
// weights widened at use. Every load of every row is issued before any compute: the slot and
// count loads first (each heads the only dependent chain, slot -> ring rows), then the filter and
// the x rows, then the ring rows.
// MODE 0: weight / bias layout and SiLU read from the arguments. MODE 1-4: contiguous 16-byte
// aligned weights, and SiLU (2, 4) and a contiguous aligned bias (3, 4) fixed at compile time.
template <typename T, int W, int NB, int R, int MODE>
__global__ void __launch_bounds__(kRingThreads) ring_kernel(const RingArgs a, bool wvec, bool bvec) {
    using RV = typename RawVec<NB>::type;
    constexpr int V = NB / (int)sizeof(T);
    constexpr int K = W - 1;
    const int64_t nvec = a.D / V;
    const int64_t j = (int64_t)blockIdx.x * kRingThreads + threadIdx.x;
    if (j >= nvec) return;
    const int64_t c0 = j * V;
    int32_t slot[R], seen[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t b = (int64_t)blockIdx.y * R + r;
        slot[r] = b < a.B ? (a.idx != nullptr ? __ldg(a.idx + b) : (int32_t)b) : a.pad;
        seen[r] = b < a.B ? __ldg(a.seen + b) : 0;
    }
    constexpr bool kFixed = MODE > 0, kSilu = MODE == 2 || MODE == 4, kBias = MODE >= 3;
    const bool use_silu = kFixed ? kSilu : a.silu != 0;
    RV wt[W], bt;
    load_filter_raw<T, W>((const T*)a.w, a.w_sd, a.w_sk,
                          kFixed && !kBias ? nullptr : (const T*)a.bias, a.bias_s, c0,
                          kFixed ? true : wvec, kFixed ? kBias : bvec, wt, bt);
    RV xr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t b = (int64_t)blockIdx.y * R + r;
        if (b < a.B) xr[r] = ldg_raw<NB>((const T*)a.x + b * a.x_sb + c0);
    }
    bool live[R];
    RV rows[R][K];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        live[r] = slot[r] != a.pad && slot[r] >= 0 && (int64_t)slot[r] < a.nslots;
        if (!live[r] && slot[r] != a.pad && j == 0) flag_status(a.status, CC1D_DEV_BAD_SLOT);
        if (live[r]) {
            const T* rb = (const T*)a.ring + (int64_t)slot[r] * a.r_slot + c0;
#pragma unroll
            for (int q = 0; q < K; ++q) rows[r][q] = ld_raw<NB>(rb + q * a.r_sk);
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (!live[r]) continue;
        const int64_t b = (int64_t)blockIdx.y * R + r;
        const int pos = ring_pos(seen[r], K);
        float acc[V];
        unpack_raw<T, NB>(bt, acc);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            int p = pos + k;
            p = p >= K ? p - K : p;
            RV v = rows[r][0];
#pragma unroll
            for (int q = 1; q < K; ++q) v = (p == q) ? rows[r][q] : v;
            float f[V], wk[V];
            unpack_raw<T, NB>(v, f);
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
        T* rb = (T*)a.ring + (int64_t)slot[r] * a.r_slot + c0;
        st_raw<NB>(rb + pos * a.r_sk, xr[r]);
        st_raw<NB>((T*)a.out + b * a.o_sb + c0, pack_raw<T, NB>(acc));
    }
}

template <typename T, int W>
__global__ void __launch_bounds__(kGenThreads) ring_generic_kernel(const RingArgs a) {
    constexpr int K = W - 1;
    const int64_t n = a.B * a.D;
    const bool use_silu = a.silu != 0;
    for (int64_t id = (int64_t)blockIdx.x * kGenThreads + threadIdx.x; id < n;
         id += (int64_t)gridDim.x * kGenThreads) {
        const int64_t c = id % a.D;
        const int64_t b = id / a.D;
        const int32_t slot = a.idx != nullptr ? a.idx[b] : (int32_t)b;
        if (slot == a.pad) continue;
        if (slot < 0 || (int64_t)slot >= a.nslots) {
            if (c == 0) flag_status(a.status, CC1D_DEV_BAD_SLOT);
            continue;
        }
        const int pos = ring_pos(a.seen[b], K);
        float w[W], bb;
        load_filter1<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c, w, bb);
        T* rb = (T*)a.ring + (int64_t)slot * a.r_slot + c * a.r_sd;
        const T xv = ((const T*)a.x)[b * a.x_sb + c * a.x_sd];
        float acc = bb;
        for (int k = 0; k < K; ++k) {
            int r = pos + k;
            r = r >= K ? r - K : r;
            acc = fmaf(to_f32<T>(rb[r * a.r_sk]), w[k], acc);
        }
        acc = fmaf(to_f32<T>(xv), w[K], acc);
        rb[pos * a.r_sk] = xv;
        ((T*)a.out)[b * a.o_sb + c * a.o_sd] = from_f32<T>(activate<T>(acc, use_silu));
    }
}

template <typename T, int W, int NB, int R>
cudaError_t launch_ring_mode(int mode, dim3 grid, const RingArgs& a, bool wvec, bool bvec,
                             cudaStream_t stream) {
    switch (mode) {
        case 1: ring_kernel<T, W, NB, R, 1><<<grid, kRingThreads, 0, stream>>>(a, wvec, bvec); break;
        case 2: ring_kernel<T, W, NB, R, 2><<<grid, kRingThreads, 0, stream>>>(a, wvec, bvec); break;
        case 3: ring_kernel<T, W, NB, R, 3><<<grid, kRingThreads, 0, stream>>>(a, wvec, bvec); break;
        case 4: ring_kernel<T, W, NB, R, 4><<<grid, kRingThreads, 0, stream>>>(a, wvec, bvec); break;
        default: ring_kernel<T, W, NB, R, 0><<<grid, kRingThreads, 0, stream>>>(a, wvec, bvec); break;
    }
    return cudaGetLastError();
}

template <typename T, int W>
cudaError_t run_ring(const RingArgs& a, cudaStream_t stream) {
    constexpr int V = Vec<T>::V;
    const int64_t e = sizeof(T);
    const bool wvec = a.w_sd == W && a.w_sk == 1 && host_aligned16(a.w);
    const bool bvec = a.bias != nullptr && a.bias_s == 1 && host_aligned16(a.bias);
    const bool vec = a.x_sd == 1 && a.o_sd == 1 && a.r_sd == 1 && a.D % V == 0 &&
                     host_aligned16(a.x) && host_aligned16(a.out) && host_aligned16(a.ring) &&
                     (a.x_sb * e) % 16 == 0 && (a.o_sb * e) % 16 == 0 &&
                     (a.r_slot * e) % 16 == 0 && (a.r_sk * e) % 16 == 0;
    if (vec && a.B <= 65535) {
        // 16-bit types: 4 channels per thread (8-byte vectors), 2 rows per thread below 128 rows
        // and 4 from 128 rows, as the lean decode. Measured on B200 (D = 8192, bf16, W = 4, CUDA
        // graphs, 256 MiB L2 flush before every call; cold / warm us, as (NB bytes, R rows), one
        // run): B = 64: (16, 1) 4.52 / 3.07, (8, 1) 4.10 / 3.01, (8, 2) 3.97 / 2.84,
        // (8, 4) 4.12 / 2.92; B = 256: (16, 1) 8.64 / 6.32, (8, 2) 7.72 / 5.79, (8, 4) 7.18 / 5.00,
        // (16, 4) 8.34 / 5.22. fp32 keeps one row of 16-byte vectors. With contiguous weights and
        // a contiguous or absent bias, the layout switches and SiLU are compile-time (MODE 1-4):
        // measured inside a torch process (CUDA graphs, the same flush), B = 64 (8, 2) 4.19 / 3.23
        // -> 3.80 / 3.01 us, B = 256 (8, 4) 7.15-7.33 / 5.56 -> 6.85-6.89 / 5.25.
        if constexpr (sizeof(T) == 2) {
            const int64_t nvec8 = a.D / (8 / (int64_t)sizeof(T));
            const int R = a.B >= 128 ? 4 : 2;
            dim3 grid((unsigned)ceil_div(nvec8, kRingThreads), (unsigned)ceil_div(a.B, (int64_t)R));
            const int mode = !(wvec && (a.bias == nullptr || bvec)) ? 0
                             : 1 + (a.silu != 0 ? 1 : 0) + (a.bias != nullptr ? 2 : 0);
            if (R == 4) return launch_ring_mode<T, W, 8, 4>(mode, grid, a, wvec, bvec, stream);
            return launch_ring_mode<T, W, 8, 2>(mode, grid, a, wvec, bvec, stream);
        }
        const int64_t nvec = a.D / V;
        dim3 grid((unsigned)ceil_div(nvec, kRingThreads), (unsigned)a.B);
        ring_kernel<T, W, 16, 1, 0><<<grid, kRingThreads, 0, stream>>>(a, wvec, bvec);
        return cudaGetLastError();
    }
    const int64_t n = a.B * a.D;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, kGenThreads), 148 * 32));
    ring_generic_kernel<T, W><<<(unsigned)blocks, kGenThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

// Ordered state <-> ring state, one 16-byte channel vector of one slot (blockIdx.y) per thread.
template <typename T, int W, bool TO_RING>
__global__ void __launch_bounds__(kRingThreads) ring_convert_kernel(const RingConvArgs a) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
    const int64_t j = (int64_t)blockIdx.x * kRingThreads + threadIdx.x;
    if (j >= a.D / V) return;
    const int64_t c0 = j * V;
    const int64_t s = blockIdx.y;
    const int pos = ring_pos(__ldg(a.seen + s), K);
    T* sp = (T*)a.state + s * a.s_slot + c0 * K;
    T* rp = (T*)a.ring + s * a.r_slot + c0;
    uint4 blk[K], tm[K];
    if (TO_RING) {
#pragma unroll
        for (int q = 0; q < K; ++q) blk[q] = ld16(sp + q * V);
        block_to_time<T, K>(blk, tm);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int r = pos + k >= K ? pos + k - K : pos + k;
            st16(rp + r * a.r_sk, tm[k]);
        }
    } else {
        // All K ring rows are read whatever the position, so the loads do not wait for `seen`;
        // the rotation to oldest-first order is done in registers.
        uint4 rows[K];
#pragma unroll
        for (int r = 0; r < K; ++r) rows[r] = ld16(rp + r * a.r_sk);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int r = pos + k >= K ? pos + k - K : pos + k;
            tm[k] = rows[0];
#pragma unroll
            for (int q = 1; q < K; ++q) tm[k] = r == q ? rows[q] : tm[k];
        }
        time_to_block<T, K>(tm, blk);
#pragma unroll
        for (int q = 0; q < K; ++q) st16(sp + q * V, blk[q]);
    }
}

// Any strides: one element per thread.
template <typename T, int W>
__global__ void __launch_bounds__(kGenThreads) ring_convert_generic_kernel(const RingConvArgs a) {
    constexpr int K = W - 1;
    const int64_t n = a.S * a.D * K;
    for (int64_t id = (int64_t)blockIdx.x * kGenThreads + threadIdx.x; id < n;
         id += (int64_t)gridDim.x * kGenThreads) {
        const int k = (int)(id % K);
        const int64_t c = (id / K) % a.D;
        const int64_t s = id / (K * a.D);
        const int p = ring_pos(a.seen[s], K) + k;
        const int r = p >= K ? p - K : p;
        T* se = (T*)a.state + s * a.s_slot + c * a.s_sd + k * a.s_sk;
        T* re = (T*)a.ring + s * a.r_slot + r * a.r_sk + c * a.r_sd;
        if (a.to_ring)
            *re = *se;
        else
            *se = *re;
    }
}

template <typename T, int W>
cudaError_t run_ring_convert(const RingConvArgs& a, cudaStream_t stream) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
    const int64_t e = sizeof(T);
    const bool vec = a.D % V == 0 && a.s_sk == 1 && a.s_sd == K && a.r_sd == 1 &&
                     host_aligned16(a.state) && host_aligned16(a.ring) &&
                     (a.s_slot * e) % 16 == 0 && (a.r_slot * e) % 16 == 0 &&
                     (a.r_sk * e) % 16 == 0 && a.S <= 65535;
    if (vec) {
        dim3 grid((unsigned)ceil_div(a.D / V, (int64_t)kRingThreads), (unsigned)a.S);
        if (a.to_ring)
            ring_convert_kernel<T, W, true><<<grid, kRingThreads, 0, stream>>>(a);
        else
            ring_convert_kernel<T, W, false><<<grid, kRingThreads, 0, stream>>>(a);
        return cudaGetLastError();
    }
    const int64_t n = a.S * a.D * K;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, kGenThreads), 148 * 32));
    ring_convert_generic_kernel<T, W><<<(unsigned)blocks, kGenThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_ring(const RingArgs& a, int width, int dtype, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    CC1D_DISPATCH_DTYPE(dtype, CC1D_DISPATCH_WIDTH(width, err = (run_ring<T, kW>(a, stream))));
    return err;
}

cudaError_t launch_ring_convert(const RingConvArgs& a, int width, int dtype, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    CC1D_DISPATCH_DTYPE(dtype,
                        CC1D_DISPATCH_WIDTH(width, err = (run_ring_convert<T, kW>(a, stream))));
    return err;
}

}  // namespace cc1d
