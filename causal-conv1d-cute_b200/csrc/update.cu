// Decode: one or several tokens per batch row against a conv-state cache updated in place
// (replaces the decode kernels of causal_conv1d_cute/update.py and ConvUpdateIndexed /
// ConvUpdateIndexedVec of varlen.py).
//
// update_kernel: one thread owns a 16-byte vector of V adjacent channels of one batch row. It
// issues every load it needs at once (the filter, the x rows, then the slot index and the
// state block of V*SS contiguous elements), so the only serial dependency is slot -> state.
// The state block is transposed in registers into SS "time-major" vectors (lane e = channel e),
// the same shape as an x row, so that stepping the window is a move of whole vectors and the
// new state, the per-step windows and the outputs are written back as whole 16-byte vectors.
// State and per-step windows are moved as raw bits: they are bit-exact copies of the inputs.
//
// update_generic_kernel: one channel per thread, any strides, any state length >= W-1.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace cc1d {

namespace {

constexpr int kUpdThreads = 128;
constexpr int kGenThreads = 256;

enum { kInterNone = 0, kInterDense = 1, kInterDedup = 2 };

// One batch row of one channel group, with its x rows (xr) and state block (sr) already loaded.
// NB: bytes of channels per thread (16, or 8 for the half-width form); R the matching vector.
template <typename T, int W, int SS, int LMAX, int IMODE, int NB>
__device__ __forceinline__ void update_row(const UpdArgs& a,
                                           const typename RawVec<NB>::type (&wt)[W],
                                           const typename RawVec<NB>::type& bt, bool use_silu,
                                           int64_t b, int64_t c0, int32_t slot,
                                           const typename RawVec<NB>::type (&xr)[LMAX],
                                           const typename RawVec<NB>::type (&sr)[SS], T* sp,
                                           typename RawVec<NB>::type* dedup_smem) {
    using R = typename RawVec<NB>::type;
    constexpr int V = NB / (int)sizeof(T);
    constexpr int K = W - 1;
    T* ib = nullptr;
    if (IMODE != kInterNone) {
        const int32_t islot = a.iidx != nullptr ? __ldg(a.iidx + b) : slot;
        if (islot < 0 || (int64_t)islot >= a.inter_nslots) {
            if (c0 == 0) flag_status(a.status, CC1D_DEV_BAD_INTER_SLOT);
        } else {
            ib = (T*)a.inter + (int64_t)islot * a.i_slot;
        }
    }
    R win[SS];
    block_to_time<T, SS>(sr, win);
    T* ob = (T*)a.out + b * a.o_sb + c0;
#pragma unroll
    for (int t = 0; t < LMAX; ++t) {
        if (t < a.L) {
            float acc[V];
            unpack_raw<T, NB>(bt, acc);
#pragma unroll
            for (int k = 0; k < K; ++k) {
                float f[V], wk[V];
                unpack_raw<T, NB>(win[SS - K + k], f);
                unpack_raw<T, NB>(wt[k], wk);
#pragma unroll
                for (int e = 0; e < V; ++e) acc[e] = fmaf(f[e], wk[e], acc[e]);
            }
            {
                float f[V], wk[V];
                unpack_raw<T, NB>(xr[t], f);
                unpack_raw<T, NB>(wt[K], wk);
#pragma unroll
                for (int e = 0; e < V; ++e) {
                    acc[e] = fmaf(f[e], wk[e], acc[e]);
                    acc[e] = activate<T>(acc[e], use_silu);
                }
            }
            st_raw<NB>(ob + t * a.o_st, pack_raw<T, NB>(acc));
#pragma unroll
            for (int s = 0; s + 1 < SS; ++s) win[s] = win[s + 1];
            win[SS - 1] = xr[t];
            if (IMODE == kInterDense && ib != nullptr) {
                R blk[K];
                time_to_block<T, K>(win + (SS - K), blk);
                T* dst = ib + t * a.i_st + c0 * K;
#pragma unroll
                for (int q = 0; q < K; ++q) st_raw<NB>(dst + q * V, blk[q]);
            }
        }
    }
    {
        R blk[SS];
        time_to_block<T, SS>(win, blk);
#pragma unroll
        for (int q = 0; q < SS; ++q) st_raw<NB>(sp + q * V, blk[q]);
    }
    if (IMODE == kInterDedup && ib != nullptr) {
        // Row of PW = L + K - 1 elements per channel: the newest K-1 old state entries, then the
        // L inputs. Staged per thread in shared memory because PW is a runtime value.
        constexpr int PWMAX = LMAX + K - 1;
        const int PW = a.L + K - 1;
        T* reg = reinterpret_cast<T*>(dedup_smem);
#pragma unroll
        for (int e = 0; e < V; ++e) {
#pragma unroll
            for (int p = 0; p + 1 < K; ++p) {
                const int flat = e * SS + (SS - K + 1 + p);
                reg[e * PW + p] = lane_of<T>(sr[flat / V], flat % V);
            }
#pragma unroll
            for (int t = 0; t < LMAX; ++t)
                if (t < a.L) reg[e * PW + K - 1 + t] = lane_of<T>(xr[t], e);
        }
        T* dst = ib + c0 * PW;
#pragma unroll
        for (int q = 0; q < PWMAX; ++q)
            if (q < PW) st_raw<NB>(dst + q * V, dedup_smem[q]);
    }
}

// General decode: one channel group of one batch row per thread (gridDim.y == B), 1..LMAX steps,
// any state length SS >= W-1, optional per-step states. Every load of the row (x rows, slot, state
// block) is issued before any compute.
template <typename T, int W, int SS, int LMAX, int IMODE, int NB>
__global__ void __launch_bounds__(kUpdThreads)
    update_kernel(const UpdArgs a, bool wvec, bool bvec) {
    using R = typename RawVec<NB>::type;
    constexpr int V = NB / (int)sizeof(T);
    constexpr int K = W - 1;
    static_assert(SS >= K, "state shorter than the filter history");
    extern __shared__ uint4 dedup_smem[];
    const int64_t nvec = a.D / V;
    const int64_t j = (int64_t)blockIdx.x * kUpdThreads + threadIdx.x;
    if (j >= nvec) return;
    const int64_t c0 = j * V;
    const int64_t b = blockIdx.y;
    // The slot load heads the dependent chain (slot -> state block): issue it first.
    const int32_t slot = a.idx != nullptr ? __ldg(a.idx + b) : (int32_t)b;
    R wt[W], bt;
    load_filter_raw<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c0, wvec,
                          bvec, wt, bt);
    R xr[LMAX];
    const T* xb = (const T*)a.x + b * a.x_sb + c0;
#pragma unroll
    for (int t = 0; t < LMAX; ++t)
        if (t < a.L) xr[t] = ldg_raw<NB>(xb + t * a.x_st);
    if (slot == a.pad) return;
    if (slot < 0 || (int64_t)slot >= a.nslots) {
        if (j == 0) flag_status(a.status, CC1D_DEV_BAD_SLOT);
        return;
    }
    T* sp = (T*)a.state + (int64_t)slot * a.s_slot + c0 * SS;
    R sr[SS];
#pragma unroll
    for (int q = 0; q < SS; ++q) sr[q] = ld_raw<NB>(sp + q * V);
    update_row<T, W, SS, LMAX, IMODE, NB>(a, wt, bt, a.silu != 0, b, c0, slot, xr, sr, sp,
                                          reinterpret_cast<R*>(dedup_smem) +
                                              threadIdx.x * (LMAX + K - 1));
}

// Single-step decode without per-step states, the serving hot case, kept lean: R batch rows per
// thread (gridDim.y == ceil(B / R)), NB bytes of channels per thread, raw tap-major weights
// widened at use, no runtime step loop (the general kernel's 90 registers halve the resident
// threads). Every load is issued before any compute: the slot loads first, since each heads the
// only dependent chain (slot -> state), then the filter and the x rows, then the state blocks of
// every row; a row with the pad slot or a slot outside the cache skips its state load and all its
// stores. CHECK (a status word was given) adds the report of slots outside the cache, which costs
// 0.35 us per call, so the unchecked variant leaves it out.
//
// Launch table (16-bit types): 4 channels per thread (8-byte vectors) and 2 rows per thread below
// 128 rows, 4 rows per thread from 128 rows. Measured on B200 at D = 8192, bf16, W = 4, CUDA
// graphs with a 256 MiB L2 flush before every call (cold) or back to back (warm), us, as
// (R rows, NB bytes): direct B = 64: (1, 16) 3.84 / 3.19, (1, 8) 3.83 / 3.05, (2, 16) 4.06 / 3.24,
// (2, 8) 3.60 / 2.72, (4, 8) 4.03 / 2.78; indexed B = 64 (1024-slot cache): (1, 16) 4.07 / 3.18,
// (2, 8) 3.77 / 2.71; direct B = 256: (1, 16) 7.99 / 6.80, (2, 16) 7.30 / 6.99, (2, 8) 7.38 / 5.95,
// (4, 8) 7.21 / 5.02; indexed B = 256: (2, 16) 7.71 / 7.26, (2, 8) 8.06 / 5.93, (4, 8) 8.15 / 5.41.
// More rows per thread keep more independent loads in flight per thread; half-width vectors double
// the threads. fp32 keeps one row of 16-byte vectors. The floor under all of them: an empty
// kernel on the same grid costs 1.3-1.8 us, and a kernel that only loads the slot, then one
// 16-byte state vector per thread, costs 5.7-6.3 us cold at B = 256 (two dependent DRAM round
// trips). Forms tried and not kept: 16 channels per thread with 32-byte accesses (32- to
// 256-thread CTAs), 8 rows per thread, the warp's state block moved through shared memory with
// 512-byte coalesced accesses.
template <typename T, int W, int SS, bool CHECK, int R, int NB>
__global__ void __launch_bounds__(kUpdThreads, R == 1 ? 1 : 7) decode1_kernel(const UpdArgs a) {
    using RV = typename RawVec<NB>::type;
    constexpr int V = NB / (int)sizeof(T);
    constexpr int K = W - 1;
    const int64_t nvec = a.D / V;
    const int64_t j = (int64_t)blockIdx.x * kUpdThreads + threadIdx.x;
    if (j >= nvec) return;
    const int64_t c0 = j * V;
    int32_t slot[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t b = (int64_t)blockIdx.y * R + r;
        slot[r] = b < a.B ? (a.idx != nullptr ? __ldg(a.idx + b) : (int32_t)b) : a.pad;
    }
    RV wt[W], bt;
    load_filter_raw<T, W>((const T*)a.w, W, 1, (const T*)a.bias, 1, c0, true, a.bias != nullptr,
                          wt, bt);
    RV xr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const int64_t b = (int64_t)blockIdx.y * R + r;
        if (b < a.B) xr[r] = ldg_raw<NB>((const T*)a.x + b * a.x_sb + c0);
    }
    bool live[R];
    RV sr[R][SS];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        live[r] = slot[r] != a.pad && slot[r] >= 0 && (int64_t)slot[r] < a.nslots;
        if (live[r]) {
            const T* sp = (const T*)a.state + (int64_t)slot[r] * a.s_slot + c0 * SS;
#pragma unroll
            for (int q = 0; q < SS; ++q) sr[r][q] = ld_raw<NB>(sp + q * V);
        }
        if (CHECK && !live[r] && slot[r] != a.pad && j == 0) flag_status(a.status, CC1D_DEV_BAD_SLOT);
    }
    const bool use_silu = a.silu != 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (!live[r]) continue;
        const int64_t b = (int64_t)blockIdx.y * R + r;
        RV win[SS];
        block_to_time<T, SS>(sr[r], win);
        float acc[V];
        unpack_raw<T, NB>(bt, acc);
#pragma unroll
        for (int k = 0; k < K; ++k) {
            float f[V], wk[V];
            unpack_raw<T, NB>(win[SS - K + k], f);
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
        st_raw<NB>((T*)a.out + b * a.o_sb + c0, pack_raw<T, NB>(acc));
#pragma unroll
        for (int s = 0; s + 1 < SS; ++s) win[s] = win[s + 1];
        win[SS - 1] = xr[r];
        RV blk[SS];
        time_to_block<T, SS>(win, blk);
        T* sp = (T*)a.state + (int64_t)slot[r] * a.s_slot + c0 * SS;
#pragma unroll
        for (int q = 0; q < SS; ++q) st_raw<NB>(sp + q * V, blk[q]);
    }
}

// Any strides, any state length S >= W-1 (the whole row shifts by L), any per-step layout.
template <typename T, int W>
__global__ void __launch_bounds__(kGenThreads) update_generic_kernel(const UpdArgs a) {
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
        float w[W], bb;
        load_filter1<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c, w, bb);
        const T* xr = (const T*)a.x + b * a.x_sb + c * a.x_sd;
        T* st = (T*)a.state + (int64_t)slot * a.s_slot + c * a.s_sd;
        const int64_t S = a.S;
        const int L = a.L;
        // hist = [state row (S) | x (L)]; element m of it:
        auto hist = [&](int64_t m) -> T { return m < S ? st[m * a.s_sk] : xr[(m - S) * a.x_st]; };
        T* orow = (T*)a.out + b * a.o_sb + c * a.o_sd;
        for (int t = 0; t < L; ++t) {
            float acc = bb;
#pragma unroll
            for (int k = 0; k < W; ++k) acc = fmaf(to_f32<T>(hist(S + t - K + k)), w[k], acc);
            orow[t * a.o_st] = from_f32<T>(activate<T>(acc, use_silu));
        }
        if (a.inter != nullptr) {
            const int32_t islot = a.iidx != nullptr ? a.iidx[b] : slot;
            if (islot < 0 || (int64_t)islot >= a.inter_nslots) {
                if (c == 0) flag_status(a.status, CC1D_DEV_BAD_INTER_SLOT);
            } else {
                T* ib = (T*)a.inter + (int64_t)islot * a.i_slot + c * a.i_sd;
                for (int t = 0; t < L; ++t)
                    for (int k = 0; k < K; ++k) ib[t * a.i_st + k * a.i_sk] = hist(S + t + 1 - K + k);
            }
        }
        // Shift the row left by L in place; ascending order reads every old entry before it is
        // overwritten.
        for (int64_t s = 0; s < S; ++s) st[s * a.s_sk] = hist(s + L);
    }
}

// Half-width form (8-byte vectors, 4 channels of a 16-bit type per thread) when the batch gives
// fewer than kHalfWidthThreads threads at 16 bytes each: the kernel is latency-bound, and twice
// the threads (48 instead of 80 registers each) keep twice the loads in flight. Measured on B200
// at B = 64, D = 8192, 4 steps, dense per-step states (CUDA graph, cold L2): 9.36 -> 7.27 us.
constexpr int64_t kHalfWidthThreads = 148LL * 1024;

template <typename T, int W, int SS, int LMAX, int IMODE>
cudaError_t launch_vec(const UpdArgs& a, bool wvec, bool bvec, cudaStream_t stream) {
    size_t smem = IMODE == kInterDedup ? (size_t)kUpdThreads * (LMAX + W - 2) * 16 : 0;
    if constexpr (sizeof(T) == 2) {
        if (a.B * (a.D / Vec<T>::V) < kHalfWidthThreads) {
            const int64_t nvec = a.D / 4;
            dim3 grid((unsigned)ceil_div(nvec, kUpdThreads), (unsigned)a.B);
            update_kernel<T, W, SS, LMAX, IMODE, 8>
                <<<grid, kUpdThreads, smem, stream>>>(a, wvec, bvec);
            return cudaGetLastError();
        }
    }
    const int64_t nvec = a.D / Vec<T>::V;
    dim3 grid((unsigned)ceil_div(nvec, kUpdThreads), (unsigned)a.B);
    update_kernel<T, W, SS, LMAX, IMODE, 16><<<grid, kUpdThreads, smem, stream>>>(a, wvec, bvec);
    return cudaGetLastError();
}

template <typename T, int W, int SS, int LMAX>
cudaError_t launch_vec_inter(const UpdArgs& a, int imode, bool wvec, bool bvec,
                             cudaStream_t stream) {
    if (imode == kInterDense) return launch_vec<T, W, SS, LMAX, kInterDense>(a, wvec, bvec, stream);
    if (imode == kInterDedup) return launch_vec<T, W, SS, LMAX, kInterDedup>(a, wvec, bvec, stream);
    return launch_vec<T, W, SS, LMAX, kInterNone>(a, wvec, bvec, stream);
}

// The lean single-step decode, R rows per thread, with or without the status report.
template <typename T, int W, int K, int P, int R, int NB>
cudaError_t launch_decode1(const UpdArgs& a, cudaStream_t stream) {
    const int64_t nvec = a.D / (NB / (int64_t)sizeof(T));
    dim3 grid((unsigned)ceil_div(nvec, kUpdThreads), (unsigned)ceil_div(a.B, (int64_t)R));
    if (a.status != nullptr) {
        if (a.S == K) decode1_kernel<T, W, K, true, R, NB><<<grid, kUpdThreads, 0, stream>>>(a);
        else decode1_kernel<T, W, P, true, R, NB><<<grid, kUpdThreads, 0, stream>>>(a);
    } else {
        if (a.S == K) decode1_kernel<T, W, K, false, R, NB><<<grid, kUpdThreads, 0, stream>>>(a);
        else decode1_kernel<T, W, P, false, R, NB><<<grid, kUpdThreads, 0, stream>>>(a);
    }
    return cudaGetLastError();
}

template <typename T, int W>
cudaError_t run_update(const UpdArgs& a, cudaStream_t stream) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
    constexpr int P = W <= 2 ? 2 : W <= 4 ? 4 : 8;  // power of two >= W (padded layout)
    const int64_t e = sizeof(T);
    const bool wvec = a.w_sd == W && a.w_sk == 1 && host_aligned16(a.w);
    const bool bvec = a.bias != nullptr && a.bias_s == 1 && host_aligned16(a.bias);
    const bool xok = a.x_sd == 1 && a.o_sd == 1 && a.D % V == 0 && host_aligned16(a.x) &&
                     host_aligned16(a.out) && (a.x_sb * e) % 16 == 0 && (a.o_sb * e) % 16 == 0 &&
                     (a.L == 1 || ((a.x_st * e) % 16 == 0 && (a.o_st * e) % 16 == 0));
    const bool sok = a.s_sk == 1 && a.s_sd == a.S && host_aligned16(a.state) &&
                     (a.s_slot * e) % 16 == 0;
    int imode = kInterNone;
    bool iok = true;
    if (a.inter != nullptr) {
        const int64_t PW = a.L + K - 1;
        iok = host_aligned16(a.inter) && (a.i_slot * e) % 16 == 0 && a.S == K;
        if (a.i_sk == 1 && a.i_sd == K && a.i_st == a.D * K) {
            imode = kInterDense;
        } else if (a.i_sk == 1 && a.i_sd == PW && a.i_st == 1) {
            imode = kInterDedup;
        } else {
            iok = false;
        }
    }
    const bool lean = wvec && (a.bias == nullptr || bvec) && a.L == 1 && imode == kInterNone;
    if (xok && sok && iok && lean && (a.S == K || a.S == P) && a.B <= 65535) {
        if constexpr (sizeof(T) == 2 && W <= 4) {
            if (a.B >= 128) return launch_decode1<T, W, K, P, 4, 8>(a, stream);
            return launch_decode1<T, W, K, P, 2, 8>(a, stream);
        }
        return launch_decode1<T, W, K, P, 1, 16>(a, stream);
    }
    if (xok && sok && iok && a.L >= 1 && a.L <= 16 && a.B <= 65535) {
        if (a.S == K) {
            if (a.L == 1) {
                // A single step: dense and dedup per-step layouts coincide.
                return launch_vec_inter<T, W, K, 1>(a, imode == kInterNone ? kInterNone : kInterDense,
                                                    wvec, bvec, stream);
            }
            if (a.L <= 4) return launch_vec_inter<T, W, K, 4>(a, imode, wvec, bvec, stream);
            if (a.L <= 8) return launch_vec_inter<T, W, K, 8>(a, imode, wvec, bvec, stream);
            return launch_vec_inter<T, W, K, 16>(a, imode, wvec, bvec, stream);
        }
        if (a.S == P && P != K && a.L == 1 && imode == kInterNone)
            return launch_vec<T, W, P, 1, kInterNone>(a, wvec, bvec, stream);
    }
    const int64_t n = a.B * a.D;
    const int64_t blocks = std::min<int64_t>(ceil_div(n, kGenThreads), 148 * 32);
    update_generic_kernel<T, W><<<(unsigned)std::max<int64_t>(blocks, 1), kGenThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_update(const UpdArgs& a, int width, int dtype, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    CC1D_DISPATCH_DTYPE(dtype, CC1D_DISPATCH_WIDTH(width, err = (run_update<T, kW>(a, stream))));
    return err;
}

}  // namespace cc1d
