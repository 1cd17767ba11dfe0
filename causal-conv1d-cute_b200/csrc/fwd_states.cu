// Prefill with initial states, final states and per-token sequence ids: the arguments of the
// Dao-AILab causal_conv1d_fn interface (seq_idx, initial_states, return_final_states /
// final_states_out) that the reference's dao_compat shim passes upstream (dao_compat.py:28-78).
//
// out[b, c, t] = act(bias[c] + sum_k w[c, k] * v(b, c, t - (W-1) + k)) where v(b, c, p) is
//   x[b, c, p]                       for 0 <= p (and seq[b, p] == seq[b, t] with sequence ids),
//   init[b, c, (W-1) + p]            for p < 0 with initial states,
//   0                                otherwise;
// a tap whose sequence id differs from the token's adds nothing (the term is skipped, not
// multiplied by zero). final[b, c, k] = the k-th of the last W-1 entries of [init[b, c, :] | x[b, c, :]]
// (zeros in place of init without initial states), copied bit for bit from the inputs.
//
// Kernels:
//   fwd_states_staged_kernel  channel-last x / out, 16-bit types, contiguous weights: the
//                           staged strips of the plain prefill (one per CTA, landed in
//                           shared memory), initial states in the halo of a row's first strip.
//   fwd_states_vec_kernel   channel-last x / out otherwise (16-byte channel vectors, the walk and
//                           grid of the plain channel-last register walk): a thread walks a share
//                           of token rows of one 16-byte channel group; a stretch that starts a
//                           row takes its history from the initial states, the one that ends it
//                           writes the final states.
//   fwd_states_generic_kernel  any strides, one channel of a strip per thread.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "walk.cuh"

namespace cc1d {

namespace {

constexpr int kStThreads = 64;
constexpr int kStGenThreads = 256;
constexpr int64_t kStStrip = 128;
constexpr int kStRows = 8;  // rows in flight per thread (U of the walk)

// The W-1 entries of history before token t0 of row b, channels c0..c0+V-1, as fp32 (oldest
// first): x rows for t >= 0, initial states (or zeros) for t < 0; with sequence ids, the id of
// each history row (rows before the start carry no id: their values are 0 or initial states, and
// sequence ids exclude initial states).
template <typename T, int W>
__device__ __forceinline__ void states_halo(const FwdStateArgs& a, int64_t b, int64_t c0,
                                            int64_t t0, float (&h)[W - 1][Vec<T>::V],
                                            int32_t (&qh)[W - 1]) {
    constexpr int V = Vec<T>::V;
    const T* xb = (const T*)a.f.x + b * a.f.x_sb + c0;
    const T* init = (const T*)a.init;
#pragma unroll
    for (int k = 0; k < W - 1; ++k) {
        const int64_t t = t0 - (W - 1) + k;
        if (t >= 0) {
            unpack16<T>(ldg16(xb + t * a.f.x_sl), h[k]);
            qh[k] = a.seq != nullptr ? __ldg(a.seq + b * a.q_sb + t * a.q_sl) : 0;
        } else {
#pragma unroll
            for (int e = 0; e < V; ++e)
                h[k][e] = init != nullptr
                              ? to_f32<T>(init[b * a.i_sb + (c0 + e) * a.i_sd + ((W - 1) + t) * a.i_sk])
                              : 0.f;
            qh[k] = INT32_MIN;  // no id: the value is 0 or an initial state, never masked in
        }
    }
}

// Final states of row b, channels c0..c0+V-1: raw copies of x rows L-(W-1)..L-1, or of the
// initial states (zeros without them) for positions before the row start.
template <typename T, int W>
__device__ __forceinline__ void states_final(const FwdStateArgs& a, int64_t b, int64_t c0, int nch) {
    const T* xb = (const T*)a.f.x + b * a.f.x_sb;
    const T* init = (const T*)a.init;
    T* fin = (T*)a.fin;
    for (int k = 0; k < W - 1; ++k) {
        const int64_t t = a.f.L - (W - 1) + k;
        for (int e = 0; e < nch; ++e) {
            const int64_t c = c0 + e;
            T v;
            if (t >= 0) {
                v = xb[c * a.f.x_sd + t * a.f.x_sl];
            } else if (init != nullptr) {
                v = init[b * a.i_sb + c * a.i_sd + ((W - 1) + t) * a.i_sk];
            } else {
                v = from_f32<T>(0.f);
            }
            fin[b * a.f_sb + c * a.f_sd + k * a.f_sk] = v;
        }
    }
}

// Channel-last: blockIdx.x is a 64-thread channel block, blockIdx.y one of gridDim.y equal shares
// of the flattened (batch, token) rows (as fwd_channel_last_share_kernel). A thread walks its
// 16-byte channel group through the share: the history of each batch stretch comes from x, or
// from the initial states before token 0; the stretch that ends a row writes its final states.
template <typename T, int W, bool SEQ>
__global__ void __launch_bounds__(kStThreads)
    fwd_states_vec_kernel(const FwdStateArgs a, bool wvec, bool bvec) {
    constexpr int V = Vec<T>::V;
    const FwdArgs& f = a.f;
    const int64_t nvec = f.D / V;
    const int64_t j = (int64_t)blockIdx.x * kStThreads + threadIdx.x;
    if (j >= nvec) return;
    const int64_t c0 = j * V;
    float w[W][V], bv[V];
    load_filter<T, W>((const T*)f.w, f.w_sd, f.w_sk, (const T*)f.bias, f.bias_s, c0, wvec, bvec,
                      w, bv);
    const bool use_silu = f.silu != 0;
    prescale_filter<T, W>(w, bv, use_silu);
    const int64_t total = f.B * f.L;
    int64_t r = total * blockIdx.y / gridDim.y;
    const int64_t end = total * (blockIdx.y + 1) / gridDim.y;
    if (f.L == 0) {
        // Nothing to convolve: the final states are the tails of the initial states.
        for (int64_t b = blockIdx.y; b < f.B; b += gridDim.y)
            if (a.fin != nullptr) states_final<T, W>(a, b, c0, V);
        return;
    }
    while (r < end) {
        const int64_t b = r / f.L;
        const int64_t t0 = r - b * f.L;
        const int64_t n = min(end - r, f.L - t0);
        const T* xb = (const T*)f.x + b * f.x_sb + c0;
        T* ob = (T*)f.out + b * f.o_sb + c0;
        float h[W - 1][V];
        int32_t qh[W - 1];
        states_halo<T, W>(a, b, c0, t0, h, qh);
        if (SEQ)
            walk_strip_seq<T, W, kStRows>(xb, f.x_sl, ob, f.o_sl, a.seq + b * a.q_sb, a.q_sl, t0,
                                          t0 + n, h, qh, w, bv, use_silu);
        else
            walk_strip<T, W, kStRows, true>(xb, f.x_sl, ob, f.o_sl, t0, t0 + n, h, w, bv, use_silu);
        if (a.fin != nullptr && t0 + n == f.L) states_final<T, W>(a, b, c0, V);
        r += n;
    }
}

// Staged form for 16-bit types (the launch table of the plain prefill, fwd.cu): one
// CTA per strip of S tokens of one batch row and NT channel vectors, the strip landed in shared
// memory by cp.async (stage_strip). History before token 0 is the initial states (zeros without
// them), written into the stage's halo rows; with sequence ids (SEQ) a tap counts only when its id
// equals the token's; the strip that ends a row writes that row's final states. FULL: a whole strip
// of S rows (no per-row guard, see the plain staged kernel).
template <typename T, int W, int S, int NT, bool SILU, bool SEQ, bool FULL>
__device__ __forceinline__ void states_strip(const FwdStateArgs& a, uint4* col, int64_t b,
                                             int64_t t0, int64_t n, int64_t c0) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
    constexpr int HALF = S / 2;
    const FwdArgs& f = a.f;
    const T* xb = (const T*)f.x + b * f.x_sb + c0;
    stage_strip<T, K, S, NT, FULL>(col, xb, f.x_sl, t0, n);
    const T* init = (const T*)a.init;
    // Sequence ids of the halo and the strip's rows (rows before token 0 carry none: their values
    // are zeros or initial states, which sequence ids exclude).
    int32_t qh[K], q[S];
    const int32_t* qb = SEQ ? a.seq + b * a.q_sb : nullptr;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int64_t t = t0 - K + k;
        if (t < 0) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (init != nullptr) {
#pragma unroll
                for (int e = 0; e < V; ++e)
                    set_lane<T>(v, e, init[b * a.i_sb + (c0 + e) * a.i_sd + (K + t) * a.i_sk]);
            }
            col[k * NT] = v;
        }
        if (SEQ) qh[k] = t >= 0 ? __ldg(qb + t * a.q_sl) : INT32_MIN;
    }
    if (SEQ) {
        const int32_t* qr = qb + t0 * a.q_sl;
        if (FULL && a.q_sl == 1 && aligned16(qr)) {
            // Contiguous, aligned ids: four to a 16-byte load.
#pragma unroll
            for (int g = 0; g < S / 4; ++g) {
                const int4 v = __ldg(reinterpret_cast<const int4*>(qr) + g);
                q[4 * g] = v.x;
                q[4 * g + 1] = v.y;
                q[4 * g + 2] = v.z;
                q[4 * g + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int r = 0; r < S; ++r)
                if (FULL || r < n) q[r] = __ldg(qr + r * a.q_sl);
        }
    }
    Pairs w2[W], b2;
    {
        float w[W][V], bv[V];
        load_filter<T, W>((const T*)f.w, f.w_sd, f.w_sk, (const T*)f.bias, f.bias_s, c0, true,
                          true, w, bv);
        prescale_filter<T, W>(w, bv, SILU);
        filter_pairs<W>(w, bv, w2, b2);
    }
    T* ob = (T*)f.out + b * f.o_sb + c0;
    Pairs h[K];
    auto row = [&](int r) {
        const Pairs xv = to_pairs<T>(col[(K + r) * NT]);
        const Pairs o = SEQ ? conv_step_x2_seq<W, SILU>(h, qh, xv, q[r], w2, b2)
                            : conv_step_x2<W, SILU>(h, xv, w2, b2);
        st16_stream(ob + (t0 + r) * f.o_sl, from_pairs<T>(o));
    };
    cp_async_wait<1>();
#pragma unroll
    for (int k = 0; k < K; ++k) h[k] = to_pairs<T>(col[k * NT]);
    if (FULL) {
#pragma unroll
        for (int r = 0; r < HALF; ++r) row(r);
        cp_async_wait<0>();
#pragma unroll
        for (int r = HALF; r < S; ++r) row(r);
    } else {
        cp_async_wait<0>();
#pragma unroll
        for (int r = 0; r < S; ++r)
            if (r < n) row(r);
    }
    if (a.fin != nullptr && t0 + n == f.L) states_final<T, W>(a, b, c0, V);
}

// Strips strip0 .. strip0 + nstrips - 1 of every batch row: whole strips (FULL) in one launch, each
// row's last partial strip in a second one, as the plain staged prefill (fwd.cu).
template <typename T, int W, int S, int NT, bool SILU, bool SEQ, bool FULL>
__global__ void __launch_bounds__(NT)
    fwd_states_staged_kernel(const FwdStateArgs a, int64_t nstrips, int64_t gx, int64_t strip0) {
    constexpr int V = Vec<T>::V;
    extern __shared__ uint4 stage[];
    const int64_t blk = blockIdx.x;
    const int64_t su = blk / gx;
    const int64_t j = (blk - su * gx) * NT + threadIdx.x;
    if (j >= a.f.D / V) return;
    const int64_t b = su / nstrips;
    const int64_t t0 = (strip0 + su - b * nstrips) * S;
    const int64_t n = FULL ? S : a.f.L - t0;
    states_strip<T, W, S, NT, SILU, SEQ, FULL>(a, stage + threadIdx.x, b, t0, n, j * V);
}

template <typename T, int W, int S, int NT, bool SILU, bool SEQ>
cudaError_t launch_states_staged(const FwdStateArgs& a, int64_t gx, cudaStream_t stream) {
    const size_t smem = (size_t)(S + W - 1) * NT * 16;
    const int64_t full = a.f.L / S;
    if (full > 0) {
        fwd_states_staged_kernel<T, W, S, NT, SILU, SEQ, true>
            <<<(unsigned)(gx * a.f.B * full), NT, smem, stream>>>(a, full, gx, 0);
    }
    if (a.f.L % S != 0) {
        fwd_states_staged_kernel<T, W, S, NT, SILU, SEQ, false>
            <<<(unsigned)(gx * a.f.B), NT, smem, stream>>>(a, 1, gx, full);
    }
    return cudaGetLastError();
}

// Any strides: thread = (row, channel, strip of kStStrip tokens).
template <typename T, int W>
__global__ void __launch_bounds__(kStGenThreads) fwd_states_generic_kernel(const FwdStateArgs a,
                                                                           int64_t nstrips) {
    constexpr int K = W - 1;
    const FwdArgs& f = a.f;
    const int64_t n = f.B * f.D * nstrips;
    const bool use_silu = f.silu != 0;
    const T* init = (const T*)a.init;
    for (int64_t id = (int64_t)blockIdx.x * kStGenThreads + threadIdx.x; id < n;
         id += (int64_t)gridDim.x * kStGenThreads) {
        const int64_t s = id % nstrips;
        const int64_t c = (id / nstrips) % f.D;
        const int64_t b = id / (nstrips * f.D);
        const int64_t t0 = s * kStStrip, t1 = min(t0 + kStStrip, f.L);
        float w[W], bb;
        load_filter1<T, W>((const T*)f.w, f.w_sd, f.w_sk, (const T*)f.bias, f.bias_s, c, w, bb);
        const T* xr = (const T*)f.x + b * f.x_sb + c * f.x_sd;
        T* orow = (T*)f.out + b * f.o_sb + c * f.o_sd;
        const int32_t* qb = a.seq != nullptr ? a.seq + b * a.q_sb : nullptr;
        float h[K > 0 ? K : 1];
        int32_t qh[K > 0 ? K : 1];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int64_t t = t0 - K + k;
            if (t >= 0) {
                h[k] = to_f32<T>(xr[t * f.x_sl]);
                qh[k] = qb != nullptr ? qb[t * a.q_sl] : 0;
            } else {
                h[k] = init != nullptr ? to_f32<T>(init[b * a.i_sb + c * a.i_sd + (K + t) * a.i_sk])
                                       : 0.f;
                qh[k] = INT32_MIN;
            }
        }
        for (int64_t t = t0; t < t1; ++t) {
            const float xv = to_f32<T>(xr[t * f.x_sl]);
            const int32_t q = qb != nullptr ? qb[t * a.q_sl] : 0;
            float acc = bb;
#pragma unroll
            for (int k = 0; k < K; ++k)
                acc = (qb == nullptr || qh[k] == q) ? fmaf(h[k], w[k], acc) : acc;
            acc = fmaf(xv, w[K], acc);
            orow[t * f.o_sl] = from_f32<T>(activate<T>(acc, use_silu));
#pragma unroll
            for (int k = 0; k + 1 < K; ++k) {
                h[k] = h[k + 1];
                qh[k] = qh[k + 1];
            }
            if (K > 0) {
                h[K - 1] = xv;
                qh[K - 1] = q;
            }
        }
        if (a.fin != nullptr && t1 == f.L) {
            T* fin = (T*)a.fin;
            for (int k = 0; k < K; ++k) {
                const int64_t t = f.L - K + k;
                T v = t >= 0 ? xr[t * f.x_sl]
                             : (init != nullptr ? init[b * a.i_sb + c * a.i_sd + (K + t) * a.i_sk]
                                                : from_f32<T>(0.f));
                fin[b * a.f_sb + c * a.f_sd + k * a.f_sk] = v;
            }
        }
    }
}

template <typename T, int W>
cudaError_t run_fwd_states(const FwdStateArgs& a, cudaStream_t stream) {
    constexpr int V = Vec<T>::V;
    const FwdArgs& f = a.f;
    const int64_t e = sizeof(T);
    const int64_t nstrips = ceil_div(std::max<int64_t>(f.L, 1), kStStrip);
    const bool wvec = f.w_sd == W && f.w_sk == 1 && host_aligned16(f.w);
    const bool bvec = f.bias != nullptr && f.bias_s == 1 && host_aligned16(f.bias);
    const bool cl = f.x_sd == 1 && f.o_sd == 1 && f.D % V == 0 && host_aligned16(f.x) &&
                    host_aligned16(f.out) && (f.x_sl * e) % 16 == 0 && (f.o_sl * e) % 16 == 0 &&
                    (f.x_sb * e) % 16 == 0 && (f.o_sb * e) % 16 == 0;
    if constexpr (sizeof(T) == 2) {
        // Staged strips of 16 tokens (32 at W = 8), one per 64-thread CTA, as the plain
        // channel-last prefill (channel pairs, compile-time SiLU).
        // Measured on B200 at the config-2 shape (bf16, W = 4), staged vs the balanced register
        // walk below: initial + final states 163.3 vs 182.9 us (172.5 with scalar FMAs and a
        // run-time SiLU); with sequence ids 170.4 vs 181.4 us (183.4 with scalar FMAs, 184.3 with
        // the 16 ids of a strip loaded one by one instead of four to a 16-byte load).
        constexpr int S = W == 8 ? 32 : 16, NT = 64;
        const int64_t gx = ceil_div(f.D / V, (int64_t)NT);
        const int64_t blocks = gx * f.B * ceil_div(f.L, (int64_t)S);
        if (cl && f.L > 0 && wvec && (f.bias == nullptr || bvec) && blocks <= 0x7fffffffLL) {
            if (a.seq != nullptr)
                return f.silu ? launch_states_staged<T, W, S, NT, true, true>(a, gx, stream)
                              : launch_states_staged<T, W, S, NT, false, true>(a, gx, stream);
            return f.silu ? launch_states_staged<T, W, S, NT, true, false>(a, gx, stream)
                          : launch_states_staged<T, W, S, NT, false, false>(a, gx, stream);
        }
    }
    if (cl) {
        // Launch table as for the plain channel-last prefill (fwd.cu): many ~128-row shares,
        // balanced by the block scheduler, for W <= 3 or short sequences when they give at least
        // half a wave of CTAs; otherwise one balanced wave.
        const int64_t gx = ceil_div(f.D / V, (int64_t)kStThreads);
        static int slot_cache[2][kSlotCacheDevices] = {};
        const bool seq = a.seq != nullptr;
        auto kern = seq ? fwd_states_vec_kernel<T, W, true> : fwd_states_vec_kernel<T, W, false>;
        const int64_t slots = device_slots((const void*)kern, kStThreads, slot_cache[seq]);
        const int64_t rows = std::max<int64_t>(f.B * f.L, 1);
        const int64_t strips = ceil_div(rows, kStStrip);
        int64_t gy = (W <= 3 || f.L <= kStStrip) && strips * gx * 2 >= slots
                         ? strips
                         : std::min<int64_t>(std::max<int64_t>(slots, 1) / gx, ceil_div(rows, (int64_t)16));
        if (f.L == 0) gy = f.B;
        gy = std::max<int64_t>(1, std::min<int64_t>(gy, 65535));
        kern<<<dim3((unsigned)gx, (unsigned)gy), kStThreads, 0, stream>>>(a, wvec, bvec);
        return cudaGetLastError();
    }
    const int64_t n = f.B * f.D * nstrips;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, kStGenThreads), 148 * 32));
    fwd_states_generic_kernel<T, W><<<(unsigned)blocks, kStGenThreads, 0, stream>>>(a, nstrips);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd_states(const FwdStateArgs& a, int width, int dtype, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    CC1D_DISPATCH_DTYPE(dtype, CC1D_DISPATCH_WIDTH(width, err = (run_fwd_states<T, kW>(a, stream))));
    return err;
}

}  // namespace cc1d
