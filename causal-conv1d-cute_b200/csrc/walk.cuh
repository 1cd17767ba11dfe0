// Token-row walk shared by the channel-last prefill and the token-major varlen kernels.
//
// A thread owns one 16-byte vector of V adjacent channels and walks consecutive token rows,
// keeping the W-1 most recent inputs of its channels in registers (fp32, oldest first).
#pragma once

#include <type_traits>

#include "common.cuh"

namespace cc1d {

// Scale applied to the filter and bias of the streaming kernels: with SiLU on a 16-bit output,
// the weights are pre-multiplied by 1/2 (exact in fp32), so the accumulator holds h = a / 2 and
// SiLU(a) = a * (tanh(a / 2) / 2 + 1/2) = h * tanh(h) + h takes one MUFU and one FMA per element.
// The sums are exactly half of the unscaled ones (power-of-two scaling commutes with rounding
// outside the fp32 subnormal range), so outputs are unchanged.
template <typename T>
__host__ __device__ constexpr bool prescaled_silu() {
    return !std::is_same<T, float>::value;
}

template <typename T, int W, int NB = 16>
__device__ __forceinline__ void prescale_filter(float (&w)[W][NB / sizeof(T)],
                                                float (&b)[NB / sizeof(T)], bool use_silu) {
    if (prescaled_silu<T>() && use_silu) {
#pragma unroll
        for (int e = 0; e < NB / (int)sizeof(T); ++e) {
#pragma unroll
            for (int k = 0; k < W; ++k) w[k][e] *= 0.5f;
            b[e] *= 0.5f;
        }
    }
}

// Activation of a prescaled accumulator (see prescale_filter).
template <typename T>
__device__ __forceinline__ float activate_prescaled(float acc, bool use_silu) {
    if (prescaled_silu<T>()) return use_silu ? fmaf(acc, tanh_approx(acc), acc) : acc;
    return activate<T>(acc, use_silu);
}

// One output vector from the fp32 window h (oldest first) and the new input xv; shifts xv into
// the window afterwards. Bias first, taps oldest first, one fused multiply-add per tap. The
// filter is prescaled (prescale_filter).
template <typename T, int W, int NB = 16>
__device__ __forceinline__ void conv_step(float (&h)[W - 1][NB / sizeof(T)], const float* xv,
                                          const float (&w)[W][NB / sizeof(T)],
                                          const float (&bv)[NB / sizeof(T)], bool use_silu,
                                          float* o) {
    constexpr int V = NB / (int)sizeof(T);
    constexpr int K = W - 1;
#pragma unroll
    for (int e = 0; e < V; ++e) {
        float acc = bv[e];
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(h[k][e], w[k][e], acc);
        acc = fmaf(xv[e], w[K][e], acc);
        o[e] = activate_prescaled<T>(acc, use_silu);
    }
#pragma unroll
    for (int k = 0; k + 1 < K; ++k)
#pragma unroll
        for (int e = 0; e < V; ++e) h[k][e] = h[k + 1][e];
#pragma unroll
    for (int e = 0; e < V; ++e) h[K - 1][e] = xv[e];
}

// Walk rows [ta, tb) of one channel group: h holds the W-1 previous inputs (fp32, oldest first).
// Rows are loaded U at a time; with PF the next U rows are requested before the current U are
// computed, so 2U 16-byte loads per thread stay in flight (bytes in flight per SM bound this
// kernel). NB: bytes of channels per thread (16, or 8 for the half-width kernels).
template <typename T, int W, int U, bool PF, int NB = 16>
__device__ __forceinline__ void walk_strip(const T* __restrict__ xb, int64_t x_st,
                                           T* __restrict__ ob, int64_t o_st, int64_t ta,
                                           int64_t tb, float (&h)[W - 1][NB / sizeof(T)],
                                           const float (&w)[W][NB / sizeof(T)],
                                           const float (&bv)[NB / sizeof(T)], bool use_silu) {
    constexpr int V = NB / (int)sizeof(T);
    using R = typename RawVec<NB>::type;
    int64_t t = ta;
    auto emit = [&](const R& r, int64_t row) {
        float xv[V], o[V];
        unpack_raw<T, NB>(r, xv);
        conv_step<T, W, NB>(h, xv, w, bv, use_silu, o);
        st_stream_raw<NB>(ob + row * o_st, pack_raw<T, NB>(o));
    };
    if (PF) {
        R nxt[U];
        bool have = t + U <= tb;
        if (have) {
#pragma unroll
            for (int i = 0; i < U; ++i) nxt[i] = ldg_stream_raw<NB>(xb + (t + i) * x_st);
        }
        while (have) {
            R cur[U];
#pragma unroll
            for (int i = 0; i < U; ++i) cur[i] = nxt[i];
            const int64_t tn = t + U;
            have = tn + U <= tb;
            if (have) {
#pragma unroll
                for (int i = 0; i < U; ++i) nxt[i] = ldg_stream_raw<NB>(xb + (tn + i) * x_st);
            }
#pragma unroll
            for (int i = 0; i < U; ++i) emit(cur[i], t + i);
            t = tn;
        }
    } else {
        for (; t + U <= tb; t += U) {
            R r[U];
#pragma unroll
            for (int i = 0; i < U; ++i) r[i] = ldg_stream_raw<NB>(xb + (t + i) * x_st);
#pragma unroll
            for (int i = 0; i < U; ++i) emit(r[i], t + i);
        }
    }
    for (; t < tb; ++t) emit(ldg_stream_raw<NB>(xb + t * x_st), t);
}

// conv_step with per-token sequence ids: a history tap counts only when its id equals the
// token's id q (a differing id adds nothing; the term is skipped, not multiplied by zero). The
// window ids qh shift with the values.
template <typename T, int W>
__device__ __forceinline__ void conv_step_seq(float (&h)[W - 1][Vec<T>::V], int32_t (&qh)[W - 1],
                                              const float* xv, int32_t q,
                                              const float (&w)[W][Vec<T>::V],
                                              const float (&bv)[Vec<T>::V], bool use_silu,
                                              float* o) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
#pragma unroll
    for (int e = 0; e < V; ++e) {
        float acc = bv[e];
#pragma unroll
        for (int k = 0; k < K; ++k) acc = qh[k] == q ? fmaf(h[k][e], w[k][e], acc) : acc;
        acc = fmaf(xv[e], w[K][e], acc);
        o[e] = activate_prescaled<T>(acc, use_silu);
    }
#pragma unroll
    for (int k = 0; k + 1 < K; ++k) {
        qh[k] = qh[k + 1];
#pragma unroll
        for (int e = 0; e < V; ++e) h[k][e] = h[k + 1][e];
    }
    qh[K - 1] = q;
#pragma unroll
    for (int e = 0; e < V; ++e) h[K - 1][e] = xv[e];
}

// walk_strip (with prefetch) for rows carrying sequence ids qb[row * q_st].
template <typename T, int W, int U>
__device__ __forceinline__ void walk_strip_seq(const T* __restrict__ xb, int64_t x_st,
                                               T* __restrict__ ob, int64_t o_st,
                                               const int32_t* __restrict__ qb, int64_t q_st,
                                               int64_t ta, int64_t tb,
                                               float (&h)[W - 1][Vec<T>::V], int32_t (&qh)[W - 1],
                                               const float (&w)[W][Vec<T>::V],
                                               const float (&bv)[Vec<T>::V], bool use_silu) {
    constexpr int V = Vec<T>::V;
    int64_t t = ta;
    auto emit = [&](const uint4& r, int32_t q, int64_t row) {
        float xv[V], o[V];
        unpack16<T>(r, xv);
        conv_step_seq<T, W>(h, qh, xv, q, w, bv, use_silu, o);
        st16_stream(ob + row * o_st, pack16<T>(o));
    };
    uint4 nxt[U];
    int32_t nq[U];
    bool have = t + U <= tb;
    if (have) {
#pragma unroll
        for (int i = 0; i < U; ++i) {
            nxt[i] = ldg16_stream(xb + (t + i) * x_st);
            nq[i] = __ldg(qb + (t + i) * q_st);
        }
    }
    while (have) {
        uint4 cur[U];
        int32_t cq[U];
#pragma unroll
        for (int i = 0; i < U; ++i) {
            cur[i] = nxt[i];
            cq[i] = nq[i];
        }
        const int64_t tn = t + U;
        have = tn + U <= tb;
        if (have) {
#pragma unroll
            for (int i = 0; i < U; ++i) {
                nxt[i] = ldg16_stream(xb + (tn + i) * x_st);
                nq[i] = __ldg(qb + (tn + i) * q_st);
            }
        }
#pragma unroll
        for (int i = 0; i < U; ++i) emit(cur[i], cq[i], t + i);
        t = tn;
    }
    for (; t < tb; ++t) emit(ldg16_stream(xb + t * x_st), __ldg(qb + t * q_st), t);
}

// Packed form of conv_step for the staged kernels: a 16-byte vector of a 16-bit type (8
// channels) as 4 channel pairs, every tap one fp32x2 fused multiply-add (__ffma2_rn, which rounds
// each lane as fmaf does, so the bits equal conv_step's) and SILU fixed at compile time. Against
// 8 scalar FMAs per tap this halves the arithmetic instructions, which bound the staged walk from
// W = 7 (measured on B200 at the config-2 shape: W = 7 211 -> 174 us, W = 8 242 -> 192 us; no
// change up to W = 6). The filter and bias are prescaled by 1/2 when SILU (prescale_filter).
constexpr int kPairs = 4;

struct Pairs {
    float2 p[kPairs];
};

template <typename T>
__device__ __forceinline__ Pairs to_pairs(const uint4& v) {
    float f[2 * kPairs];
    unpack16<T>(v, f);
    Pairs r;
#pragma unroll
    for (int q = 0; q < kPairs; ++q) r.p[q] = make_float2(f[2 * q], f[2 * q + 1]);
    return r;
}

template <typename T>
__device__ __forceinline__ uint4 from_pairs(const Pairs& v) {
    float f[2 * kPairs];
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
        f[2 * q] = v.p[q].x;
        f[2 * q + 1] = v.p[q].y;
    }
    return pack16<T>(f);
}

// The prescaled fp32 filter and bias of load_filter / prescale_filter as channel pairs.
template <int W>
__device__ __forceinline__ void filter_pairs(const float (&w)[W][2 * kPairs],
                                             const float (&b)[2 * kPairs], Pairs (&w2)[W],
                                             Pairs& b2) {
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
        b2.p[q] = make_float2(b[2 * q], b[2 * q + 1]);
#pragma unroll
        for (int k = 0; k < W; ++k) w2[k].p[q] = make_float2(w[k][2 * q], w[k][2 * q + 1]);
    }
}

template <int W, bool SILU>
__device__ __forceinline__ Pairs conv_step_x2(Pairs (&h)[W - 1], const Pairs& xv,
                                              const Pairs (&w)[W], const Pairs& b) {
    constexpr int K = W - 1;
    Pairs o;
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
        float2 acc = b.p[q];
#pragma unroll
        for (int k = 0; k < K; ++k) acc = __ffma2_rn(h[k].p[q], w[k].p[q], acc);
        acc = __ffma2_rn(xv.p[q], w[K].p[q], acc);
        if (SILU) acc = __ffma2_rn(acc, make_float2(tanh_approx(acc.x), tanh_approx(acc.y)), acc);
        o.p[q] = acc;
    }
#pragma unroll
    for (int k = 0; k + 1 < K; ++k) h[k] = h[k + 1];
    h[K - 1] = xv;
    return o;
}

// conv_step_x2 with per-token sequence ids: a history tap counts only when its id equals the
// token's id q (the term is skipped, as in conv_step_seq); the window ids qh shift with the values.
template <int W, bool SILU>
__device__ __forceinline__ Pairs conv_step_x2_seq(Pairs (&h)[W - 1], int32_t (&qh)[W - 1],
                                                  const Pairs& xv, int32_t q, const Pairs (&w)[W],
                                                  const Pairs& b) {
    constexpr int K = W - 1;
    Pairs o;
#pragma unroll
    for (int p = 0; p < kPairs; ++p) {
        float2 acc = b.p[p];
#pragma unroll
        for (int k = 0; k < K; ++k)
            if (qh[k] == q) acc = __ffma2_rn(h[k].p[p], w[k].p[p], acc);
        acc = __ffma2_rn(xv.p[p], w[K].p[p], acc);
        if (SILU) acc = __ffma2_rn(acc, make_float2(tanh_approx(acc.x), tanh_approx(acc.y)), acc);
        o.p[p] = acc;
    }
#pragma unroll
    for (int k = 0; k + 1 < K; ++k) {
        h[k] = h[k + 1];
        qh[k] = qh[k + 1];
    }
    h[K - 1] = xv;
    qh[K - 1] = q;
    return o;
}

// Stage of a short strip in shared memory, for the staged kernels: a thread's 16-byte column of
// the K rows before t0 and of the strip's rows t0.. t0+n-1 (n == S when FULL) lies at
// col[r * NT], halo rows first. The halo rows at t >= 0 and the strip's first half are one
// cp.async group, the second half another, so cp_async_wait<1>() makes the halo and the first half
// readable while the rest lands. Halo rows at t < 0 are not touched: the caller fills them.
template <typename T, int K, int S, int NT, bool FULL>
__device__ __forceinline__ void stage_strip(uint4* col, const T* xb, int64_t x_st, int64_t t0,
                                            int64_t n) {
    constexpr int HALF = S / 2;
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int64_t t = t0 - K + k;
        if (t >= 0) cp_async16(col + k * NT, xb + t * x_st);
    }
#pragma unroll
    for (int i = 0; i < HALF; ++i)
        if (FULL || i < n) cp_async16(col + (K + i) * NT, xb + (t0 + i) * x_st);
    cp_async_commit();
#pragma unroll
    for (int i = HALF; i < S; ++i)
        if (FULL || i < n) cp_async16(col + (K + i) * NT, xb + (t0 + i) * x_st);
    cp_async_commit();
}

// Window of the W-1 rows before t0 (zeros before the sequence start).
template <typename T, int W, int NB = 16>
__device__ __forceinline__ void load_halo(const T* xb, int64_t x_st, int64_t t0,
                                          float (&h)[W - 1][NB / sizeof(T)]) {
#pragma unroll
    for (int k = 0; k < W - 1; ++k) {
        const int64_t t = t0 - (W - 1) + k;
        if (t >= 0) {
            unpack_raw<T, NB>(ldg_raw<NB>(xb + t * x_st), h[k]);
        } else {
#pragma unroll
            for (int e = 0; e < NB / (int)sizeof(T); ++e) h[k][e] = 0.f;
        }
    }
}

}  // namespace cc1d
