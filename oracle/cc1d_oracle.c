/*
 * CPU port of the reference's fallback algorithm (TEST INFRASTRUCTURE ONLY: the CPU baseline that
 * bench.py times, and a second checker for the tests). Not part of the library.
 *
 * Restates causal_conv1d_cute/fallback.py: fwd (fallback.py:49-74), varlen (fallback.py:77-114)
 * and update (fallback.py:117-164) with fp32 accumulation (bias first, taps oldest first) and
 * round-to-nearest-even to bf16, multithreaded with OpenMP over independent (row, channel) work.
 * bf16 tensors are uint16 bit patterns. Layouts: channel-last (batch, seqlen, dim) rows for fwd
 * and token-major (ntokens, dim) rows for varlen, which is how the benchmark stores them.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

static inline float bf2f(uint16_t v) {
    uint32_t u = (uint32_t)v << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f2bf(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float silu(float a) { return a / (1.0f + expf(-a)); }

int oracle_threads(void) { return omp_get_max_threads(); }

void oracle_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

/* Prefill over channel-last bf16: x, out (B, L, D) contiguous; w (D, W); bias (D) or NULL. */
void oracle_fwd_cl_bf16(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* out,
                        int64_t B, int64_t L, int64_t D, int W, int use_silu) {
    const int K = W - 1;
    const int64_t CH = 64; /* tokens per work item */
    const int64_t chunks = (L + CH - 1) / CH;
#pragma omp parallel
    {
        float acc[1024];
#pragma omp for schedule(static)
        for (int64_t item = 0; item < B * chunks; ++item) {
            const int64_t b = item / chunks;
            const int64_t t0 = (item % chunks) * CH;
            const int64_t t1 = t0 + CH < L ? t0 + CH : L;
            for (int64_t t = t0; t < t1; ++t) {
                for (int64_t c0 = 0; c0 < D; c0 += 1024) {
                    const int64_t n = D - c0 < 1024 ? D - c0 : 1024;
                    for (int64_t c = 0; c < n; ++c)
                        acc[c] = bias ? bf2f(bias[c0 + c]) : 0.0f;
                    for (int k = 0; k < W; ++k) {
                        const int64_t src = t - K + k;
                        if (src < 0) continue;
                        const uint16_t* xr = x + (b * L + src) * D + c0;
                        for (int64_t c = 0; c < n; ++c)
                            acc[c] += bf2f(w[(c0 + c) * W + k]) * bf2f(xr[c]);
                    }
                    uint16_t* orow = out + (b * L + t) * D + c0;
                    for (int64_t c = 0; c < n; ++c)
                        orow[c] = f2bf(use_silu ? silu(acc[c]) : acc[c]);
                }
            }
        }
    }
}

/* Packed prefill over token-major bf16 x (T, D); states (slots, D, K) updated in place. */
void oracle_varlen_bf16(const uint16_t* x, const uint16_t* w, const uint16_t* bias, uint16_t* out,
                        const int32_t* qsl, int64_t nseq, int64_t D, int W, const int32_t* cidx,
                        const uint8_t* hinit, uint16_t* states, int32_t pad, int use_silu) {
    const int K = W - 1;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int64_t s = 0; s < nseq; ++s) {
        for (int64_t c = 0; c < D; ++c) {
            const int64_t a = qsl[s], e = qsl[s + 1];
            const int32_t slot = cidx ? cidx[s] : (int32_t)s;
            if (e <= a || (states && slot == pad)) continue;
            float init[8] = {0};
            uint16_t init_bits[8] = {0};
            if (states && hinit && hinit[s])
                for (int k = 0; k < K; ++k) {
                    init_bits[k] = states[((int64_t)slot * D + c) * K + k];
                    init[k] = bf2f(init_bits[k]);
                }
            for (int64_t t = a; t < e; ++t) {
                float acc = bias ? bf2f(bias[c]) : 0.0f;
                for (int k = 0; k < W; ++k) {
                    const int64_t p = t - K + k;
                    const float v = p >= a ? bf2f(x[p * D + c]) : init[K + (p - a)];
                    acc += bf2f(w[c * W + k]) * v;
                }
                out[t * D + c] = f2bf(use_silu ? silu(acc) : acc);
            }
            if (states) {
                uint16_t* st = states + ((int64_t)slot * D + c) * K;
                for (int k = 0; k < K; ++k) {
                    const int64_t p = e - K + k;
                    st[k] = p >= a ? x[p * D + c] : init_bits[k + (e - a)];
                }
            }
        }
    }
}

/* Single-token indexed decode: x (B, D), state (slots, D, K) in place, out (B, D). */
void oracle_update_bf16(const uint16_t* x, uint16_t* state, const uint16_t* w, const uint16_t* bias,
                        uint16_t* out, const int32_t* idx, int64_t B, int64_t D, int W, int32_t pad,
                        int use_silu) {
    const int K = W - 1;
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t b = 0; b < B; ++b) {
        for (int64_t c = 0; c < D; ++c) {
            const int32_t slot = idx ? idx[b] : (int32_t)b;
            if (slot == pad) continue;
            uint16_t* st = state + ((int64_t)slot * D + c) * K;
            float acc = bias ? bf2f(bias[c]) : 0.0f;
            for (int k = 0; k < K; ++k) acc += bf2f(w[c * W + k]) * bf2f(st[k]);
            acc += bf2f(w[c * W + K]) * bf2f(x[b * D + c]);
            for (int k = 0; k + 1 < K; ++k) st[k] = st[k + 1];
            st[K - 1] = x[b * D + c];
            out[b * D + c] = f2bf(use_silu ? silu(acc) : acc);
        }
    }
}
