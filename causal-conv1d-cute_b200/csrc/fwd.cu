// Prefill over dense batched sequences (replaces causal_conv1d_cute/fwd.py).
//
// Kernels, chosen by layout and width in run_fwd:
//   fwd_channel_last_staged  (B, L, D) storage, 16-bit types: one CTA per strip of 16 (32 at
//                      W = 8) tokens of one batch row and 64 16-byte channel vectors; each thread lands
//                      its column of the strip (and the W-1 rows before it) in shared memory with
//                      cp.async and walks it there. Many short-lived CTAs, several waves.
//   fwd_channel_last   (B, L, D) storage otherwise (x_sd == 1): every thread owns one 16-byte (or
//   _share             8-byte) vector of channels and walks a run of tokens from registers,
//                      keeping the W-1 most recent inputs; a run re-reads only the W-1 rows
//                      before it, which its neighbour has just pulled into L2. Runs are fixed
//                      strips (several waves) or balanced shares (one wave), per the launch table.
//   fwd_channel_first  (B, D, L) contiguous storage: the tensor is one flat stream; every lane of
//                      a warp owns 16 or 32 consecutive elements and receives the W-1 elements
//                      before them from the lane to its left by a warp shuffle, so HBM is read once.
//   fwd_generic        any other strides, one channel per thread (correctness path).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "walk.cuh"

namespace cc1d {

namespace {

constexpr int kClThreads = 64;
constexpr int kCfThreads = 256;
constexpr int kGenThreads = 256;

template <typename T, int W, int U, bool PF, int NT>
__global__ void __launch_bounds__(NT)
    fwd_channel_last_kernel(const FwdArgs a, int strip, int nstrips, bool wvec, bool bvec) {
    constexpr int V = Vec<T>::V;
    const int64_t nvec = a.D / V;
    const int64_t j = (int64_t)blockIdx.x * NT + threadIdx.x;
    if (j >= nvec) return;
    const int64_t c0 = j * V;
    float w[W][V], bv[V];
    load_filter<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c0, wvec, bvec,
                      w, bv);
    const bool use_silu = a.silu != 0;
    prescale_filter<T, W>(w, bv, use_silu);
    const int64_t units = (int64_t)nstrips * a.B;
    for (int64_t u = blockIdx.y; u < units; u += gridDim.y) {
        const int64_t b = u / nstrips;
        const int64_t t0 = (u - b * nstrips) * (int64_t)strip;
        const int64_t t1 = min(t0 + strip, a.L);
        const T* xb = (const T*)a.x + b * a.x_sb + c0;
        T* ob = (T*)a.out + b * a.o_sb + c0;
        float h[W - 1][V];
        load_halo<T, W>(xb, a.x_sl, t0, h);
        walk_strip<T, W, U, PF>(xb, a.x_sl, ob, a.o_sl, t0, t1, h, w, bv, use_silu);
    }
}

// Balanced variant: blockIdx.x is the channel block (NT vectors) and blockIdx.y one of gridDim.y
// equal contiguous shares of the flattened (batch, token) rows; the grid is sized to the CTAs the
// GPU holds at once. A thread walks its channel vector through the share's rows, re-reading the
// W-1 rows before each batch stretch. Every CTA does the same work whatever B and L are (no
// partial last wave), and the CTAs of one share, launched back to back, read the same token rows
// at about the same time, so each DRAM page is opened once for all its channel blocks.
template <typename T, int W, int U, bool PF, int NT, int MINB, int NB = 16>
__global__ void __launch_bounds__(NT, MINB)
    fwd_channel_last_share_kernel(const FwdArgs a, bool wvec, bool bvec) {
    constexpr int V = NB / (int)sizeof(T);
    const int64_t nvec = a.D / V;
    const int64_t j = (int64_t)blockIdx.x * NT + threadIdx.x;
    if (j >= nvec) return;
    const int64_t total = a.B * a.L;
    int64_t r = total * blockIdx.y / gridDim.y;
    const int64_t end = total * (blockIdx.y + 1) / gridDim.y;
    const bool use_silu = a.silu != 0;
    const int64_t c0 = j * V;
    float w[W][V], bv[V];
    load_filter<T, W, NB>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c0, wvec,
                          bvec, w, bv);
    prescale_filter<T, W, NB>(w, bv, use_silu);
    while (r < end) {
        const int64_t b = r / a.L;
        const int64_t t0 = r - b * a.L;
        const int64_t n = min(end - r, a.L - t0);
        const T* xb = (const T*)a.x + b * a.x_sb + c0;
        T* ob = (T*)a.out + b * a.o_sb + c0;
        float h[W - 1][V];
        load_halo<T, W, NB>(xb, a.x_sl, t0, h);
        walk_strip<T, W, U, PF, NB>(xb, a.x_sl, ob, a.o_sl, t0, t0 + n, h, w, bv, use_silu);
        r += n;
    }
}

// The staged walk (one strip of 16 tokens, 32 at W = 8, per 64-thread CTA, rows landed in shared
// memory by cp.async, channel pairs by packed FMAs) serves 16-bit types at every width. Measured on
// B200 at the config-2 shape (8 x 4096 x 8192 bf16, one launch at a time; staged vs the register
// walk below, us): W = 2: 163.7 vs 174.1; 3: 163.9 vs 176.6; 4: 162.3 vs 184.1; 5: 161.8 vs 185.5;
// 6: 162.0 vs 185.5 (175.2 with the default budget of 130 registers, 7 CTAs per SM; a separate
// kernel asks for 8); 7: 179.7 vs 186.6; 8: 189.2 vs 198.7. The library's copy of the same bytes
// takes 160-161 us. Longer strips
// lost at W <= 7 (W = 4: 32 tokens 175.7 us, 64: 256.5 us: fewer CTAs fit and each lives longer)
// and 16 tokens lost at W = 8 (222-248 us: the 7 halo rows are a larger share of each strip); so
// did the same strips walked from registers (16 tokens, all loads up front: 210 us at W = 4,
// spilling), one-thread bulk copies of whole 1 KB row segments on an mbarrier (164.8 us, no gain),
// scalar FMAs (W = 7: 211 us, W = 8: 242 us), SiLU tested at run time (W = 5: 183.6 us), run-time
// weight and bias layout flags (W = 8: 196 -> 190 us when constant) and a minimum of 9-12
// resident CTAs in the launch bounds at W <= 5 (it spills). fp32 keeps the register walk.
constexpr int kStageThreads = 64;
template <typename T, int W>
constexpr bool staged_prefill() {
    return sizeof(T) == 2;
}
template <int W>
constexpr int stage_rows() {
    return W == 8 ? 32 : 16;
}

// One strip of n rows (n == S when FULL): copies, filter, then the walk from shared memory in
// channel pairs (conv_step_x2). The full-strip form has no per-row guard, so the window shift of
// every row is a static register renaming; a guard on each row turns it into a select per window
// register (the W = 4 kernel took 243 instead of 164 us at the config-2 shape that way), so only a
// batch row's last strip, when L is not a multiple of S, takes the guarded form.
template <typename T, int W, int S, int NT, bool SILU, bool FULL>
__device__ __forceinline__ void staged_strip(const FwdArgs& a, uint4* col, const T* xb, T* ob,
                                             int64_t t0, int64_t n, int64_t c0) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
    constexpr int HALF = S / 2;
    stage_strip<T, K, S, NT, FULL>(col, xb, a.x_sl, t0, n);
#pragma unroll
    for (int k = 0; k < K; ++k)
        if (t0 - K + k < 0) col[k * NT] = make_uint4(0u, 0u, 0u, 0u);
    Pairs w2[W], b2;
    {
        float w[W][V], bv[V];
        load_filter<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c0, true,
                          true, w, bv);
        prescale_filter<T, W>(w, bv, SILU);
        filter_pairs<W>(w, bv, w2, b2);
    }
    Pairs h[K];
    auto row = [&](int r) {
        const Pairs o = conv_step_x2<W, SILU>(h, to_pairs<T>(col[(K + r) * NT]), w2, b2);
        st16_stream(ob + (t0 + r) * a.o_sl, from_pairs<T>(o));
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
        for (int r = 0; r < n; ++r) row(r);
    }
}

// Staged variant, one short strip per CTA: blockIdx.x = strip * gx + channel block, where a strip
// is S consecutive tokens of one batch row and a channel block NT 16-byte vectors. Each thread
// copies its own 16-byte column of the W-1 rows before the strip and of the strip's S rows into
// shared memory with cp.async (the bytes in flight hold no registers), loads the filter while
// they land, waits for its own copies (in two groups: the first half is computed while the second
// lands) and walks the rows from shared memory. No thread reads another's column, so there is no
// barrier. The grid runs many short-lived CTAs back to back, which keeps the bytes requested from
// DRAM at any moment within a narrow window of consecutive rows, as a copy does; the halo rows
// were just read by the neighbouring strip's CTA and come from L2. 16-bit types only (the pair
// arithmetic takes 8 channels per 16-byte vector); the weights are the contiguous (dim, W) tensor
// and the bias, if any, is contiguous (the host sends other layouts to the register walk).
//
// One launch covers strips strip0 .. strip0 + nstrips - 1 of every batch row. FULL launches cover
// the whole strips; a second, guarded launch (FULL false, nstrips 1) covers each row's last strip
// when L is not a multiple of S. The two forms are separate kernels because the guarded form's
// registers would otherwise be the whole kernel's (W = 8: 250 instead of 166 registers, 210 instead
// of 196 us at the config-2 shape).
template <typename T, int W, int S, int NT, bool SILU, bool FULL>
__device__ __forceinline__ void staged_cta(const FwdArgs& a, int64_t nstrips, int64_t gx,
                                           int64_t strip0) {
    constexpr int V = Vec<T>::V;
    extern __shared__ uint4 stage[];
    const int64_t blk = blockIdx.x;
    const int64_t su = blk / gx;
    const int64_t j = (blk - su * gx) * NT + threadIdx.x;
    if (j >= a.D / V) return;
    const int64_t b = su / nstrips;
    const int64_t t0 = (strip0 + su - b * nstrips) * S;
    const int64_t n = FULL ? S : a.L - t0;
    const int64_t c0 = j * V;
    const T* xb = (const T*)a.x + b * a.x_sb + c0;
    T* ob = (T*)a.out + b * a.o_sb + c0;
    uint4* col = stage + threadIdx.x;  // row r of the stage (halo rows first) at col[r * NT]
    staged_strip<T, W, S, NT, SILU, FULL>(a, col, xb, ob, t0, n, c0);
}

// The launch bounds name no minimum of resident CTAs: with an explicit minimum of 1 the compiler
// spends registers freely (W = 4: 194 instead of 98, W = 2: 174 instead of 60) and the kernel
// fits half as many CTAs per SM (W = 4: 198 instead of 163 us at the config-2 shape).
template <typename T, int W, int S, int NT, bool SILU, bool FULL>
__global__ void __launch_bounds__(NT)
    fwd_channel_last_staged_kernel(const FwdArgs a, int64_t nstrips, int64_t gx, int64_t strip0) {
    staged_cta<T, W, S, NT, SILU, FULL>(a, nstrips, gx, strip0);
}

// W = 6 with SiLU, whole strips: the default budget (130 registers) leaves 7 CTAs per SM; a
// minimum of 8 fits it in 128 registers without spilling.
template <typename T, int S, int NT>
__global__ void __launch_bounds__(NT, 8)
    fwd_channel_last_staged_w6_kernel(const FwdArgs a, int64_t nstrips, int64_t gx) {
    staged_cta<T, 6, S, NT, true, true>(a, nstrips, gx, 0);
}

// The full-strip launch and, when L is not a multiple of S, the last-strip launch.
template <typename T, int W, int S, bool SILU>
cudaError_t launch_staged(const FwdArgs& a, int64_t gx, cudaStream_t stream) {
    const size_t smem = (size_t)(S + W - 1) * kStageThreads * 16;
    const int64_t full = a.L / S;
    if (full > 0) {
        if constexpr (W == 6 && SILU)
            fwd_channel_last_staged_w6_kernel<T, S, kStageThreads>
                <<<(unsigned)(gx * a.B * full), kStageThreads, smem, stream>>>(a, full, gx);
        else
            fwd_channel_last_staged_kernel<T, W, S, kStageThreads, SILU, true>
                <<<(unsigned)(gx * a.B * full), kStageThreads, smem, stream>>>(a, full, gx, 0);
    }
    if (a.L % S != 0) {
        fwd_channel_last_staged_kernel<T, W, S, kStageThreads, SILU, false>
            <<<(unsigned)(gx * a.B), kStageThreads, smem, stream>>>(a, 1, gx, full);
    }
    return cudaGetLastError();
}

// Flat-stream kernel for contiguous (B, D, L) with L >= EPT. Element f sits at row f / L (channel
// (f / L) % D) and position t = f % L; tap k of its output reads element f - (W-1) + k when that
// lies in the same row (t >= W-1-k), zero otherwise. A lane owns EPT (16 or 32, at most L)
// consecutive elements (16-byte vectors) and receives the W-1 elements before them
// from the lane to its left by a warp shuffle; lane 0 gets them from lane 31 of the previous
// iteration, so every element is read from HBM once. The next iteration's vectors are requested
// before the current ones are computed. A lane's elements straddle at most one row boundary.
template <typename T, int W, bool V32, int EPT>
__global__ void __launch_bounds__(kCfThreads)
    fwd_channel_first_kernel(const FwdArgs a, int64_t total, int iters) {
    constexpr int K = W - 1;
    constexpr int PER = 16 / (int)sizeof(T);
    constexpr int NV = EPT / PER;
    constexpr int WSPAN = 32 * EPT;  // elements per warp iteration
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    // A programmatic dependent (the channel-first varlen boundary pass) may start as this grid's
    // CTAs retire; it waits for this grid before writing anything this grid writes.
    allow_dependent_launch();
    const int64_t gw = ((int64_t)blockIdx.x * kCfThreads + threadIdx.x) >> 5;
    const int64_t base = gw * (int64_t)iters * WSPAN;
    if (base >= total) return;  // warp-uniform
    const T* x = (const T*)a.x;
    T* out = (T*)a.out;
    const T* wt = (const T*)a.w;
    const T* bs = (const T*)a.bias;
    const int64_t L = a.L, D = a.D;
    const bool use_silu = a.silu != 0;
    // SiLU on a prescaled accumulator (walk.cuh: exactly half the sums, same outputs).
    const float scale = (prescaled_silu<T>() && use_silu) ? 0.5f : 1.0f;

    int64_t f = base + lane * EPT;
    int64_t row = f / L;
    int64_t t = f - row * L;
    int64_t c = row % D;

    float carry[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int64_t p = base - K + k;
        carry[k] = (lane == 0 && p >= 0) ? to_f32<T>(x[p]) : 0.f;
    }
    auto load = [&](int64_t g, uint4 (&v)[NV]) {
        if (g + EPT <= total) {
            if (V32) {
#pragma unroll
                for (int q = 0; q < NV; q += 2) ldg32_stream(x + g + q * PER, v[q], v[q + 1]);
            } else {
#pragma unroll
                for (int q = 0; q < NV; ++q) v[q] = ldg16_stream(x + g + q * PER);
            }
        } else {
#pragma unroll
            for (int q = 0; q < NV; ++q) {
                v[q] = make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int i = 0; i < PER; ++i)
                    if (g + q * PER + i < total) set_lane<T>(v[q], i, x[g + q * PER + i]);
            }
        }
    };
    uint4 cur[NV];
    load(f, cur);
    int64_t wc = -1;
    float w0[W], b0 = 0.f;
    for (int it = 0; it < iters; ++it) {
        f = base + (int64_t)it * WSPAN + lane * EPT;
        uint4 nxt[NV];
        if (it + 1 < iters) load(f + WSPAN, nxt);
        float xv[EPT];
#pragma unroll
        for (int q = 0; q < NV; ++q) unpack16<T>(cur[q], xv + q * PER);
        float win[K + EPT];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const float up = __shfl_up_sync(FULL, xv[EPT - K + k], 1);
            const float last = __shfl_sync(FULL, xv[EPT - K + k], 31);
            win[k] = lane == 0 ? carry[k] : up;
            carry[k] = last;
        }
#pragma unroll
        for (int e = 0; e < EPT; ++e) win[K + e] = xv[e];
        const bool full = f + EPT <= total;
        if (f < total) {
            if (c != wc) {
                load_filter1<T, W>(wt, a.w_sd, a.w_sk, bs, a.bias_s, c, w0, b0);
#pragma unroll
                for (int k = 0; k < W; ++k) w0[k] *= scale;
                b0 *= scale;
                wc = c;
            }
            float o[EPT];
            if (full && t + EPT <= L) {
                // Fast path: the elements lie in one row. At a row start (t < W-1) the window
                // entries before the row are zeroed, which is the slow path's causal padding (a
                // zero tap still goes through the same fused multiply-add, so the bits agree).
                if (t < K) {
#pragma unroll
                    for (int i = 0; i < K; ++i)
                        if (i < K - t) win[i] = 0.f;
                }
#pragma unroll
                for (int e = 0; e < EPT; ++e) {
                    float acc = b0;
#pragma unroll
                    for (int k = 0; k < W; ++k) acc = fmaf(win[e + k], w0[k], acc);
                    o[e] = activate_prescaled<T>(acc, use_silu);
                }
                if (V32) {
#pragma unroll
                    for (int q = 0; q < NV; q += 2)
                        st32_stream(out + f + q * PER, pack16<T>(o + q * PER),
                                    pack16<T>(o + (q + 1) * PER));
                } else {
#pragma unroll
                    for (int q = 0; q < NV; ++q)
                        st16_stream(out + f + q * PER, pack16<T>(o + q * PER));
                }
            } else {
                float w1[W], b1 = 0.f;
                const bool straddle = t + EPT > L;
                if (straddle) {
                    const int64_t c1 = (c + 1 == D) ? 0 : c + 1;
                    load_filter1<T, W>(wt, a.w_sd, a.w_sk, bs, a.bias_s, c1, w1, b1);
#pragma unroll
                    for (int k = 0; k < W; ++k) w1[k] *= scale;
                    b1 *= scale;
                }
#pragma unroll
                for (int e = 0; e < EPT; ++e) {
                    const bool second = straddle && (t + e >= L);
                    const int64_t te = second ? t + e - L : t + e;
                    float acc = second ? b1 : b0;
#pragma unroll
                    for (int k = 0; k < W; ++k) {
                        const float v = (te >= K - k) ? win[e + k] : 0.f;
                        acc = fmaf(v, second ? w1[k] : w0[k], acc);
                    }
                    o[e] = activate_prescaled<T>(acc, use_silu);
                }
                if (full) {
#pragma unroll
                    for (int q = 0; q < NV; ++q)
                        st16_stream(out + f + q * PER, pack16<T>(o + q * PER));
                } else {
#pragma unroll
                    for (int e = 0; e < EPT; ++e)
                        if (f + e < total) out[f + e] = from_f32<T>(o[e]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < NV; ++q) cur[q] = nxt[q];
        // Advance this lane by one warp stride.
        if (L >= WSPAN) {
            t += WSPAN;
            if (t >= L) {
                t -= L;
                c = (c + 1 == D) ? 0 : c + 1;
            }
        } else {
            const int64_t f2 = f + WSPAN;
            row = f2 / L;
            t = f2 - row * L;
            c = row % D;
        }
    }
}

template <typename T, int W>
__global__ void __launch_bounds__(kGenThreads)
    fwd_generic_kernel(const FwdArgs a, int strip, int nstrips) {
    constexpr int K = W - 1;
    const int64_t n = a.B * a.D * nstrips;
    const T* x = (const T*)a.x;
    T* out = (T*)a.out;
    const bool use_silu = a.silu != 0;
    for (int64_t idx = (int64_t)blockIdx.x * kGenThreads + threadIdx.x; idx < n;
         idx += (int64_t)gridDim.x * kGenThreads) {
        const int64_t c = idx % a.D;
        const int64_t r = idx / a.D;
        const int64_t s = r % nstrips;
        const int64_t b = r / nstrips;
        float w[W], bb;
        load_filter1<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c, w, bb);
        const int64_t t0 = s * strip;
        const int64_t t1 = min(t0 + strip, a.L);
        const T* xr = x + b * a.x_sb + c * a.x_sd;
        T* orow = out + b * a.o_sb + c * a.o_sd;
        float h[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int64_t t = t0 - K + k;
            h[k] = t >= 0 ? to_f32<T>(xr[t * a.x_sl]) : 0.f;
        }
        for (int64_t t = t0; t < t1; ++t) {
            const float xv = to_f32<T>(xr[t * a.x_sl]);
            float acc = bb;
#pragma unroll
            for (int k = 0; k < K; ++k) acc = fmaf(h[k], w[k], acc);
            acc = fmaf(xv, w[K], acc);
            orow[t * a.o_sl] = from_f32<T>(activate<T>(acc, use_silu));
#pragma unroll
            for (int k = 0; k + 1 < K; ++k) h[k] = h[k + 1];
            h[K - 1] = xv;
        }
    }
}

// Launch table for the channel-last walk: strips (one CTA row per (batch, strip of at most
// kStripRows tokens), scheduled by the hardware in several waves) or balanced shares (one wave of
// resident CTAs, equal work each). Measured on B200 (bf16, 64-thread CTAs), strips / balanced:
//   shape (B x L x D)        W = 2              W = 4              W = 8
//   8 x 4096 x 8192     182.5 / 196.6 us   193.3 / 190.4 us   251.1 / 224.5 us
//   4 x 2048 x 8192      53.8 /  55.8 us    67.7 /  59.1 us    76.4 /  71.5 us
//   3 x 1000 x 2304      22.6 /  16.5 us    24.5 /  14.5 us    30.6 /  20.5 us
//   64 x 128 x 4096      33.0 /  33.7 us    33.8 /  35.7 us    38.9 /  44.9 us
// (L2 flushed between launches.) Strips win for W <= 3 (the lightest walks, where the scheduler's
// dynamic balancing across SMs is worth more than a strip restart; W = 3 at the config-2 shape:
// 178.0 vs 199.1 us) and for short sequences (a share would restart its walk at every sequence),
// as long as they give at least half a wave of CTAs; otherwise balanced shares.
constexpr int64_t kStripRows = 128;
constexpr int64_t kMinShareRows = 16;

// Launch table of the balanced walk: bytes of channels per thread (NB), rows in flight per thread
// (U), CTA size and minimum resident CTAs per SM in the launch bounds (0: the compiler's own
// register budget). With 16-byte vectors (8 bf16 channels per thread) the filter and window of a
// wide filter take most of the registers: at W = 8 the walk needed 234 registers, so only 8 warps
// per SM held loads in flight. From W = 5, 16-bit types use 8-byte vectors (4 channels per
// thread) with 16 rows in flight. Measured on B200 at the config-2 shape, one launch at a time
// (16-byte / 8-byte vectors, us): W = 4: 182.0 / 183.9; 5: 188.0 / 184.4 (128-thread CTAs);
// 6: 204.9 / 185.7 (minimum 6 CTAs); 8: 210.2 / 196.2. Earlier 16-byte measurements (W: U = 8
// with the compiler's budget / U = 8 with minimum 1 / U = 6 with minimum 1): 4: 182.6 / 196.2 /
// 183.1; 5: 200.5 / 197.4 / 184.4; 6: 204.6 / 201.6 / 218.7; 7: 206.1 / 202.1 / 219.3;
// 8: 217.9 / 207.7 / 227.0. fp32 keeps 16-byte vectors, which hold 4 channels already.
template <typename T, int W>
constexpr int share_bytes() {
    return sizeof(T) == 2 && W >= 5 ? 8 : 16;
}
template <typename T, int W>
constexpr int share_rows() {
    return share_bytes<T, W>() == 8 ? 16 : (W == 5 ? 6 : 8);
}
template <typename T, int W>
constexpr int share_threads() {
    return share_bytes<T, W>() == 8 && W == 5 ? 128 : 64;
}
template <typename T, int W>
constexpr int share_min_ctas() {
    if (share_bytes<T, W>() == 8) return W == 6 ? 6 : 1;
    return W >= 5 ? 1 : 0;
}

// Elements per lane of the flat-stream kernel. 32 (four 16-byte vectors, 123-128 registers, two
// CTAs per SM) halves the warp-shuffle halo and loop overhead per element against 16 (64-88
// registers, three CTAs per SM). Measured on B200, bf16, 8192 channels, 16 -> 32 elements (us):
// (8, 4096): W = 3: 220.2 -> 215.7 (1 x 40807), W = 4: 179.9 -> 175.5, W = 8: 193.5 -> 181.8
// (204.0 before the prescaled SiLU), W = 2: 179.5 -> 174.8, W = 5: 184.6 -> 177.1, W = 6:
// 186.8 -> 178.2; (1, 40807): W = 2: 220.5 -> 214.4, W = 4: 221.7 -> 216.9, W = 8: 238.8 ->
// 225.6. W = 7 lost (189.5 -> 230.7) and keeps 16; W = 2 at 32 elements needs the cap of two
// CTAs per SM (three: 197.8). Packed fp32x2 FMAs (__ffma2_rn, elements e and e + EPT/2 paired)
// were slower at every width (W = 8, (8, 4096): 220.7 us at 16 elements) for their registers.
template <typename T, int W>
constexpr int cf_elems_per_lane() {
    return sizeof(T) == 2 && W != 7 ? 32 : 16;
}

template <typename T, int W, int EPT>
cudaError_t launch_channel_first(const FwdArgs& a, cudaStream_t stream) {
    const int64_t total = a.B * a.D * a.L;
    const int64_t chunks = ceil_div(total, 32 * EPT);  // one warp iteration each
    // One wave: every resident warp walks an equal run of chunks (measured on B200 at the
    // config-2 sizes, 16 elements per lane: 8 chunks per warp 196.5 us, 16: 189.8, 32: 188.1, one
    // wave: 187.4). 32-byte accesses when both streams are 32-byte aligned (a lane's elements are).
    const bool v32 = host_aligned32(a.x) && host_aligned32(a.out);
    auto kern = v32 ? fwd_channel_first_kernel<T, W, true, EPT>
                    : fwd_channel_first_kernel<T, W, false, EPT>;
    static int slot_cache[2][kSlotCacheDevices] = {};
    int64_t slots = std::max(1, device_slots((const void*)kern, kCfThreads, slot_cache[v32]));
    // At most 3 resident CTAs per SM (the 16-bit kernels for W <= 4 at 16 elements fit 4).
    // Measured on B200 (bf16, W = 4, 8192 channels, 16 elements; 4 -> 3 CTAs per SM, us):
    // B x L = 1 x 20000: 126.8 -> 113.5; 1 x 40807: 243.6 -> 221.4; 1 x 65536: 381.5 -> 345.9;
    // 8 x 4096: 199.1 -> 179.6; 4 x 8192: 198.7 -> 179.1; 16 x 2048: 193.5 -> 179.2;
    // 2 x 16384: 197.2 -> 178.0; 8 x 7000: 314.8 -> 302.2; 6 x 5000: 165.8 -> 169.7 (the one
    // shape of 14 that lost).
    // With 32 elements per lane, at most 2 (the occupancy of every width but W = 2 anyway).
    const int64_t cap = EPT == 32 ? 2 : 3;
    const int sms = device_sm_count();
    if (sms > 0 && slots > cap * sms) slots = cap * sms;
    const int64_t wave_warps = slots * (kCfThreads / 32);
    const int iters = (int)std::max<int64_t>(1, ceil_div(chunks, wave_warps));
    const int64_t warps = ceil_div(chunks, iters);
    const int64_t blocks = ceil_div(warps * 32, kCfThreads);
    kern<<<(unsigned)blocks, kCfThreads, 0, stream>>>(a, total, iters);
    return cudaGetLastError();
}

template <typename T, int W>
cudaError_t run_fwd(const FwdArgs& a, cudaStream_t stream) {
    constexpr int V = Vec<T>::V;
    const int64_t e = sizeof(T);
    const bool wvec = a.w_sd == W && a.w_sk == 1 && host_aligned16(a.w);
    const bool bvec = a.bias != nullptr && a.bias_s == 1 && host_aligned16(a.bias);
    const bool cl = a.x_sd == 1 && a.o_sd == 1 && a.D % V == 0 && host_aligned16(a.x) &&
                    host_aligned16(a.out) && (a.x_sl * e) % 16 == 0 && (a.o_sl * e) % 16 == 0 &&
                    (a.x_sb * e) % 16 == 0 && (a.o_sb * e) % 16 == 0;
    if (cl) {
        const int64_t nvec = a.D / V;
        if constexpr (staged_prefill<T, W>()) {
            constexpr int S = stage_rows<W>();
            const int64_t sgx = ceil_div(nvec, (int64_t)kStageThreads);
            const int64_t blocks = sgx * a.B * ceil_div(a.L, (int64_t)S);
            if (wvec && (a.bias == nullptr || bvec) && blocks <= 0x7fffffffLL)
                return a.silu ? launch_staged<T, W, S, true>(a, sgx, stream)
                              : launch_staged<T, W, S, false>(a, sgx, stream);
        }
        const int64_t gx = ceil_div(nvec, (int64_t)kClThreads);
        constexpr int SB = share_bytes<T, W>();
        constexpr int SNT = share_threads<T, W>();
        const int64_t sgx = ceil_div(a.D / (SB / (int64_t)sizeof(T)), (int64_t)SNT);
        static int slot_cache[kSlotCacheDevices] = {};
        auto share = fwd_channel_last_share_kernel<T, W, share_rows<T, W>(), true, SNT,
                                                   share_min_ctas<T, W>(), SB>;
        const int64_t slots = device_slots((const void*)share, SNT, slot_cache);
        const int64_t strip = std::max<int64_t>(1, std::min<int64_t>(a.L, kStripRows));
        const int64_t nstrips = ceil_div(a.L, strip);
        if ((W <= 3 || a.L <= kStripRows) && a.B * nstrips * gx * 2 >= slots) {
            dim3 grid((unsigned)gx, (unsigned)std::min<int64_t>(a.B * nstrips, 65535));
            fwd_channel_last_kernel<T, W, 8, true, kClThreads>
                <<<grid, kClThreads, 0, stream>>>(a, (int)strip, (int)nstrips, wvec, bvec);
            return cudaGetLastError();
        }
        const int64_t gy = std::max<int64_t>(
            1, std::min<int64_t>({std::max<int64_t>(slots, 1) / sgx,
                                  ceil_div(a.B * a.L, kMinShareRows), 65535}));
        share<<<dim3((unsigned)sgx, (unsigned)gy), SNT, 0, stream>>>(a, wvec, bvec);
        return cudaGetLastError();
    }
    const bool rows_dense = a.x_sl == 1 && a.o_sl == 1 && a.x_sd == a.L && a.o_sd == a.L &&
                            (a.B == 1 || (a.x_sb == a.D * a.L && a.o_sb == a.D * a.L));
    if (rows_dense && a.L >= 16 && host_aligned16(a.x) && host_aligned16(a.out)) {
        // 32 elements per lane for 16-bit types on rows of 32+ elements (cf_elems_per_lane),
        // else 16.
        if (cf_elems_per_lane<T, W>() == 32 && a.L >= 32)
            return launch_channel_first<T, W, cf_elems_per_lane<T, W>()>(a, stream);
        return launch_channel_first<T, W, 16>(a, stream);
    }
    const int strip = 64;
    const int nstrips = (int)ceil_div(a.L, strip);
    const int64_t n = a.B * a.D * nstrips;
    const int64_t blocks = std::min<int64_t>(ceil_div(n, kGenThreads), 148 * 64);
    fwd_generic_kernel<T, W><<<(unsigned)blocks, kGenThreads, 0, stream>>>(a, strip, nstrips);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_fwd(const FwdArgs& a, int width, int dtype, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    CC1D_DISPATCH_DTYPE(dtype, CC1D_DISPATCH_WIDTH(width, err = (run_fwd<T, kW>(a, stream))));
    return err;
}

}  // namespace cc1d
