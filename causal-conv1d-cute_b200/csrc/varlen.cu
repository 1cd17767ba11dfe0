// Packed variable-length prefill in one launch (replaces the strip walk + ConvSeqBoundary /
// ConvSeqBoundaryVec pair of causal_conv1d_cute/varlen.py, which needs two launches for more
// than one sequence).
//
// The packed stream of T tokens is cut into strips of S tokens; a thread owns one strip of one
// channel group. Sequence bounds come from query_start_loc on the device (binary search for the
// strip start, then a walk), so the call needs no host synchronisation.
//
// Ownership. The first W-1 outputs of a sequence depend on its initial state, and its final
// state is written into the same cache slot. Both belong to the thread whose strip holds the
// sequence's first token (its "owner"): it reads the initial state, computes the head outputs
// (running past its strip end when the sequence starts in the last W-2 tokens of the strip),
// then writes the final state. Every other strip of the sequence starts W-1 tokens after the
// sequence start at the earliest and reads only the sequence's own inputs. No slot is read by one
// thread and written by another, so one launch suffices.
//
// The final state is the last W-1 inputs of [initial state | sequence]; it is copied as raw bits
// from x (or from the initial state when the sequence is shorter than W-1 tokens).
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "seq.cuh"
#include "walk.cuh"

namespace cc1d {

namespace {

constexpr int kVarThreads = 64;
constexpr int kBoundaryThreads = 128;
constexpr int kGenThreads = 256;

// ---------------------------------------------------------------------------------------------
// Token-major: x rows of D adjacent channels, x_st elements apart
// ---------------------------------------------------------------------------------------------

// Owner work of sequence s for one channel group: read the initial state (zeros without one),
// write the final state (the last W-1 inputs of [initial state | sequence], as raw bits) and leave
// the initial state in the fp32 window h. The final state is written before the walk, so the
// raw initial state does not stay live across it.
template <typename T, int W, int NB>
__device__ __forceinline__ void owner_state(const VarArgs& a, const T* xb, int64_t c0, int64_t s,
                                            int64_t bos, int64_t eos, bool report,
                                            float (&h)[W - 1][NB / sizeof(T)]) {
    constexpr int V = NB / (int)sizeof(T);
    constexpr int K = W - 1;
    using R = typename RawVec<NB>::type;
    if (report) check_bounds(a, s);
    const SeqSlot ss = seq_slot(a, s, report);
    T* sp = ss.live ? (T*)a.states + ss.slot * a.s_slot + c0 * K : nullptr;
    R init[K];
    if (ss.use_init) {
        R blk[K];
#pragma unroll
        for (int q = 0; q < K; ++q) blk[q] = ld_raw<NB>(sp + q * V);
#pragma unroll
        for (int ee = 0; ee < V; ++ee)
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int flat = ee * K + k;
                set_lane<T>(init[k], ee, lane_of<T>(blk[flat / V], flat % V));
            }
    } else {
#pragma unroll
        for (int k = 0; k < K; ++k) init[k] = R{};
    }
#pragma unroll
    for (int k = 0; k < K; ++k) unpack_raw<T, NB>(init[k], h[k]);
    if (!ss.live) return;
    const int64_t n = eos - bos;
    R fin[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int64_t pos = eos - K + k;
        if (pos >= bos) {
            fin[k] = ldg_raw<NB>(xb + pos * a.x_st);
        } else {
            // n < K: entry k + n of the initial state.
            const int64_t m = k + n;
            R v = init[0];
#pragma unroll
            for (int q = 1; q < K; ++q) v = (m == q) ? init[q] : v;
            fin[k] = v;
        }
    }
    R blk[K];
#pragma unroll
    for (int q = 0; q < K; ++q)
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int flat = q * V + i;
            set_lane<T>(blk[q], i, lane_of<T>(fin[flat % K], flat / K));
        }
#pragma unroll
    for (int q = 0; q < K; ++q) st_raw<NB>(sp + q * V, blk[q]);
}

// NB: bytes of channels per thread (16, or 8 for wide filters; see the launch table).
template <typename T, int W, int U, bool PF, int NT, int MINB, int NB>
__global__ void __launch_bounds__(NT, MINB)
    varlen_token_major_kernel(const VarArgs a, bool wvec, bool bvec) {
    constexpr int V = NB / (int)sizeof(T);
    constexpr int K = W - 1;
    const int64_t nvec = a.D / V;
    const int64_t j = (int64_t)blockIdx.x * NT + threadIdx.x;
    if (j >= nvec) return;
    const int64_t c0 = j * V;
    float w[W][V], bv[V];
    load_filter<T, W, NB>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c0, wvec,
                          bvec, w, bv);
    const bool use_silu = a.silu != 0;
    prescale_filter<T, W, NB>(w, bv, use_silu);
    const T* xb = (const T*)a.x + c0;
    T* ob = (T*)a.out + c0;
    // This CTA's share of the packed tokens: [t0, t1), one of gridDim.y equal parts.
    {
        const int64_t t0 = a.T * blockIdx.y / gridDim.y;
        const int64_t t1 = a.T * (blockIdx.y + 1) / gridDim.y;
        int64_t s = seq_of(a, t0);
        int64_t t = t0;
        if (s < 0) {
            t = min(t1, qsl_at(a, 0));
            s = 0;
        }
        while (t < t1 && s < a.nseq) {
            const int64_t bos = qsl_at(a, s);
            const int64_t eos = max(qsl_at(a, s + 1), bos);
            if (eos <= t) {
                ++s;
                continue;
            }
            const int64_t e = min(t1, eos);
            float h[K][V];
            int64_t ta, tb;
            if (t == bos) {
                // Owner of sequence s: initial state in, final state out, then the walk starts
                // at the sequence start and runs past the strip end over the first W-1 tokens.
                owner_state<T, W, NB>(a, xb, c0, s, bos, eos, j == 0, h);
                ta = bos;
                tb = min(eos, max(e, bos + K));
            } else {
                // Tokens less than W-1 after the sequence start belong to its owner.
                ta = max(t, bos + K);
                tb = e;
                if (ta < tb) load_halo<T, W, NB>(xb, a.x_st, ta, h);  // rows >= bos
            }
            if (ta < tb)
                walk_strip<T, W, U, PF, NB>(xb, a.x_st, ob, a.o_st, ta, tb, h, w, bv, use_silu);
            t = e;
            if (e == eos) ++s;
        }
    }
}

// Staged form for 16-bit types (as the plain channel-last prefill, fwd.cu): one CTA
// per strip of S packed tokens and NT channel vectors, the strip and the W-1 rows before it landed
// in shared memory by cp.async (stage_strip), walked in channel pairs (conv_step_x2); contiguous
// weights and bias (the host sends other layouts to the register walk). The sequence search for
// the strip start runs while
// the rows land. A strip that lies inside one sequence at least W-1 tokens after its start (all
// but the few strips at sequence starts) walks its S rows with no per-row guard. Any other strip
// takes the ownership rules of the register walk above: the thread whose strip holds a sequence's
// first token reads its initial state, writes its final state and computes its first W-1 outputs
// (reading the rows past the strip end from global memory), so no cache slot is read by one CTA
// and written by another.
template <typename T, int W, int S, int NT, bool SILU>
__global__ void __launch_bounds__(NT)
    varlen_staged_kernel(const VarArgs a, int64_t gx) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
    constexpr int HALF = S / 2;
    extern __shared__ uint4 stage[];
    const int64_t blk = blockIdx.x;
    const int64_t su = blk / gx;
    const int64_t j = (blk - su * gx) * NT + threadIdx.x;
    if (j >= a.D / V) return;
    const int64_t c0 = j * V;
    const int64_t t0 = su * S;
    const int64_t t1 = min(t0 + S, a.T);
    const int64_t n = t1 - t0;
    const T* xb = (const T*)a.x + c0;
    T* ob = (T*)a.out + c0;
    uint4* col = stage + threadIdx.x;  // row t at col[(t - t0 + K) * NT]
    if (n == S) stage_strip<T, K, S, NT, true>(col, xb, a.x_st, t0, n);
    else stage_strip<T, K, S, NT, false>(col, xb, a.x_st, t0, n);
    const int64_t s0 = seq_of(a, t0);
    Pairs w2[W], b2;
    {
        float w[W][V], bv[V];
        load_filter<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c0, true,
                          true, w, bv);
        prescale_filter<T, W>(w, bv, SILU);
        filter_pairs<W>(w, bv, w2, b2);
    }
    Pairs h[K];
    auto emit = [&](const uint4& r, int64_t t) {
        const Pairs o = conv_step_x2<W, SILU>(h, to_pairs<T>(r), w2, b2);
        st16_stream(ob + t * a.o_st, from_pairs<T>(o));
    };
    auto staged = [&](int64_t t) -> const uint4& { return col[(t - t0 + K) * NT]; };
    if (n == S && s0 >= 0 && s0 < a.nseq && qsl_at(a, s0) + K <= t0 && qsl_at(a, s0 + 1) >= t1) {
        // The whole strip continues one sequence: history from the staged rows before it.
        cp_async_wait<1>();
#pragma unroll
        for (int k = 0; k < K; ++k) h[k] = to_pairs<T>(col[k * NT]);
#pragma unroll
        for (int r = 0; r < HALF; ++r) emit(col[(K + r) * NT], t0 + r);
        cp_async_wait<0>();
#pragma unroll
        for (int r = HALF; r < S; ++r) emit(col[(K + r) * NT], t0 + r);
        return;
    }
    cp_async_wait<0>();
    int64_t s = s0;
    int64_t t = t0;
    if (s < 0) {
        t = min(t1, qsl_at(a, 0));
        s = 0;
    }
    while (t < t1 && s < a.nseq) {
        const int64_t bos = qsl_at(a, s);
        const int64_t eos = max(qsl_at(a, s + 1), bos);
        if (eos <= t) {
            ++s;
            continue;
        }
        const int64_t e = min(t1, eos);
        int64_t ta, tb;
        if (t == bos) {
            float hf[K][V];
            owner_state<T, W, 16>(a, xb, c0, s, bos, eos, j == 0, hf);
#pragma unroll
            for (int k = 0; k < K; ++k)
#pragma unroll
                for (int q = 0; q < kPairs; ++q) h[k].p[q] = make_float2(hf[k][2 * q], hf[k][2 * q + 1]);
            ta = bos;
            tb = min(eos, max(e, bos + K));
        } else {
            ta = max(t, bos + K);
            tb = e;
            if (ta < tb) {
#pragma unroll
                for (int k = 0; k < K; ++k) h[k] = to_pairs<T>(staged(ta - K + k));
            }
        }
        for (int64_t u = ta; u < tb; ++u)
            emit(u < t1 ? staged(u) : ldg16(xb + u * a.x_st), u);
        t = e;
        if (e == eos) ++s;
    }
}

// ---------------------------------------------------------------------------------------------
// Channel-first: x is contiguous (D, T), one packed stream per channel. The bulk pass is the
// channel-first prefill of a (1, D, T) batch (launch_fwd): it computes every output as if each
// channel row were one sequence, so every output whose W-1 predecessors lie in its own sequence is
// final. The others are the first W-1 outputs of each sequence, which a second, small launch with
// one thread per (channel, sequence) pair (varlen_boundary_kernel) recomputes from the initial
// state and overwrites, stream order placing it after the bulk pass; and outputs of tokens outside
// every sequence, which are undefined. The boundary launch also reads and writes the cache, which
// the bulk pass never touches. Tracking sequence bounds inside the stream pass instead cost a
// quarter of its time at the config-5 shape: with 1.3k-token sequences, 40 % of the 512-token warp
// steps meet a boundary and diverge into masked stores.
// ---------------------------------------------------------------------------------------------

// Owner work of sequence s in channel c of a contiguous (D, T) stream: initial state in, final
// state out, and the first W-1 outputs. Every load (inputs at both ends of the sequence, filter,
// initial state) is issued before the first store, so a thread waits for memory once rather than
// once per element (the compiler cannot move a load of x above a store to out by itself).
template <typename T, int W>
__device__ __forceinline__ void owner_channel(const VarArgs& a, int64_t c, int64_t s) {
    constexpr int K = W - 1;
    const int64_t bos = qsl_at(a, s);
    const int64_t eos = max(qsl_at(a, s + 1), bos);
    const int64_t n = eos - bos;
    if (c == 0) check_bounds(a, s);
    const SeqSlot ss = seq_slot(a, s, c == 0);
    const T* xr = (const T*)a.x + c * a.T;
    T* orow = (T*)a.out + c * a.T;
    T* sp = ss.live ? (T*)a.states + ss.slot * a.s_slot + c * a.s_sd : nullptr;
    T head[K], tail[K], init[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
        head[k] = k < n ? __ldg(xr + bos + k) : from_f32<T>(0.f);
        const int64_t pos = eos - K + k;
        tail[k] = pos >= bos ? __ldg(xr + pos) : from_f32<T>(0.f);
        init[k] = ss.use_init ? sp[k * a.s_sk] : from_f32<T>(0.f);
    }
    float wf[W], bf;
    load_filter1<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c, wf, bf);
    const bool use_silu = a.silu != 0;
    float h[K];
#pragma unroll
    for (int k = 0; k < K; ++k) h[k] = to_f32<T>(init[k]);
    T o[K];
#pragma unroll
    for (int j = 0; j < K; ++j) {
        const float xv = to_f32<T>(head[j]);
        float acc = bf;
#pragma unroll
        for (int k = 0; k < K; ++k) acc = fmaf(h[k], wf[k], acc);
        acc = fmaf(xv, wf[K], acc);
        o[j] = from_f32<T>(activate<T>(acc, use_silu));
#pragma unroll
        for (int k = 0; k + 1 < K; ++k) h[k] = h[k + 1];
        h[K - 1] = xv;
    }
    if (ss.live) {
        // The last K inputs of [initial state | sequence]: entry k is x[eos - K + k] when that
        // lies in the sequence, else initial-state entry k + n.
#pragma unroll
        for (int k = 0; k < K; ++k) {
            T v = tail[k];
            if (eos - K + k < bos) {
                const int64_t m = k + n;
#pragma unroll
                for (int q = 0; q < K; ++q) v = (m == q) ? init[q] : v;
            }
            sp[k * a.s_sk] = v;
        }
    }
    // The head outputs replace the bulk pass's values, so they wait for it; everything above
    // (reads of x and of the cache, the final state) is independent of the bulk pass.
    grid_dependency_wait();
#pragma unroll
    for (int j = 0; j < K; ++j)
        if (j < n) orow[bos + j] = o[j];
}

// Second launch of the channel-first path: one thread per (channel, sequence) does the owner work
// (initial state in, final state out, first W-1 outputs, which replace the bulk pass's values).
// It is launched as a programmatic dependent of the bulk pass: its CTAs start as the bulk pass's
// CTAs retire, issue their loads and write the final states at once, and wait for the bulk pass
// only before writing the head outputs (owner_channel).
template <typename T, int W>
__global__ void __launch_bounds__(kBoundaryThreads) varlen_boundary_kernel(const VarArgs a) {
    const int64_t c = (int64_t)blockIdx.x * kBoundaryThreads + threadIdx.x;
    const int64_t s = blockIdx.y;
    if (c >= a.D || qsl_at(a, s + 1) <= qsl_at(a, s)) return;
    owner_channel<T, W>(a, c, s);
}

// ---------------------------------------------------------------------------------------------
// Any strides: one channel per thread, same ownership rules.
// ---------------------------------------------------------------------------------------------

template <typename T, int W>
__global__ void __launch_bounds__(kGenThreads) varlen_generic_kernel(const VarArgs a, int strip) {
    constexpr int K = W - 1;
    const int64_t nstrips = ceil_div(a.T, strip);
    const int64_t n = nstrips * a.D;
    const bool use_silu = a.silu != 0;
    const T* x = (const T*)a.x;
    T* out = (T*)a.out;
    for (int64_t id = (int64_t)blockIdx.x * kGenThreads + threadIdx.x; id < n;
         id += (int64_t)gridDim.x * kGenThreads) {
        const int64_t c = id % a.D;
        const int64_t u = id / a.D;
        float w[W], bb;
        load_filter1<T, W>((const T*)a.w, a.w_sd, a.w_sk, (const T*)a.bias, a.bias_s, c, w, bb);
        const T* xr = x + c * a.x_sd;
        T* orow = out + c * a.o_sd;
        auto walk = [&](int64_t ta, int64_t tb, float (&h)[K]) {
            for (int64_t t = ta; t < tb; ++t) {
                const float xv = to_f32<T>(xr[t * a.x_st]);
                float acc = bb;
#pragma unroll
                for (int k = 0; k < K; ++k) acc = fmaf(h[k], w[k], acc);
                acc = fmaf(xv, w[K], acc);
                orow[t * a.o_st] = from_f32<T>(activate<T>(acc, use_silu));
#pragma unroll
                for (int k = 0; k + 1 < K; ++k) h[k] = h[k + 1];
                h[K - 1] = xv;
            }
        };
        const int64_t t0 = u * strip;
        const int64_t t1 = min(t0 + strip, a.T);
        int64_t s = seq_of(a, t0);
        int64_t t = t0;
        if (s < 0) {
            t = min(t1, qsl_at(a, 0));
            s = 0;
        }
        while (t < t1 && s < a.nseq) {
            const int64_t bos = qsl_at(a, s);
            const int64_t eos = max(qsl_at(a, s + 1), bos);
            if (eos <= t) {
                ++s;
                continue;
            }
            const int64_t e = min(t1, eos);
            float h[K];
            if (t == bos) {
                if (c == 0) check_bounds(a, s);
                const SeqSlot ss = seq_slot(a, s, c == 0);
                T* sp = ss.live ? (T*)a.states + ss.slot * a.s_slot + c * a.s_sd : nullptr;
                T init[K];
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    init[k] = ss.use_init ? sp[k * a.s_sk] : from_f32<T>(0.f);
                    h[k] = to_f32<T>(init[k]);
                }
                walk(bos, min(eos, max(e, bos + K)), h);
                if (ss.live) {
                    const int64_t nn = eos - bos;
#pragma unroll
                    for (int k = 0; k < K; ++k) {
                        const int64_t pos = eos - K + k;
                        T v;
                        if (pos >= bos) {
                            v = xr[pos * a.x_st];
                        } else {
                            const int64_t m = k + nn;
                            v = init[0];
#pragma unroll
                            for (int q = 1; q < K; ++q) v = (m == q) ? init[q] : v;
                        }
                        sp[k * a.s_sk] = v;
                    }
                }
            } else {
                const int64_t start = max(t, bos + K);
                if (start < e) {
#pragma unroll
                    for (int k = 0; k < K; ++k) h[k] = to_f32<T>(xr[(start - K + k) * a.x_st]);
                    walk(start, e, h);
                }
            }
            t = e;
            if (e == eos) ++s;
        }
    }
}

// Token shares of the token-major walk, as for the channel-last prefill (fwd.cu): strips of at most
// kStripTokens tokens for W = 2, else one balanced wave of resident CTAs. Measured on B200 with the
// config-5 batch (32 lognormal sequences, 40807 tokens x 8192 channels, bf16):
//   width                       2          3          4          8
//   128-token strips         219.9 us   248 us     232.2 us   304.6 us
//   one balanced wave        232.2 us   225.6 us   230.5 us   258.4 us
// From W = 3 on a share saves the per-strip halo, owner and sequence-search work that grows with W.
constexpr int64_t kStripTokens = 128;
constexpr int64_t kMinShareTokens = 16;

// Launch table of the token-major walk: bytes of channels per thread (NB), rows in flight per
// thread (U), CTA size and minimum resident CTAs per SM in the launch bounds (0: the compiler's own
// register budget). As in the channel-last prefill, 16-bit types switch to 8-byte vectors
// (4 channels per thread, 16 rows in flight) from W = 5, where the filter and window of 8 channels
// left too few warps per SM. Earlier 16-byte measurements on B200 with the config-5 batch, one
// balanced wave (W: us with U = 8 / U = 6, minimum 1 CTA; U = 6 with minimum 6 CTAs):
// 4: 230.4 / 231.2; 5: 244.6 / 231.1; 6: 248.3 / 268.0, 236.2 with minimum 6; 8: 256.1 / 278.3.
template <typename T, int W>
constexpr int var_bytes() {
    return sizeof(T) == 2 && W >= 5 ? 8 : 16;
}
template <typename T, int W>
constexpr int var_rows() {
    return var_bytes<T, W>() == 8 ? 16 : (W == 5 || W == 6 ? 6 : 8);
}
template <typename T, int W>
constexpr int var_threads() {
    return var_bytes<T, W>() == 8 && W == 5 ? 128 : kVarThreads;
}
template <typename T, int W>
constexpr int var_min_ctas() {
    if (var_bytes<T, W>() == 8) return W == 6 ? 6 : 1;
    return W == 6 ? 6 : 0;
}

template <typename T, int W>
cudaError_t run_varlen(const VarArgs& a, int dtype, cudaStream_t stream) {
    constexpr int V = Vec<T>::V;
    constexpr int K = W - 1;
    const int64_t e = sizeof(T);
    const bool wvec = a.w_sd == W && a.w_sk == 1 && host_aligned16(a.w);
    const bool bvec = a.bias != nullptr && a.bias_s == 1 && host_aligned16(a.bias);
    const bool sok = a.states == nullptr ||
                     (a.s_sk == 1 && a.s_sd == K && host_aligned16(a.states) &&
                      (a.s_slot * e) % 16 == 0);
    const bool tm = a.x_sd == 1 && a.o_sd == 1 && a.D % V == 0 && host_aligned16(a.x) &&
                    host_aligned16(a.out) && (a.x_st * e) % 16 == 0 && (a.o_st * e) % 16 == 0;
    if constexpr (sizeof(T) == 2 && W <= 7) {
        // Staged strips of 16 tokens, one per 64-thread CTA (varlen_staged_kernel), as the plain
        // channel-last prefill, up to W = 7. Measured on B200 with the config-5 batch (bf16, 32
        // sequences, 40807 tokens x 8192 channels), staged (channel pairs, compile-time SiLU) vs
        // the register walk below, us: W = 2: 203.1 vs 217.7; 3: 201.8 vs 223.6; 4: 202.3 vs
        // 226.4; 5: 213.9 vs 235.7; 6: 224.0 vs 238.7; 7: 236.7 vs 239.1; 8 (32-token strips):
        // 243.8-248.7 vs 240.7, so W = 8 keeps the register walk. A minimum of 9-12 resident CTAs
        // in the launch bounds made every width slower (W = 4: 338.5 -> 397 us on a 66k-token
        // batch) by capping registers.
        constexpr int S = 16, NT = 64;
        const int64_t gx = ceil_div(a.D / V, (int64_t)NT);
        const int64_t blocks = gx * ceil_div(a.T, (int64_t)S);
        if (tm && sok && wvec && (a.bias == nullptr || bvec) && blocks <= 0x7fffffffLL) {
            const size_t smem = (size_t)(S + K) * NT * 16;
            auto kern = a.silu ? varlen_staged_kernel<T, W, S, NT, true>
                               : varlen_staged_kernel<T, W, S, NT, false>;
            kern<<<(unsigned)blocks, NT, smem, stream>>>(a, gx);
            return cudaGetLastError();
        }
    }
    if (tm && sok) {
        constexpr int NB = var_bytes<T, W>();
        constexpr int NT = var_threads<T, W>();
        const int64_t gx = ceil_div(a.D / (NB / e), (int64_t)NT);
        static int slot_cache[kSlotCacheDevices] = {};
        auto kern = varlen_token_major_kernel<T, W, var_rows<T, W>(), true, NT,
                                              var_min_ctas<T, W>(), NB>;
        const int64_t slots = device_slots((const void*)kern, NT, slot_cache);
        const int64_t strips = ceil_div(a.T, kStripTokens);
        const int64_t shares = W == 2 && strips * gx * 2 >= slots
                                   ? strips
                                   : std::min<int64_t>(std::max<int64_t>(slots, 1) / gx,
                                                       ceil_div(a.T, kMinShareTokens));
        const int64_t gy = std::max<int64_t>(1, std::min<int64_t>(shares, 65535));
        kern<<<dim3((unsigned)gx, (unsigned)gy), NT, 0, stream>>>(a, wvec, bvec);
        return cudaGetLastError();
    }
    if (a.x_st == 1 && a.o_st == 1 && a.x_sd == a.T && a.o_sd == a.T && a.nseq <= 65535) {
        // Contiguous (D, T): the prefill of one (D, T) batch row, then the boundary pass.
        FwdArgs f{};
        f.x = a.x;
        f.x_sb = a.D * a.T;
        f.x_sd = a.T;
        f.x_sl = 1;
        f.w = a.w;
        f.w_sd = a.w_sd;
        f.w_sk = a.w_sk;
        f.bias = a.bias;
        f.bias_s = a.bias_s;
        f.out = a.out;
        f.o_sb = a.D * a.T;
        f.o_sd = a.T;
        f.o_sl = 1;
        f.B = 1;
        f.D = a.D;
        f.L = a.T;
        f.silu = a.silu;
        cudaError_t err = launch_fwd(f, W, dtype, stream);
        if (err != cudaSuccess) return err;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)ceil_div(a.D, kBoundaryThreads), (unsigned)a.nseq);
        cfg.blockDim = dim3(kBoundaryThreads);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, varlen_boundary_kernel<T, W>, a);
    }
    const int strip = 64;
    const int64_t n = ceil_div(a.T, strip) * a.D;
    const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, kGenThreads), 148 * 32));
    varlen_generic_kernel<T, W><<<(unsigned)blocks, kGenThreads, 0, stream>>>(a, strip);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_varlen(const VarArgs& a, int width, int dtype, cudaStream_t stream) {
    cudaError_t err = cudaErrorInvalidValue;
    CC1D_DISPATCH_DTYPE(dtype, CC1D_DISPATCH_WIDTH(width, err = (run_varlen<T, kW>(a, dtype, stream))));
    return err;
}

}  // namespace cc1d
