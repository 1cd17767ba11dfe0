// extern "C" entry points of libcc1d.so (declared in include/cc1d.h). Each one validates its
// arguments on the host, returns a status code instead of throwing, and enqueues one kernel on
// the caller's stream. Nothing is allocated and nothing is synchronised.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"
#include "kernels.h"

namespace {

thread_local char g_last_error[512] = "";

cc1d_status_t fail(cc1d_status_t code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

cc1d_status_t ok() {
    g_last_error[0] = '\0';
    return CC1D_OK;
}

cc1d_status_t from_cuda(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return ok();
    return fail(CC1D_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

cc1d_status_t check_common(int32_t width, int32_t dtype) {
    if (dtype != CC1D_BF16 && dtype != CC1D_F16 && dtype != CC1D_F32)
        return fail(CC1D_ERR_DTYPE, "dtype %d is not bf16 (0), fp16 (1) or fp32 (2)", dtype);
    if (width < 2 || width > 8) return fail(CC1D_ERR_WIDTH, "kernel width %d is outside 2..8", width);
    return CC1D_OK;
}

// Make the stream's device current on this thread, so a launch from any host thread lands on
// the device that owns the stream (the legacy default stream keeps the current device). While the
// stream is being captured into a CUDA graph the device query is not permitted, and the capturing
// thread already works on the stream's device, so nothing is changed then.
cc1d_status_t bind_stream(void* stream) {
    if (stream == nullptr) return CC1D_OK;
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    cudaError_t err = cudaStreamIsCapturing((cudaStream_t)stream, &capture);
    if (err != cudaSuccess) return from_cuda(err, "cudaStreamIsCapturing");
    if (capture != cudaStreamCaptureStatusNone) return CC1D_OK;
    int dev = -1, cur = -1;
    err = cudaStreamGetDevice((cudaStream_t)stream, &dev);
    if (err != cudaSuccess) return from_cuda(err, "cudaStreamGetDevice");
    err = cudaGetDevice(&cur);
    if (err != cudaSuccess) return from_cuda(err, "cudaGetDevice");
    if (cur != dev) {
        err = cudaSetDevice(dev);
        if (err != cudaSuccess) return from_cuda(err, "cudaSetDevice");
    }
    return CC1D_OK;
}

// Bytes spanned by a (n0, n1, n2) tensor with non-negative element strides.
int64_t span_bytes(int64_t n0, int64_t s0, int64_t n1, int64_t s1, int64_t n2, int64_t s2,
                   int64_t esize) {
    return ((n0 - 1) * s0 + (n1 - 1) * s1 + (n2 - 1) * s2 + 1) * esize;
}

bool overlap(const void* p, int64_t np, const void* q, int64_t nq) {
    const char* a = (const char*)p;
    const char* b = (const char*)q;
    return a < b + nq && b < a + np;
}

}  // namespace

extern "C" {

int32_t cc1d_abi_version(void) { return 1; }

const char* cc1d_status_string(cc1d_status_t code) {
    switch (code) {
        case CC1D_OK: return "ok";
        case CC1D_ERR_INVALID: return "invalid argument";
        case CC1D_ERR_DTYPE: return "unsupported dtype";
        case CC1D_ERR_WIDTH: return "unsupported kernel width";
        case CC1D_ERR_LAYOUT: return "unsupported tensor layout";
        case CC1D_ERR_CUDA: return "CUDA launch failed";
        default: return "unknown status";
    }
}

const char* cc1d_last_error(void) { return g_last_error; }

cc1d_status_t cc1d_fwd(const void* x, int64_t x_sb, int64_t x_sd, int64_t x_sl,
                       const void* weight, int64_t w_sd, int64_t w_sk,
                       const void* bias, int64_t bias_s,
                       void* out, int64_t o_sb, int64_t o_sd, int64_t o_sl,
                       int64_t batch, int64_t dim, int64_t seqlen, int32_t width,
                       int32_t dtype, int32_t silu, void* stream) {
    if (cc1d_status_t s = check_common(width, dtype)) return s;
    if (batch < 0 || dim < 0 || seqlen < 0)
        return fail(CC1D_ERR_INVALID, "negative size (batch %lld, dim %lld, seqlen %lld)",
                    (long long)batch, (long long)dim, (long long)seqlen);
    if (batch == 0 || dim == 0 || seqlen == 0) return ok();
    if (x == nullptr || weight == nullptr || out == nullptr)
        return fail(CC1D_ERR_INVALID, "x, weight and out must not be NULL");
    cc1d::FwdArgs a{x, x_sb, x_sd, x_sl, weight, w_sd, w_sk, bias, bias_s,
                    out, o_sb, o_sd, o_sl, batch, dim, seqlen, silu != 0};
    if (cc1d_status_t s = bind_stream(stream)) return s;
    return from_cuda(cc1d::launch_fwd(a, width, dtype, (cudaStream_t)stream), "cc1d_fwd");
}

cc1d_status_t cc1d_fwd_states(const void* x, int64_t x_sb, int64_t x_sd, int64_t x_sl,
                              const void* weight, int64_t w_sd, int64_t w_sk,
                              const void* bias, int64_t bias_s,
                              void* out, int64_t o_sb, int64_t o_sd, int64_t o_sl,
                              const int32_t* seq_idx, int64_t q_sb, int64_t q_sl,
                              const void* initial_states, int64_t i_sb, int64_t i_sd, int64_t i_sk,
                              void* final_states, int64_t f_sb, int64_t f_sd, int64_t f_sk,
                              int64_t batch, int64_t dim, int64_t seqlen, int32_t width,
                              int32_t dtype, int32_t silu, void* stream) {
    if (cc1d_status_t s = check_common(width, dtype)) return s;
    if (batch < 0 || dim < 0 || seqlen < 0)
        return fail(CC1D_ERR_INVALID, "negative size (batch %lld, dim %lld, seqlen %lld)",
                    (long long)batch, (long long)dim, (long long)seqlen);
    if (seq_idx != nullptr && (initial_states != nullptr || final_states != nullptr))
        return fail(CC1D_ERR_INVALID, "sequence ids exclude initial and final states");
    if (batch == 0 || dim == 0) return ok();
    if (weight == nullptr || (seqlen > 0 && (x == nullptr || out == nullptr)))
        return fail(CC1D_ERR_INVALID, "x, weight and out must not be NULL");
    if (i_sb < 0 || i_sd < 0 || i_sk < 0 || f_sb < 0 || f_sd < 0 || f_sk < 0)
        return fail(CC1D_ERR_LAYOUT, "state strides must not be negative");
    const int64_t e = dtype == CC1D_F32 ? 4 : 2;
    const int64_t K = width - 1;
    if (final_states != nullptr && initial_states != nullptr &&
        overlap(final_states, span_bytes(batch, f_sb, dim, f_sd, K, f_sk, e), initial_states,
                span_bytes(batch, i_sb, dim, i_sd, K, i_sk, e)))
        return fail(CC1D_ERR_INVALID, "final states overlap the initial states");
    cc1d::FwdStateArgs a{{x, x_sb, x_sd, x_sl, weight, w_sd, w_sk, bias, bias_s,
                          out, o_sb, o_sd, o_sl, batch, dim, seqlen, silu != 0},
                         seq_idx, q_sb, q_sl, initial_states, i_sb, i_sd, i_sk,
                         final_states, f_sb, f_sd, f_sk};
    if (seqlen == 0 && final_states == nullptr) return ok();
    if (cc1d_status_t s = bind_stream(stream)) return s;
    return from_cuda(cc1d::launch_fwd_states(a, width, dtype, (cudaStream_t)stream),
                     "cc1d_fwd_states");
}

}  // extern "C"

namespace {

cc1d_status_t ring_convert(bool to_ring, const void* state, int64_t s_slot, int64_t s_sd,
                           int64_t s_sk, const void* ring, int64_t r_slot, int64_t r_sk,
                           int64_t r_sd, const int32_t* cache_seqlens, int64_t slots, int64_t dim,
                           int32_t width, int32_t dtype, void* stream, const char* what) {
    if (cc1d_status_t s = check_common(width, dtype)) return s;
    if (slots < 0 || dim < 0)
        return fail(CC1D_ERR_INVALID, "negative size (slots %lld, dim %lld)", (long long)slots,
                    (long long)dim);
    if (slots == 0 || dim == 0) return ok();
    if (state == nullptr || ring == nullptr || cache_seqlens == nullptr)
        return fail(CC1D_ERR_INVALID, "state, ring and cache_seqlens must not be NULL");
    if (s_slot < 0 || s_sd < 0 || s_sk < 0 || r_slot < 0 || r_sk < 0 || r_sd < 0)
        return fail(CC1D_ERR_LAYOUT, "strides must not be negative");
    const int64_t e = dtype == CC1D_F32 ? 4 : 2;
    const int64_t K = width - 1;
    if (overlap(state, span_bytes(slots, s_slot, dim, s_sd, K, s_sk, e), ring,
                span_bytes(slots, r_slot, K, r_sk, dim, r_sd, e)))
        return fail(CC1D_ERR_INVALID, "the ring and the ordered state overlap");
    cc1d::RingConvArgs a{state, s_slot, s_sd, s_sk, const_cast<void*>(ring), r_slot, r_sk, r_sd,
                         cache_seqlens, slots, dim, to_ring};
    if (cc1d_status_t s = bind_stream(stream)) return s;
    return from_cuda(cc1d::launch_ring_convert(a, width, dtype, (cudaStream_t)stream), what);
}

}  // namespace

extern "C" {

cc1d_status_t cc1d_to_ring(const void* state, int64_t s_slot, int64_t s_sd, int64_t s_sk,
                           void* ring, int64_t r_slot, int64_t r_sk, int64_t r_sd,
                           const int32_t* cache_seqlens, int64_t slots, int64_t dim,
                           int32_t width, int32_t dtype, void* stream) {
    return ring_convert(true, state, s_slot, s_sd, s_sk, ring, r_slot, r_sk, r_sd, cache_seqlens,
                        slots, dim, width, dtype, stream, "cc1d_to_ring");
}

cc1d_status_t cc1d_from_ring(const void* ring, int64_t r_slot, int64_t r_sk, int64_t r_sd,
                             void* state, int64_t s_slot, int64_t s_sd, int64_t s_sk,
                             const int32_t* cache_seqlens, int64_t slots, int64_t dim,
                             int32_t width, int32_t dtype, void* stream) {
    return ring_convert(false, state, s_slot, s_sd, s_sk, ring, r_slot, r_sk, r_sd, cache_seqlens,
                        slots, dim, width, dtype, stream, "cc1d_from_ring");
}

cc1d_status_t cc1d_update(const void* x, int64_t x_sb, int64_t x_sd, int64_t x_st,
                          void* state, int64_t s_slot, int64_t s_sd, int64_t s_sk,
                          int64_t state_len, int64_t nslots,
                          const void* weight, int64_t w_sd, int64_t w_sk,
                          const void* bias, int64_t bias_s,
                          void* out, int64_t o_sb, int64_t o_sd, int64_t o_st,
                          const int32_t* state_indices, int32_t pad_slot_id,
                          void* inter, int64_t i_slot, int64_t i_st, int64_t i_sd, int64_t i_sk,
                          int64_t inter_nslots, const int32_t* inter_indices,
                          int64_t batch, int64_t dim, int32_t steps, int32_t width,
                          int32_t dtype, int32_t silu, int32_t* dev_status, void* stream) {
    if (cc1d_status_t s = check_common(width, dtype)) return s;
    if (batch < 0 || dim < 0 || steps < 1)
        return fail(CC1D_ERR_INVALID, "bad sizes (batch %lld, dim %lld, steps %d)",
                    (long long)batch, (long long)dim, steps);
    if (state_len < width - 1)
        return fail(CC1D_ERR_INVALID, "state length %lld is shorter than width - 1 = %d",
                    (long long)state_len, width - 1);
    if (batch == 0 || dim == 0) return ok();
    if (x == nullptr || weight == nullptr || out == nullptr || state == nullptr)
        return fail(CC1D_ERR_INVALID, "x, state, weight and out must not be NULL");
    if (state_indices == nullptr && nslots < batch)
        return fail(CC1D_ERR_INVALID, "without state indices the cache needs >= %lld slots, has %lld",
                    (long long)batch, (long long)nslots);
    if (inter != nullptr && inter_nslots < 1)
        return fail(CC1D_ERR_INVALID, "the per-step state cache has no slots");
    cc1d::UpdArgs a{x, x_sb, x_sd, x_st, state, s_slot, s_sd, s_sk, state_len, nslots,
                    weight, w_sd, w_sk, bias, bias_s, out, o_sb, o_sd, o_st,
                    state_indices, pad_slot_id, inter, i_slot, i_st, i_sd, i_sk, inter_nslots,
                    inter_indices, batch, dim, steps, silu != 0, dev_status};
    if (cc1d_status_t s = bind_stream(stream)) return s;
    return from_cuda(cc1d::launch_update(a, width, dtype, (cudaStream_t)stream), "cc1d_update");
}

cc1d_status_t cc1d_update_ring(const void* x, int64_t x_sb, int64_t x_sd,
                               void* ring, int64_t r_slot, int64_t r_sk, int64_t r_sd,
                               int64_t nslots,
                               const void* weight, int64_t w_sd, int64_t w_sk,
                               const void* bias, int64_t bias_s,
                               void* out, int64_t o_sb, int64_t o_sd,
                               const int32_t* cache_seqlens, const int32_t* state_indices,
                               int32_t pad_slot_id, int64_t batch, int64_t dim, int32_t width,
                               int32_t dtype, int32_t silu, int32_t* dev_status, void* stream) {
    if (cc1d_status_t s = check_common(width, dtype)) return s;
    if (batch < 0 || dim < 0)
        return fail(CC1D_ERR_INVALID, "negative size (batch %lld, dim %lld)", (long long)batch,
                    (long long)dim);
    if (batch == 0 || dim == 0) return ok();
    if (x == nullptr || ring == nullptr || weight == nullptr || out == nullptr ||
        cache_seqlens == nullptr)
        return fail(CC1D_ERR_INVALID, "x, ring, weight, out and cache_seqlens must not be NULL");
    if (state_indices == nullptr && nslots < batch)
        return fail(CC1D_ERR_INVALID, "without state indices the ring needs >= %lld slots, has %lld",
                    (long long)batch, (long long)nslots);
    cc1d::RingArgs a{x, x_sb, x_sd, ring, r_slot, r_sk, r_sd, nslots, weight, w_sd, w_sk,
                     bias, bias_s, out, o_sb, o_sd, cache_seqlens, state_indices, pad_slot_id,
                     batch, dim, silu != 0, dev_status};
    if (cc1d_status_t s = bind_stream(stream)) return s;
    return from_cuda(cc1d::launch_ring(a, width, dtype, (cudaStream_t)stream), "cc1d_update_ring");
}

cc1d_status_t cc1d_varlen(const void* x, int64_t x_sd, int64_t x_st,
                          const void* weight, int64_t w_sd, int64_t w_sk,
                          const void* bias, int64_t bias_s,
                          void* out, int64_t o_sd, int64_t o_st,
                          const int32_t* query_start_loc, int64_t nseq, int64_t ntokens,
                          const int32_t* cache_indices, const uint8_t* has_initial_state,
                          void* conv_states, int64_t s_slot, int64_t s_sd, int64_t s_sk,
                          int64_t nslots, int32_t pad_slot_id, int64_t dim, int32_t width,
                          int32_t dtype, int32_t silu, int32_t* dev_status, void* stream) {
    if (cc1d_status_t s = check_common(width, dtype)) return s;
    if (nseq < 0 || ntokens < 0 || dim < 0)
        return fail(CC1D_ERR_INVALID, "negative size (nseq %lld, ntokens %lld, dim %lld)",
                    (long long)nseq, (long long)ntokens, (long long)dim);
    if (nseq == 0 || ntokens == 0 || dim == 0) return ok();
    if (ntokens > INT32_MAX)
        return fail(CC1D_ERR_INVALID, "%lld tokens exceed the int32 range of query_start_loc",
                    (long long)ntokens);
    if (x == nullptr || weight == nullptr || out == nullptr || query_start_loc == nullptr)
        return fail(CC1D_ERR_INVALID, "x, weight, out and query_start_loc must not be NULL");
    if (conv_states != nullptr && nslots < 1)
        return fail(CC1D_ERR_INVALID, "the conv state cache has no slots");
    cc1d::VarArgs a{x, x_sd, x_st, weight, w_sd, w_sk, bias, bias_s, out, o_sd, o_st,
                    query_start_loc, nseq, ntokens, cache_indices, has_initial_state,
                    conv_states, s_slot, s_sd, s_sk, nslots, pad_slot_id, dim, silu != 0,
                    dev_status};
    if (cc1d_status_t s = bind_stream(stream)) return s;
    return from_cuda(cc1d::launch_varlen(a, width, dtype, (cudaStream_t)stream), "cc1d_varlen");
}

cc1d_status_t cc1d_update_unpack(const void* qkvz, int64_t q_sb, const void* ba, int64_t ba_sb,
                                 void* state, int64_t nslots,
                                 const void* weight, const void* bias,
                                 void* out, void* z, void* b, void* a,
                                 const int32_t* state_indices, int32_t pad_slot_id,
                                 int64_t batch, int64_t dim, int64_t zdim, int64_t heads,
                                 int32_t width, int32_t dtype, int32_t gdtype, int32_t silu,
                                 void* stream) {
    if (cc1d_status_t s = check_common(width, dtype)) return s;
    if (gdtype != CC1D_BF16 && gdtype != CC1D_F16 && gdtype != CC1D_F32)
        return fail(CC1D_ERR_DTYPE, "gate dtype %d is not bf16, fp16 or fp32", gdtype);
    if (batch < 0 || dim < 0 || zdim < 0 || heads < 0)
        return fail(CC1D_ERR_INVALID, "negative size");
    if (batch == 0) return ok();
    if (batch > 65535) return fail(CC1D_ERR_INVALID, "batch %lld exceeds 65535", (long long)batch);
    if (!qkvz || !ba || !state || !weight || !out || !z || !b || !a || !state_indices)
        return fail(CC1D_ERR_INVALID, "a required pointer is NULL");
    const int64_t e = dtype == CC1D_F32 ? 4 : 2;
    const int64_t V = 16 / e;
    const int64_t ge = gdtype == CC1D_F32 ? 4 : 2;
    if (dim % V || zdim % V || (q_sb * e) % 16 || !cc1d::host_aligned16(qkvz) ||
        !cc1d::host_aligned16(state) || !cc1d::host_aligned16(weight) ||
        !cc1d::host_aligned16(out) || !cc1d::host_aligned16(z) ||
        (bias != nullptr && !cc1d::host_aligned16(bias)) || q_sb < dim + zdim ||
        ba_sb < 2 * heads || ((uintptr_t)ba % ge) != 0)
        return fail(CC1D_ERR_LAYOUT,
                    "fused decode needs dim and zdim multiples of %lld, 16-byte aligned rows and "
                    "contiguous state, weight and outputs",
                    (long long)V);
    cc1d::UnpackArgs args{qkvz, q_sb, ba, ba_sb, state, nslots, weight, bias, out, z, b, a,
                          state_indices, pad_slot_id, batch, dim, zdim, heads, (int)ge,
                          silu != 0};
    if (cc1d_status_t s = bind_stream(stream)) return s;
    return from_cuda(cc1d::launch_unpack(args, width, dtype, (cudaStream_t)stream),
                     "cc1d_update_unpack");
}

cc1d_status_t cc1d_copy(void* dst, const void* src, int64_t bytes, void* stream) {
    if (bytes < 0) return fail(CC1D_ERR_INVALID, "negative size");
    if (bytes == 0) return ok();
    if (!dst || !src) return fail(CC1D_ERR_INVALID, "a required pointer is NULL");
    if (overlap(dst, bytes, src, bytes)) return fail(CC1D_ERR_INVALID, "dst overlaps src");
    if (!cc1d::host_aligned32(dst) || !cc1d::host_aligned32(src))
        return fail(CC1D_ERR_LAYOUT, "the copy needs 32-byte aligned pointers");
    if (cc1d_status_t s = bind_stream(stream)) return s;
    return from_cuda(cc1d::launch_copy(dst, src, bytes, (cudaStream_t)stream), "cc1d_copy");
}

}  // extern "C"
