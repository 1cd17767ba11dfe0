// Host-side launchers of the sm_100a kernels. api.cu validates the C-ABI arguments and calls
// these; each launcher picks the kernel variant for the layout it is given (the sm_100 launch
// table) and returns the launch status.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace cc1d {

struct FwdArgs {
    const void* x;
    int64_t x_sb, x_sd, x_sl;
    const void* w;
    int64_t w_sd, w_sk;
    const void* bias;
    int64_t bias_s;
    void* out;
    int64_t o_sb, o_sd, o_sl;
    int64_t B, D, L;
    int silu;
};

// Prefill with the Dao-interface extras: per-token sequence ids (taps reach back only to tokens
// with the same id), initial states (the W-1 inputs before token 0 of each batch row) and final
// states (the last W-1 inputs of [initial | x] of each row). Each pointer may be NULL.
struct FwdStateArgs {
    FwdArgs f;
    const int32_t* seq;
    int64_t q_sb, q_sl;
    const void* init;
    int64_t i_sb, i_sd, i_sk;
    void* fin;
    int64_t f_sb, f_sd, f_sk;
};

struct UpdArgs {
    const void* x;
    int64_t x_sb, x_sd, x_st;
    void* state;
    int64_t s_slot, s_sd, s_sk, S, nslots;
    const void* w;
    int64_t w_sd, w_sk;
    const void* bias;
    int64_t bias_s;
    void* out;
    int64_t o_sb, o_sd, o_st;
    const int32_t* idx;
    int32_t pad;
    void* inter;
    int64_t i_slot, i_st, i_sd, i_sk, inter_nslots;
    const int32_t* iidx;
    int64_t B, D;
    int L;
    int silu;
    int32_t* status;
};

struct RingArgs {
    const void* x;
    int64_t x_sb, x_sd;
    void* ring;
    int64_t r_slot, r_sk, r_sd, nslots;
    const void* w;
    int64_t w_sd, w_sk;
    const void* bias;
    int64_t bias_s;
    void* out;
    int64_t o_sb, o_sd;
    const int32_t* seen;
    const int32_t* idx;
    int32_t pad;
    int64_t B, D;
    int silu;
    int32_t* status;
};

// Conversion between the ordered conv state (slots, dim, W-1) and the ring state
// (slots, W-1, dim): ring row (seen[s] + k) % (W-1) holds ordered entry k.
struct RingConvArgs {
    const void* state;
    int64_t s_slot, s_sd, s_sk;
    void* ring;
    int64_t r_slot, r_sk, r_sd;
    const int32_t* seen;
    int64_t S, D;
    bool to_ring;  // state -> ring; otherwise ring -> state
};

struct VarArgs {
    const void* x;
    int64_t x_sd, x_st;
    const void* w;
    int64_t w_sd, w_sk;
    const void* bias;
    int64_t bias_s;
    void* out;
    int64_t o_sd, o_st;
    const int32_t* qsl;
    int64_t nseq, T;
    const int32_t* cidx;
    const uint8_t* hinit;
    void* states;
    int64_t s_slot, s_sd, s_sk, nslots;
    int32_t pad;
    int64_t D;
    int silu;
    int32_t* status;
};

struct UnpackArgs {
    const void* qkvz;
    int64_t q_sb;
    const void* ba;
    int64_t ba_sb;
    void* state;
    int64_t nslots;
    const void* w;
    const void* bias;
    void* out;
    void* z;
    void* b;
    void* a;
    const int32_t* idx;
    int32_t pad;
    int64_t B, D, zdim, heads;
    int gsize;  // bytes per element of the [B|A] rows
    int silu;
};

cudaError_t launch_fwd(const FwdArgs& a, int width, int dtype, cudaStream_t stream);
cudaError_t launch_fwd_states(const FwdStateArgs& a, int width, int dtype, cudaStream_t stream);
cudaError_t launch_update(const UpdArgs& a, int width, int dtype, cudaStream_t stream);
cudaError_t launch_ring(const RingArgs& a, int width, int dtype, cudaStream_t stream);
cudaError_t launch_ring_convert(const RingConvArgs& a, int width, int dtype, cudaStream_t stream);
cudaError_t launch_varlen(const VarArgs& a, int width, int dtype, cudaStream_t stream);
cudaError_t launch_unpack(const UnpackArgs& a, int width, int dtype, cudaStream_t stream);
cudaError_t launch_copy(void* dst, const void* src, int64_t bytes, cudaStream_t stream);

}  // namespace cc1d
