/*
 * cc1d.h - C ABI of libcc1d.so, the B200 (sm_100a) depthwise causal conv1d kernels.
 *
 * The operator is out[b,c,t] = act(bias[c] + sum_k w[c,k] * x[b,c,t-(W-1)+k]) with x taken as
 * zero (or as the cached conv state) before the start of each sequence, act = SiLU or identity,
 * fp32 accumulation, and outputs rounded to the storage dtype.
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are DEVICE pointers. Every tensor is described by its element
 *     strides (int64, in elements, not bytes), so views of wider buffers are consumed in place.
 *   - `dtype` is one of CC1D_BF16 / CC1D_F16 / CC1D_F32. x, weight, bias, states and outputs
 *     share it.
 *   - `width` is the kernel width W, 2..8. K = W - 1 is the conv state length.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Work is enqueued on it and the
 *     call returns without synchronising, so every call may be captured in a CUDA graph.
 *   - The library allocates nothing and keeps no state between calls; calls are thread-safe.
 *   - Kernels launch on the device that owns the calling thread's current CUDA context.
 *   - `dev_status`, when not NULL, is a device int32 that kernels OR CC1D_DEV_* bits into when
 *     they meet an index they refuse (a slot outside the cache, sequence bounds outside the
 *     packed tokens). The offending work item is skipped; nothing is read or written out of
 *     range. The caller clears the word and reads it back when it chooses to.
 *   - The return value is CC1D_OK or a CC1D_ERR_* code; cc1d_last_error() describes the most
 *     recent failure on the calling thread.
 */
#ifndef CC1D_H
#define CC1D_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t cc1d_status_t;

enum {
    CC1D_OK = 0,
    CC1D_ERR_INVALID = 1, /* null pointer, negative size, inconsistent shape */
    CC1D_ERR_DTYPE = 2,   /* dtype not bf16 / fp16 / fp32 */
    CC1D_ERR_WIDTH = 3,   /* width outside 2..8 */
    CC1D_ERR_LAYOUT = 4,  /* a stride pattern the kernels do not address */
    CC1D_ERR_CUDA = 5     /* the launch itself failed (see cc1d_last_error) */
};

enum { CC1D_BF16 = 0, CC1D_F16 = 1, CC1D_F32 = 2 };

enum {
    CC1D_DEV_BAD_SLOT = 1,       /* a conv-state / ring slot outside [0, nslots) and != pad */
    CC1D_DEV_BAD_QSL = 2,        /* query_start_loc outside [0, ntokens] or decreasing */
    CC1D_DEV_BAD_INTER_SLOT = 4  /* a per-step state slot outside [0, inter_nslots) */
};

/* ABI revision; bumped on any signature change. */
int32_t cc1d_abi_version(void);

/* Static description of a status code. */
const char* cc1d_status_string(cc1d_status_t code);

/* Detail of the last failing call on this thread ("" if none). */
const char* cc1d_last_error(void);

/*
 * Prefill over batched dense sequences: x and out are (batch, dim, seqlen) with arbitrary
 * strides. Channel-last storage (x_sd == 1, token rows x_sl >= dim apart) and channel-first
 * storage (x_sl == 1) take vectorised kernels; any other stride pattern takes a generic one.
 * out must not overlap x.
 * Replaces: causal_conv1d_fn (causal_conv1d_cute/functional.py:315-347) -> CausalConv1d.fwd
 * (api.py:257-338) -> the fwd.py kernels ConvFwdRowMajor (fwd.py:81-234), ConvFwdRowMajorRagged
 * (fwd.py:1033-1178), ConvFwdChannelLast (fwd.py:360-469), ConvFwdChannelLastStrip
 * (fwd.py:623-842).
 */
cc1d_status_t cc1d_fwd(const void* x, int64_t x_sb, int64_t x_sd, int64_t x_sl,
                       const void* weight, int64_t w_sd, int64_t w_sk,
                       const void* bias, int64_t bias_s,
                       void* out, int64_t o_sb, int64_t o_sd, int64_t o_sl,
                       int64_t batch, int64_t dim, int64_t seqlen, int32_t width,
                       int32_t dtype, int32_t silu, void* stream);

/*
 * Prefill with the Dao-AILab causal_conv1d_fn extras. Shapes and x / weight / bias / out as in
 * cc1d_fwd, plus (each may be NULL):
 *   seq_idx         int32 (batch, seqlen), strides (q_sb, q_sl): a tap reaches back only to
 *                   tokens with the same id as the output token (a different id adds nothing);
 *   initial_states  (batch, dim, W-1), strides (i_sb, i_sd, i_sk): the W-1 inputs before token 0
 *                   of each row (zeros when NULL);
 *   final_states    (batch, dim, W-1), strides (f_sb, f_sd, f_sk), written: the last W-1 entries
 *                   of [initial_states | x] of each row, bit for bit (seqlen may be 0).
 * seq_idx excludes both states (as upstream); final_states must not overlap initial_states.
 * Replaces: the upstream causal_conv1d_fn(x, weight, bias, seq_idx, initial_states,
 * return_final_states, final_states_out, activation) that dao_compat.around_fn passes these
 * calls to (dao_compat.py:28-78).
 */
cc1d_status_t cc1d_fwd_states(const void* x, int64_t x_sb, int64_t x_sd, int64_t x_sl,
                              const void* weight, int64_t w_sd, int64_t w_sk,
                              const void* bias, int64_t bias_s,
                              void* out, int64_t o_sb, int64_t o_sd, int64_t o_sl,
                              const int32_t* seq_idx, int64_t q_sb, int64_t q_sl,
                              const void* initial_states, int64_t i_sb, int64_t i_sd, int64_t i_sk,
                              void* final_states, int64_t f_sb, int64_t f_sd, int64_t f_sk,
                              int64_t batch, int64_t dim, int64_t seqlen, int32_t width,
                              int32_t dtype, int32_t silu, void* stream);

/*
 * Decode of `steps` tokens per batch row (1..16) against a conv-state cache updated in place.
 * x and out are (batch, dim, steps). state is (nslots, dim, state_len) with state_len >= W-1:
 * the last W-1 entries of a channel row are the history, and the whole row shifts left by
 * `steps` (state_len > W-1 covers the power-of-two padded layout). Row b uses slot
 * state_indices[b] (b when NULL); rows whose slot equals pad_slot_id are skipped and their
 * outputs are left unwritten.
 * When inter is not NULL, the conv state after every token t is written to
 * inter[inter_indices[b], t, :, :] (inter_indices defaults to state_indices), a
 * (inter_nslots, steps, dim, W-1) tensor given by its strides: contiguous ("dense") or the
 * overlapping view with strides (dim*(steps+W-2), 1, steps+W-2, 1) ("dedup").
 * Replaces: causal_conv1d_update / _update (functional.py:711-858) -> ConvUpdateIndexedVec
 * (varlen.py:627-815), ConvUpdateIndexed (varlen.py:512-624), and the direct-state kernels
 * ConvUpdateVec / ConvUpdatePadded / ConvUpdatePaddedVec / ConvUpdateStd2D (update.py:43-483)
 * reached through CausalConv1d.update (api.py:419-479).
 */
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
                          int32_t dtype, int32_t silu, int32_t* dev_status, void* stream);

/*
 * Single-token decode on a ring conv state (nslots, W-1, dim): row cache_seqlens[b] % (W-1)
 * holds the oldest input of batch row b; it is overwritten with x[b] and the other rows are
 * left in place. Slot mapping and padding as in cc1d_update.
 * Replaces: causal_conv1d_update_ring (functional.py:861-930) -> CausalConv1d.update_ring
 * (api.py:346-398) -> ConvUpdateRing (ring.py:70-217).
 */
cc1d_status_t cc1d_update_ring(const void* x, int64_t x_sb, int64_t x_sd,
                               void* ring, int64_t r_slot, int64_t r_sk, int64_t r_sd,
                               int64_t nslots,
                               const void* weight, int64_t w_sd, int64_t w_sk,
                               const void* bias, int64_t bias_s,
                               void* out, int64_t o_sb, int64_t o_sd,
                               const int32_t* cache_seqlens, const int32_t* state_indices,
                               int32_t pad_slot_id, int64_t batch, int64_t dim, int32_t width,
                               int32_t dtype, int32_t silu, int32_t* dev_status, void* stream);

/*
 * Layout conversion between the ordered conv state (slots, dim, W-1) (the prefill / decode
 * layout, oldest entry first) and the ring state (slots, W-1, dim) of cc1d_update_ring: ring row
 * (cache_seqlens[s] + k) mod (W-1) of slot s holds ordered entry k. width is W (2..8); the two
 * tensors, given by element strides, must not overlap.
 * Replaces: to_ring / from_ring (ring.py:33-67), torch gathers in the reference.
 */
cc1d_status_t cc1d_to_ring(const void* state, int64_t s_slot, int64_t s_sd, int64_t s_sk,
                           void* ring, int64_t r_slot, int64_t r_sk, int64_t r_sd,
                           const int32_t* cache_seqlens, int64_t slots, int64_t dim,
                           int32_t width, int32_t dtype, void* stream);
cc1d_status_t cc1d_from_ring(const void* ring, int64_t r_slot, int64_t r_sk, int64_t r_sd,
                             void* state, int64_t s_slot, int64_t s_sd, int64_t s_sk,
                             const int32_t* cache_seqlens, int64_t slots, int64_t dim,
                             int32_t width, int32_t dtype, void* stream);

/*
 * Packed variable-length prefill. x and out are (dim, ntokens). Token-major views (x_sd == 1,
 * the serving layout) take ONE vectorised launch for any number of sequences; contiguous
 * channel-first storage (x_st == 1) takes a vectorised stream pass plus a per-(channel, sequence)
 * boundary launch; other strides take a scalar kernel.
 * Sequence i spans tokens [query_start_loc[i], query_start_loc[i+1]); tokens outside every
 * sequence keep their previous output contents. When conv_states (nslots, dim, W-1) is given,
 * sequence i starts from conv_states[cache_indices[i]] if has_initial_state[i] != 0 (from zeros
 * otherwise) and that slot receives the last W-1 inputs of [initial state | sequence] after the
 * call; sequences of zero tokens and sequences whose slot equals pad_slot_id leave the cache
 * untouched. Without conv_states every sequence starts from zeros.
 * Replaces: causal_conv1d_varlen_fn / _varlen / _varlen_token_major (functional.py:350-573)
 * -> ConvFwdChannelLastStripSeq (varlen.py:382-509) + ConvSeqBoundaryVec (varlen.py:209-379),
 * or the channel-first bulk pass + ConvSeqBoundary (varlen.py:26-206).
 */
cc1d_status_t cc1d_varlen(const void* x, int64_t x_sd, int64_t x_st,
                          const void* weight, int64_t w_sd, int64_t w_sk,
                          const void* bias, int64_t bias_s,
                          void* out, int64_t o_sd, int64_t o_st,
                          const int32_t* query_start_loc, int64_t nseq, int64_t ntokens,
                          const int32_t* cache_indices, const uint8_t* has_initial_state,
                          void* conv_states, int64_t s_slot, int64_t s_sd, int64_t s_sk,
                          int64_t nslots, int32_t pad_slot_id, int64_t dim, int32_t width,
                          int32_t dtype, int32_t silu, int32_t* dev_status, void* stream);

/*
 * Fused single-token decode of a Gated DeltaNet layer: the conv reads the leading `dim` columns
 * of each [Q|K|V|Z] projection row in place, updates conv_state (nslots, dim, W-1, contiguous
 * per slot) and writes out (batch, dim); the Z columns (zdim after dim) and the B and A halves of
 * each [B|A] row (2*heads wide, dtype gdtype) are copied to contiguous z (batch, zdim),
 * b (batch, heads) and a (batch, heads). Rows whose slot is the pad slot or lies outside the
 * cache keep their state and have their conv input copied to out unchanged. weight (dim, W) and
 * bias (dim,) are the model's own contiguous tensors.
 * Replaces: causal_conv1d_update_unpack (unpack.py:328-374) -> ConvUpdateUnpack
 * (unpack.py:33-222), reached from sglang_compat.around_unpack (sglang_compat.py:245-326).
 */
cc1d_status_t cc1d_update_unpack(const void* qkvz, int64_t q_sb, const void* ba, int64_t ba_sb,
                                 void* state, int64_t nslots,
                                 const void* weight, const void* bias,
                                 void* out, void* z, void* b, void* a,
                                 const int32_t* state_indices, int32_t pad_slot_id,
                                 int64_t batch, int64_t dim, int64_t zdim, int64_t heads,
                                 int32_t width, int32_t dtype, int32_t gdtype, int32_t silu,
                                 void* stream);

/*
 * Device-to-device copy of `bytes` bytes (src and dst on the stream's device, 32-byte aligned,
 * not overlapping) with 32-byte accesses from one wave of CTAs. It is the
 * measured ceiling the streaming kernels are reported against: a prefill moves the same bytes
 * (each input read once, each output written once) and adds only its arithmetic.
 * Replaces: the reference's copy ceiling, benchmarks/copy_baseline.py:38-90 (a D2D copy of a
 * prefill's bytes timed beside every prefill kernel, benchmarks/BASELINES.md:44).
 */
cc1d_status_t cc1d_copy(void* dst, const void* src, int64_t bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CC1D_H */
