// Sequence bounds and cache slots of a packed (varlen) batch, shared by the varlen kernels.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace cc1d {

// query_start_loc[s] clamped into [0, T].
__device__ __forceinline__ int64_t qsl_at(const VarArgs& a, int64_t s) {
    const int64_t v = __ldg(a.qsl + s);
    return v < 0 ? 0 : (v > a.T ? a.T : v);
}

// Largest s in [0, nseq] with query_start_loc[s] <= t, or -1 when t precedes the first sequence.
// Empty sequences are skipped because the largest index wins.
__device__ inline int64_t seq_of(const VarArgs& a, int64_t t) {
    if (qsl_at(a, 0) > t) return -1;
    int64_t lo = 0, hi = a.nseq;
    while (lo < hi) {
        const int64_t mid = (lo + hi + 1) >> 1;
        if (qsl_at(a, mid) <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

__device__ __forceinline__ void check_bounds(const VarArgs& a, int64_t s) {
    const int32_t lo = __ldg(a.qsl + s), hi = __ldg(a.qsl + s + 1);
    if (lo < 0 || hi > a.T || hi < lo) flag_status(a.status, CC1D_DEV_BAD_QSL);
}

struct SeqSlot {
    bool live;      // the cache slot is read and written
    bool use_init;  // the sequence starts from the cached state
    int64_t slot;
};

__device__ __forceinline__ SeqSlot seq_slot(const VarArgs& a, int64_t s, bool report) {
    SeqSlot r{false, false, 0};
    if (a.states == nullptr) return r;
    const int32_t slot = a.cidx != nullptr ? __ldg(a.cidx + s) : (int32_t)s;
    if (slot == a.pad) return r;
    if (slot < 0 || (int64_t)slot >= a.nslots) {
        if (report) flag_status(a.status, CC1D_DEV_BAD_SLOT);
        return r;
    }
    r.live = true;
    r.slot = slot;
    r.use_init = a.hinit != nullptr && __ldg(a.hinit + s) != 0;
    return r;
}

}  // namespace cc1d
