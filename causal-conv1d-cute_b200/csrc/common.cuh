// Shared device helpers for the depthwise causal conv1d kernels (sm_100a).
//
// Every kernel moves data in 16-byte vectors: V = 16 / sizeof(T) adjacent elements (8 for
// bf16/fp16, 4 for fp32), accumulates in fp32 with the bias first and the taps in order
// k = 0..W-1 (oldest input first), then applies SiLU and rounds to the storage dtype. This is
// the accumulation order of the reference kernels (causal_conv1d_cute/fwd.py:217-225).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/cc1d.h"

namespace cc1d {

using bf16 = __nv_bfloat16;
using f16 = __half;

template <typename T>
struct Vec {
    static constexpr int V = 16 / (int)sizeof(T);  // elements per 16-byte vector
};

// ---------------------------------------------------------------------------------------------
// 16-byte vector <-> fp32 lanes
// ---------------------------------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, float* f);

template <>
__device__ __forceinline__ void unpack16<bf16>(const uint4& v, float* f) {
    // A bf16 is the high half of an fp32: widening is a shift or a mask.
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

template <>
__device__ __forceinline__ void unpack16<f16>(const uint4& v, float* f) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        float2 p = __half22float2(h);
        f[2 * i] = p.x;
        f[2 * i + 1] = p.y;
    }
}

template <>
__device__ __forceinline__ void unpack16<float>(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* f);

template <>
__device__ __forceinline__ uint4 pack16<bf16>(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <>
__device__ __forceinline__ uint4 pack16<f16>(const float* f) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

template <>
__device__ __forceinline__ uint4 pack16<float>(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
}

// Element <-> fp32 for the scalar paths.
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<bf16>(bf16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<f16>(f16 v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ bf16 from_f32<bf16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ f16 from_f32<f16>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }

// Raw element i (0..V-1) of a 16-byte vector, kept in the storage type (bit-exact copies).
template <typename T>
__device__ __forceinline__ T lane_of(const uint4& v, int i) {
    return reinterpret_cast<const T*>(&v)[i];
}
template <typename T>
__device__ __forceinline__ void set_lane(uint4& v, int i, T val) {
    reinterpret_cast<T*>(&v)[i] = val;
}
template <typename T>
__device__ __forceinline__ T lane_of(const uint2& v, int i) {
    return reinterpret_cast<const T*>(&v)[i];
}
template <typename T>
__device__ __forceinline__ void set_lane(uint2& v, int i, T val) {
    reinterpret_cast<T*>(&v)[i] = val;
}

// ---------------------------------------------------------------------------------------------
// Global memory access
// ---------------------------------------------------------------------------------------------

// Read-only data that this kernel never writes (inputs, weights): non-coherent path.
__device__ __forceinline__ uint4 ldg16(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}

// Streamed input read once: do not keep it in L1.
__device__ __forceinline__ uint4 ldg16_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Data that the same kernel later overwrites (conv state caches): coherent load.
__device__ __forceinline__ uint4 ld16(const void* p) {
    return *reinterpret_cast<const uint4*>(p);
}

__device__ __forceinline__ void st16(void* p, const uint4& v) {
    *reinterpret_cast<uint4*>(p) = v;
}

// Streamed output written once: evict-first so it does not displace reusable lines in L2.
// 32-byte vector load / store (sm_100 has 256-bit global accesses; the address must be 32-byte
// aligned): one instruction moves what two 16-byte accesses do. A copy kernel measured on B200
// moved 512 MiB in 164.8 us with these against 168.7 us with 16-byte vectors.
__device__ __forceinline__ void ldg32_stream(const void* p, uint4& lo, uint4& hi) {
    asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y),
                   "=r"(hi.z), "=r"(hi.w)
                 : "l"(p));
}

__device__ __forceinline__ void st32_stream(void* p, const uint4& lo, const uint4& hi) {
    asm volatile("st.global.cs.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(lo.x),
                 "r"(lo.y), "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
                 : "memory");
}

__device__ __forceinline__ void st16_stream(void* p, const uint4& v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Asynchronous 16-byte copy global -> shared (cached in L2 only), and its group fences. The bytes
// in flight hold no registers: a thread waits for its own copies with cp_async_wait<N>() (at most
// N of its committed groups still pending) and then reads them from shared memory.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Programmatic dependent launch. A kernel launched with programmatic stream serialisation may
// start once every CTA of the kernel before it in the stream has called allow_dependent_launch()
// (or exited); grid_dependency_wait() then blocks until that kernel has completed and its memory
// writes are visible. Both are hardware dependency controls, not spin loops, and are no-ops for a
// kernel launched the ordinary way.
__device__ __forceinline__ void allow_dependent_launch() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// A thread's channel vector of NB bytes (16: uint4, 8: uint2) for the kernels that can run with
// half-width vectors (fewer registers per thread when the filter is wide).
template <int NB>
struct RawVec;
template <>
struct RawVec<16> {
    using type = uint4;
};
template <>
struct RawVec<8> {
    using type = uint2;
};

template <int NB>
__device__ __forceinline__ typename RawVec<NB>::type ldg_stream_raw(const void* p) {
    if constexpr (NB == 16) {
        return ldg16_stream(p);
    } else {
        uint2 v;
        asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                     : "=r"(v.x), "=r"(v.y)
                     : "l"(p));
        return v;
    }
}

template <int NB>
__device__ __forceinline__ void st_stream_raw(void* p, const typename RawVec<NB>::type& v) {
    if constexpr (NB == 16) {
        st16_stream(p, v);
    } else {
        asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y)
                     : "memory");
    }
}

template <int NB>
__device__ __forceinline__ typename RawVec<NB>::type ldg_raw(const void* p) {
    return __ldg(reinterpret_cast<const typename RawVec<NB>::type*>(p));
}

// Coherent NB-byte load and store (conv state caches, which the same kernel writes).
template <int NB>
__device__ __forceinline__ typename RawVec<NB>::type ld_raw(const void* p) {
    return *reinterpret_cast<const typename RawVec<NB>::type*>(p);
}
template <int NB>
__device__ __forceinline__ void st_raw(void* p, const typename RawVec<NB>::type& v) {
    *reinterpret_cast<typename RawVec<NB>::type*>(p) = v;
}

// NB-byte vector <-> NB / sizeof(T) fp32 lanes.
template <typename T, int NB>
__device__ __forceinline__ void unpack_raw(const typename RawVec<NB>::type& v, float* f) {
    if constexpr (NB == 16) {
        unpack16<T>(v, f);
    } else {
        float g[Vec<T>::V];
        unpack16<T>(make_uint4(v.x, v.y, 0u, 0u), g);
#pragma unroll
        for (int i = 0; i < NB / (int)sizeof(T); ++i) f[i] = g[i];
    }
}

template <typename T, int NB>
__device__ __forceinline__ typename RawVec<NB>::type pack_raw(const float* f) {
    if constexpr (NB == 16) {
        return pack16<T>(f);
    } else {
        float g[Vec<T>::V];
#pragma unroll
        for (int i = 0; i < Vec<T>::V; ++i) g[i] = i < NB / (int)sizeof(T) ? f[i] : 0.f;
        const uint4 u = pack16<T>(g);
        return make_uint2(u.x, u.y);
    }
}

__device__ __forceinline__ bool aligned16(const void* p) {
    return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// ---------------------------------------------------------------------------------------------
// Activation
// ---------------------------------------------------------------------------------------------

// Hardware tanh approximation (PTX tanh.approx.f32, sm_75+).
__device__ __forceinline__ float tanh_approx(float x) {
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// SiLU a * sigmoid(a). For 16-bit outputs sigmoid(a) = 0.5 * tanh(a / 2) + 0.5 evaluated with the
// hardware approximation, written as h * tanh(h) + h with h = a / 2; its error is far below one
// bf16/fp16 ulp. fp32 outputs use the library expf.
template <typename T>
__device__ __forceinline__ float silu(float a) {
    if constexpr (std::is_same<T, float>::value) {
        return a / (1.0f + expf(-a));
    } else {
        const float h = 0.5f * a;
        return fmaf(h, tanh_approx(h), h);
    }
}

template <typename T>
__device__ __forceinline__ float activate(float a, bool use_silu) {
    return use_silu ? silu<T>(a) : a;
}

// State blocks: transpose between the channel-major state block (element e*SS + s of the block, V*SS
// elements in SS vectors) and SS time-major vectors (vector s, lane e). R is the vector type
// (uint4, or uint2 for the half-width kernels); V = sizeof(R) / sizeof(T).
template <typename T, int SS, typename R>
__device__ __forceinline__ void block_to_time(const R (&blk)[SS], R (&tm)[SS]) {
    constexpr int V = (int)(sizeof(R) / sizeof(T));
#pragma unroll
    for (int e = 0; e < V; ++e)
#pragma unroll
        for (int s = 0; s < SS; ++s) {
            const int flat = e * SS + s;
            set_lane<T>(tm[s], e, lane_of<T>(blk[flat / V], flat % V));
        }
}

template <typename T, int N, typename R>
__device__ __forceinline__ void time_to_block(const R* tm, R (&blk)[N]) {
    constexpr int V = (int)(sizeof(R) / sizeof(T));
#pragma unroll
    for (int q = 0; q < N; ++q)
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int flat = q * V + i;
            set_lane<T>(blk[q], i, lane_of<T>(tm[flat % N], flat / N));
        }
}

// CTAs of `kern` (launched with `threads` threads, no dynamic shared memory) that the current
// device holds at once: SM count x resident CTAs per SM. Cached per device in `cache`, an array
// of kSlotCacheDevices zero-initialised ints owned by the caller; 0 when the query fails.
constexpr int kSlotCacheDevices = 64;

// Streaming multiprocessors of the current device (0 when the query fails), cached per device.
inline int device_sm_count() {
    static int cache[kSlotCacheDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kSlotCacheDevices) return 0;
    if (cache[dev] == 0) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
        cache[dev] = sms;
    }
    return cache[dev];
}

inline int device_slots(const void* kern, int threads, int* cache) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kSlotCacheDevices) return 0;
    if (cache[dev] == 0) {
        int sms = 0, per_sm = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, 0) !=
                cudaSuccess)
            return 0;
        cache[dev] = sms * per_sm;
    }
    return cache[dev];
}

__device__ __forceinline__ void flag_status(int32_t* status, int32_t bits) {
    if (status != nullptr) atomicOr(status, bits);
}

// ---------------------------------------------------------------------------------------------
// Filter weights and bias of V adjacent channels, widened to fp32 registers
// ---------------------------------------------------------------------------------------------

// w[k][e] = weight[c0 + e, k]; b[e] = bias[c0 + e] (0 without bias). The weights are the caller's
// own (dim, W) tensor read in place: when it is contiguous and 16-byte aligned (wvec) the V*W
// elements of a channel group are W whole 16-byte vectors, otherwise they are read one by one.
// bvec: the bias is contiguous and 16-byte aligned.
// NB: bytes of channels per thread (16, or 8 for the half-width kernels); V = NB / sizeof(T).
template <typename T, int W, int NB = 16>
__device__ __forceinline__ void load_filter(const T* __restrict__ weight, int64_t w_sd,
                                            int64_t w_sk, const T* __restrict__ bias,
                                            int64_t bias_s, int64_t c0, bool wvec, bool bvec,
                                            float (&w)[W][NB / sizeof(T)],
                                            float (&b)[NB / sizeof(T)]) {
    constexpr int V = NB / (int)sizeof(T);
    if (wvec) {
        const T* base = weight + c0 * W;
#pragma unroll
        for (int q = 0; q < W; ++q) {
            float f[V];
            unpack_raw<T, NB>(ldg_raw<NB>(base + q * V), f);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const int flat = q * V + i;  // = e * W + k
                w[flat % W][flat / W] = f[i];
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < V; ++e)
#pragma unroll
            for (int k = 0; k < W; ++k)
                w[k][e] = to_f32<T>(__ldg(weight + (c0 + e) * w_sd + k * w_sk));
    }
    if (bias == nullptr) {
#pragma unroll
        for (int e = 0; e < V; ++e) b[e] = 0.f;
    } else if (bvec) {
        unpack_raw<T, NB>(ldg_raw<NB>(bias + c0), b);
    } else {
#pragma unroll
        for (int e = 0; e < V; ++e) b[e] = to_f32<T>(__ldg(bias + (c0 + e) * bias_s));
    }
}

// The same filter kept as raw storage-type vectors (W tap-major vectors wt[k], lane e = channel
// c0 + e, plus the bias vector): a quarter of the registers of the fp32 form for bf16/fp16. Decode
// kernels use each weight once per row, so widening at use costs nothing extra.
template <typename T, int W, typename R>
__device__ __forceinline__ void load_filter_raw(const T* __restrict__ weight, int64_t w_sd,
                                                int64_t w_sk, const T* __restrict__ bias,
                                                int64_t bias_s, int64_t c0, bool wvec, bool bvec,
                                                R (&wt)[W], R& bt) {
    constexpr int V = (int)(sizeof(R) / sizeof(T));
    if (wvec) {
        R blk[W];
#pragma unroll
        for (int q = 0; q < W; ++q) blk[q] = __ldg(reinterpret_cast<const R*>(weight + c0 * W + q * V));
#pragma unroll
        for (int e = 0; e < V; ++e)
#pragma unroll
            for (int k = 0; k < W; ++k) {
                const int flat = e * W + k;
                set_lane<T>(wt[k], e, lane_of<T>(blk[flat / V], flat % V));
            }
    } else {
#pragma unroll
        for (int e = 0; e < V; ++e)
#pragma unroll
            for (int k = 0; k < W; ++k) set_lane<T>(wt[k], e, __ldg(weight + (c0 + e) * w_sd + k * w_sk));
    }
    if (bias == nullptr) {
        bt = R{};
    } else if (bvec) {
        bt = __ldg(reinterpret_cast<const R*>(bias + c0));
    } else {
#pragma unroll
        for (int e = 0; e < V; ++e) set_lane<T>(bt, e, __ldg(bias + (c0 + e) * bias_s));
    }
}

// Weights of one channel, for the scalar kernels.
template <typename T, int W>
__device__ __forceinline__ void load_filter1(const T* __restrict__ weight, int64_t w_sd,
                                             int64_t w_sk, const T* __restrict__ bias,
                                             int64_t bias_s, int64_t c, float (&w)[W],
                                             float& b) {
#pragma unroll
    for (int k = 0; k < W; ++k) w[k] = to_f32<T>(__ldg(weight + c * w_sd + k * w_sk));
    b = bias == nullptr ? 0.f : to_f32<T>(__ldg(bias + c * bias_s));
}

// ---------------------------------------------------------------------------------------------
// Host-side dispatch
// ---------------------------------------------------------------------------------------------

#define CC1D_DISPATCH_WIDTH(width, ...)            \
    switch (width) {                               \
        case 2: { constexpr int kW = 2; __VA_ARGS__; } break; \
        case 3: { constexpr int kW = 3; __VA_ARGS__; } break; \
        case 4: { constexpr int kW = 4; __VA_ARGS__; } break; \
        case 5: { constexpr int kW = 5; __VA_ARGS__; } break; \
        case 6: { constexpr int kW = 6; __VA_ARGS__; } break; \
        case 7: { constexpr int kW = 7; __VA_ARGS__; } break; \
        case 8: { constexpr int kW = 8; __VA_ARGS__; } break; \
        default: break;                            \
    }

#define CC1D_DISPATCH_DTYPE(dtype, ...)                              \
    switch (dtype) {                                                 \
        case CC1D_BF16: { using T = ::cc1d::bf16; __VA_ARGS__; } break; \
        case CC1D_F16: { using T = ::cc1d::f16; __VA_ARGS__; } break;   \
        case CC1D_F32: { using T = float; __VA_ARGS__; } break;         \
        default: break;                                              \
    }

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool host_aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool host_aligned32(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 31u) == 0; }

}  // namespace cc1d
