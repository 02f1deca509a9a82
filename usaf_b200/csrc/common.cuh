// Shared device helpers for the usaf_b200 kernels (sm_100a).
#pragma once
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <type_traits>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/usaf_b200.h"

#define USAF_CHECK_LAUNCH()                                         \
    do {                                                            \
        if (cudaPeekAtLastError() != cudaSuccess) {                 \
            (void)cudaGetLastError();                               \
            return USAF_ECUDA;                                      \
        }                                                           \
    } while (0)

#define USAF_REQUIRE(cond) \
    do {                   \
        if (!(cond)) return USAF_EINVAL; \
    } while (0)

namespace usaf {

static inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }
static inline unsigned cdiv(int64_t a, int64_t b) { return (unsigned)((a + b - 1) / b); }

// Plans whose pair capacity is at most this many pairs per expert (about half
// of it routed: batches of up to ~32 tokens per expert) take the CUDA-core
// expert-weight gradient kernel: the tensor-core SDDMM spends a fixed cost
// per 128 x 256 tile whatever the expert's slot count (C2 layer, measured:
// T = 256 459 -> 225 us, T = 512 460 -> 280 us, T = 1 213 -> 74 us).
constexpr int kSimtMaxPairsPerExpert = 64;
static inline bool small_plan(const usaf_route_plan *pl) {
    return (int64_t)pl->P_cap <= (int64_t)kSimtMaxPairsPerExpert * pl->E;
}

// ---- activation dtype plumbing -------------------------------------------
// Values move through fp32 registers; `Act` is the storage type.
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// round an fp32 value to the activation dtype and back (the reference stores
// intermediates in the activation dtype)
template <typename T> __device__ __forceinline__ float round_to(float v) { return to_f(from_f<T>(v)); }

// ---- int4 codes -----------------------------------------------------------
// fp16(fp16(q*s) + z): separately rounded multiply and add, as the
// reference's half-precision elementwise ops (usaf/quantization.py:129).
__device__ __forceinline__ __half dq_half(uint32_t code, __half s, __half z) {
    __half qh = __ushort2half_rn((unsigned short)code);  // exact, 0..15
    __half p = __hmul_rn(qh, s);
    return __hadd_rn(p, z);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Effective weight of storage element (e, r, c) of a projection, looked up
// through the CSR overlay when the coordinate is trained.  Used by the
// generic (SIMT) paths; the tensor-core kernels patch tiles instead.
__device__ __forceinline__ float qweight_base(const usaf_qweight &w, int64_t flat) {
    uint8_t byte = (uint8_t)w.q[flat >> 1];
    uint32_t code = (flat & 1) ? (byte >> 4) : (byte & 0xF);
    int64_t g = flat / w.group_size;
    __half s = __ushort_as_half(w.s[g]);
    __half z = __ushort_as_half(w.z[g]);
    return __half2float(dq_half(code, s, z));
}

}  // namespace usaf
