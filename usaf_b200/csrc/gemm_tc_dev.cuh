// Device helpers of the grouped int4 GEMM kernels (gemm_tc.cu): the int4 -> bf16 dequant
// of a 32-element half k-block with the overlay patch, packed fp32 pair
// arithmetic for the SwiGLU epilogues, and the tile decoder.
#pragma once
#include "tc_common.cuh"

namespace usaf {
namespace gemm_dev {
using namespace tc;

// time-bounded wait that ignores the abort flag (used to drain in-flight work)
static __device__ __forceinline__ void drain_wait(uint64_t *bar, uint32_t parity, int *err) {
    uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > kWaitBudgetNs) {
            atomicOr(err, USAF_ERR_WAIT_TIMEOUT);
            return;
        }
    }
}

// Dequantize 32 elements (16 pairs) from 4 code words in the repacked
// order: pair i = nibbles (i%4, i%4+4) of word i/4.  fp16(fp16(q*s)+z) per
// element (separately rounded multiply and add, the reference's rounding),
// then bf16.  SCALE_PER_ROW: pair i has its own scales and zeros, szr[2i] and
// szr[2i+1] as half2 (transposed weights); otherwise one (scale, zero) for the
// whole block.
// A pending trained coordinate at pair pj is blended in after the bf16
// conversion: m2 holds its bf16 value in both halves, hm selects the half.
// One compare and one predicated bit select per pair.
template <bool SCALE_PER_ROW>
static __device__ __forceinline__ void dequant16(uint4 codes, uint32_t szw, const uint32_t *szr, int pj,
                                          uint32_t m2, uint32_t hm, uint32_t (&r)[16]) {
    const uint32_t w[4] = {codes.x, codes.y, codes.z, codes.w};
    const __half2 magic = __half2half2(__ushort_as_half((unsigned short)0x6400));
    __half2 s2 = __half2half2(__ushort_as_half((unsigned short)(szw & 0xFFFF)));
    __half2 z2 = __half2half2(__ushort_as_half((unsigned short)(szw >> 16)));
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        uint32_t u = ((w[i >> 2] >> (4 * (i & 3))) & 0x000F000Fu) | 0x64006400u;
        __half2 c = __hsub2(*reinterpret_cast<__half2 *>(&u), magic);
        if (SCALE_PER_ROW) {
            // the pair's scales and zeros arrive packed as half2 words
            uint32_t su = szr[2 * i], zu = szr[2 * i + 1];
            s2 = *reinterpret_cast<__half2 *>(&su);
            z2 = *reinterpret_cast<__half2 *>(&zu);
        }
        __half2 v = __hadd2_rn(__hmul2_rn(c, s2), z2);
        float2 f = __half22float2(v);
        __nv_bfloat162 bb = __floats2bfloat162_rn(f.x, f.y);
        uint32_t rv = *reinterpret_cast<uint32_t *>(&bb);
        asm("{\n .reg .pred p;\n setp.eq.s32 p, %1, %2;\n @p lop3.b32 %0, %0, %3, %4, 0xD8;\n}\n"
            : "+r"(rv)
            : "r"(pj), "r"(i), "r"(m2), "r"(hm));
        r[i] = rv;
    }
}

// slow path for a second trained coordinate in the same 32-wide block: one
// compare and one predicated bit select (lop3 "c ? b : a") per register keeps
// r[] in registers
static __device__ __forceinline__ void patch_elem16(uint32_t (&r)[16], int c, uint32_t vb) {
    const uint32_t pi = (uint32_t)c >> 1;
    const uint32_t v2 = vb | (vb << 16);
    const uint32_t hm = (c & 1) ? 0xFFFF0000u : 0x0000FFFFu;
#pragma unroll
    for (int i = 0; i < 16; ++i)
        asm("{\n .reg .pred p;\n setp.eq.u32 p, %1, %2;\n @p lop3.b32 %0, %0, %3, %4, 0xD8;\n}\n"
            : "+r"(r[i])
            : "r"(pi), "r"((uint32_t)i), "r"(v2), "r"(hm));
}

// packed fp32 pairs (sm_100 f32x2 arithmetic, round to nearest even)
static __device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
static __device__ __forceinline__ float f2_lo(uint64_t a) { return __uint_as_float((uint32_t)a); }
static __device__ __forceinline__ float f2_hi(uint64_t a) { return __uint_as_float((uint32_t)(a >> 32)); }
static __device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
static __device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
static __device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// bf16 pair (low half = first element) <-> packed fp32 pair
static __device__ __forceinline__ uint64_t bf2_to_f2(uint32_t w) {
    return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
static __device__ __forceinline__ uint32_t f2_to_bf2(uint64_t a) {
    const __nv_bfloat162 r = __floats2bfloat162_rn(f2_lo(a), f2_hi(a));
    return *reinterpret_cast<const uint32_t *>(&r);
}

static __device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// Tile `tile` of the grouped problem: expert e, first slot t0 inside the
// expert's segment and ntok slots.  An expert with cnt slots is cut into
// ntt = tile_off[e+1] - tile_off[e] tiles of equal size rounded up to ALIGN.
template <int ALIGN = 16>
static __device__ __forceinline__ void decode_tile(const int *tile_off, const int *cnts, int E, int tile,
                                            int &e, int &t0, int &ntok) {
    int lo = 0, hi = E;  // first expert with tile_off[e+1] > tile
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (tile_off[mid + 1] > tile) hi = mid;
        else lo = mid + 1;
    }
    e = lo;
    int cnt = cnts[e];
    int ntt = tile_off[e + 1] - tile_off[e];
    int tt = tile - tile_off[e];
    int per = (((cnt + ntt - 1) / ntt) + ALIGN - 1) & ~(ALIGN - 1);
    t0 = tt * per;
    ntok = min(per, cnt - t0);
}

}  // namespace gemm_dev
}  // namespace usaf
