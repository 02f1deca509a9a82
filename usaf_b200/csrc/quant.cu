// int4 (usaf.quantization layout) dequantize / quantize kernels.
//
// Layout (usaf/quantization.py:21-85): flat groups of `gs` consecutive
// elements, codes packed two per byte (even element in the low nibble),
// fp16 scale and zero per group.  Dequantization is the reference's fp16
// arithmetic, fp16(fp16(q*s)+z), done with separately rounded half multiply
// and add so it is bit-exact.  Both kernels are HBM-bound streaming kernels:
// 16-byte loads of packed codes, one group's scale/zero per 8 bytes.
#include "common.cuh"

namespace usaf {

// 16 elements (8 packed bytes) per thread; all 16 share one group because
// gs % 16 == 0 is required on this path.
template <typename Out>
__global__ void __launch_bounds__(256) dequant_vec16(const uint2 *__restrict__ q,
                                                     const __half *__restrict__ s,
                                                     const __half *__restrict__ z,
                                                     int64_t n16, int gs,
                                                     Out *__restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i < n16; i += (int64_t)gridDim.x * blockDim.x) {
        uint2 p = __ldg(q + i);
        int64_t g = (i * 16) / gs;
        __half2 s2 = __half2half2(s[g]);
        __half2 z2 = __half2half2(z[g]);
        uint32_t w[2] = {p.x, p.y};
        __half2 h[8];
#pragma unroll
        for (int b = 0; b < 2; ++b) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t byte = (w[b] >> (8 * j)) & 0xFF;
                __half2 c = __halves2half2(__ushort2half_rn((unsigned short)(byte & 0xF)),
                                           __ushort2half_rn((unsigned short)(byte >> 4)));
                h[b * 4 + j] = __hadd2_rn(__hmul2_rn(c, s2), z2);
            }
        }
        if constexpr (sizeof(Out) == 2 && std::is_same<Out, __half>::value) {
            uint4 *o = reinterpret_cast<uint4 *>(out + i * 16);
            const uint4 *src = reinterpret_cast<const uint4 *>(h);
            o[0] = src[0];
            o[1] = src[1];
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                out[i * 16 + 2 * j] = from_f<Out>(__low2float(h[j]));
                out[i * 16 + 2 * j + 1] = from_f<Out>(__high2float(h[j]));
            }
        }
    }
}

// generic element-wise path (any even group size, any numel)
template <typename Out>
__global__ void dequant_scalar(const int8_t *__restrict__ q, const __half *__restrict__ s,
                               const __half *__restrict__ z, int64_t numel, int gs,
                               Out *__restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i < numel; i += (int64_t)gridDim.x * blockDim.x) {
        uint8_t byte = (uint8_t)q[i >> 1];
        uint32_t code = (i & 1) ? (byte >> 4) : (byte & 0xF);
        int64_t g = i / gs;
        out[i] = from_f<Out>(__half2float(dq_half(code, s[g], z[g])));
    }
}
template <>
__global__ void dequant_scalar<__half>(const int8_t *__restrict__ q, const __half *__restrict__ s,
                                       const __half *__restrict__ z, int64_t numel, int gs,
                                       __half *__restrict__ out) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i < numel; i += (int64_t)gridDim.x * blockDim.x) {
        uint8_t byte = (uint8_t)q[i >> 1];
        uint32_t code = (i & 1) ? (byte >> 4) : (byte & 0xF);
        int64_t g = i / gs;
        out[i] = dq_half(code, s[g], z[g]);
    }
}

// One warp per group: min/max, fp32 scale = (max-min)/15 clamped to 1e-12,
// codes = clamp(rint((x-min)/scale), 0, 15), packed even|odd<<4.
// Elements past numel are the reference's zero padding (:54-55).
template <typename In>
__global__ void quant_groups(const In *__restrict__ x, int64_t numel, int egs, int64_t ngroups,
                             uint8_t *__restrict__ q, __half *__restrict__ s,
                             __half *__restrict__ z) {
    int lane = threadIdx.x & 31;
    int64_t g = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int64_t gstride = ((int64_t)gridDim.x * blockDim.x) >> 5;
    int half_len = (egs + 1) / 2;
    for (; g < ngroups; g += gstride) {
        int64_t base = g * egs;
        float mn = INFINITY, mx = -INFINITY;
        for (int j = lane; j < egs; j += 32) {
            int64_t idx = base + j;
            float v = idx < numel ? to_f(x[idx]) : 0.0f;
            mn = fminf(mn, v);
            mx = fmaxf(mx, v);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        float scale = __fdiv_rn(__fsub_rn(mx, mn), 15.0f);
        scale = fmaxf(scale, 1e-12f);
        for (int b = lane; b < half_len; b += 32) {
            uint32_t codes[2] = {0, 0};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                int j = 2 * b + h;
                if (j < egs) {
                    int64_t idx = base + j;
                    float v = idx < numel ? to_f(x[idx]) : 0.0f;
                    float qf = rintf(__fdiv_rn(__fsub_rn(v, mn), scale));
                    qf = fminf(fmaxf(qf, 0.0f), 15.0f);
                    codes[h] = (uint32_t)qf;
                }
            }
            q[g * half_len + b] = (uint8_t)(codes[0] | (codes[1] << 4));
        }
        if (lane == 0) {
            s[g] = __float2half_rn(scale);
            z[g] = __float2half_rn(mn);
        }
    }
}

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_dequant_int4(const void *q, const void *s, const void *z, int64_t numel,
                                 int32_t group_size, int32_t out_dtype, void *out,
                                 void *stream) {
    USAF_REQUIRE(q && s && z && out && numel >= 1 && group_size >= 1);
    int64_t egs = group_size < numel ? group_size : numel;
    int64_t ng = (numel + egs - 1) / egs;
    if (egs % 2 != 0 && ng > 1) return USAF_EUNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    const __half *sh = reinterpret_cast<const __half *>(s);
    const __half *zh = reinterpret_cast<const __half *>(z);
    bool vec = (egs % 16 == 0) && (numel % 16 == 0) &&
               ((reinterpret_cast<uintptr_t>(q) & 7) == 0) &&
               ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
    int64_t n16 = numel / 16;
    unsigned grid_v = (unsigned)std::min<int64_t>((n16 + 255) / 256, 148 * 16);
    unsigned grid_s = (unsigned)std::min<int64_t>((numel + 255) / 256, 148 * 32);
    switch (out_dtype) {
        case USAF_F16:
            if (vec) dequant_vec16<__half><<<grid_v, 256, 0, st>>>((const uint2 *)q, sh, zh, n16, (int)egs, (__half *)out);
            else dequant_scalar<__half><<<grid_s, 256, 0, st>>>((const int8_t *)q, sh, zh, numel, (int)egs, (__half *)out);
            break;
        case USAF_F32:
            if (vec) dequant_vec16<float><<<grid_v, 256, 0, st>>>((const uint2 *)q, sh, zh, n16, (int)egs, (float *)out);
            else dequant_scalar<float><<<grid_s, 256, 0, st>>>((const int8_t *)q, sh, zh, numel, (int)egs, (float *)out);
            break;
        case USAF_BF16:
            if (vec) dequant_vec16<__nv_bfloat16><<<grid_v, 256, 0, st>>>((const uint2 *)q, sh, zh, n16, (int)egs, (__nv_bfloat16 *)out);
            else dequant_scalar<__nv_bfloat16><<<grid_s, 256, 0, st>>>((const int8_t *)q, sh, zh, numel, (int)egs, (__nv_bfloat16 *)out);
            break;
        default:
            return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_quant_int4(const void *x, int32_t x_dtype, int64_t numel, int32_t group_size,
                               void *q, void *s, void *z, void *stream) {
    USAF_REQUIRE(x && q && s && z && numel >= 1 && group_size >= 1);
    int64_t egs = group_size < numel ? group_size : numel;
    int64_t ng = (numel + egs - 1) / egs;
    cudaStream_t st = as_stream(stream);
    unsigned grid = (unsigned)std::min<int64_t>((ng * 32 + 255) / 256, 148 * 32);
    auto *qq = reinterpret_cast<uint8_t *>(q);
    auto *ss = reinterpret_cast<__half *>(s);
    auto *zz = reinterpret_cast<__half *>(z);
    switch (x_dtype) {
        case USAF_F32: quant_groups<float><<<grid, 256, 0, st>>>((const float *)x, numel, (int)egs, ng, qq, ss, zz); break;
        case USAF_BF16: quant_groups<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16 *)x, numel, (int)egs, ng, qq, ss, zz); break;
        case USAF_F16: quant_groups<__half><<<grid, 256, 0, st>>>((const __half *)x, numel, (int)egs, ng, qq, ss, zz); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

// ---- column-major copy for the backward GEMMs ------------------------------
namespace usaf {
// qT: storage column c of expert e, codes along rows r, 8 rows per 32-bit
// word in the dequant order e0 e2 e4 e6 | e1 e3 e5 e7 (see usaf_int4_repack)
__global__ void int4_transpose_codes(const uint8_t *__restrict__ q, int E, int R, int C,
                                     uint32_t *__restrict__ qT) {
    const int64_t total = (int64_t)E * C * (R / 8);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r8 = i % (R / 8);
        int64_t ec = i / (R / 8);
        int64_t c = ec % C, e = ec / C;
        uint32_t out = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            int64_t f = (e * R + r8 * 8 + k) * C + c;
            uint32_t code = (q[f >> 1] >> ((f & 1) * 4)) & 0xF;
            int slot = (k & 1) ? 4 + (k >> 1) : (k >> 1);
            out |= code << (4 * slot);
        }
        qT[i] = out;
    }
}
// Per (expert, column group), two words per pair of rows 2p, 2p+1:
// szT[(e*(C/gs) + cb)*R + 2p]     = s[row 2p] | s[row 2p+1] << 16,
// szT[(e*(C/gs) + cb)*R + 2p + 1] = z[row 2p] | z[row 2p+1] << 16
// (the half2 scale and zero operands of a dequantized element pair as they are)
__global__ void int4_transpose_scales(const uint16_t *__restrict__ s, const uint16_t *__restrict__ z,
                                      int E, int R, int C, int gs, uint32_t *__restrict__ szT) {
    const int ncb = C / gs;
    const int64_t total = (int64_t)E * ncb * R;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i % R;
        const int64_t ecb = i / R;
        const int64_t cb = ecb % ncb, e = ecb / ncb;
        const int64_t r0 = r & ~(int64_t)1;
        const uint16_t *src = (r & 1) ? z : s;
        szT[i] = (uint32_t)src[(e * R + r0) * ncb + cb] | ((uint32_t)src[(e * R + r0 + 1) * ncb + cb] << 16);
    }
}
}  // namespace usaf

extern "C" int usaf_int4_transpose(const void *q, const void *s, const void *z, int32_t E, int32_t R,
                                   int32_t C, int32_t group_size, void *qT, void *szT, void *stream) {
    USAF_REQUIRE(q && s && z && qT && szT && E >= 1 && R >= 2 && C >= 1 && group_size >= 1);
    if (R % 8 || C % group_size) return USAF_EUNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    unsigned grid = 148 * 16;
    int4_transpose_codes<<<grid, 256, 0, st>>>((const uint8_t *)q, E, R, C, (uint32_t *)qT);
    int4_transpose_scales<<<grid, 256, 0, st>>>((const uint16_t *)s, (const uint16_t *)z, E, R, C,
                                                group_size, (uint32_t *)szT);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

// ---- dequant-friendly nibble order for the tensor-core producers ------------
// Within every 32-bit word (8 consecutive elements e0..e7) the codes are
// stored as  e0 e2 e4 e6 | e1 e3 e5 e7  (nibble k at bits 4k), so that
// ((w >> 4i) & 0x000F000F) holds the pair (e_2i, e_2i+1) in the two fp16
// lanes -- one shift and one LOP3 per pair with the 0x6400 magic number.
namespace usaf {
__device__ __forceinline__ uint32_t repack_word(uint32_t w) {
    uint32_t out = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t byte = (w >> (8 * i)) & 0xFF;      // e_2i (low) | e_2i+1 (high)
        out |= (byte & 0xF) << (4 * i);
        out |= (byte >> 4) << (16 + 4 * i);
    }
    return out;
}
__global__ void int4_repack_words(const uint32_t *__restrict__ in, int64_t nwords,
                                  uint32_t *__restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nwords;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = repack_word(in[i]);
}
}  // namespace usaf

extern "C" int usaf_int4_repack(const void *q, int64_t numel, void *qp, void *stream) {
    USAF_REQUIRE(q && qp && numel >= 0);
    if (numel % 8) return USAF_EUNSUPPORTED;
    if (numel == 0) return USAF_OK;
    int4_repack_words<<<148 * 16, 256, 0, as_stream(stream)>>>((const uint32_t *)q, numel / 8,
                                                                (uint32_t *)qp);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
