// Expert-weight gradients at the selected coordinates only (SDDMM), and the
// dense per-expert |gradient| used by the importance pass.
//
// The reference materialises the dense per-expert gradient dW_e = gout_e^T gin_e
// (F.linear backward, rounded to the parameter dtype), then gathers the
// active coordinates and index-adds them into compact fp32 vectors
// (usaf/qwen3moe_dml.py:43-56, usaf/moe_loader.py:564-578).  Here only the
// selected coordinates are computed: for coordinate (e, r, c)
//   g = dtype( sum over expert e's slots s of gout[s, r] * gin[s, c] )
// in a fixed slot order (deterministic), then compact[pos] += scale * g.
//
// Work item = (expert, block of 256 storage rows); one thread per row walks
// that row's CSR entries.  Token chunks of gin (all columns) and gout (the
// block's rows) are staged transposed in shared memory so every coordinate
// reads contiguous token runs; per-chunk partial sums go to an fp32 scratch
// vector owned one-to-one by coordinates (no atomics).
#include "common.cuh"

namespace usaf {

constexpr int kRowsPerBlock = 256;

template <typename Act, int TC>
__global__ void __launch_bounds__(kRowsPerBlock) sddmm_kernel(
    usaf_route_plan pl, usaf_qweight w, const Act *__restrict__ gout,
    const Act *__restrict__ gin, const int32_t *__restrict__ csr_to_compact, float scale,
    float *__restrict__ compact, float *__restrict__ scratch) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Act *ginT = reinterpret_cast<Act *>(smem_raw);              // [C][TC]
    Act *goutT = ginT + (size_t)w.C * TC;                       // [256][TC]
    const int e = blockIdx.y;
    const int R = w.R, C = w.C;
    const int cnt = pl.expert_cnt[e];
    if (cnt == 0) return;
    const int seg0 = pl.expert_off[e];
    const int r_local = threadIdx.x;
    const int r = blockIdx.x * kRowsPerBlock + r_local;
    const int rows_here = min(kRowsPerBlock, R - (int)blockIdx.x * kRowsPerBlock);
    int jb = 0, je = 0;
    if (r < R) {
        jb = w.row_ptr[(int64_t)e * R + r];
        je = w.row_ptr[(int64_t)e * R + r + 1];
    }
    for (int t0 = 0; t0 < cnt; t0 += TC) {
        int tn = min(TC, cnt - t0);
        __syncthreads();
        for (int i = threadIdx.x; i < TC * C; i += blockDim.x) {
            int t = i / C, c = i - t * C;
            ginT[(size_t)c * TC + t] =
                t < tn ? gin[(int64_t)(seg0 + t0 + t) * C + c] : from_f<Act>(0.0f);
        }
        for (int i = threadIdx.x; i < TC * rows_here; i += blockDim.x) {
            int t = i / rows_here, rr = i - t * rows_here;
            goutT[(size_t)rr * TC + t] =
                t < tn ? gout[(int64_t)(seg0 + t0 + t) * R + blockIdx.x * kRowsPerBlock + rr]
                       : from_f<Act>(0.0f);
        }
        __syncthreads();
        if (r < R && jb < je) {
            float a[TC];
#pragma unroll
            for (int t = 0; t < TC; ++t) a[t] = to_f(goutT[(size_t)r_local * TC + t]);
            for (int j = jb; j < je; ++j) {
                const Act *col = ginT + (size_t)w.col[j] * TC;
                float d = 0.0f;
#pragma unroll
                for (int t = 0; t < TC; ++t) d = fmaf(a[t], to_f(col[t]), d);
                scratch[j] = t0 == 0 ? d : __fadd_rn(scratch[j], d);
            }
        }
    }
    if (r < R) {
        for (int j = jb; j < je; ++j) {
            int pos = csr_to_compact[j];
            compact[pos] = __fadd_rn(compact[pos], __fmul_rn(scale, round_to<Act>(scratch[j])));
        }
    }
}

// dense |dW_e| for the importance pass: out[e][r][c] = |dtype(sum_s gout[s,r] gin[s,c])|
template <typename Act>
__global__ void __launch_bounds__(256) dense_dw_kernel(usaf_route_plan pl, int R, int C,
                                                       const Act *__restrict__ gout,
                                                       const Act *__restrict__ gin,
                                                       float *__restrict__ out) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const int e = blockIdx.z;
    const int cnt = pl.expert_cnt[e], seg0 = pl.expert_off[e];
    const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < cnt; k0 += 16) {
        for (int i = threadIdx.x; i < 16 * 64; i += 256) {
            int mm = i & 63, kk = i >> 6;
            int k = k0 + kk;
            As[kk][mm] = (k < cnt && r0 + mm < R) ? to_f(gout[(int64_t)(seg0 + k) * R + r0 + mm]) : 0.0f;
            Bs[kk][mm] = (k < cnt && c0 + mm < C) ? to_f(gin[(int64_t)(seg0 + k) * C + c0 + mm]) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int rr = r0 + ty * 4 + i, cc = c0 + tx * 4 + j;
            if (rr < R && cc < C) out[((int64_t)e * R + rr) * C + cc] = fabsf(round_to<Act>(acc[i][j]));
        }
}

template <typename Act>
static int sddmm_launch(const usaf_route_plan *pl, const usaf_qweight *w, const Act *gout,
                        const Act *gin, const int32_t *c2c, float scale, float *compact,
                        float *scratch, cudaStream_t st) {
    const size_t budget = 200 * 1024;
    dim3 grid(cdiv(w->R, kRowsPerBlock), w->E);
    auto bytes = [&](int tc) { return ((size_t)w->C + kRowsPerBlock) * tc * sizeof(Act); };
#define SDDMM_TRY(TC)                                                                            \
    if (bytes(TC) <= budget) {                                                                   \
        cudaFuncSetAttribute(sddmm_kernel<Act, TC>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                             (int)bytes(TC));                                                    \
        sddmm_kernel<Act, TC><<<grid, kRowsPerBlock, bytes(TC), st>>>(*pl, *w, gout, gin, c2c,   \
                                                                      scale, compact, scratch);  \
        USAF_CHECK_LAUNCH();                                                                     \
        return USAF_OK;                                                                          \
    }
    SDDMM_TRY(32)
    SDDMM_TRY(16)
    SDDMM_TRY(8)
#undef SDDMM_TRY
    return USAF_EUNSUPPORTED;
}

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_sparse_dw(const usaf_route_plan *plan, const usaf_qweight *w, const void *gout,
                              const void *gin, int32_t dtype, const int32_t *csr_to_compact,
                              float scale, float *compact, float *scratch, void *stream) {
    USAF_REQUIRE(plan && w && gout && gin);
    if (w->n_ov == 0) return USAF_OK;
    USAF_REQUIRE(csr_to_compact && compact && scratch && w->row_ptr && w->col);
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case USAF_F32: return sddmm_launch<float>(plan, w, (const float *)gout, (const float *)gin, csr_to_compact, scale, compact, scratch, st);
        case USAF_BF16: return sddmm_launch<__nv_bfloat16>(plan, w, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin, csr_to_compact, scale, compact, scratch, st);
        default: return USAF_EINVAL;
    }
}

extern "C" int usaf_expert_dense_dw(const usaf_route_plan *plan, int32_t R, int32_t C,
                                    const void *gout, const void *gin, int32_t dtype, float *out,
                                    void *stream) {
    USAF_REQUIRE(plan && gout && gin && out && R >= 1 && C >= 1);
    cudaStream_t st = as_stream(stream);
    dim3 grid(cdiv(C, 64), cdiv(R, 64), plan->E);
    switch (dtype) {
        case USAF_F32: dense_dw_kernel<float><<<grid, 256, 0, st>>>(*plan, R, C, (const float *)gout, (const float *)gin, out); break;
        case USAF_BF16: dense_dw_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(*plan, R, C, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin, out); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
