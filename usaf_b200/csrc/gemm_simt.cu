// Grouped expert GEMMs over int4 weights on CUDA cores, and the SwiGLU
// element-wise forward/backward.
//
// This is the fp32 path (the CPU-runnable configuration computes in fp32,
// which tensor cores would round to tf32).  The bf16 path uses the tcgen05
// kernels in gemm_tc.cu.  Weights are dequantized into shared memory as
// fp16(fp16(q*s)+z) converted to the compute dtype, and trained coordinates
// are patched from the overlay (CSR for W, CSC for W^T) before use, which is
// the effective weight of usaf/moe_loader.py:241-247.
#include "common.cuh"

namespace usaf {

// m-tile -> (expert, first row inside the expert's segment)
__device__ __forceinline__ bool find_mtile(const usaf_route_plan &pl, int tile, int bm, int &e_out,
                                           int &m0_out) {
    int acc = 0;
    for (int e = 0; e < pl.E; ++e) {
        int n = (pl.expert_cnt[e] + bm - 1) / bm;
        if (tile < acc + n) {
            e_out = e;
            m0_out = (tile - acc) * bm;
            return true;
        }
        acc += n;
    }
    return false;
}

__device__ __forceinline__ int lower_bound_i32(const int32_t *a, int lo, int hi, int key) {
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (a[mid] < key) lo = mid + 1;
        else hi = mid;
    }
    return lo;
}

// out[s][n] = sum_k A[s][k] * W(e; n, k) with W(e;n,k) = TRANS ? Wst[e][k][n] : Wst[e][n][k]
template <typename Act, bool TRANS>
__global__ void __launch_bounds__(256) grouped_gemm_simt(usaf_route_plan pl, usaf_qweight w,
                                                         const Act *__restrict__ A, int K, int N,
                                                         Act *__restrict__ out, int ldo) {
    constexpr int BM = 64, BN = 64, BK = 16;
    __shared__ float As[BK][BM + 4];
    __shared__ float Ws[BK][BN + 4];
    __shared__ int s_e, s_m0;
    if (threadIdx.x == 0) {
        int e, m0;
        if (!find_mtile(pl, blockIdx.y, BM, e, m0)) e = -1, m0 = 0;
        s_e = e;
        s_m0 = m0;
    }
    __syncthreads();
    const int e = s_e, m0 = s_m0;
    if (e < 0) return;
    const int seg0 = pl.expert_off[e], cnt = pl.expert_cnt[e];
    const int n0 = blockIdx.x * BN;
    const int R = w.R, C = w.C;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
        for (int i = threadIdx.x; i < BK * BM; i += 256) {
            int kk = i % BK, mm = i / BK;
            int m = m0 + mm, k = k0 + kk;
            As[kk][mm] = (m < cnt && k < K) ? to_f(A[(int64_t)(seg0 + m) * K + k]) : 0.0f;
        }
        for (int i = threadIdx.x; i < BK * BN; i += 256) {
            int kk, nn;
            if (TRANS) { nn = i % BN; kk = i / BN; }   // storage row = k, consecutive n contiguous
            else { kk = i % BK; nn = i / BK; }
            int n = n0 + nn, k = k0 + kk;
            float v = 0.0f;
            if (n < N && k < K) {
                int64_t flat = TRANS ? (((int64_t)e * R + k) * C + n) : (((int64_t)e * R + n) * C + k);
                v = round_to<Act>(qweight_base(w, flat));
            }
            Ws[kk][nn] = v;
        }
        __syncthreads();
        if (w.n_ov > 0 && threadIdx.x < BN) {
            int n = n0 + threadIdx.x;
            if (n < N) {
                const int half = (k0 >> 5) & 1;   // the 16-wide k tile lies in one 32-wide half
                if (!TRANS) {
                    int r = (e * R + n) * 2 + half;
                    int b = w.row_ptr[r], en = w.row_ptr[r + 1];
                    for (int j = lower_bound_i32(w.col, b, en, k0); j < en && w.col[j] < k0 + BK; ++j)
                        Ws[w.col[j] - k0][threadIdx.x] = w.val[j];
                } else {
                    int c = (e * C + n) * 2 + half;
                    int b = w.colT_ptr[c], en = w.colT_ptr[c + 1];
                    for (int j = lower_bound_i32(w.rowT, b, en, k0); j < en && w.rowT[j] < k0 + BK; ++j)
                        Ws[w.rowT[j] - k0][threadIdx.x] = w.valT[j];
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Ws[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        int m = m0 + ty * 4 + i;
        if (m >= cnt) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int n = n0 + tx * 4 + j;
            if (n < N) out[(int64_t)(seg0 + m) * ldo + n] = from_f<Act>(acc[i][j]);
        }
    }
}

// silu as the reference's CPU kernel: x / (1 + exp(-x)) in fp32
__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// h = act(act(silu(gate)) * up); gu is [P, 2I] with gate = [:, :I], up = [:, I:]
template <typename Act>
__global__ void swiglu_fwd_kernel(const int32_t *__restrict__ n_pairs, const Act *__restrict__ gu,
                                  int I, Act *__restrict__ h) {
    int64_t total = (int64_t)(*n_pairs) * I;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t s = i / I;
        int c = (int)(i - s * I);
        float g = to_f(gu[s * 2 * I + c]);
        float u = to_f(gu[s * 2 * I + I + c]);
        float sg = round_to<Act>(silu_f(g));
        h[i] = from_f<Act>(__fmul_rn(sg, u));
    }
}

// autograd of h = silu(gate) * up (each op rounded to the activation dtype):
//   ds = act(dh*u), du = act(dh*s), dgate = act(ds * sig * (1 + g*(1-sig)))
template <typename Act>
__device__ __forceinline__ void swiglu_bwd_elem(float dh, float g, float u, float &dg, float &du) {
    float sg = round_to<Act>(silu_f(g));
    float ds = round_to<Act>(__fmul_rn(dh, u));
    du = round_to<Act>(__fmul_rn(dh, sg));
    float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    float t = __fadd_rn(1.0f, __fmul_rn(g, __fsub_rn(1.0f, sig)));
    dg = round_to<Act>(__fmul_rn(__fmul_rn(ds, sig), t));
}

template <typename Act>
__global__ void swiglu_bwd_kernel(const int32_t *__restrict__ n_pairs, const Act *dh, int ldh,
                                  const Act *__restrict__ gu, int I, Act *dgu) {
    int64_t total = (int64_t)(*n_pairs) * I;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t s = i / I;
        int c = (int)(i - s * I);
        float g = to_f(gu[s * 2 * I + c]);
        float u = to_f(gu[s * 2 * I + I + c]);
        float dg, du;
        swiglu_bwd_elem<Act>(to_f(dh[s * ldh + c]), g, u, dg, du);
        dgu[s * 2 * I + c] = from_f<Act>(dg);
        dgu[s * 2 * I + I + c] = from_f<Act>(du);
    }
}

template <typename Act, bool TRANS>
int launch_simt(const usaf_route_plan *pl, const usaf_qweight *w, const Act *A, int K, int N,
                Act *out, int ldo, cudaStream_t st) {
    int tiles = (pl->P_cap + 63) / 64 + pl->E;
    dim3 grid(cdiv(N, 64), tiles);
    grouped_gemm_simt<Act, TRANS><<<grid, 256, 0, st>>>(*pl, *w, A, K, N, out, ldo);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

// explicit instantiations used by the C ABI in expert_api.cu
template int launch_simt<float, false>(const usaf_route_plan *, const usaf_qweight *, const float *, int, int, float *, int, cudaStream_t);
template int launch_simt<float, true>(const usaf_route_plan *, const usaf_qweight *, const float *, int, int, float *, int, cudaStream_t);
template int launch_simt<__nv_bfloat16, false>(const usaf_route_plan *, const usaf_qweight *, const __nv_bfloat16 *, int, int, __nv_bfloat16 *, int, cudaStream_t);
template int launch_simt<__nv_bfloat16, true>(const usaf_route_plan *, const usaf_qweight *, const __nv_bfloat16 *, int, int, __nv_bfloat16 *, int, cudaStream_t);

template <typename Act>
int launch_swiglu_fwd(const usaf_route_plan *pl, const Act *gu, int I, Act *h, cudaStream_t st) {
    swiglu_fwd_kernel<Act><<<148 * 16, 256, 0, st>>>(pl->n_pairs, gu, I, h);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
template <typename Act>
int launch_swiglu_bwd(const usaf_route_plan *pl, const Act *dh, int ldh, const Act *gu, int I,
                      Act *dgu, cudaStream_t st) {
    swiglu_bwd_kernel<Act><<<148 * 16, 256, 0, st>>>(pl->n_pairs, dh, ldh, gu, I, dgu);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
template int launch_swiglu_fwd<float>(const usaf_route_plan *, const float *, int, float *, cudaStream_t);
template int launch_swiglu_fwd<__nv_bfloat16>(const usaf_route_plan *, const __nv_bfloat16 *, int, __nv_bfloat16 *, cudaStream_t);
template int launch_swiglu_bwd<float>(const usaf_route_plan *, const float *, int, const float *, int, float *, cudaStream_t);
template int launch_swiglu_bwd<__nv_bfloat16>(const usaf_route_plan *, const __nv_bfloat16 *, int, const __nv_bfloat16 *, int, __nv_bfloat16 *, cudaStream_t);

}  // namespace usaf
