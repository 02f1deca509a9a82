// Router of the Qwen3-MoE block (usaf/qwen3moe_dml.py:72-83) and its backward.
//
// Forward: logits = X W_r^T (fp32 accumulate, rounded to the activation
// dtype), fp32 softmax, k-th largest probability (counting duplicates) as the
// threshold, mask = probs >= threshold, renormalised weights cast to the
// activation dtype.  One warp per token for everything after the logits.
// Backward: per token through renorm + mask + softmax (the autograd of the
// same lines), then dW_r = dlogits^T X and dX_r = dlogits W_r.
#include "common.cuh"

namespace usaf {

// ---- dense tile GEMM on CUDA cores -----------------------------------------
// C[M,N] (+)= sum_k A(m,k) B(n,k); A and B are read through functors so the
// same tile routine serves logits (X W^T), dX_r (dL W) and dW_r (dL^T X).
// 64x64 tile, BK = 16, 256 threads, 4x4 per thread, fixed k order.
template <typename LA, typename LB, typename ST>
__device__ __forceinline__ void tile_gemm_64x64(int M, int N, int K, int m0, int n0, LA la, LB lb,
                                                ST st) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 16 * 64; i += 256) {
            int kk = i & 15, mm = i >> 4;
            int gm = m0 + mm, gk = k0 + kk;
            As[kk][mm] = (gm < M && gk < K) ? la(gm, gk) : 0.0f;
            int gn = n0 + mm;
            Bs[kk][mm] = (gn < N && gk < K) ? lb(gn, gk) : 0.0f;
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
            int gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
            if (gm < M && gn < N) st(gm, gn, acc[i][j]);
        }
}

template <typename Act>
__global__ void __launch_bounds__(256) logits_kernel(const Act *__restrict__ x,
                                                     const Act *__restrict__ w, int T, int H,
                                                     int E, float *__restrict__ logits) {
    tile_gemm_64x64(
        T, E, H, blockIdx.y * 64, blockIdx.x * 64,
        [&](int m, int k) { return to_f(x[(int64_t)m * H + k]); },
        [&](int n, int k) { return to_f(w[(int64_t)n * H + k]); },
        [&](int m, int n, float v) { logits[(int64_t)m * E + n] = round_to<Act>(v); });
}

// ---- per-token selection -------------------------------------------------
// EPL = experts per lane (E <= 32*EPL).  Threshold = value of the k-th largest
// probability counting duplicates (torch.topk(probs,k)[0][:,-1]).
template <typename Act, int EPL>
__global__ void __launch_bounds__(256) select_kernel(const float *__restrict__ logits, int T,
                                                     int E, int k, int norm,
                                                     float *__restrict__ probs,
                                                     float *__restrict__ wsum,
                                                     Act *__restrict__ weights) {
    int lane = threadIdx.x & 31;
    int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= T) return;
    const float *lg = logits + (int64_t)t * E;
    float v[EPL];
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        int e = lane + 32 * j;
        v[j] = e < E ? lg[e] : -INFINITY;
        mx = fmaxf(mx, v[j]);
    }
    mx = warp_max(mx);
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        int e = lane + 32 * j;
        v[j] = e < E ? expf(__fsub_rn(v[j], mx)) : 0.0f;
        sum = __fadd_rn(sum, v[j]);
    }
    sum = warp_sum(sum);
    float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
    for (int j = 0; j < EPL; ++j) v[j] = __fmul_rn(v[j], inv);
    // k-th largest with multiplicity: remove one max instance (lowest index) k-1 times
    uint32_t taken = 0;
    float thr = 0.0f;
    for (int it = 0; it < k; ++it) {
        float best = -INFINITY;
        int bidx = 0x7fffffff;
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
            int e = lane + 32 * j;
            if (e < E && !((taken >> j) & 1u)) {
                if (v[j] > best) { best = v[j]; bidx = e; }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ob = __shfl_xor_sync(0xffffffffu, best, o);
            int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
            if (ob > best || (ob == best && oi < bidx)) { best = ob; bidx = oi; }
        }
        thr = best;
        if ((bidx & 31) == lane) taken |= 1u << (bidx >> 5);
    }
    float wm[EPL];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        int e = lane + 32 * j;
        wm[j] = (e < E && v[j] >= thr) ? v[j] : 0.0f;
        s = __fadd_rn(s, wm[j]);
    }
    s = warp_sum(s);
    float denom = fmaxf(s, 1e-9f);
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        int e = lane + 32 * j;
        if (e < E) {
            probs[(int64_t)t * E + e] = v[j];
            float w = norm ? __fdiv_rn(wm[j], denom) : wm[j];
            weights[(int64_t)t * E + e] = from_f<Act>(w);
        }
    }
    if (lane == 0) wsum[t] = s;
}

// ---- backward: dlogits per token ----------------------------------------
// weights = (wm / clamp_min(S,1e-9)).to(act), wm = probs*mask, S = sum(wm).
// autograd: d(wm)_j = dw_j / Sc + [S >= 1e-9] * sum_i(-dw_i * ((wm_i / Sc) / Sc))
//           dprobs = d(wm) * mask
//           dlogits = act((dprobs - sum_i dprobs_i p_i) * p)
template <typename Act, int EPL>
__global__ void __launch_bounds__(256) router_bwd_token(
    const int32_t *__restrict__ tok_off, const int32_t *__restrict__ pair_exp,
    const float *__restrict__ dw_pair, const float *__restrict__ probs,
    const float *__restrict__ wsum, const Act *__restrict__ weights, int T, int E, int norm,
    float *__restrict__ dlogits, __nv_bfloat16 *__restrict__ dl_bf, __nv_bfloat16 *__restrict__ dlT,
    int ldT) {
    int lane = threadIdx.x & 31;
    int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (t >= T) return;
    float p[EPL], dw[EPL], msk[EPL];
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        int e = lane + 32 * j;
        p[j] = e < E ? probs[(int64_t)t * E + e] : 0.0f;
        dw[j] = 0.0f;
        msk[j] = 0.0f;
    }
    // pairs of this token carry the mask (nonzero routing weight) and dw
    int b = tok_off[t], en = tok_off[t + 1];
    for (int q = b; q < en; ++q) {
        int e = pair_exp[q];
        if ((e & 31) == lane) {
#pragma unroll
            for (int j = 0; j < EPL; ++j)
                if ((e >> 5) == j) { dw[j] = dw_pair[q]; msk[j] = 1.0f; }
        }
    }
    float S = wsum[t];
    float Sc = fmaxf(S, 1e-9f);
    float dsum = 0.0f;
    if (norm) {
#pragma unroll
        for (int j = 0; j < EPL; ++j) {
            float wmj = __fmul_rn(p[j], msk[j]);
            float r = __fdiv_rn(__fdiv_rn(wmj, Sc), Sc);
            dsum = __fadd_rn(dsum, __fmul_rn(-dw[j], r));
        }
        dsum = warp_sum(dsum);
        if (!(S >= 1e-9f)) dsum = 0.0f;
    }
    float dp[EPL];
    float sdp = 0.0f;
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        float dwm = norm ? __fadd_rn(__fdiv_rn(dw[j], Sc), dsum) : dw[j];
        dp[j] = __fmul_rn(dwm, msk[j]);
        sdp = __fadd_rn(sdp, __fmul_rn(dp[j], p[j]));
    }
    sdp = warp_sum(sdp);
#pragma unroll
    for (int j = 0; j < EPL; ++j) {
        int e = lane + 32 * j;
        if (e < E) {
            const float d = round_to<Act>(__fmul_rn(__fsub_rn(dp[j], sdp), p[j]));
            dlogits[(int64_t)t * E + e] = d;
            if (dl_bf) dl_bf[(int64_t)t * E + e] = __float2bfloat16_rn(d);
            if (dlT) dlT[(int64_t)e * ldT + t] = __float2bfloat16_rn(d);
        }
    }
    (void)weights;
}

template <typename Act>
__global__ void __launch_bounds__(256) dwr_kernel(const float *__restrict__ dl,
                                                  const Act *__restrict__ x, int T, int H, int E,
                                                  Act *__restrict__ dwr) {
    // dW_r[e,h] = sum_t dl[t,e] x[t,h]   (M=E, N=H, K=T)
    tile_gemm_64x64(
        E, H, T, blockIdx.y * 64, blockIdx.x * 64,
        [&](int m, int k) { return dl[(int64_t)k * E + m]; },
        [&](int n, int k) { return to_f(x[(int64_t)k * H + n]); },
        [&](int m, int n, float v) { dwr[(int64_t)m * H + n] = from_f<Act>(v); });
}

template <typename Act>
__global__ void __launch_bounds__(256) dxr_kernel(const float *__restrict__ dl,
                                                  const Act *__restrict__ w, int T, int H, int E,
                                                  float *__restrict__ dx) {
    // dX_r[t,h] = sum_e dl[t,e] W[e,h]   (M=T, N=H, K=E), kept in fp32
    tile_gemm_64x64(
        T, H, E, blockIdx.y * 64, blockIdx.x * 64,
        [&](int m, int k) { return dl[(int64_t)m * E + k]; },
        [&](int n, int k) { return to_f(w[(int64_t)k * H + n]); },
        [&](int m, int n, float v) { dx[(int64_t)m * H + n] = v; });
}

template <typename Act>
static int launch_select(const float *logits, int T, int E, int k, int norm, float *probs,
                         float *wsum, Act *w, cudaStream_t st) {
    unsigned grid = cdiv((int64_t)T * 32, 256);
    if (E <= 32) select_kernel<Act, 1><<<grid, 256, 0, st>>>(logits, T, E, k, norm, probs, wsum, w);
    else if (E <= 64) select_kernel<Act, 2><<<grid, 256, 0, st>>>(logits, T, E, k, norm, probs, wsum, w);
    else if (E <= 128) select_kernel<Act, 4><<<grid, 256, 0, st>>>(logits, T, E, k, norm, probs, wsum, w);
    else if (E <= 256) select_kernel<Act, 8><<<grid, 256, 0, st>>>(logits, T, E, k, norm, probs, wsum, w);
    else if (E <= 512) select_kernel<Act, 16><<<grid, 256, 0, st>>>(logits, T, E, k, norm, probs, wsum, w);
    else return USAF_EUNSUPPORTED;
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

template <typename Act>
static int launch_router_bwd_token(const usaf_route_plan *pl, const float *dw_pair,
                                   const float *probs, const float *wsum, const Act *w, int norm,
                                   float *dl, __nv_bfloat16 *dl_bf, __nv_bfloat16 *dlT, int ldT,
                                   cudaStream_t st) {
    int T = pl->T, E = pl->E;
    unsigned grid = cdiv((int64_t)T * 32, 256);
#define RB_LAUNCH(EPL) router_bwd_token<Act, EPL><<<grid, 256, 0, st>>>(pl->tok_off, pl->pair_exp, dw_pair, probs, wsum, w, T, E, norm, dl, dl_bf, dlT, ldT)
    if (E <= 32) RB_LAUNCH(1);
    else if (E <= 64) RB_LAUNCH(2);
    else if (E <= 128) RB_LAUNCH(4);
    else if (E <= 256) RB_LAUNCH(8);
    else if (E <= 512) RB_LAUNCH(16);
    else return USAF_EUNSUPPORTED;
#undef RB_LAUNCH
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}


// ---- tensor-core path (bf16): dense GEMMs and split-K finalize -------------
// b_mn: B is [K, N] row-major (read transposed by the MMA), else [N, K]
int dense_tc_partials(const __nv_bfloat16 *A, int a_rows, int a_cols, int lda,
                      const __nv_bfloat16 *B, int b_rows, int b_cols, int ldb, int Mp, int Np,
                      int Kp, int splits, float *part, int *err, cudaStream_t st, bool b_mn);
bool dense_tc_available();
int dense_tc_direct(const __nv_bfloat16 *A, int a_rows, int a_cols, int lda, const __nv_bfloat16 *B,
                    int b_rows, int b_cols, int ldb, int Mp, int Np, int Kp, float *out, int64_t ldo,
                    int m_valid, int *err, cudaStream_t st, bool b_mn);

static inline int64_t rup(int64_t x, int64_t m) { return (x + m - 1) / m * m; }

// out[m][n] = round(sum_s part[s][m][n]) in split order; optional transpose
// (out[n][m]); rounding to bf16 kept as fp32 (logits), bf16 storage (dW_r)
// or none (dX_r accumulator).
enum { FIN_F32_ROUND_BF16 = 0, FIN_BF16 = 1, FIN_F32 = 2 };
__global__ void finalize_partials(const float *__restrict__ part, int splits, int Mp, int Np, int M,
                                  int N, int transpose, int mode, void *out, int ldo) {
    int64_t total = (int64_t)M * N;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t m, n, o;
        if (transpose) { n = i / M; m = i % M; o = n * ldo + m; }   // coalesced output writes
        else { m = i / N; n = i % N; o = m * ldo + n; }
        float acc = 0.0f;
        for (int s_ = 0; s_ < splits; ++s_) acc = __fadd_rn(acc, part[((int64_t)s_ * Mp + m) * Np + n]);
        if (mode == FIN_F32_ROUND_BF16) reinterpret_cast<float *>(out)[o] = __bfloat162float(__float2bfloat16_rn(acc));
        else if (mode == FIN_BF16) reinterpret_cast<__nv_bfloat16 *>(out)[o] = __float2bfloat16_rn(acc);
        else reinterpret_cast<float *>(out)[o] = acc;
    }
}

struct RouterWs {
    float *part;
    __nv_bfloat16 *dl_bf, *dlT;
    int64_t Tp;
};

static int64_t router_ws_bytes(int T, int H, int E) {
    int64_t Tp = rup(T, 128), Hp = rup(H, 128), Ep = rup(E, 128);
    int64_t part = std::max({(int64_t)4 * Tp * Ep, Hp * Tp, (int64_t)8 * Ep * Hp});
    return part * 4 + (Tp * Ep + Ep * Tp) * 2 + 3 * 256;
}

static RouterWs carve(void *ws, int T, int H, int E) {
    int64_t Tp = rup(T, 128), Hp = rup(H, 128), Ep = rup(E, 128);
    int64_t part = std::max({(int64_t)4 * Tp * Ep, Hp * Tp, (int64_t)8 * Ep * Hp});
    char *p = static_cast<char *>(ws);
    auto take = [&](int64_t bytes) { char *r = p; p += (bytes + 255) / 256 * 256; return r; };
    RouterWs w;
    w.part = reinterpret_cast<float *>(take(part * 4));
    w.dl_bf = reinterpret_cast<__nv_bfloat16 *>(take(Tp * Ep * 2));
    w.dlT = reinterpret_cast<__nv_bfloat16 *>(take(Ep * Tp * 2));
    w.Tp = Tp;
    return w;
}

// E a multiple of 8: the [T][E] bf16 dlogits rows start on 16-byte boundaries
// (TMA); tiles past E and H read as zero.
static bool router_tc_ok(int T, int H, int E, const void *ws) {
    return ws && dense_tc_available() && H % 64 == 0 && E % 8 == 0 && T >= 1;
}

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_router_select(const float *logits, int32_t dtype, int32_t T, int32_t E,
                                  int32_t top_k, int32_t norm, float *probs, float *wsum,
                                  void *weights, void *stream) {
    USAF_REQUIRE(logits && probs && wsum && weights && T >= 0 && E >= 1);
    USAF_REQUIRE(top_k >= 1 && top_k <= E);
    if (T == 0) return USAF_OK;
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case USAF_F32: return launch_select<float>(logits, T, E, top_k, norm, probs, wsum, (float *)weights, st);
        case USAF_BF16: return launch_select<__nv_bfloat16>(logits, T, E, top_k, norm, probs, wsum, (__nv_bfloat16 *)weights, st);
        default: return USAF_EINVAL;
    }
}

extern "C" int64_t usaf_router_workspace_bytes(int32_t T, int32_t H, int32_t E) {
    if (T < 0 || H < 1 || E < 1) return -1;
    return router_ws_bytes(T, H, E);
}

extern "C" int usaf_router_fwd(const void *x, const void *w_r, int32_t dtype, int32_t T, int32_t H,
                               int32_t E, int32_t top_k, int32_t norm, float *logits,
                               float *probs, float *wsum, void *weights, void *ws, int32_t *err,
                               void *stream) {
    USAF_REQUIRE(x && w_r && logits && T >= 0 && H >= 1 && E >= 1);
    if (T == 0) return USAF_OK;
    cudaStream_t st = as_stream(stream);
    if (dtype == USAF_BF16 && err && router_tc_ok(T, H, E, ws)) {
        // logits = X W_r^T on tensor cores (split-K 4, fixed-order finalize)
        RouterWs w = carve(ws, T, H, E);
        int64_t Tp = rup(T, 128), Ep = rup(E, 128);
        int rc = dense_tc_partials((const __nv_bfloat16 *)x, T, H, H, (const __nv_bfloat16 *)w_r, E, H, H,
                                   (int)Tp, (int)Ep, H, 4, w.part, err, st, false);
        if (rc) return rc;
        finalize_partials<<<cdiv((int64_t)T * E, 256), 256, 0, st>>>(w.part, 4, (int)Tp, (int)Ep, T, E, 0,
                                                                     FIN_F32_ROUND_BF16, logits, E);
        USAF_CHECK_LAUNCH();
        return usaf_router_select(logits, dtype, T, E, top_k, norm, probs, wsum, weights, stream);
    }
    dim3 grid(cdiv(E, 64), cdiv(T, 64));
    switch (dtype) {
        case USAF_F32: logits_kernel<float><<<grid, 256, 0, st>>>((const float *)x, (const float *)w_r, T, H, E, logits); break;
        case USAF_BF16: logits_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16 *)x, (const __nv_bfloat16 *)w_r, T, H, E, logits); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return usaf_router_select(logits, dtype, T, E, top_k, norm, probs, wsum, weights, stream);
}

extern "C" int usaf_router_bwd(const usaf_route_plan *plan, const void *x, const void *w_r,
                               int32_t dtype, int32_t H, int32_t norm, const float *probs,
                               const float *wsum, const void *weights, const float *dw_pair,
                               float *dlogits, void *dw_r, float *dx_acc, void *ws, void *stream) {
    USAF_REQUIRE(plan && x && w_r && probs && wsum && dw_pair && dlogits && dw_r && dx_acc);
    int T = plan->T, E = plan->E;
    if (T == 0) return USAF_OK;
    cudaStream_t st = as_stream(stream);
    int rc;
    if (dtype == USAF_BF16 && router_tc_ok(T, H, E, ws)) {
        RouterWs w = carve(ws, T, H, E);
        const int64_t Tp = w.Tp, Hp = rup(H, 128), Ep = rup(E, 128);
        const auto *xb = (const __nv_bfloat16 *)x;
        const auto *wb = (const __nv_bfloat16 *)w_r;
        rc = launch_router_bwd_token<__nv_bfloat16>(plan, dw_pair, probs, wsum, (const __nv_bfloat16 *)weights,
                                                    norm, dlogits, w.dl_bf, w.dlT, (int)Tp, st);
        if (rc) return rc;
        // dX_r [T][H] = dl [T][E] * W_r [E][H]   (K = E, W_r read MN-major), straight
        // into dx_acc when its rows hold whole 128-column tiles
        if (H % 128 == 0) {
            rc = dense_tc_direct(w.dl_bf, T, E, E, wb, E, H, H, (int)Tp, (int)Hp, (int)rup(E, 64), dx_acc,
                                 H, T, plan->err, st, true);
            if (rc) return rc;
        } else {
            rc = dense_tc_partials(w.dl_bf, T, E, E, wb, E, H, H, (int)Tp, (int)Hp, (int)rup(E, 64), 1, w.part,
                                   plan->err, st, true);
            if (rc) return rc;
            finalize_partials<<<cdiv((int64_t)T * H, 256), 256, 0, st>>>(w.part, 1, (int)Tp, (int)Hp, T, H, 0,
                                                                         FIN_F32, dx_acc, H);
        }
        // dW_r [E][H] = dl^T [E][T] * X [T][H]   (K = T, X read MN-major, split-K 8)
        rc = dense_tc_partials(w.dlT, E, T, (int)Tp, xb, T, H, H, (int)Ep, (int)Hp, (int)rup(T, 64), 8,
                               w.part, plan->err, st, true);
        if (rc) return rc;
        finalize_partials<<<cdiv((int64_t)E * H, 256), 256, 0, st>>>(w.part, 8, (int)Ep, (int)Hp, E, H, 0,
                                                                     FIN_BF16, dw_r, H);
        USAF_CHECK_LAUNCH();
        return USAF_OK;
    }
    dim3 gw(cdiv(H, 64), cdiv(E, 64)), gx(cdiv(H, 64), cdiv(T, 64));
    switch (dtype) {
        case USAF_F32:
            rc = launch_router_bwd_token<float>(plan, dw_pair, probs, wsum, (const float *)weights, norm, dlogits, nullptr, nullptr, 0, st);
            if (rc) return rc;
            dwr_kernel<float><<<gw, 256, 0, st>>>(dlogits, (const float *)x, T, H, E, (float *)dw_r);
            dxr_kernel<float><<<gx, 256, 0, st>>>(dlogits, (const float *)w_r, T, H, E, dx_acc);
            break;
        case USAF_BF16:
            rc = launch_router_bwd_token<__nv_bfloat16>(plan, dw_pair, probs, wsum, (const __nv_bfloat16 *)weights, norm, dlogits, nullptr, nullptr, 0, st);
            if (rc) return rc;
            dwr_kernel<__nv_bfloat16><<<gw, 256, 0, st>>>(dlogits, (const __nv_bfloat16 *)x, T, H, E, (__nv_bfloat16 *)dw_r);
            dxr_kernel<__nv_bfloat16><<<gx, 256, 0, st>>>(dlogits, (const __nv_bfloat16 *)w_r, T, H, E, dx_acc);
            break;
        default:
            return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
