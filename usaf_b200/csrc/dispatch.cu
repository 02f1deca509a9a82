// Token dispatch into per-expert segments, weighted combine and their backward.
//
// Dispatch restates benchmarks/kaggle_t4_bench.py:293-306 deterministically:
// pairs = nonzero(weights) in token-major order, bincount per expert,
// exclusive cumsum, stable (ascending-token) slot assignment.  Three passes:
// per-256-token-chunk histograms (shared-memory atomics), one scan block,
// then a rank pass (warp ballots) that writes both index maps.  The combine
// sums each token's expert outputs in ascending expert order in fp32
// (usaf/qwen3moe_dml.py:62), so it is deterministic and needs no atomics.
#include "common.cuh"

namespace usaf {

constexpr int kChunk = 256;

template <typename Act>
__global__ void __launch_bounds__(kChunk) count_kernel(const Act *__restrict__ w, int T, int E,
                                                       int32_t *__restrict__ tok_cnt,
                                                       int32_t *__restrict__ chunk_cnt) {
    extern __shared__ int32_t hist[];
    for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
    __syncthreads();
    int t = blockIdx.x * kChunk + threadIdx.x;
    if (t < T) {
        int c = 0;
        const Act *row = w + (int64_t)t * E;
        for (int e = 0; e < E; ++e) {
            if (to_f(row[e]) != 0.0f) {
                ++c;
                atomicAdd(&hist[e], 1);
            }
        }
        tok_cnt[t] = c;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x)
        chunk_cnt[(int64_t)blockIdx.x * E + e] = hist[e];
}

// block-wide exclusive scan of one int per thread (blockDim = 1024)
__device__ int block_excl_scan(int v, int *smem_warp, int &total) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) smem_warp[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int nw = blockDim.x >> 5;
        int s = lane < nw ? smem_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        if (lane < nw) smem_warp[lane] = s;
    }
    __syncthreads();
    int base = wid ? smem_warp[wid - 1] : 0;
    total = smem_warp[(blockDim.x >> 5) - 1];
    __syncthreads();
    return base + x - v;
}

__global__ void __launch_bounds__(1024) scan_kernel(usaf_route_plan pl, int nchunks) {
    __shared__ int warp_s[32];
    int T = pl.T, E = pl.E;
    // per-expert totals and exclusive prefix over chunks (in place -> chunk bases)
    int tot_e = 0;
    if ((int)threadIdx.x < E) {
        int e = threadIdx.x;
        int run = 0;
        for (int c = 0; c < nchunks; ++c) {
            int v = pl.chunk_cnt[(int64_t)c * E + e];
            pl.chunk_cnt[(int64_t)c * E + e] = run;
            run += v;
        }
        tot_e = run;
    }
    int total;
    int off_e = block_excl_scan((int)threadIdx.x < E ? tot_e : 0, warp_s, total);
    bool overflow = total > pl.P_cap;
    if ((int)threadIdx.x < E) {
        pl.expert_cnt[threadIdx.x] = overflow ? 0 : tot_e;
        pl.expert_off[threadIdx.x] = overflow ? 0 : off_e;
        for (int c = 0; c < nchunks; ++c) pl.chunk_cnt[(int64_t)c * E + threadIdx.x] += off_e;
    }
    if (threadIdx.x == 0) {
        pl.expert_off[E] = overflow ? 0 : total;
        pl.n_pairs[0] = overflow ? 0 : total;
        if (overflow) atomicOr(pl.err, USAF_ERR_PAIR_OVERFLOW);
    }
    // token offsets
    int carry = 0;
    for (int t0 = 0; t0 < T; t0 += blockDim.x) {
        int t = t0 + threadIdx.x;
        int v = t < T ? pl.tok_cnt[t] : 0;
        int tot;
        int ex = block_excl_scan(v, warp_s, tot);
        if (t < T) pl.tok_off[t] = overflow ? 0 : carry + ex;
        carry += tot;
    }
    if (threadIdx.x == 0) pl.tok_off[T] = overflow ? 0 : carry;
}

template <typename Act>
__global__ void __launch_bounds__(kChunk) scatter_kernel(usaf_route_plan pl,
                                                         const Act *__restrict__ w) {
    __shared__ int warp_cnt[kChunk / 32];
    int T = pl.T, E = pl.E;
    int t = blockIdx.x * kChunk + threadIdx.x;
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int32_t *base = pl.chunk_cnt + (int64_t)blockIdx.x * E;
    int p = t < T ? pl.tok_off[t] : 0;
    for (int e = 0; e < E; ++e) {
        float wv = t < T ? to_f(w[(int64_t)t * E + e]) : 0.0f;
        bool f = wv != 0.0f;
        unsigned bal = __ballot_sync(0xffffffffu, f);
        if (lane == 0) warp_cnt[wid] = __popc(bal);
        __syncthreads();
        int before = 0;
        for (int i = 0; i < wid; ++i) before += warp_cnt[i];
        __syncthreads();
        if (f) {
            int rank = before + __popc(bal & ((1u << lane) - 1));
            int slot = base[e] + rank;
            if (slot < pl.P_cap && p < pl.P_cap) {
                pl.seg_tok[slot] = t;
                pl.seg_pair[slot] = p;
                pl.seg_w[slot] = wv;
                pl.pair_exp[p] = e;
                pl.pair_slot[p] = slot;
            }
            ++p;
        }
    }
}

// x_perm[slot] = x[seg_tok[slot]]; one warp per slot, 16-byte vectors
__global__ void gather_rows_kernel(const int32_t *__restrict__ n_pairs,
                                   const int32_t *__restrict__ seg_tok,
                                   const uint4 *__restrict__ x, int row_vec,
                                   uint4 *__restrict__ xp) {
    int P = *n_pairs;
    int lane = threadIdx.x & 31;
    for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < P;
         s += (gridDim.x * blockDim.x) >> 5) {
        const uint4 *src = x + (int64_t)seg_tok[s] * row_vec;
        uint4 *dst = xp + (int64_t)s * row_vec;
        for (int i = lane; i < row_vec; i += 32) dst[i] = __ldg(src + i);
    }
}

template <typename Act>
__global__ void gather_rows_scalar(const int32_t *__restrict__ n_pairs,
                                   const int32_t *__restrict__ seg_tok, const Act *__restrict__ x,
                                   int H, Act *__restrict__ xp) {
    int P = *n_pairs;
    int lane = threadIdx.x & 31;
    for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < P;
         s += (gridDim.x * blockDim.x) >> 5) {
        const Act *src = x + (int64_t)seg_tok[s] * H;
        for (int i = lane; i < H; i += 32) xp[(int64_t)s * H + i] = src[i];
    }
}

// y[t] = act( sum_{pairs of t, ascending expert} fp32(y_seg[slot]) * w )
template <typename Act>
__global__ void __launch_bounds__(256) combine_kernel(usaf_route_plan pl,
                                                      const Act *__restrict__ yseg, int H,
                                                      Act *__restrict__ y) {
    int t = blockIdx.x;
    int b = pl.tok_off[t], e = pl.tok_off[t + 1];
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
        float acc = 0.0f;
        for (int q = b; q < e; ++q) {
            int s = pl.pair_slot[q];
            acc = __fadd_rn(acc, __fmul_rn(to_f(yseg[(int64_t)s * H + h]), pl.seg_w[s]));
        }
        y[(int64_t)t * H + h] = from_f<Act>(acc);
    }
}

// per slot: dcur = act(dy[t] * w); dw_pair = act(sum_h dy[t,h] * y_seg[s,h])
template <typename Act>
__global__ void __launch_bounds__(256) combine_bwd_kernel(usaf_route_plan pl,
                                                          const Act *__restrict__ dy,
                                                          const Act *__restrict__ yseg, int H,
                                                          Act *__restrict__ dcur,
                                                          float *__restrict__ dw_pair) {
    int P = *pl.n_pairs;
    int lane = threadIdx.x & 31;
    for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < P;
         s += (gridDim.x * blockDim.x) >> 5) {
        int t = pl.seg_tok[s];
        float w = pl.seg_w[s];
        float dot = 0.0f;
        for (int h = lane; h < H; h += 32) {
            float g = to_f(dy[(int64_t)t * H + h]);
            dot = fmaf(g, to_f(yseg[(int64_t)s * H + h]), dot);
            dcur[(int64_t)s * H + h] = from_f<Act>(__fmul_rn(g, w));
        }
        dot = warp_sum(dot);
        if (lane == 0) dw_pair[pl.seg_pair[s]] = round_to<Act>(dot);
    }
}

template <typename Act>
__global__ void __launch_bounds__(256) gather_dx_kernel(usaf_route_plan pl,
                                                        const Act *__restrict__ dxseg,
                                                        const float *__restrict__ dxacc, int H,
                                                        Act *__restrict__ dx) {
    int t = blockIdx.x;
    int b = pl.tok_off[t], e = pl.tok_off[t + 1];
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
        float acc = 0.0f;
        for (int q = b; q < e; ++q) {
            int s = pl.pair_slot[q];
            acc = __fadd_rn(acc, to_f(dxseg[(int64_t)s * H + h]));
        }
        if (dxacc) acc = __fadd_rn(acc, dxacc[(int64_t)t * H + h]);
        dx[(int64_t)t * H + h] = from_f<Act>(acc);
    }
}

template <typename Act>
static int dispatch_impl(const usaf_route_plan *pl, const Act *w, const Act *x, int H, Act *xp,
                         cudaStream_t st) {
    int T = pl->T, E = pl->E;
    if (E > 1024) return USAF_EUNSUPPORTED;
    int nchunks = (T + kChunk - 1) / kChunk;
    if (nchunks > 0)
        count_kernel<Act><<<nchunks, kChunk, E * sizeof(int32_t), st>>>(w, T, E, pl->tok_cnt, pl->chunk_cnt);
    scan_kernel<<<1, 1024, 0, st>>>(*pl, nchunks);
    if (nchunks > 0) scatter_kernel<Act><<<nchunks, kChunk, 0, st>>>(*pl, w);
    if (x && xp) {
        size_t row_bytes = (size_t)H * sizeof(Act);
        unsigned grid = 148 * 8;
        if (row_bytes % 16 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)xp & 15) == 0)
            gather_rows_kernel<<<grid, 256, 0, st>>>(pl->n_pairs, pl->seg_tok, (const uint4 *)x, (int)(row_bytes / 16), (uint4 *)xp);
        else
            gather_rows_scalar<Act><<<grid, 256, 0, st>>>(pl->n_pairs, pl->seg_tok, x, H, xp);
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_dispatch(const usaf_route_plan *plan, const void *weights, const void *x,
                             int32_t dtype, int32_t H, void *x_perm, void *stream) {
    USAF_REQUIRE(plan && weights && plan->T >= 0 && plan->E >= 1 && plan->P_cap >= 0);
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case USAF_F32: return dispatch_impl<float>(plan, (const float *)weights, (const float *)x, H, (float *)x_perm, st);
        case USAF_BF16: return dispatch_impl<__nv_bfloat16>(plan, (const __nv_bfloat16 *)weights, (const __nv_bfloat16 *)x, H, (__nv_bfloat16 *)x_perm, st);
        default: return USAF_EINVAL;
    }
}

extern "C" int usaf_combine(const usaf_route_plan *plan, const void *y_seg, int32_t dtype,
                            int32_t H, void *y, void *stream) {
    USAF_REQUIRE(plan && y_seg && y && H >= 1);
    if (plan->T == 0) return USAF_OK;
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case USAF_F32: combine_kernel<float><<<plan->T, 256, 0, st>>>(*plan, (const float *)y_seg, H, (float *)y); break;
        case USAF_BF16: combine_kernel<__nv_bfloat16><<<plan->T, 256, 0, st>>>(*plan, (const __nv_bfloat16 *)y_seg, H, (__nv_bfloat16 *)y); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_combine_bwd(const usaf_route_plan *plan, const void *dy, const void *y_seg,
                                int32_t dtype, int32_t H, void *dcur, float *dw_pair,
                                void *stream) {
    USAF_REQUIRE(plan && dy && y_seg && dcur && dw_pair && H >= 1);
    cudaStream_t st = as_stream(stream);
    unsigned grid = 148 * 8;
    switch (dtype) {
        case USAF_F32: combine_bwd_kernel<float><<<grid, 256, 0, st>>>(*plan, (const float *)dy, (const float *)y_seg, H, (float *)dcur, dw_pair); break;
        case USAF_BF16: combine_bwd_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(*plan, (const __nv_bfloat16 *)dy, (const __nv_bfloat16 *)y_seg, H, (__nv_bfloat16 *)dcur, dw_pair); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_gather_dx(const usaf_route_plan *plan, const void *dx_seg, const float *dx_acc,
                              int32_t dtype, int32_t H, void *dx, void *stream) {
    USAF_REQUIRE(plan && dx_seg && dx && H >= 1);
    if (plan->T == 0) return USAF_OK;
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case USAF_F32: gather_dx_kernel<float><<<plan->T, 256, 0, st>>>(*plan, (const float *)dx_seg, dx_acc, H, (float *)dx); break;
        case USAF_BF16: gather_dx_kernel<__nv_bfloat16><<<plan->T, 256, 0, st>>>(*plan, (const __nv_bfloat16 *)dx_seg, dx_acc, H, (__nv_bfloat16 *)dx); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
