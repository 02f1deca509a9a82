// Token dispatch into per-expert segments, weighted combine and their backward.
//
// Dispatch restates benchmarks/kaggle_t4_bench.py:293-306 deterministically:
// pairs = nonzero(weights) in token-major order, bincount per expert,
// exclusive cumsum, stable (ascending-token) slot assignment.  Three passes:
// per-chunk expert histograms (one warp walks 16 consecutive tokens, each
// lane owning E/32 experts' counters in registers), one scan block, then a
// rank pass over the same chunks that writes both index maps.  The combine
// sums each token's expert outputs in ascending expert order in fp32
// (usaf/qwen3moe_dml.py:62), so it is deterministic and needs no atomics.
#include "common.cuh"

namespace usaf {

constexpr int kChunk = 16;   // tokens per dispatch chunk (one warp)

// per chunk: tok_cnt[t] = #nonzero weights of token t, chunk_cnt[c][e] = #tokens
// of the chunk routed to expert e.  Lane l owns experts [l*EPL, l*EPL+EPL).
template <typename Act, int EPL>
__global__ void __launch_bounds__(256) count_kernel(const Act *__restrict__ w, int T, int E,
                                                    int32_t *__restrict__ tok_cnt,
                                                    int32_t *__restrict__ chunk_cnt) {
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (c * kChunk >= T) return;
    int cnt[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) cnt[i] = 0;
    int my_tok = 0;   // lane tt keeps token tt's count
#pragma unroll 4
    for (int tt = 0; tt < kChunk; ++tt) {
        const int t = c * kChunk + tt;
        if (t >= T) break;
        const Act *row = w + (int64_t)t * E;
        int mine = 0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const int e = lane * EPL + i;
            const int f = (e < E && to_f(row[e]) != 0.0f) ? 1 : 0;
            cnt[i] += f;
            mine += f;
        }
        const int tot = __reduce_add_sync(0xffffffffu, mine);
        if (lane == tt) my_tok = tot;
    }
    if (lane < kChunk && c * kChunk + lane < T) tok_cnt[c * kChunk + lane] = my_tok;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int e = lane * EPL + i;
        if (e < E) chunk_cnt[(int64_t)c * E + e] = cnt[i];
    }
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

// Expert totals, expert offsets, chunk bases (in place in chunk_cnt) and
// token offsets.  blockDim / E thread groups split the chunks of every expert
// so the per-chunk loads run in parallel.
__global__ void __launch_bounds__(1024) scan_kernel(usaf_route_plan pl, int nchunks) {
    __shared__ int warp_s[32];
    __shared__ int part_s[1024];
    __shared__ int eoff_s[1024];
    const int T = pl.T, E = pl.E;
    const int nparts = blockDim.x / E;              // E <= 1024
    const int e = threadIdx.x % E, part = threadIdx.x / E;
    const bool active = part < nparts;
    const int cpp = (nchunks + nparts - 1) / nparts;
    const int c0 = part * cpp, c1 = min(nchunks, c0 + cpp);
    int sum = 0;
    if (active)
        for (int c = c0; c < c1; ++c) sum += pl.chunk_cnt[(int64_t)c * E + e];
    part_s[threadIdx.x] = active ? sum : 0;
    __syncthreads();
    int before = 0, tot_e = 0;
    if (active) {
        for (int q = 0; q < nparts; ++q) {
            const int v = part_s[q * E + e];
            if (q < part) before += v;
            tot_e += v;
        }
    }
    int total;
    const int off_e = block_excl_scan((int)threadIdx.x < E ? tot_e : 0, warp_s, total);
    const bool overflow = total > pl.P_cap;
    if ((int)threadIdx.x < E) {
        eoff_s[e] = off_e;
        pl.expert_cnt[e] = overflow ? 0 : tot_e;
        pl.expert_off[e] = overflow ? 0 : off_e;
    }
    if (threadIdx.x == 0) {
        pl.expert_off[E] = overflow ? 0 : total;
        pl.n_pairs[0] = overflow ? 0 : total;
        if (overflow) atomicOr(pl.err, USAF_ERR_PAIR_OVERFLOW);
    }
    __syncthreads();
    if (active) {
        // chunk base = expert offset + tokens of this expert in earlier chunks
        int run = eoff_s[e] + before;
        for (int cb = c0; cb < c1; cb += 16) {
            int v[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) v[i] = cb + i < c1 ? pl.chunk_cnt[(int64_t)(cb + i) * E + e] : 0;
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (cb + i < c1) {
                    pl.chunk_cnt[(int64_t)(cb + i) * E + e] = run;
                    run += v[i];
                }
        }
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

// rank pass: the chunk's warp walks its tokens in order; each lane advances
// the slot counters of its experts (chunk base after the scan), and a token's
// pairs are numbered in ascending expert order from tok_off[t].
template <typename Act, int EPL>
__global__ void __launch_bounds__(256) scatter_kernel(usaf_route_plan pl, const Act *__restrict__ w) {
    const int T = pl.T, E = pl.E;
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (c * kChunk >= T) return;
    int run[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
        const int e = lane * EPL + i;
        run[i] = e < E ? pl.chunk_cnt[(int64_t)c * E + e] : 0;
    }
#pragma unroll 2
    for (int tt = 0; tt < kChunk; ++tt) {
        const int t = c * kChunk + tt;
        if (t >= T) break;
        const Act *row = w + (int64_t)t * E;
        float wv[EPL];
        int mine = 0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            const int e = lane * EPL + i;
            wv[i] = e < E ? to_f(row[e]) : 0.0f;
            mine += wv[i] != 0.0f;
        }
        int incl = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int p = pl.tok_off[t] + incl - mine;
#pragma unroll
        for (int i = 0; i < EPL; ++i) {
            if (wv[i] != 0.0f) {
                const int e = lane * EPL + i;
                const int slot = run[i]++;
                if (slot < pl.P_cap && p < pl.P_cap) {
                    pl.seg_tok[slot] = t;
                    pl.seg_pair[slot] = p;
                    pl.seg_w[slot] = wv[i];
                    pl.pair_exp[p] = e;
                    pl.pair_slot[p] = slot;
                }
                ++p;
            }
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

// 16-byte vector of activations <-> fp32 lanes
template <typename Act> struct Vec16 {
    static constexpr int N = 16 / sizeof(Act);
};
template <typename Act>
__device__ __forceinline__ void unpack16(const uint4 &u, float (&f)[16 / sizeof(Act)]) {
    const Act *a = reinterpret_cast<const Act *>(&u);
#pragma unroll
    for (int i = 0; i < Vec16<Act>::N; ++i) f[i] = to_f(a[i]);
}
template <typename Act>
__device__ __forceinline__ uint4 pack16(const float (&f)[16 / sizeof(Act)]) {
    uint4 u;
    Act *a = reinterpret_cast<Act *>(&u);
#pragma unroll
    for (int i = 0; i < Vec16<Act>::N; ++i) a[i] = from_f<Act>(f[i]);
    return u;
}

constexpr int kMaxTokPairs = 1024;   // pairs of one token staged in shared memory (<= E)

// y[t] = act( sum_{pairs of t, ascending expert} fp32(y_seg[slot]) * w )
// one block per token; each thread owns 16-byte column vectors
template <typename Act>
__global__ void __launch_bounds__(256) combine_kernel(usaf_route_plan pl,
                                                      const Act *__restrict__ yseg, int H,
                                                      Act *__restrict__ y) {
    constexpr int V = Vec16<Act>::N;
    __shared__ int s_slot[kMaxTokPairs];
    __shared__ float s_w[kMaxTokPairs];
    const int t = blockIdx.x;
    const int b = pl.tok_off[t], n = min(pl.tok_off[t + 1] - b, kMaxTokPairs);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int sl = pl.pair_slot[b + i];
        s_slot[i] = sl;
        s_w[i] = pl.seg_w[sl];
    }
    __syncthreads();
    const int nv = H / V;
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        float acc[V];
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = 0.0f;
        for (int q = 0; q < n; ++q) {
            float f[V];
            unpack16<Act>(__ldg(reinterpret_cast<const uint4 *>(yseg + (int64_t)s_slot[q] * H) + v), f);
            const float wq = s_w[q];
#pragma unroll
            for (int i = 0; i < V; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(f[i], wq));
        }
        reinterpret_cast<uint4 *>(y + (int64_t)t * H)[v] = pack16<Act>(acc);
    }
}

// per slot: dcur = act(dy[t] * w); dw_pair = act(sum_h dy[t,h] * y_seg[s,h])
// one warp per slot, 16-byte vectors
template <typename Act>
__global__ void __launch_bounds__(256) combine_bwd_kernel(usaf_route_plan pl,
                                                          const Act *__restrict__ dy,
                                                          const Act *__restrict__ yseg, int H,
                                                          Act *__restrict__ dcur,
                                                          float *__restrict__ dw_pair) {
    constexpr int V = Vec16<Act>::N;
    const int P = *pl.n_pairs;
    const int lane = threadIdx.x & 31;
    const int nv = H / V;
    for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < P;
         s += (gridDim.x * blockDim.x) >> 5) {
        const int t = pl.seg_tok[s];
        const float w = pl.seg_w[s];
        const uint4 *dyr = reinterpret_cast<const uint4 *>(dy + (int64_t)t * H);
        const uint4 *ysr = reinterpret_cast<const uint4 *>(yseg + (int64_t)s * H);
        uint4 *dcr = reinterpret_cast<uint4 *>(dcur + (int64_t)s * H);
        float dot = 0.0f;
        for (int v = lane; v < nv; v += 32) {
            float g[V], yv[V], o[V];
            unpack16<Act>(__ldg(dyr + v), g);
            unpack16<Act>(__ldg(ysr + v), yv);
#pragma unroll
            for (int i = 0; i < V; ++i) {
                dot = fmaf(g[i], yv[i], dot);
                o[i] = __fmul_rn(g[i], w);
            }
            dcr[v] = pack16<Act>(o);
        }
        dot = warp_sum(dot);
        if (lane == 0) dw_pair[pl.seg_pair[s]] = round_to<Act>(dot);
    }
}

// dx[t] = act( sum_{pairs of t, ascending expert} dx_seg[slot] (+ dx_acc[t]) )
template <typename Act>
__global__ void __launch_bounds__(256) gather_dx_kernel(usaf_route_plan pl,
                                                        const Act *__restrict__ dxseg,
                                                        const float *__restrict__ dxacc, int H,
                                                        Act *__restrict__ dx) {
    constexpr int V = Vec16<Act>::N;
    __shared__ int s_slot[kMaxTokPairs];
    const int t = blockIdx.x;
    const int b = pl.tok_off[t], n = min(pl.tok_off[t + 1] - b, kMaxTokPairs);
    for (int i = threadIdx.x; i < n; i += blockDim.x) s_slot[i] = pl.pair_slot[b + i];
    __syncthreads();
    const int nv = H / V;
    for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        float acc[V];
#pragma unroll
        for (int i = 0; i < V; ++i) acc[i] = 0.0f;
        for (int q = 0; q < n; ++q) {
            float f[V];
            unpack16<Act>(__ldg(reinterpret_cast<const uint4 *>(dxseg + (int64_t)s_slot[q] * H) + v), f);
#pragma unroll
            for (int i = 0; i < V; ++i) acc[i] = __fadd_rn(acc[i], f[i]);
        }
        if (dxacc) {
#pragma unroll
            for (int i = 0; i < V; ++i) acc[i] = __fadd_rn(acc[i], dxacc[(int64_t)t * H + v * V + i]);
        }
        reinterpret_cast<uint4 *>(dx + (int64_t)t * H)[v] = pack16<Act>(acc);
    }
}

template <typename Act>
static int dispatch_impl(const usaf_route_plan *pl, const Act *w, const Act *x, int H, Act *xp,
                         cudaStream_t st) {
    int T = pl->T, E = pl->E;
    if (E > 1024) return USAF_EUNSUPPORTED;
    const int nchunks = (T + kChunk - 1) / kChunk;
    const unsigned grid = cdiv(nchunks, 8);    // 8 warps (chunks) per block
    if (nchunks > 0) {
#define USAF_CNT(EPL) count_kernel<Act, EPL><<<grid, 256, 0, st>>>(w, T, E, pl->tok_cnt, pl->chunk_cnt)
        if (E <= 32) USAF_CNT(1);
        else if (E <= 64) USAF_CNT(2);
        else if (E <= 128) USAF_CNT(4);
        else if (E <= 256) USAF_CNT(8);
        else if (E <= 512) USAF_CNT(16);
        else USAF_CNT(32);
#undef USAF_CNT
    }
    scan_kernel<<<1, 1024, 0, st>>>(*pl, nchunks);
    if (nchunks > 0) {
#define USAF_SCT(EPL) scatter_kernel<Act, EPL><<<grid, 256, 0, st>>>(*pl, w)
        if (E <= 32) USAF_SCT(1);
        else if (E <= 64) USAF_SCT(2);
        else if (E <= 128) USAF_SCT(4);
        else if (E <= 256) USAF_SCT(8);
        else if (E <= 512) USAF_SCT(16);
        else USAF_SCT(32);
#undef USAF_SCT
    }
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

// rows of H activations must start on 16-byte boundaries for the vector kernels
static bool vec_ok(const void *a, const void *b, int H, int dtype) {
    const int esz = dtype == USAF_F32 ? 4 : 2;
    return ((uintptr_t)a & 15) == 0 && ((uintptr_t)b & 15) == 0 && ((int64_t)H * esz) % 16 == 0;
}

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
    if (!vec_ok(y_seg, y, H, dtype) || plan->E > kMaxTokPairs) return USAF_EUNSUPPORTED;
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
    if (!vec_ok(dy, y_seg, H, dtype) || !vec_ok(dcur, dcur, H, dtype)) return USAF_EUNSUPPORTED;
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
    if (!vec_ok(dx_seg, dx, H, dtype) || plan->E > kMaxTokPairs) return USAF_EUNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case USAF_F32: gather_dx_kernel<float><<<plan->T, 256, 0, st>>>(*plan, (const float *)dx_seg, dx_acc, H, (float *)dx); break;
        case USAF_BF16: gather_dx_kernel<__nv_bfloat16><<<plan->T, 256, 0, st>>>(*plan, (const __nv_bfloat16 *)dx_seg, dx_acc, H, (__nv_bfloat16 *)dx); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
