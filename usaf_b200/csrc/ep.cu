// Row regrouping for expert parallelism.
//
// Rank r of W owns experts [r*El, (r+1)*El).  Every rank dispatches its own
// tokens over all E experts (x_perm is expert-major, so the rows bound for
// rank d are one contiguous range), and an all-to-all delivers them: the
// receive buffer of rank r holds, for source s = 0..W-1, the rows of s for
// each local expert e = 0..El-1 in s's slot order -- block order (s, e).
// The grouped GEMMs need expert-major segments (e, s): within an expert,
// source rank first, then the source's slot order, which is ascending token
// order of the concatenation of the ranks' token batches.  These kernels
// move rows between the two orders and build the owner-side expert counts.
//
// counts[s*El + e] = rows received from source s for local expert e.
#include "common.cuh"

namespace usaf {

constexpr int kEpMaxBlocks = 4096;   // W * El

// exclusive prefix of the W*El block sizes in source-major order (src_start)
// and the start of each block in expert-major order (dst_start), by one warp
__device__ void ep_block_starts(const int32_t *__restrict__ counts, int W, int El, int *src_start,
                                int *dst_start) {
    const int lane = threadIdx.x & 31;
    const int nb = W * El;
    int run = 0;
    for (int b0 = 0; b0 < nb; b0 += 32) {
        const int b = b0 + lane;
        const int v = b < nb ? counts[b] : 0;
        int x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (b < nb) src_start[b] = run + x - v;
        run += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) src_start[nb] = run;
    run = 0;
    for (int b0 = 0; b0 < nb; b0 += 32) {
        const int bt = b0 + lane;                 // expert-major index e*W + s
        const int e = bt / W, s = bt % W;
        const int v = bt < nb ? counts[s * El + e] : 0;
        int x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (bt < nb) dst_start[s * El + e] = run + x - v;
        run += __shfl_sync(0xffffffffu, x, 31);
    }
}

// forward (inverse == 0): out[dst(i)] = in[i] for received row i;
// inverse: out[i] = in[dst(i)].  One warp per row, 16-byte vectors.
__global__ void __launch_bounds__(256) ep_permute_kernel(const int32_t *__restrict__ counts, int W, int El,
                                                         int64_t n_rows, const uint4 *__restrict__ in,
                                                         uint4 *__restrict__ out, int vec_per_row,
                                                         int inverse, int32_t *err) {
    extern __shared__ int ep_sm[];
    const int nb = W * El;
    int *src_start = ep_sm;              // [nb + 1]
    int *dst_start = ep_sm + nb + 1;     // [nb]
    if (threadIdx.x < 32) ep_block_starts(counts, W, El, src_start, dst_start);
    __syncthreads();
    if ((int64_t)src_start[nb] != n_rows) {   // counts and the row count disagree
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(err, USAF_ERR_BAD_INDEX);
        return;
    }
    const int lane = threadIdx.x & 31;
    const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < n_rows; row += nw) {
        // last block whose start is <= row
        int lo = 0, hi = nb - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (src_start[mid] <= row) lo = mid; else hi = mid - 1;
        }
        const int64_t dst = dst_start[lo] + (row - src_start[lo]);
        const uint4 *src = in + (inverse ? dst : row) * vec_per_row;
        uint4 *d = out + (inverse ? row : dst) * vec_per_row;
        for (int v = lane; v < vec_per_row; v += 32) d[v] = __ldg(src + v);
    }
}

// expert_cnt[e] = sum_s counts[s][e]; expert_off = exclusive prefix (El + 1)
__global__ void ep_owner_counts_kernel(const int32_t *__restrict__ counts, int W, int El,
                                       int32_t *__restrict__ expert_cnt, int32_t *__restrict__ expert_off,
                                       int32_t *__restrict__ n_rows) {
    const int lane = threadIdx.x & 31;
    int run = 0;
    for (int e0 = 0; e0 < El; e0 += 32) {
        const int e = e0 + lane;
        int v = 0;
        if (e < El)
            for (int s = 0; s < W; ++s) v += counts[s * El + e];
        int x = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (e < El) {
            expert_cnt[e] = v;
            expert_off[e] = run + x - v;
        }
        run += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) {
        expert_off[El] = run;
        if (n_rows) n_rows[0] = run;
    }
}

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_ep_permute(const int32_t *counts, int32_t W, int32_t El, int64_t n_rows,
                               const void *in, void *out, int64_t row_bytes, int32_t inverse,
                               int32_t *err, void *stream) {
    USAF_REQUIRE(counts && W >= 1 && El >= 1 && n_rows >= 0 && err);
    USAF_REQUIRE(W * El <= kEpMaxBlocks);
    if (n_rows == 0) return USAF_OK;
    USAF_REQUIRE(in && out && in != out && row_bytes > 0);
    if (row_bytes % 16 || ((uintptr_t)in & 15) || ((uintptr_t)out & 15)) return USAF_EUNSUPPORTED;
    const int nb = W * El;
    const size_t smem = (size_t)(2 * nb + 1) * sizeof(int);
    const int64_t warps = std::min<int64_t>(n_rows, 148 * 64);
    const unsigned grid = (unsigned)((warps * 32 + 255) / 256);
    ep_permute_kernel<<<grid, 256, smem, as_stream(stream)>>>(counts, W, El, n_rows, (const uint4 *)in,
                                                             (uint4 *)out, (int)(row_bytes / 16),
                                                             inverse, err);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_ep_owner_counts(const int32_t *counts, int32_t W, int32_t El, int32_t *expert_cnt,
                                    int32_t *expert_off, int32_t *n_rows, void *stream) {
    USAF_REQUIRE(counts && expert_cnt && expert_off && W >= 1 && El >= 1);
    ep_owner_counts_kernel<<<1, 32, 0, as_stream(stream)>>>(counts, W, El, expert_cnt, expert_off, n_rows);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
