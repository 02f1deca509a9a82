// Small utilities of the C ABI: a deterministic dot product (the step's
// scalar readback; its block partials live in a fixed array of this library,
// so two dot products in flight at once on one device race), CSR row pointers
// from sorted row keys, the overlay's per-column-block positions, and the
// version.
#include "common.cuh"

namespace usaf {

constexpr int kDotBlocks = 296;   // two per SM
__device__ float g_dot_partials[kDotBlocks];

// block-level fp32 partial sums in a fixed order (16-byte vector loads when the
// inputs allow), then one block adds the partials in block order: the scalar
// is reproducible run to run
template <typename T>
__global__ void __launch_bounds__(256) dot_partial_kernel(const T *__restrict__ a, const T *__restrict__ b,
                                                          int64_t n, int vec) {
    __shared__ float ws[8];
    float acc = 0.0f;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t nthr = (int64_t)gridDim.x * blockDim.x;
    constexpr int V = 16 / sizeof(T);
    int64_t done = 0;
    if (vec) {
        const int64_t nv = n / V;
        for (int64_t i = tid; i < nv; i += nthr) {
            const uint4 ua = __ldg(reinterpret_cast<const uint4 *>(a) + i);
            const uint4 ub = __ldg(reinterpret_cast<const uint4 *>(b) + i);
            const T *ta = reinterpret_cast<const T *>(&ua);
            const T *tb = reinterpret_cast<const T *>(&ub);
#pragma unroll
            for (int k = 0; k < V; ++k) acc = fmaf(to_f(ta[k]), to_f(tb[k]), acc);
        }
        done = nv * V;
    }
    for (int64_t i = done + tid; i < n; i += nthr) acc = fmaf(to_f(a[i]), to_f(b[i]), acc);
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float v = 0.0f;
        for (int w = 0; w < 8; ++w) v += ws[w];
        g_dot_partials[blockIdx.x] = v;
    }
}

__global__ void dot_final_kernel(float *__restrict__ out) {
    float v = 0.0f;
    for (int i = threadIdx.x; i < kDotBlocks; i += 32) v += g_dot_partials[i];
    v = warp_sum(v);
    if (threadIdx.x == 0) *out = v;
}

__global__ void rowptr_kernel(const int64_t *__restrict__ keys, int64_t n, int64_t n_rows,
                              int32_t *__restrict__ row_ptr) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r <= n_rows;
         r += (int64_t)gridDim.x * blockDim.x) {
        int64_t lo = 0, hi = n;
        while (lo < hi) {
            int64_t mid = (lo + hi) >> 1;
            if (keys[mid] < r) lo = mid + 1;
            else hi = mid;
        }
        row_ptr[r] = (int32_t)lo;
    }
}

// one thread per CSR segment (row, half): the first position of each
// 256-column block inside the segment (columns ascend within a segment)
__global__ void ov_cbptr_kernel(const int32_t *__restrict__ row_ptr, const int32_t *__restrict__ col,
                                int64_t n_seg, int ncb, int32_t *__restrict__ out) {
    for (int64_t sg = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; sg < n_seg;
         sg += (int64_t)gridDim.x * blockDim.x) {
        int p = row_ptr[sg];
        const int end = row_ptr[sg + 1];
        const int64_t row = sg >> 1, h = sg & 1;
        for (int b = 0; b < ncb; ++b) {
            while (p < end && col[p] < 256 * b) ++p;
            out[(row * ncb + b) * 2 + h] = p;
        }
    }
}

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_dot(const void *a, const void *b, int32_t dtype, int64_t n, float *out,
                        void *stream) {
    USAF_REQUIRE(out && n >= 0 && (n == 0 || (a && b)));
    cudaStream_t st = as_stream(stream);
    const int vec = ((uintptr_t)a & 15) == 0 && ((uintptr_t)b & 15) == 0;
    switch (dtype) {
        case USAF_F32: dot_partial_kernel<float><<<kDotBlocks, 256, 0, st>>>((const float *)a, (const float *)b, n, vec); break;
        case USAF_BF16: dot_partial_kernel<__nv_bfloat16><<<kDotBlocks, 256, 0, st>>>((const __nv_bfloat16 *)a, (const __nv_bfloat16 *)b, n, vec); break;
        default: return USAF_EINVAL;
    }
    dot_final_kernel<<<1, 32, 0, st>>>(out);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_build_rowptr(const int64_t *keys, int64_t n, int64_t n_rows, int32_t *row_ptr,
                                 void *stream) {
    USAF_REQUIRE(row_ptr && n >= 0 && n_rows >= 0 && (keys || n == 0));
    cudaStream_t st = as_stream(stream);
    unsigned grid = (unsigned)std::min<int64_t>((n_rows + 256) / 256, 148 * 8);
    rowptr_kernel<<<grid, 256, 0, st>>>(keys, n, n_rows, row_ptr);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_build_ov_cbptr(const int32_t *row_ptr, const int32_t *col, int32_t E, int32_t R,
                                   int32_t C, int32_t *out, void *stream) {
    USAF_REQUIRE(row_ptr && out && E >= 0 && R >= 0 && C >= 1);
    const int64_t n_seg = (int64_t)E * R * 2;
    if (n_seg == 0) return USAF_OK;
    cudaStream_t st = as_stream(stream);
    unsigned grid = (unsigned)std::min<int64_t>((n_seg + 255) / 256, 148 * 8);
    ov_cbptr_kernel<<<grid, 256, 0, st>>>(row_ptr, col, n_seg, (C + 255) / 256, out);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" const char *usaf_version(void) { return "usaf_b200 0.1 sm_100a"; }
