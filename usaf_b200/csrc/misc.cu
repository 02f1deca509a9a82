// Small utilities of the C ABI: a deterministic dot product (the step's
// scalar readback), CSR row pointers from sorted row keys, and the version.
#include "common.cuh"

namespace usaf {

template <typename T>
__global__ void __launch_bounds__(1024) dot_kernel(const T *__restrict__ a, const T *__restrict__ b,
                                                   int64_t n, float *__restrict__ out) {
    // single block: fixed reduction order, so the scalar is reproducible
    __shared__ float ws[32];
    float acc = 0.0f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) acc = fmaf(to_f(a[i]), to_f(b[i]), acc);
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = ws[threadIdx.x];
        v = warp_sum(v);
        if (threadIdx.x == 0) *out = v;
    }
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

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_dot(const void *a, const void *b, int32_t dtype, int64_t n, float *out,
                        void *stream) {
    USAF_REQUIRE(a && b && out && n >= 0);
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case USAF_F32: dot_kernel<float><<<1, 1024, 0, st>>>((const float *)a, (const float *)b, n, out); break;
        case USAF_BF16: dot_kernel<__nv_bfloat16><<<1, 1024, 0, st>>>((const __nv_bfloat16 *)a, (const __nv_bfloat16 *)b, n, out); break;
        default: return USAF_EINVAL;
    }
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

extern "C" const char *usaf_version(void) { return "usaf_b200 0.1 sm_100a"; }
