// Fused SparseAdam (usaf/sparse_optim.py:86-134) over the selected-index list.
//
// One HBM-bound pass per element: grad (divided by the loss-scale
// denominator, train.py:661-662), L2 weight decay added to the gradient,
// m/v update, bias-corrected step, master update, and the write-back of the
// new value into the GEMM overlay (fp16 of the master, then the compute
// dtype), which is sync_resident (usaf/moe_loader.py:425-443) fused in.
// The fp32 operation sequence follows the reference's CPU kernels exactly:
//   m = fma(g, 1-b1, m*b1)            (add_ with alpha is a fused multiply-add)
//   v = fma((1-b2)*g, g, v*b2)        (addcmul_)
//   upd = (m / bias1) / (sqrt(v / bias2) + eps);  delta = (-lr) * upd
#include "common.cuh"

namespace usaf {

struct AdamConsts {
    float b1, omb1, b2, omb2, bias1, bias2, eps, neg_lr, wd, gdiv;
};

static AdamConsts make_consts(int step, double lr, double b1, double b2, double eps, double wd,
                              double gdiv) {
    AdamConsts c;
    c.b1 = (float)b1;
    c.omb1 = (float)(1.0 - b1);
    c.b2 = (float)b2;
    c.omb2 = (float)(1.0 - b2);
    c.bias1 = (float)(1.0 - std::pow(b1, (double)step));
    c.bias2 = (float)(1.0 - std::pow(b2, (double)step));
    c.eps = (float)eps;
    c.neg_lr = (float)(-lr);
    c.wd = (float)wd;
    c.gdiv = (float)gdiv;
    return c;
}

__device__ __forceinline__ float adam_delta(float p, float g, float &m, float &v,
                                            const AdamConsts &c) {
    if (c.wd > 0.0f) g = __fadd_rn(g, __fmul_rn(c.wd, p));
    m = __fmaf_rn(g, c.omb1, __fmul_rn(m, c.b1));
    v = __fmaf_rn(__fmul_rn(c.omb2, g), g, __fmul_rn(v, c.b2));
    float upd = __fdiv_rn(__fdiv_rn(m, c.bias1), __fadd_rn(__fsqrt_rn(__fdiv_rn(v, c.bias2)), c.eps));
    return __fmul_rn(c.neg_lr, upd);
}

template <typename Act>
__global__ void adam_compact_kernel(int64_t n, float *__restrict__ p, float *__restrict__ m,
                                    float *__restrict__ v, const float *__restrict__ grad,
                                    AdamConsts c, float *__restrict__ ov_val,
                                    const int32_t *__restrict__ ov_pos,
                                    float *__restrict__ ov_valT,
                                    const int32_t *__restrict__ ov_posT) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        float g = c.gdiv == 1.0f ? grad[i] : __fdiv_rn(grad[i], c.gdiv);
        float pi = p[i], mi = m[i], vi = v[i];
        float d = adam_delta(pi, g, mi, vi, c);
        float np = __fadd_rn(pi, d);
        p[i] = np;
        m[i] = mi;
        v[i] = vi;
        // the resident weight holds fp16(master) (usaf/moe_loader.py:442)
        float ev = to_f(from_f<Act>(__half2float(__float2half_rn(np))));
        if (ov_val) ov_val[ov_pos ? ov_pos[i] : i] = ev;   // NULL map: CSR order
        if (ov_valT) ov_valT[ov_posT[i]] = ev;
    }
}

template <typename P>
__global__ void adam_gather_kernel(int64_t n, const int64_t *__restrict__ idx, P *__restrict__ param,
                                   const P *__restrict__ grad, float *__restrict__ m,
                                   float *__restrict__ v, AdamConsts c) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t j = idx[i];
        float g = to_f(grad[j]);
        if (c.gdiv != 1.0f) g = to_f(from_f<P>(__fdiv_rn(g, c.gdiv)));  // grad.div_ in its dtype
        float pi = to_f(param[j]);
        float mi = m[i], vi = v[i];
        float d = adam_delta(pi, g, mi, vi, c);
        // delta is cast to the parameter dtype, then added in that dtype (:127, :134)
        param[j] = from_f<P>(__fadd_rn(pi, to_f(from_f<P>(d))));
        m[i] = mi;
        v[i] = vi;
    }
}

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_sparse_adam(int64_t n, float *p, float *m, float *v, const float *grad,
                                double grad_div, int32_t step, double lr, double beta1,
                                double beta2, double eps, double weight_decay, int32_t dtype,
                                float *ov_val, const int32_t *ov_pos, float *ov_valT,
                                const int32_t *ov_posT, void *stream) {
    USAF_REQUIRE(n >= 0 && step >= 1);
    if (n == 0) return USAF_OK;
    USAF_REQUIRE(p && m && v && grad);
    USAF_REQUIRE(ov_val != nullptr || ov_pos == nullptr);
    USAF_REQUIRE((ov_valT == nullptr) == (ov_posT == nullptr));
    AdamConsts c = make_consts(step, lr, beta1, beta2, eps, weight_decay, grad_div);
    cudaStream_t st = as_stream(stream);
    unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
    switch (dtype) {
        case USAF_F32: adam_compact_kernel<float><<<grid, 256, 0, st>>>(n, p, m, v, grad, c, ov_val, ov_pos, ov_valT, ov_posT); break;
        case USAF_BF16: adam_compact_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(n, p, m, v, grad, c, ov_val, ov_pos, ov_valT, ov_posT); break;
        case USAF_F16: adam_compact_kernel<__half><<<grid, 256, 0, st>>>(n, p, m, v, grad, c, ov_val, ov_pos, ov_valT, ov_posT); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_sparse_adam_gather(int64_t n, const int64_t *idx, void *param, const void *grad,
                                       int32_t dtype, double grad_div, float *m, float *v,
                                       int32_t step, double lr, double beta1, double beta2,
                                       double eps, double weight_decay, void *stream) {
    USAF_REQUIRE(n >= 0 && step >= 1);
    if (n == 0) return USAF_OK;
    USAF_REQUIRE(idx && param && grad && m && v);
    AdamConsts c = make_consts(step, lr, beta1, beta2, eps, weight_decay, grad_div);
    cudaStream_t st = as_stream(stream);
    unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
    switch (dtype) {
        case USAF_F32: adam_gather_kernel<float><<<grid, 256, 0, st>>>(n, idx, (float *)param, (const float *)grad, m, v, c); break;
        case USAF_BF16: adam_gather_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(n, idx, (__nv_bfloat16 *)param, (const __nv_bfloat16 *)grad, m, v, c); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
