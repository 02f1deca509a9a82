// C ABI of the grouped expert GEMMs: routes each call to the kernel for its
// dtype (fp32 -> CUDA-core kernels of gemm_simt.cu; bf16 -> tcgen05 kernels
// of gemm_tc.cu) and checks the shapes those kernels accept.
#include "common.cuh"
#include "gemm_tc.cuh"

namespace usaf {
template <typename Act, bool TRANS>
int launch_simt(const usaf_route_plan *, const usaf_qweight *, const Act *, int, int, Act *, int,
                cudaStream_t);
template <typename Act>
int launch_swiglu_fwd(const usaf_route_plan *, const Act *, int, Act *, cudaStream_t);
template <typename Act>
int launch_swiglu_bwd(const usaf_route_plan *, const Act *, int, const Act *, int, Act *,
                      cudaStream_t);
}  // namespace usaf

using namespace usaf;
using bf16 = __nv_bfloat16;

static bool qweight_ok(const usaf_qweight *w) {
    return w && w->q && w->s && w->z && w->E >= 1 && w->R >= 1 && w->C >= 1 &&
           w->group_size >= 2 && w->C % w->group_size == 0 && (w->n_ov == 0 || (w->row_ptr && w->col && w->val));
}

extern "C" int usaf_expert_gate_up_fwd(const usaf_route_plan *plan, const usaf_qweight *w_gu,
                                       const void *x_perm, int32_t dtype, void *gu, void *h,
                                       void *stream) {
    USAF_REQUIRE(plan && qweight_ok(w_gu) && x_perm && gu && h && w_gu->R % 2 == 0 && plan->E == w_gu->E);
    cudaStream_t st = as_stream(stream);
    const int K = w_gu->C, N = w_gu->R, I = N / 2;
    int rc;
    if (dtype == USAF_F32) {
        rc = launch_simt<float, false>(plan, w_gu, (const float *)x_perm, K, N, (float *)gu, N, st);
        if (rc) return rc;
        return launch_swiglu_fwd<float>(plan, (const float *)gu, I, (float *)h, st);
    }
    if (dtype == USAF_BF16) {
        if (tc_supported_gate_up(w_gu)) return tc_gate_up_fwd(plan, w_gu, (const bf16 *)x_perm, (bf16 *)gu, (bf16 *)h, st);
        rc = launch_simt<bf16, false>(plan, w_gu, (const bf16 *)x_perm, K, N, (bf16 *)gu, N, st);
        if (rc) return rc;
        return launch_swiglu_fwd<bf16>(plan, (const bf16 *)gu, I, (bf16 *)h, st);
    }
    return USAF_EINVAL;
}

extern "C" int usaf_expert_down_fwd(const usaf_route_plan *plan, const usaf_qweight *w_dn,
                                    const void *h, int32_t dtype, void *y_seg, void *stream) {
    USAF_REQUIRE(plan && qweight_ok(w_dn) && h && y_seg && plan->E == w_dn->E);
    cudaStream_t st = as_stream(stream);
    const int K = w_dn->C, N = w_dn->R;
    if (dtype == USAF_F32) return launch_simt<float, false>(plan, w_dn, (const float *)h, K, N, (float *)y_seg, N, st);
    if (dtype == USAF_BF16) {
        if (tc_supported_down(w_dn)) return tc_down_fwd(plan, w_dn, (const bf16 *)h, (bf16 *)y_seg, st);
        return launch_simt<bf16, false>(plan, w_dn, (const bf16 *)h, K, N, (bf16 *)y_seg, N, st);
    }
    return USAF_EINVAL;
}

extern "C" int usaf_expert_down_bwd(const usaf_route_plan *plan, const usaf_qweight *w_dn,
                                    const void *dcur, const void *gu, int32_t dtype, void *dgu,
                                    void *stream) {
    USAF_REQUIRE(plan && qweight_ok(w_dn) && dcur && gu && dgu && plan->E == w_dn->E);
    USAF_REQUIRE(w_dn->n_ov == 0 || (w_dn->colT_ptr && w_dn->rowT && w_dn->valT));
    cudaStream_t st = as_stream(stream);
    // dh = dcur @ W_dn[e] (storage [E,H,I]: K = H = R, N = I = C), written
    // into the gate half of dgu, then SwiGLU backward in place
    const int K = w_dn->R, N = w_dn->C, I = N;
    int rc;
    if (dtype == USAF_F32) {
        rc = launch_simt<float, true>(plan, w_dn, (const float *)dcur, K, N, (float *)dgu, 2 * I, st);
        if (rc) return rc;
        return launch_swiglu_bwd<float>(plan, (const float *)dgu, 2 * I, (const float *)gu, I, (float *)dgu, st);
    }
    if (dtype == USAF_BF16) {
        if (tc_supported_down_bwd(w_dn)) return tc_down_bwd(plan, w_dn, (const bf16 *)dcur, (const bf16 *)gu, (bf16 *)dgu, st);
        rc = launch_simt<bf16, true>(plan, w_dn, (const bf16 *)dcur, K, N, (bf16 *)dgu, 2 * I, st);
        if (rc) return rc;
        return launch_swiglu_bwd<bf16>(plan, (const bf16 *)dgu, 2 * I, (const bf16 *)gu, I, (bf16 *)dgu, st);
    }
    return USAF_EINVAL;
}

extern "C" int usaf_expert_gate_up_bwd(const usaf_route_plan *plan, const usaf_qweight *w_gu,
                                       const void *dgu, int32_t dtype, void *dx_seg,
                                       void *stream) {
    USAF_REQUIRE(plan && qweight_ok(w_gu) && dgu && dx_seg && plan->E == w_gu->E);
    USAF_REQUIRE(w_gu->n_ov == 0 || (w_gu->colT_ptr && w_gu->rowT && w_gu->valT));
    cudaStream_t st = as_stream(stream);
    // dx = dgu @ W_gu[e] (storage [E,2I,H]: K = 2I = R, N = H = C)
    const int K = w_gu->R, N = w_gu->C;
    if (dtype == USAF_F32) return launch_simt<float, true>(plan, w_gu, (const float *)dgu, K, N, (float *)dx_seg, N, st);
    if (dtype == USAF_BF16) {
        if (tc_supported_gate_up_bwd(w_gu)) return tc_gate_up_bwd(plan, w_gu, (const bf16 *)dgu, (bf16 *)dx_seg, st);
        return launch_simt<bf16, true>(plan, w_gu, (const bf16 *)dgu, K, N, (bf16 *)dx_seg, N, st);
    }
    return USAF_EINVAL;
}
