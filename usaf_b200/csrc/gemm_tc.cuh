// tcgen05 grouped expert GEMMs (bf16, int4 weights dequantized on the fly).
#pragma once
#include "common.cuh"

namespace usaf {
bool tc_supported_gate_up(const usaf_qweight *w);
bool tc_supported_down(const usaf_qweight *w);
bool tc_supported_down_bwd(const usaf_qweight *w);
bool tc_supported_gate_up_bwd(const usaf_qweight *w);
int tc_gate_up_fwd(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *x_perm,
                   __nv_bfloat16 *gu, __nv_bfloat16 *h, cudaStream_t st);
int tc_down_fwd(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *h,
                __nv_bfloat16 *y_seg, cudaStream_t st);
int tc_down_bwd(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *dcur,
                const __nv_bfloat16 *gu, __nv_bfloat16 *dgu, cudaStream_t st);
int tc_gate_up_bwd(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *dgu,
                   __nv_bfloat16 *dx_seg, cudaStream_t st);

}  // namespace usaf
