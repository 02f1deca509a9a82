// tcgen05 grouped expert GEMMs -- placeholder until the sm_100a kernels land.
#include "gemm_tc.cuh"

namespace usaf {
bool tc_supported_gate_up(const usaf_qweight *) { return false; }
bool tc_supported_down(const usaf_qweight *) { return false; }
bool tc_supported_down_bwd(const usaf_qweight *) { return false; }
bool tc_supported_gate_up_bwd(const usaf_qweight *) { return false; }
int tc_gate_up_fwd(const usaf_route_plan *, const usaf_qweight *, const __nv_bfloat16 *, __nv_bfloat16 *, __nv_bfloat16 *, cudaStream_t) { return USAF_EUNSUPPORTED; }
int tc_down_fwd(const usaf_route_plan *, const usaf_qweight *, const __nv_bfloat16 *, __nv_bfloat16 *, cudaStream_t) { return USAF_EUNSUPPORTED; }
int tc_down_bwd(const usaf_route_plan *, const usaf_qweight *, const __nv_bfloat16 *, const __nv_bfloat16 *, __nv_bfloat16 *, cudaStream_t) { return USAF_EUNSUPPORTED; }
int tc_gate_up_bwd(const usaf_route_plan *, const usaf_qweight *, const __nv_bfloat16 *, __nv_bfloat16 *, cudaStream_t) { return USAF_EUNSUPPORTED; }
}  // namespace usaf
