// Importance candidates without the dense |grad| buffer (bf16, tensor cores).
//
// TopKImportanceStore.add (usaf/moe_loader.py:604-611) keeps, for every expert
// that received tokens, the top k = max(1, int(numel_e * frac * cand_mult))
// entries of |grad_e| with their flat indices.  Here the gradient tiles are
// formed three times by the tensor-core SDDMM (sddmm_tc.cu) and never written
// out; what leaves the SM per pass is:
//   pass 1  a histogram per expert of the 8 exponent bits of the 15-bit key of
//           |bf16(g)| (the key orders like the value);
//   pick    per expert the exponent bucket that holds the k-th largest key;
//   pass 2  a histogram of the keys inside that bucket (its 7 mantissa bits);
//   pick    the k-th largest key itself (the threshold), the number of keys
//           equal to it and how many of those the list takes;
//   pass 3  every key above the threshold into the expert's candidate list,
//           every key equal to it into the expert's tie list;
//   ties    the tie lists ordered by flat index (usaf_sort_u32) and the lowest
//           indices appended to each candidate list (ties resolve to the
//           lowest flat index, as usaf_topk_desc does);
//   order   each list sorted by descending value, ties by ascending index.
// An expert whose slots span several SDDMM chunks is summed chunk after chunk
// in TMEM (usaf_importance_chunk_slots() slots per chunk).
#include "common.cuh"

namespace usaf {

int sddmm_tc_key_hist(const usaf_route_plan *pl, int R, int C, const __nv_bfloat16 *gout,
                      const __nv_bfloat16 *gin, int shift, int pmask, const int32_t *pval,
                      unsigned int *hist, cudaStream_t st);
int sddmm_tc_key_emit(const usaf_route_plan *pl, int R, int C, const __nv_bfloat16 *gout,
                      const __nv_bfloat16 *gin, const int32_t *thr, int64_t k, const int32_t *cand_row,
                      int32_t *n_gt, int32_t *n_eq, float *gt_val, int64_t *gt_idx, const int64_t *eq_off,
                      float *eq_val, int64_t *eq_idx, cudaStream_t st);
int sddmm_tc_chunk_slots();
bool sddmm_tc_supported(int R, int C);

namespace {

constexpr int kBins = 256;

// One block per expert.  level 1: hist holds every key of the expert binned
// by exponent; the bucket b with the k-th largest key gives pval[e] = b << 7
// and need[e] = k - (keys in higher buckets).  level 2: hist holds the keys
// of that bucket binned by their low 8 bits; the bin with the need[e]-th
// largest gives thr[e], the count of keys equal to it (n_eq[e]) and need[e]
// becomes the number of those the list takes.  Experts without slots
// (level 1) or left out (pval < 0, level 2) get -1.
__global__ void __launch_bounds__(kBins) imp_pick(const unsigned int *__restrict__ hist, int64_t k,
                                                  const int32_t *__restrict__ cnt, int level, int32_t *pval,
                                                  int64_t *need, int32_t *thr, int64_t *n_eq) {
    const int e = blockIdx.x, t = threadIdx.x;
    __shared__ unsigned long long suf[kBins + 1];
    if ((level == 1 && cnt[e] <= 0) || (level == 2 && pval[e] < 0)) {
        if (t == 0) {
            if (level == 1) {
                pval[e] = -1;
                need[e] = 0;
            } else {
                thr[e] = -1;
                n_eq[e] = 0;
                need[e] = 0;
            }
        }
        return;
    }
    const unsigned long long h = hist[(int64_t)e * kBins + t];
    suf[t] = h;
    if (t == 0) suf[kBins] = 0;
    __syncthreads();
    // suffix sums over the bins (Hillis-Steele from the top)
    for (int o = 1; o < kBins; o <<= 1) {
        const unsigned long long add = t + o < kBins ? suf[t + o] : 0ull;
        __syncthreads();
        suf[t] += add;
        __syncthreads();
    }
    const long long target = level == 1 ? k : need[e];
    // the unique bin whose suffix reaches the target and whose next does not
    if ((long long)suf[t] >= target && (long long)suf[t + 1] < target) {
        if (level == 1) {
            pval[e] = t << 7;
            need[e] = target - (long long)suf[t + 1];
        } else {
            thr[e] = (pval[e] & ~0xFF) | t;
            n_eq[e] = (long long)h;
            need[e] = target - (long long)suf[t + 1];
        }
    }
}

// the lowest-index need[e] ties of expert e (its tie list already ordered by
// index) fill the end of its candidate list
__global__ void imp_take_ties(int64_t k, const int32_t *__restrict__ cand_row, const int64_t *__restrict__ need,
                              const int64_t *__restrict__ eq_off, const float *__restrict__ eq_val,
                              const int64_t *__restrict__ eq_idx, float *gt_val, int64_t *gt_idx) {
    const int e = blockIdx.y;
    const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int row = cand_row[e];
    if (row < 0) return;
    const int64_t nt = need[e];
    if (j >= nt) return;
    const int64_t dst = (int64_t)row * k + (k - nt) + j;
    gt_val[dst] = eq_val[eq_off[e] + j];
    gt_idx[dst] = eq_idx[eq_off[e] + j];
}

// optional gather through perm, then sort keys of the result:
// mode 0 the flat index, mode 1 (list << 15) | (0x7FFF - value key) (list =
// position / k: ascending list, descending value), mode 2 no keys
__global__ void imp_keys(const float *__restrict__ vin, const int64_t *__restrict__ iin,
                         const int64_t *__restrict__ perm, int64_t n, int64_t k, int mode, float *vout,
                         int64_t *iout, uint32_t *keys, int64_t *pos) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t src = perm ? perm[i] : i;
        const float v = vin[src];
        const int64_t ix = iin[src];
        if (vout) vout[i] = v;
        if (iout) iout[i] = ix;
        if (mode == 0) keys[i] = (uint32_t)ix;
        else if (mode == 1)
            keys[i] = ((uint32_t)(i / k) << 15) | (0x7FFFu - ((__float_as_uint(v) >> 16) & 0x7FFFu));
        if (pos) pos[i] = i;
    }
}

}  // namespace
}  // namespace usaf

using namespace usaf;

extern "C" int32_t usaf_importance_chunk_slots(void) { return sddmm_tc_chunk_slots(); }

extern "C" int usaf_importance_supported(int32_t R, int32_t C, int32_t dtype) {
    return dtype == USAF_BF16 && sddmm_tc_supported(R, C) ? 1 : 0;
}

extern "C" int usaf_importance_hist(const usaf_route_plan *plan, int32_t R, int32_t C, const void *gout,
                                    const void *gin, int32_t dtype, int32_t level, const int32_t *pval,
                                    uint32_t *hist, void *stream) {
    USAF_REQUIRE(plan && gout && gin && hist && R >= 1 && C >= 1 && (level == 1 || (level == 2 && pval)));
    if (!usaf_importance_supported(R, C, dtype)) return USAF_EUNSUPPORTED;
    // level 1: every key, binned by its exponent; level 2: the keys of the chosen
    // exponent bucket, binned by their low 8 bits
    const int shift = level == 1 ? 7 : 0, pmask = level == 1 ? 0 : 0x7F80;
    return sddmm_tc_key_hist(plan, R, C, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin, shift, pmask,
                             level == 1 ? nullptr : pval, hist, as_stream(stream));
}

extern "C" int usaf_importance_pick(const uint32_t *hist, int32_t E, int64_t k, const int32_t *expert_cnt,
                                    int32_t level, int32_t *pval, int64_t *need, int32_t *thr, int64_t *n_eq,
                                    void *stream) {
    USAF_REQUIRE(hist && E >= 1 && k >= 1 && pval && need && (level == 1 ? expert_cnt != nullptr : (thr && n_eq)));
    USAF_REQUIRE(level == 1 || level == 2);
    imp_pick<<<E, kBins, 0, as_stream(stream)>>>(hist, k, expert_cnt, level, pval, need, thr, n_eq);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_importance_emit(const usaf_route_plan *plan, int32_t R, int32_t C, const void *gout,
                                    const void *gin, int32_t dtype, const int32_t *thr, int64_t k,
                                    const int32_t *cand_row, int32_t *n_gt, int32_t *n_eq, float *cand_val,
                                    int64_t *cand_idx, const int64_t *eq_off, float *eq_val, int64_t *eq_idx,
                                    void *stream) {
    USAF_REQUIRE(plan && gout && gin && thr && k >= 1 && cand_row && n_gt && n_eq && cand_val && cand_idx &&
                 eq_off && R >= 1 && C >= 1);
    if (!usaf_importance_supported(R, C, dtype)) return USAF_EUNSUPPORTED;
    return sddmm_tc_key_emit(plan, R, C, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin, thr, k, cand_row,
                             n_gt, n_eq, cand_val, cand_idx, eq_off, eq_val, eq_idx, as_stream(stream));
}

extern "C" int usaf_importance_take_ties(int32_t E, int64_t k, const int32_t *cand_row, const int64_t *need,
                                         const int64_t *eq_off, const float *eq_val, const int64_t *eq_idx,
                                         float *cand_val, int64_t *cand_idx, void *stream) {
    USAF_REQUIRE(E >= 1 && k >= 1 && cand_row && need && eq_off && cand_val && cand_idx);
    dim3 grid(cdiv(k, 256), E);
    imp_take_ties<<<grid, 256, 0, as_stream(stream)>>>(k, cand_row, need, eq_off, eq_val, eq_idx, cand_val, cand_idx);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_importance_keys(const float *val, const int64_t *idx, const int64_t *perm, int64_t n,
                                    int64_t k, int32_t mode, float *val_out, int64_t *idx_out, uint32_t *keys,
                                    int64_t *pos, void *stream) {
    USAF_REQUIRE(n >= 0 && k >= 1 && mode >= 0 && mode <= 2);
    if (n == 0) return USAF_OK;
    USAF_REQUIRE(val && idx && (mode == 2 || keys));
    if (mode == 1) USAF_REQUIRE(n / k < (1 << 16));
    const unsigned grid = std::max(1u, std::min(cdiv(n, 256), 148u * 8u));
    imp_keys<<<grid, 256, 0, as_stream(stream)>>>(val, idx, perm, n, k, mode, val_out, idx_out, keys, pos);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
