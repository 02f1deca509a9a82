/*
 * usaf_b200.h -- C ABI of the B200-native MoE expert hot path.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream (passed as void*), enqueues its kernels on that stream and returns
 * an int status (USAF_OK or one of the USAF_E* codes below).  Nothing here
 * allocates device memory or synchronizes the host; buffers are owned by the
 * caller.  Device-side failures (an overflowing pair buffer, a wait that ran
 * out) are recorded in the caller's `err` word, which the caller reads back
 * when it syncs.
 *
 * Each function names the reference interface it replaces
 * (tsuyu122/usaf, path:line within that project).
 */
#ifndef USAF_B200_H
#define USAF_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define USAF_OK            0
#define USAF_EINVAL        1   /* bad argument (null pointer, negative size, bad dtype) */
#define USAF_EUNSUPPORTED  2   /* shape the kernels do not handle (e.g. K % 64 != 0) */
#define USAF_ECUDA         3   /* a CUDA launch failed */

/* device error-word bits (set with atomicOr by kernels) */
#define USAF_ERR_PAIR_OVERFLOW  1   /* more routed pairs than the pair buffer holds */
#define USAF_ERR_WAIT_TIMEOUT   2   /* a bounded device-side wait gave up */
#define USAF_ERR_BAD_INDEX      4   /* an index outside its tensor was skipped */

/* activation / compute dtypes */
#define USAF_F32   0
#define USAF_BF16  1
#define USAF_F16   2

/* Routing plan: the dispatch of (token, expert) pairs into per-expert
 * contiguous segments.  Pairs are the nonzero entries of the dense routing
 * weights in token-major order (benchmarks/kaggle_t4_bench.py:293); slots are
 * the same pairs stably sorted by expert (:298), ascending token within an
 * expert. */
typedef struct {
    int32_t  T, E, P_cap;
    int32_t *tok_cnt;     /* [T]      pairs per token                          */
    int32_t *tok_off;     /* [T+1]    exclusive scan of tok_cnt                */
    int32_t *expert_cnt;  /* [E]      tokens per expert (bincount, :296)      */
    int32_t *expert_off;  /* [E+1]    exclusive scan of expert_cnt (:300-301) */
    int32_t *seg_tok;     /* [P_cap]  token of each slot                       */
    int32_t *seg_pair;    /* [P_cap]  token-major pair index of each slot      */
    float   *seg_w;       /* [P_cap]  routing weight of each slot              */
    int32_t *pair_exp;    /* [P_cap]  expert of each token-major pair          */
    int32_t *pair_slot;   /* [P_cap]  slot of each token-major pair            */
    int32_t *n_pairs;     /* [1]                                               */
    int32_t *chunk_cnt;   /* [ceil(T/16)*E] scratch                            */
    int32_t *err;         /* [1]      device error word                        */
    int32_t *sched;       /* [16] or NULL: work counters of the grouped expert
                           * GEMMs (one pair per entry point).  Zeroed once by
                           * the caller; every launch hands its work items out
                           * from them longest first and leaves them zeroed.
                           * Launches that share a plan must not overlap on
                           * the GPU.  NULL: a fixed round-robin assignment. */
} usaf_route_plan;

/* One int4 expert projection in the usaf.quantization layout
 * (usaf/quantization.py:21-85) with its sparse overlay of trained values
 * (usaf/moe_loader.py:241-247).  Storage shape [E, R, C], groups of
 * `group_size` consecutive elements along C (C % group_size == 0).
 * The overlay is held twice: CSR by storage row and CSC by storage column,
 * each split into two sorted segments per row (column): entries whose
 * column (row) index has bit 5 clear, then those with bit 5 set -- the two
 * 32-wide halves of every 64-wide k-block.  Values are already rounded the
 * way the reference rounds them (fp16 of the master, then the compute dtype). */
typedef struct {
    int32_t E, R, C, group_size;
    const int8_t   *q;        /* [E*R*C/2] packed codes, low nibble = even element */
    const uint16_t *s;        /* [E*R*C/group_size] fp16 scales                   */
    const uint16_t *z;        /* [E*R*C/group_size] fp16 zeros                    */
    int32_t n_ov;
    const int32_t *row_ptr;   /* [E*R*2+1] CSR offsets, segment (row, half)         */
    const int32_t *col;       /* [n_ov]   column of each CSR entry                 */
    const float   *val;       /* [n_ov]   effective value of each CSR entry        */
    const int32_t *colT_ptr;  /* [E*C*2+1] CSC offsets, segment (column, half)      */
    const int32_t *rowT;      /* [n_ov]   row of each CSC entry                    */
    const float   *valT;      /* [n_ov]   effective value of each CSC entry        */
    /* copies for the tensor-core GEMMs, codes in the usaf_int4_repack order:
     * qP [E*R*C/2] row-major (forward), qT [E*C*R/2] column-major (backward,
     * usaf_int4_transpose), szT [E*(C/group_size)*R] uint32: per (column
     * group, pair of rows 2p, 2p+1) the words scale[2p] | scale[2p+1] << 16
     * and zero[2p] | zero[2p+1] << 16 */
    const int8_t   *qT;
    const uint32_t *szT;
    const int8_t   *qP;
    /* overlay bitmap [E*R*C/32]: bit (c % 32) of word (e*R + r)*(C/32) + c/32
     * is set for every overlay coordinate (e, r, c).  Optional (NULL selects
     * the SIMT gradient kernel); the tensor-core usaf_sparse_dw reads it. */
    const uint32_t *ov_mask;
    /* overlay positions per 256-column block [E*R*ceil(C/256)*2]: entry
     * ((e*R + r)*ceil(C/256) + b)*2 + h is the CSR position of the first entry
     * of segment (row e*R + r, half h) whose column is >= 256*b
     * (usaf_build_ov_cbptr).  The tensor-core usaf_sparse_dw needs it with
     * ov_mask; NULL selects the SIMT gradient kernel. */
    const int32_t *ov_cbptr;
    /* [E] or NULL: the largest number of overlay coordinates in one storage
     * row (ov_emax) / storage column (ov_emaxT) of each expert.  The grouped
     * GEMMs order their work by it besides the token count: a heavily
     * trained row or column slows the whole item it belongs to. */
    const int32_t *ov_emax;
    const int32_t *ov_emaxT;
} usaf_qweight;

/* ---- int4 format ---------------------------------------------------------
 * usaf_dequant_int4 replaces dequantize_4bit (usaf/quantization.py:88-132):
 * out = fp16(fp16(q*s) + z), written as fp16 (out_dtype USAF_F16) or that
 * fp16 value converted to fp32/bf16.  Bit-exact with the reference.
 * usaf_quant_int4 replaces quantize_4bit (usaf/quantization.py:21-85);
 * x is fp32/bf16/fp16, numel >= 1. */
int usaf_dequant_int4(const void *q, const void *s, const void *z, int64_t numel,
                      int32_t group_size, int32_t out_dtype, void *out, void *stream);
int usaf_quant_int4(const void *x, int32_t x_dtype, int64_t numel, int32_t group_size,
                    void *q, void *s, void *z, void *stream);

/* usaf_int4_transpose: build the column-major copy (qT, szT) of a projection
 * [E, R, C] for the tensor-core backward GEMMs.  Same codes, scales and
 * zeros, re-laid so a storage column's codes are contiguous. */
int usaf_int4_transpose(const void *q, const void *s, const void *z, int32_t E, int32_t R,
                        int32_t C, int32_t group_size, void *qT, void *szT, void *stream);

/* usaf_int4_repack: copy of the packed codes with the nibbles of every 32-bit
 * word (8 elements) reordered to e0 e2 e4 e6 e1 e3 e5 e7, the order the
 * tensor-core producers dequantize from (numel % 8 == 0).  The backward copy
 * of usaf_int4_transpose is written in the same order. */
int usaf_int4_repack(const void *q, int64_t numel, void *qp, void *stream);

/* ---- router ----------------------------------------------------------------
 * usaf_router_fwd replaces the router of dml_qwen3_moe_block_forward
 * (usaf/qwen3moe_dml.py:72-83): logits = X W_r^T rounded to the activation
 * dtype, fp32 softmax, threshold mask probs >= k-th largest (ties admit more
 * than k), renormalisation, weights cast to the activation dtype.
 * logits/probs: fp32 [T,E]; wsum: fp32 [T] (the renormaliser); weights:
 * activation dtype [T,E].
 * usaf_router_select runs the same selection from given logits.
 * ws: usaf_router_workspace_bytes(T, H, E) bytes or NULL; err: device error word. */
int usaf_router_fwd(const void *x, const void *w_r, int32_t dtype, int32_t T, int32_t H,
                    int32_t E, int32_t top_k, int32_t norm_topk_prob, float *logits,
                    float *probs, float *wsum, void *weights, void *ws, int32_t *err,
                    void *stream);
int usaf_router_select(const float *logits, int32_t dtype, int32_t T, int32_t E,
                       int32_t top_k, int32_t norm_topk_prob, float *probs, float *wsum,
                       void *weights, void *stream);

/* usaf_router_bwd replaces autograd through the router (renorm, mask, fp32
 * softmax and F.linear; usaf/qwen3moe_dml.py:73-83, trained by train.py:147-152).
 * dw_pair: fp32 [P] gradient of each pair's routing weight (activation-dtype
 * value).  Writes dlogits (activation dtype rounded, fp32 storage) [T,E],
 * dW_r (activation dtype) [E,H] and adds dlogits W_r into dx_acc (fp32 [T,H]). */
int usaf_router_bwd(const usaf_route_plan *plan, const void *x, const void *w_r,
                    int32_t dtype, int32_t H, int32_t norm_topk_prob, const float *probs,
                    const float *wsum, const void *weights, const float *dw_pair,
                    float *dlogits, void *dw_r, float *dx_acc, void *ws, void *stream);
/* Workspace of the router GEMMs (bf16 runs them on tensor cores: logits,
 * dX_r and dW_r with split-K partials summed in a fixed order).  ws may be
 * NULL (CUDA-core path); err receives device-side wait timeouts. */
int64_t usaf_router_workspace_bytes(int32_t T, int32_t H, int32_t E);

/* ---- dispatch / combine ---------------------------------------------------
 * usaf_dispatch replaces the nonzero / bincount / stable argsort / cumsum
 * dispatch of batched_sparse_experts_forward (benchmarks/kaggle_t4_bench.py:
 * 293-306) and gathers the routed rows: x_perm[slot] = x[seg_tok[slot]]. */
int usaf_dispatch(const usaf_route_plan *plan, const void *weights, const void *x,
                  int32_t dtype, int32_t H, void *x_perm, void *stream);

/* usaf_combine replaces the weighted combine (usaf/qwen3moe_dml.py:62,
 * benchmarks/kaggle_t4_bench.py:280-281): y[t] = sum over t's pairs in
 * ascending expert order of fp32(y_seg[slot]) * w, fp32 accumulation, cast
 * to the activation dtype.  usaf_combine, usaf_combine_bwd and usaf_gather_dx
 * move rows as 16-byte vectors: H * sizeof(dtype) % 16 == 0 and 16-byte
 * aligned row buffers, else USAF_EUNSUPPORTED; E <= 1024. */
int usaf_combine(const usaf_route_plan *plan, const void *y_seg, int32_t dtype, int32_t H,
                 void *y, void *stream);

/* usaf_combine_bwd: dcur[slot] = dtype(dy[t] * w) and
 * dw_pair[p] = dtype(sum_h dy[t,h] * y_seg[slot,h]) (autograd of :62). */
int usaf_combine_bwd(const usaf_route_plan *plan, const void *dy, const void *y_seg,
                     int32_t dtype, int32_t H, void *dcur, float *dw_pair, void *stream);

/* usaf_gather_dx: dx[t] = dtype(sum over t's pairs (ascending expert) of
 * dx_seg[slot] + dx_acc[t]). */
int usaf_gather_dx(const usaf_route_plan *plan, const void *dx_seg, const float *dx_acc,
                   int32_t dtype, int32_t H, void *dx, void *stream);

/* ---- grouped expert GEMMs over int4 weights --------------------------------
 * Replace the per-expert F.linear pairs of usaf/qwen3moe_dml.py:58-61 and
 * their autograd (dX).  Activations are in slot order (expert segments).
 *   usaf_expert_gate_up_fwd: gu = act @ W_gu[e]^T, h = silu(gate) * up
 *       (gu: [P, 2I], h: [P, I], activation dtype, rounded like the reference)
 *   usaf_expert_down_fwd:    y_seg = h @ W_dn[e]^T              ([P, H])
 *   usaf_expert_down_bwd:    dh = dcur @ W_dn[e]; dgu = SwiGLU backward(dh, gu)
 *   usaf_expert_gate_up_bwd: dx_seg = dgu @ W_gu[e]             ([P, H])
 * plan->E must equal the projection's E (USAF_EINVAL otherwise); the
 * tensor-core kernels take E <= 1024. */
int usaf_expert_gate_up_fwd(const usaf_route_plan *plan, const usaf_qweight *w_gu,
                            const void *x_perm, int32_t dtype, void *gu, void *h, void *stream);
int usaf_expert_down_fwd(const usaf_route_plan *plan, const usaf_qweight *w_dn,
                         const void *h, int32_t dtype, void *y_seg, void *stream);
int usaf_expert_down_bwd(const usaf_route_plan *plan, const usaf_qweight *w_dn,
                         const void *dcur, const void *gu, int32_t dtype, void *dgu,
                         void *stream);
int usaf_expert_gate_up_bwd(const usaf_route_plan *plan, const usaf_qweight *w_gu,
                            const void *dgu, int32_t dtype, void *dx_seg, void *stream);

/* ---- sparse expert-weight gradients -----------------------------------------
 * usaf_sparse_dw replaces the dense per-expert weight gradient + gather +
 * index_add of the capture protocol (usaf/qwen3moe_dml.py:43-56,
 * usaf/moe_loader.py:564-578).  For every overlay coordinate (e, r, c) of w:
 *   g = dtype( sum over expert e's slots s of gout[s, r] * gin[s, c] )
 *   compact[pos] += scale * g        (pos = compact position of the entry)
 * gout: [P, R] (dgu or dcur), gin: [P, C] (x_perm or h).
 * csr_to_compact: [n_ov] compact position of each CSR entry, or NULL when
 * the compact vector is kept in CSR order (identity map); scratch: fp32
 * [n_ov] per-coordinate partial sums.  bf16 with w->ov_mask runs on the
 * tensor cores unless the plan holds at most 64 pair slots per expert
 * (P_cap <= 64 * E, decode-sized batches), which take the CUDA-core kernel;
 * the results agree to bf16 rounding.  On the tensor cores an expert of up to
 * 320 slots keeps its gin block resident across row blocks; when the plan
 * may hold larger experts (plan->T > 320, or T == 0 for an unknown count) a
 * second, streaming kernel takes those (plan->E <= 1024 then, else
 * USAF_EUNSUPPORTED). */
int usaf_sparse_dw(const usaf_route_plan *plan, const usaf_qweight *w, const void *gout,
                   const void *gin, int32_t dtype, const int32_t *csr_to_compact,
                   float scale, float *compact, float *scratch, void *stream);

/* usaf_sparse_dw_noalloc: usaf_sparse_dw for callers that cannot allocate
 * device memory at call time (a process working inside a pool it reserved at
 * start-up, or a foreign-language host that can only pass buffers it already
 * owns).  No counterpart in the reference.  The per-coordinate scratch is a
 * fixed array inside this library (2,097,152 fp32 slots = 8 MiB, resident on
 * every GPU that loads the library until exit); a projection with more
 * overlay coordinates returns USAF_EUNSUPPORTED.  The first call on a device
 * looks the array up (cudaGetSymbolAddress) with that device current, so make
 * that first call before any stream capture.  The looked-up address is kept
 * for the life of the process and is not refreshed after cudaDeviceReset:
 * do not call this entry point on a device after resetting it.  All calls
 * share the one array: calls that may overlap on the GPU (different streams,
 * several threads) race and must be serialized by the caller.  Allocates
 * nothing. */
int usaf_sparse_dw_noalloc(const usaf_route_plan *plan, const usaf_qweight *w, const void *gout,
                           const void *gin, int32_t dtype, const int32_t *csr_to_compact,
                           float scale, float *compact, void *stream);

/* ---- optimizer ------------------------------------------------------------
 * usaf_sparse_adam replaces SparseAdam.step (usaf/sparse_optim.py:86-134) in
 * compact mode: p = fp32 master [n]; m, v fp32 [n]; grad fp32 [n] (divided by
 * grad_div first, as train.py:662 divides by loss_scale*ACCUM).  Hyper-
 * parameters are doubles, converted the way Python scalars meet fp32 tensors.
 * If ov_val is given, the new value rounded the way the GEMMs consume it
 * (fp16, then `dtype`) is written to ov_val[ov_pos[i]] -- ov_val[i] when
 * ov_pos is NULL (masters in CSR order) -- and to ov_valT[ov_posT[i]], as
 * sync_resident does (usaf/moe_loader.py:425-443). */
int usaf_sparse_adam(int64_t n, float *p, float *m, float *v, const float *grad,
                     double grad_div, int32_t step, double lr, double beta1, double beta2,
                     double eps, double weight_decay, int32_t dtype, float *ov_val,
                     const int32_t *ov_pos, float *ov_valT, const int32_t *ov_posT,
                     void *stream);

/* usaf_sparse_adam_gather: gather/scatter mode (usaf/sparse_optim.py:110-134)
 * on a parameter of dtype `dtype` (fp32/bf16): idx int64 [n] flat indices,
 * grad = the dense gradient of the same dtype. */
int usaf_sparse_adam_gather(int64_t n, const int64_t *idx, void *param, const void *grad,
                            int32_t dtype, double grad_div, float *m, float *v, int32_t step,
                            double lr, double beta1, double beta2, double eps,
                            double weight_decay, void *stream);

/* ---- selection ------------------------------------------------------------
 * usaf_topk_desc: the k largest of vals[n] (fp32, non-negative or any), in
 * descending order; ties at equal value are taken in ascending index order.
 * Writes out_vals[k], out_idx[k] (int64: idx_base + position, or
 * idx_map[position] when idx_map is given).  Scratch: usaf_topk_scratch_bytes.
 * Replaces torch.topk in TopKImportanceStore.add/select (usaf/moe_loader.py:
 * 607-609, 626). */
int64_t usaf_topk_scratch_bytes(int64_t n, int64_t k);
int usaf_topk_desc(const float *vals, int64_t n, int64_t k, const int64_t *idx_map,
                   int64_t idx_base, float *out_vals, int64_t *out_idx, void *scratch,
                   void *stream);

/* usaf_kth_largest: value of the k-th largest element (1-based, counting
 * duplicates) of vals[n]; replaces the np.partition threshold of
 * usaf/selector.py:6-14.  Writes one fp32 to out (device). */
int usaf_kth_largest(const float *vals, int64_t n, int64_t k, float *out, void *scratch,
                     void *stream);

/* usaf_expert_dense_dw: dense per-expert |weight gradient| for the importance
 * pass (usaf/moe_loader.py:604-611 receives the dense grad): for expert e,
 * out[e][r][c] = |dtype(sum_s gout[s,r] * gin[s,c])| as fp32, [E, R, C]. */
int usaf_expert_dense_dw(const usaf_route_plan *plan, int32_t R, int32_t C, const void *gout,
                         const void *gin, int32_t dtype, float *out, void *stream);

/* Importance candidates without the dense |grad| buffer (bf16 gradients on
 * tensor cores): the per-expert top-k of TopKImportanceStore.add
 * (usaf/moe_loader.py:604-611, k = max(1, int(numel_e*frac*cand_mult)),
 * experts without routed tokens contribute nothing) computed by three passes
 * of the SDDMM over the same plan and operands as usaf_expert_dense_dw, none
 * of which writes the gradient out.  Keys are the 15 magnitude bits of
 * |bf16(g)| (they order like the values).  Sequence, one projection:
 *   usaf_importance_hist(level 1)  hist[E*256] zeroed: keys by exponent;
 *   usaf_importance_pick(level 1)  pval[e], need[e];
 *   usaf_importance_hist(level 2)  hist zeroed again: the keys of bucket pval[e];
 *   usaf_importance_pick(level 2)  thr[e] (the k-th largest key), n_eq[e] keys
 *                                  equal to it, need[e] of those to take;
 *   usaf_importance_emit           keys > thr[e] into candidate row
 *                                  cand_row[e] (k entries a row), keys == thr[e]
 *                                  into the tie list at eq_off[e] (exclusive
 *                                  scan of n_eq); n_gt / n_eq zeroed first;
 *   usaf_sort_u32 of the tie lists by flat index (usaf_importance_keys mode 0
 *   builds the keys, mode 2 gathers), then usaf_importance_take_ties appends
 *   the need[e] lowest-index ties to each row;
 *   usaf_importance_keys mode 0 + usaf_sort_u32, then mode 1 + usaf_sort_u32,
 *   then mode 2: rows ordered by descending value, ties by ascending index.
 * cand_row[e] < 0 or thr[e] < 0 leaves expert e out.  Flat indices are
 * e*R*C + r*C + c.  usaf_importance_chunk_slots(): slots of one SDDMM chunk
 * (an expert with more is summed over several in the accumulator). */
int32_t usaf_importance_chunk_slots(void);
int usaf_importance_supported(int32_t R, int32_t C, int32_t dtype);
int usaf_importance_hist(const usaf_route_plan *plan, int32_t R, int32_t C, const void *gout,
                         const void *gin, int32_t dtype, int32_t level, const int32_t *pval,
                         uint32_t *hist, void *stream);
int usaf_importance_pick(const uint32_t *hist, int32_t E, int64_t k, const int32_t *expert_cnt,
                         int32_t level, int32_t *pval, int64_t *need, int32_t *thr, int64_t *n_eq,
                         void *stream);
int usaf_importance_emit(const usaf_route_plan *plan, int32_t R, int32_t C, const void *gout,
                         const void *gin, int32_t dtype, const int32_t *thr, int64_t k,
                         const int32_t *cand_row, int32_t *n_gt, int32_t *n_eq, float *cand_val,
                         int64_t *cand_idx, const int64_t *eq_off, float *eq_val, int64_t *eq_idx,
                         void *stream);
int usaf_importance_take_ties(int32_t E, int64_t k, const int32_t *cand_row, const int64_t *need,
                              const int64_t *eq_off, const float *eq_val, const int64_t *eq_idx,
                              float *cand_val, int64_t *cand_idx, void *stream);
int usaf_importance_keys(const float *val, const int64_t *idx, const int64_t *perm, int64_t n,
                         int64_t k, int32_t mode, float *val_out, int64_t *idx_out, uint32_t *keys,
                         int64_t *pos, void *stream);

/* usaf_sort_u32: stable LSD radix sort of (uint32 key, int64 payload) pairs,
 * ascending (descending != 0: descending) by key; equal keys keep input
 * order.  Used to build the overlay CSR/CSC from selected flat indices.
 * Scratch: usaf_sort_scratch_bytes(n). */
int64_t usaf_sort_scratch_bytes(int64_t n);
int usaf_sort_u32(const uint32_t *keys_in, const int64_t *vals_in, int64_t n, uint32_t *keys_out,
                  int64_t *vals_out, int32_t descending, void *scratch, void *stream);

/* ---- misc ------------------------------------------------------------------ */
/* usaf_dot: out[0] = sum_i a[i]*b[i] in fp32 (a, b of dtype), reproducible
 * (fixed reduction order).  Its block partials sit in a fixed array inside
 * the library: do not run two usaf_dot calls on one device concurrently. */
int usaf_dot(const void *a, const void *b, int32_t dtype, int64_t n, float *out, void *stream);
/* usaf_build_rowptr: row_ptr[r] = first position of row r in the sorted
 * row keys (n_rows + 1 entries). */
int usaf_build_rowptr(const int64_t *keys, int64_t n, int64_t n_rows, int32_t *row_ptr,
                      void *stream);
/* usaf_build_ov_cbptr: usaf_qweight.ov_cbptr from the overlay's CSR
 * (row_ptr [E*R*2+1], col [n_ov]) of a projection [E, R, C]; out holds
 * E*R*ceil(C/256)*2 int32. */
int usaf_build_ov_cbptr(const int32_t *row_ptr, const int32_t *col, int32_t E, int32_t R, int32_t C,
                        int32_t *out, void *stream);
const char *usaf_version(void);

/* ---- expert parallelism ------------------------------------------------------
 * No counterpart in the reference (it runs in a single process).  Plan:
 * rank r of W owns experts [r*El, (r+1)*El), tokens stay data-parallel and an
 * all-to-all delivers each rank's routed rows (x_perm is expert-major, so the
 * rows bound for one rank are contiguous).  counts[s*El + e] = rows received
 * from source rank s for local expert e; the receive buffer is in block order
 * (s, e), the grouped GEMMs want (e, s).
 * usaf_ep_permute: inverse == 0 moves received rows into expert-major order
 * (out[dst(i)] = in[i]); inverse == 1 moves them back (out[i] = in[dst(i)]).
 * n_rows must equal sum(counts) (else USAF_ERR_BAD_INDEX in *err, nothing
 * moved); row_bytes % 16 == 0, 16-byte aligned buffers, W*El <= 4096.
 * usaf_ep_owner_counts: expert_cnt[e] = sum_s counts[s][e], expert_off its
 * exclusive prefix [El+1], *n_rows (optional) the total. */
int usaf_ep_permute(const int32_t *counts, int32_t W, int32_t El, int64_t n_rows, const void *in,
                    void *out, int64_t row_bytes, int32_t inverse, int32_t *err, void *stream);
int usaf_ep_owner_counts(const int32_t *counts, int32_t W, int32_t El, int32_t *expert_cnt,
                         int32_t *expert_off, int32_t *n_rows, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* USAF_B200_H */
