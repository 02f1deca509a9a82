// Expert-weight gradients on tcgen05 (bf16 activations).
//
// For expert e the weight gradient is the product over its routed slots
//   D_e[r][c] = sum_{s in slots of e} gout[s][r] * gin[s][c]
// (gout = dgu / dcur [P, R], gin = x_perm / h [P, C], both slot-major).  The
// reference forms D_e densely (F.linear backward, usaf/qwen3moe_dml.py:43-56)
// and keeps only the selected coordinates (usaf/moe_loader.py:564-578).  Here
// D_e is formed tile by tile in TMEM and never written out: the epilogue
// keeps what the caller needs.
//   EPI_SPARSE   : the selected coordinates, read from the overlay bitmap, as
//                  dtype(D) into a CSR-ordered fp32 vector (stores only: a
//                  read-modify-write of the compact vector here would wait on
//                  each scattered load in turn); a second kernel adds
//                  scale * that value to the compact vector.
//   EPI_DENSE_ABS: |dtype(D)| at every coordinate (importance pass,
//                  usaf/importance.py).
//   EPI_HIST     : the importance candidates without writing D out
//                  (TopKImportanceStore, usaf/moe_loader.py:604-611): a
//                  histogram per expert of the 15-bit keys of |bf16(D)|
//                  (exponent and mantissa bits, ordered like the values),
//                  restricted to the keys with a given prefix, counted in
//                  per-warp shared-memory histograms and folded into global
//                  memory once per run of tiles;
//   EPI_EMIT     : the same keys against a threshold per expert: every
//                  coordinate above it goes to the expert's candidate list,
//                  every one equal to it to the expert's tie list.
//   In the sparse mode an expert above one resident chunk (320 slots) is
//   left to the streaming kernel of sddmm_stream.cu, launched after this one
//   (it streams both operands and sums all of a tile's slots in one
//   accumulator); the dense and importance modes sum such an expert chunk
//   after chunk in the row block's TMEM accumulator (its gin chunks reloaded
//   for every row block), so no partial sums leave the SM in any mode.
//
// Tile = 128 storage rows x 256 columns (MMA M x N), K = the expert's slots in
// blocks of 64.  Both operands reach shared memory as TMA boxes of 64 slots x
// 64 rows/columns with the 128-byte swizzle, MN-major for the MMA (rows r /
// columns c contiguous, slots along K), so no transpose is needed.
//
// Work order: the tiles are numbered column-block-major, then expert, then
// row block, and every CTA (one per SM, persistent) takes one contiguous
// range of them, cut so that the ranges cost the same (a tile's cost grows
// with its expert's slot count).  Inside a range, a run of row blocks of one
// (expert, column block) keeps the gin block -- 256 columns x up to 320
// slots -- resident in shared memory and streams only the 128-row gout
// blocks, so the operand traffic per tile is about a third of loading both.
// (Expert-major numbering measured slower: each CTA then streams one
// expert's gout once per column block, and 148 of those no longer fit in L2;
// processing the experts in waves of 32 measured the same as this order.)
//
// Warp 0 issues TMA; warp 18 zeroes the slots past an expert's end inside its
// last 16-slot group (they belong to the next expert) and forwards those
// stages (and every resident gin block) to the MMA, so the MMA issuer -- lane
// 0 of warp 1, which also owns TMEM -- runs a lean loop of waits, MMAs and
// commits (its own per-k-block bookkeeping otherwise outlasts the four MMAs
// it issues) and takes every other stage straight from its TMA barrier; warps
// 2-17 drain the accumulators, four per TMEM lane quarter (64 columns each),
// so every scheduler has four drain warps to interleave.  TMEM holds two
// 256-column accumulators, so the drain of one tile overlaps the MMAs of the
// next.
#include <climits>
#include <cudaTypedefs.h>

#include "tc_common.cuh"

namespace usaf {
using namespace tc;

namespace {

constexpr int kSM = 128;                 // storage rows per tile (MMA M)
constexpr int kSN = 256;                 // columns per tile (MMA N)
constexpr int kSK = 64;                  // slots per k-block
constexpr int kAStages = 4;              // gout ring
constexpr int kBMaxKb = 5;               // resident gin k-blocks (320 slots)
constexpr int kSThreads = 608;           // 19 warps
constexpr int kEpiThreads = 512;         // warps 2-17
constexpr int kFwdWarp = 18;             // the stage forwarder
constexpr int kBox = kSK * 64 * 2;       // one TMA box: 64 slots x 64 bf16 = 8 KB
constexpr int kAStage = 2 * kBox;        // 128 rows
constexpr int kBKb = 4 * kBox;           // 256 columns
constexpr uint32_t kFull = 0xffffffffu;

enum : int { EPI_SPARSE = 0, EPI_DENSE_ABS = 1, EPI_HIST = 2, EPI_EMIT = 3 };
constexpr int kHistBins = 256;

struct alignas(8) SShared {
    uint64_t a_full[kAStages];
    uint64_t a_empty[kAStages];
    uint64_t a_ready[kAStages];   // a ragged fill, zeroed by the forwarder
    uint64_t a_tail[kAStages];    // a ragged fill was issued
    uint64_t b_full[kBMaxKb];
    uint64_t b_ready[kBMaxKb];
    uint64_t b_empty;
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort_flag;
    int t_lo, t_hi;                          // this CTA's tile range
};

constexpr size_t kSSmem = (size_t)kAStages * kAStage + (size_t)kBMaxKb * kBKb + sizeof(SShared) + 1024;
static_assert(kSSmem <= 232448, "SDDMM shared memory above the per-block limit");

__device__ __forceinline__ void s_drain(uint64_t *bar, uint32_t parity, int *err) {
    uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > kWaitBudgetNs) {
            atomicOr(err, USAF_ERR_WAIT_TIMEOUT);
            return;
        }
    }
}

__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// MN-major operand with the 128-byte swizzle: 64-element MN blocks LBO = 8 KB
// apart (one TMA box each), 8-slot groups SBO = 1 KB apart, version 1 (sm_100)
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(kBox >> 4) << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// bf16 x bf16 -> fp32, A and B MN-major (transpose bits 15 and 16)
__host__ __device__ constexpr uint32_t idesc_mn(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ float round_bf16(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
}

// ---- work order ----------------------------------------------------------------

// cost of one tile of an expert with `cnt` slots, in units of one 16-slot MMA
// step (the fixed part stands for the epilogue and the stream of gout); an
// expert above max_cnt slots is left to the streaming kernel (no cost here)
__device__ __forceinline__ int64_t tile_cost(int cnt, int dense, int max_cnt) {
    if (cnt > max_cnt) return 0;
    if (cnt <= 0) return dense == 2 ? 0 : dense ? 40 : 2;
    return (cnt + 15) / 16 + (dense ? 40 : 6);
}

// tiles of one (column block, expert) run (nrb of them, `wt` each, the first
// at cost prefix `cum`) whose cost prefix lies below x
__device__ __forceinline__ int64_t tiles_below(int64_t x, int64_t cum, int64_t wt, int nrb) {
    if (x <= cum) return 0;
    if (wt == 0) return nrb;
    return min((int64_t)nrb, (x - cum + wt - 1) / wt);
}

__device__ __forceinline__ int64_t warp_sum64(int64_t v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    return v;
}

// one warp: this CTA's tile range [t_lo, t_hi) -- the tiles whose cost prefix
// falls in the CTA's equal share of the total
__device__ void tile_range(const usaf_route_plan &pl, int nrb, int ncb, int dense, int max_cnt, int lane,
                           int *t_lo, int *t_hi) {
    const int E = pl.E;
    int64_t We = 0;   // cost of one column block over all experts
    for (int e0 = 0; e0 < E; e0 += 32) {
        const int e = e0 + lane;
        We += e < E ? tile_cost(__ldg(pl.expert_cnt + e), dense, max_cnt) * nrb : 0;
    }
    We = warp_sum64(We);
    const int64_t W = We * ncb, G = gridDim.x, b = blockIdx.x;
    const int64_t x0 = W * b / G, x1 = W * (b + 1) / G;
    int64_t n0 = 0, n1 = 0;
    for (int cb = 0; cb < ncb; ++cb) {
        int64_t carry = We * cb;
        if (carry >= x1) break;   // this column block and the later ones lie above both bounds
        if (carry + We <= x0) {   // the whole column block lies below both bounds
            if (lane == 0) {
                n0 += (int64_t)E * nrb;
                n1 += (int64_t)E * nrb;
            }
            continue;
        }
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const int64_t wt = e < E ? tile_cost(__ldg(pl.expert_cnt + e), dense, max_cnt) : 0;
            const int64_t w = wt * nrb;
            int64_t incl = w;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t y = __shfl_up_sync(kFull, incl, o);
                if (lane >= o) incl += y;
            }
            const int64_t cum = carry + incl - w;
            carry += __shfl_sync(kFull, incl, 31);
            if (e < E) {
                n0 += tiles_below(x0, cum, wt, nrb);
                n1 += tiles_below(x1, cum, wt, nrb);
            }
        }
    }
    n0 = warp_sum64(n0);
    n1 = warp_sum64(n1);
    // (the last CTA's bound W counts every tile of nonzero cost; trailing tiles
    // of zero cost -- experts left to the streaming kernel, experts without
    // slots in the histogram mode -- have no work and no CTA walks them)
    *t_lo = (int)n0;
    *t_hi = (int)n1;
}

// a run of row blocks [rb0, rb1) of one (column block, expert) inside [t, t_hi)
struct Run {
    int e, cb, rb0, rb1;
};

__device__ __forceinline__ Run run_at(int t, int t_hi, int nrb, int E) {
    Run s;
    const int per_cb = nrb * E;
    s.cb = t / per_cb;
    const int r = t - s.cb * per_cb;
    s.e = r / nrb;
    s.rb0 = r - s.e * nrb;
    s.rb1 = min(nrb, s.rb0 + (t_hi - t));
    return s;
}

// an expert's k-blocks in slot chunks of at most kBMaxKb k-blocks
struct Chunks {
    int nk, n, per;
};

__device__ __forceinline__ Chunks chunks_of(int cnt) {
    Chunks c;
    c.nk = (cnt + kSK - 1) / kSK;
    c.n = (c.nk + kBMaxKb - 1) / kBMaxKb;
    c.per = c.n ? (c.nk + c.n - 1) / c.n : 0;
    return c;
}

// ---- MMA-side helpers ----------------------------------------------------------

// all lanes of the warp wait; the answer is the same for every lane
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *err) {
    return __all_sync(kFull, mbar_wait(bar, parity, abort_flag, err));
}

// zero slot rows [rem, round16(rem)) of `nbox` consecutive 64-slot boxes: a
// full 128-byte slot row holds exactly that slot's 64 elements under the
// 128-byte swizzle, whatever their order inside the row
__device__ __forceinline__ void zero_tail(unsigned char *base, int nbox, int rem, int lane) {
    const int per_box = (((rem + 15) & ~15) - rem) * 8;   // 16-byte chunks per box
    for (int i = lane; i < nbox * per_box; i += 32) {
        const int bx = i / per_box, k = i - bx * per_box;
        *reinterpret_cast<uint4 *>(base + bx * kBox + rem * 128 + k * 16) = make_uint4(0, 0, 0, 0);
    }
}

// ---- epilogue helpers ------------------------------------------------------------

// global store that does not allocate a line in L1: the drain's stores are
// scattered 4-byte writes nothing on this SM reads again (allocating them
// measured ~25 % slower)
__device__ __forceinline__ void st_na(float *p, float v) {
    asm volatile("st.global.L1::no_allocate.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// the selected columns of one 32-column chunk of this thread's row (values v,
// bitmap word m), in ascending column order from CSR position p on: one
// predicated store per column, straight-line code without a dependence from
// one column to the next but the position counter
__device__ __forceinline__ void drain_sparse(const uint32_t (&v)[32], uint32_t m, int &p,
                                             float *__restrict__ out) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
        if (m & (1u << i)) st_na(out + p++, round_bf16(__uint_as_float(v[i])));
}

// raw bitmap words and block start positions of one row's column block (the
// loads of slice_start, issued one tile ahead of their use)
struct SliceRaw {
    uint4 lo, hi;
    int2 pp;
};

__device__ __forceinline__ SliceRaw slice_load(const uint32_t *__restrict__ mask, const int32_t *__restrict__ cbptr,
                                               int64_t grow, int C, int ncb, int cb, int slice) {
    SliceRaw r;
    const uint32_t *mrow = mask + grow * (C / 32) + cb * 8;
    r.lo = __ldg(reinterpret_cast<const uint4 *>(mrow));
    r.hi = slice >= 2 ? __ldg(reinterpret_cast<const uint4 *>(mrow) + 1) : make_uint4(0, 0, 0, 0);
    r.pp = __ldg(reinterpret_cast<const int2 *>(cbptr + (grow * ncb + cb) * 2));
    return r;
}

__device__ __forceinline__ void slice_decode(const SliceRaw &r, int slice, uint2 &w, int &p0, int &p1) {
    int b0 = 0, b1 = 0;
    if (slice >= 1) { b0 += __popc(r.lo.x); b1 += __popc(r.lo.y); }
    if (slice >= 2) { b0 += __popc(r.lo.z); b1 += __popc(r.lo.w); }
    if (slice >= 3) { b0 += __popc(r.hi.x); b1 += __popc(r.hi.y); }
    w = slice == 0 ? make_uint2(r.lo.x, r.lo.y) : slice == 1 ? make_uint2(r.lo.z, r.lo.w)
      : slice == 2 ? make_uint2(r.hi.x, r.hi.y) : make_uint2(r.hi.z, r.hi.w);
    p0 = r.pp.x + b0;
    p1 = r.pp.y + b1;
}

// bitmap words of chunks 2 slice and 2 slice + 1 of the row's column block
// (w.x even chunk, w.y odd chunk) and the CSR positions where they start in
// the row's two halves (p0 even chunks, p1 odd chunks): the block's start
// positions plus the selected entries of the block's earlier chunks
__device__ __forceinline__ void slice_start(const uint32_t *__restrict__ mask, const int32_t *__restrict__ cbptr,
                                            int64_t grow, int C, int ncb, int cb, int slice, uint2 &w, int &p0,
                                            int &p1) {
    const uint32_t *mrow = mask + grow * (C / 32) + cb * 8;
    const uint4 mlo = __ldg(reinterpret_cast<const uint4 *>(mrow));
    const uint4 mhi = slice >= 2 ? __ldg(reinterpret_cast<const uint4 *>(mrow) + 1) : make_uint4(0, 0, 0, 0);
    const int2 pp = __ldg(reinterpret_cast<const int2 *>(cbptr + (grow * ncb + cb) * 2));
    int b0 = 0, b1 = 0;
    if (slice >= 1) { b0 += __popc(mlo.x); b1 += __popc(mlo.y); }
    if (slice >= 2) { b0 += __popc(mlo.z); b1 += __popc(mlo.w); }
    if (slice >= 3) { b0 += __popc(mhi.x); b1 += __popc(mhi.y); }
    w = slice == 0 ? make_uint2(mlo.x, mlo.y) : slice == 1 ? make_uint2(mlo.z, mlo.w)
      : slice == 2 ? make_uint2(mhi.x, mhi.y) : make_uint2(mhi.z, mhi.w);
    p0 = pp.x + b0;
    p1 = pp.y + b1;
}

__device__ __forceinline__ void drain_dense(const uint32_t (&v)[32], float *o) {
    float4 *o4 = reinterpret_cast<float4 *>(o);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        o4[i] = make_float4(fabsf(round_bf16(__uint_as_float(v[4 * i]))), fabsf(round_bf16(__uint_as_float(v[4 * i + 1]))),
                            fabsf(round_bf16(__uint_as_float(v[4 * i + 2]))),
                            fabsf(round_bf16(__uint_as_float(v[4 * i + 3]))));
}

// ---- importance epilogues ---------------------------------------------------

// Arguments of EPI_HIST / EPI_EMIT (zero for the other modes).
struct ImpArgs {
    int shift, pmask;            // HIST: key counted in bin (key >> shift) & 255 if (key & pmask) == pval[e]
    const int32_t *pval;         // [E]
    unsigned int *hist;          // [E * 256]
    const int32_t *thr;          // EMIT: [E] threshold key, < 0: the expert emits nothing
    int64_t k;                   // EMIT: candidate list capacity per expert
    const int32_t *cand_row;     // EMIT: [E] first row of e's candidate list (in units of k)
    int32_t *n_gt, *n_eq;        // EMIT: [E] list fills (zeroed by the caller)
    float *gt_val;               // EMIT: candidate values / flat indices
    int64_t *gt_idx;
    const int64_t *eq_off;       // EMIT: [E] start of e's tie list
    float *eq_val;
    int64_t *eq_idx;
};

// 15-bit order key of |bf16(v)|: exponent and mantissa bits of the rounded value
__device__ __forceinline__ int abs_key(float v) {
    return (int)((__float_as_uint(round_bf16(v)) >> 16) & 0x7FFFu);
}

__device__ __forceinline__ void hist_chunk(const uint32_t (&v)[32], unsigned int *h, int shift, int pmask, int pv) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const int key = abs_key(__uint_as_float(v[i]));
        if ((key & pmask) == pv) atomicAdd(&h[(key >> shift) & (kHistBins - 1)], 1u);
    }
}

// candidates of one chunk: the warp reserves list room with one atomic per list,
// every lane then stores its own entries in column order
__device__ __forceinline__ void emit_chunk(const uint32_t (&v)[32], int e, int64_t flat0, int thr,
                                           const ImpArgs &ia, int lane) {
    uint32_t mg = 0, me = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const int key = abs_key(__uint_as_float(v[i]));
        mg |= (uint32_t)(key > thr) << i;
        me |= (uint32_t)(key == thr) << i;
    }
    const int ng = __popc(mg), ne = __popc(me);
    int sg = ng, se = ne;   // inclusive scans over the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int yg = __shfl_up_sync(kFull, sg, o), ye = __shfl_up_sync(kFull, se, o);
        if (lane >= o) { sg += yg; se += ye; }
    }
    int bg = 0, be = 0;
    if (lane == 31) {
        if (sg) bg = atomicAdd(ia.n_gt + e, sg);
        if (se) be = atomicAdd(ia.n_eq + e, se);
    }
    bg = __shfl_sync(kFull, bg, 31) + sg - ng;
    be = __shfl_sync(kFull, be, 31) + se - ne;
    if (!(ng | ne)) return;
    float *gv = ia.gt_val + (int64_t)ia.cand_row[e] * ia.k;
    int64_t *gi = ia.gt_idx + (int64_t)ia.cand_row[e] * ia.k;
    float *ev = ia.eq_val + ia.eq_off[e];
    int64_t *ei = ia.eq_idx + ia.eq_off[e];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        const float a = fabsf(round_bf16(__uint_as_float(v[i])));
        if ((mg >> i) & 1u) {
            gv[bg] = a;
            gi[bg] = flat0 + i;
            ++bg;
        }
        if ((me >> i) & 1u) {
            ev[be] = a;
            ei[be] = flat0 + i;
            ++be;
        }
    }
}

// Tile order inside a run (one expert and column block, row blocks rb0..rb1,
// the expert's slots in n chunks).  The sparse mode only sees experts of one
// chunk (larger ones go to the streaming kernel), kept resident across the
// run's row blocks (chunk outer, row block inner); the dense and importance
// modes take row block outer, chunk inner, and sum the chunks in the row
// block's TMEM accumulator (the chunks are reloaded per row block).
struct TileOrder {
    bool rb_outer, multi;
    int rb0, rb1, n;
    __device__ __forceinline__ int n_outer() const { return rb_outer ? rb1 - rb0 : n; }
    __device__ __forceinline__ int n_inner() const { return rb_outer ? n : rb1 - rb0; }
    __device__ __forceinline__ void at(int i, int j, int &rb, int &kc) const {
        rb = rb0 + (rb_outer ? i : j);
        kc = rb_outer ? j : i;
    }
    // the tile (rb, kc) loads its chunk / is the last to use it
    __device__ __forceinline__ bool loads_b(int rb) const { return (rb_outer && multi) || rb == rb0; }
    __device__ __forceinline__ bool frees_b(int rb) const { return (rb_outer && multi) || rb == rb1 - 1; }
    // the tile starts / completes an accumulator
    __device__ __forceinline__ bool acc_start(int kc) const { return !rb_outer || kc == 0; }
    __device__ __forceinline__ bool acc_end(int kc) const { return !rb_outer || kc == n - 1; }
};

template <int EPI>
__global__ void __launch_bounds__(kSThreads, 1)
    sddmm_tc_kernel(const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_in,
                    usaf_route_plan pl, int R, int C, const uint32_t *__restrict__ mask,
                    const int32_t *__restrict__ cbptr, float *__restrict__ out, const ImpArgs ia,
                    int max_cnt) {
    // the histogram mode gives up one gout stage for the per-warp histograms
    constexpr int AST = EPI == EPI_HIST ? kAStages - 1 : kAStages;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *sb = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    unsigned char *a_ring = sb;
    unsigned char *b_res = sb + (size_t)kAStages * kAStage;   // the layout keeps every stage
    SShared &S = *reinterpret_cast<SShared *>(b_res + (size_t)kBMaxKb * kBKb);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nrb = R / kSM;
    const int ncb = (C + kSN - 1) / kSN;
    int *err = pl.err;
    if (warp == 0) {
        if (lane == 0) {
            S.abort_flag = 0;
            for (int s = 0; s < kAStages; ++s) {   // (all barriers exist)
                mbar_init(&S.a_full[s], 1);
                mbar_init(&S.a_empty[s], 1);
                mbar_init(&S.a_ready[s], 1);
                mbar_init(&S.a_tail[s], 1);
            }
            for (int k = 0; k < kBMaxKb; ++k) {
                mbar_init(&S.b_full[k], 1);
                mbar_init(&S.b_ready[k], 1);
            }
            mbar_init(&S.b_empty, 1);
            for (int b = 0; b < 2; ++b) {
                mbar_init(&S.acc_full[b], 1);
                mbar_init(&S.acc_empty[b], kEpiThreads);
            }
            mbar_init(&S.mma_done, 1);
            fence_barrier_init();
        }
        int lo, hi;
        tile_range(pl, nrb, ncb, EPI == EPI_SPARSE ? 0 : EPI == EPI_DENSE_ABS ? 1 : 2, max_cnt, lane, &lo, &hi);
        if (lane == 0) {
            S.t_lo = lo;
            S.t_hi = hi;
        }
    } else if (warp == 1) {
        tmem_alloc(&S.tmem_base, 512);
    }
    __syncthreads();
    tc_fence_after();
    volatile int *abort_flag = &S.abort_flag;
    const uint32_t tbase = S.tmem_base;
    const int t_lo = S.t_lo, t_hi = S.t_hi;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            prefetch_tmap(&tm_out);
            prefetch_tmap(&tm_in);
            int ga = 0, bc = 0;
            bool ok = true;
            for (int t = t_lo; t < t_hi && ok;) {
                const Run s = run_at(t, t_hi, nrb, pl.E);
                t += s.rb1 - s.rb0;
                const int cnt = pl.expert_cnt[s.e];
                if (cnt > max_cnt) continue;   // the streaming kernel's expert
                const int row0 = pl.expert_off[s.e];
                const Chunks ch = chunks_of(cnt);
                const int c0 = s.cb * kSN;
                const int nb = min(4, (C - c0) / 64);
                const bool ragged = ch.nk > 0 && ((cnt - (ch.nk - 1) * kSK) & 15) != 0;
                const TileOrder to{EPI != EPI_SPARSE, ch.n > 1, s.rb0, s.rb1, ch.n};
                for (int i = 0; i < to.n_outer() && ok && ch.n; ++i) {
                    for (int j = 0; j < to.n_inner() && ok; ++j) {
                        int rb, kc;
                        to.at(i, j, rb, kc);
                        const int kb0 = kc * ch.per, kb1 = min(ch.nk, kb0 + ch.per);
                        if (to.loads_b(rb)) {
                            // the previous chunk's MMAs have read the resident block
                            if (!mbar_wait(&S.b_empty, (bc & 1) ^ 1, abort_flag, err)) {
                                ok = false;
                                break;
                            }
                            // every b_full barrier completes once per chunk load, so their
                            // phases stay in step with the load count: the ones this chunk
                            // leaves unused get a plain arrive, before any load is issued (a
                            // waiter that saw b_full[0] complete knows they have completed too)
                            for (int k = kb1 - kb0; k < kBMaxKb; ++k) mbar_arrive(&S.b_full[k]);
                            for (int k = 0; k < kb1 - kb0; ++k) {
                                mbar_arrive_expect_tx(&S.b_full[k], (uint32_t)(nb * kBox));
                                const int y = row0 + (kb0 + k) * kSK;
                                for (int j = 0; j < nb; ++j)
                                    tma_load_2d(b_res + (size_t)k * kBKb + j * kBox, &tm_in, &S.b_full[k], c0 + 64 * j, y);
                            }
                            ++bc;
                        }
                        for (int kb = kb0; kb < kb1; ++kb, ++ga) {
                            const int st = ga % AST;
                            if (!mbar_wait(&S.a_empty[st], ((ga / AST) & 1) ^ 1, abort_flag, err)) {
                                ok = false;
                                break;
                            }
                            mbar_arrive_expect_tx(&S.a_full[st], (uint32_t)(2 * kBox));
                            unsigned char *dst = a_ring + (size_t)st * kAStage;
                            const int y = row0 + kb * kSK;
                            tma_load_2d(dst, &tm_out, &S.a_full[st], rb * kSM, y);
                            tma_load_2d(dst + kBox, &tm_out, &S.a_full[st], rb * kSM + 64, y);
                            if (ragged && kb == ch.nk - 1) mbar_arrive(&S.a_tail[st]);
                        }
                    }
                }
            }
            if (*abort_flag) {
                // loads in flight land before the CTA's shared memory is released
                for (int g = max(0, ga - AST); g < ga; ++g)
                    s_drain(&S.a_full[g % AST], (g / AST) & 1, err);
                if (bc > 0)
                    for (int k = 0; k < kBMaxKb; ++k) s_drain(&S.b_full[k], (bc - 1) & 1, err);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (lane 0) ----------------
        if (lane == 0) {
            // descriptors of the ring's and the resident block's first boxes: the
            // start-address field (address / 16, low 14 bits) of the others is reached
            // by adding their offset / 16 (shared addresses stay below 256 KB)
            const uint64_t dA0 = desc_mn_sw128(smem_u32(a_ring)), dB0 = desc_mn_sw128(smem_u32(b_res));
            int ga = 0, bc = 0, it = 0;
            uint32_t tail_par = 0;   // bit st: parity of the next a_ready[st] completion
            bool ok = true;
            for (int t = t_lo; t < t_hi && ok;) {
                const Run s = run_at(t, t_hi, nrb, pl.E);
                t += s.rb1 - s.rb0;
                const int cnt = pl.expert_cnt[s.e];
                if (cnt > max_cnt) continue;
                const Chunks ch = chunks_of(cnt);
                const int nb = min(4, (C - s.cb * kSN) / 64);
                const uint32_t idesc = idesc_mn(kSM, nb * 64);
                const bool ragged = ch.nk > 0 && ((cnt - (ch.nk - 1) * kSK) & 15) != 0;
                const TileOrder to{EPI != EPI_SPARSE, ch.n > 1, s.rb0, s.rb1, ch.n};
                // (an expert without slots has no tiles: nothing to issue or drain)
                for (int i = 0; i < to.n_outer() && ok && ch.n; ++i) {
                    for (int j = 0; j < to.n_inner() && ok; ++j) {
                        int rb, kc;
                        to.at(i, j, rb, kc);
                        const int kb0 = kc * ch.per, kb1 = min(ch.nk, kb0 + ch.per);
                        const bool new_b = to.loads_b(rb);
                        const int buf = it & 1;
                        if (to.acc_start(kc)) {
                            if (!(ok = mbar_wait(&S.acc_empty[buf], ((it >> 1) & 1) ^ 1, abort_flag, err))) break;
                            tc_fence_after();
                        }
                        for (int kb = kb0; kb < kb1; ++kb, ++ga) {
                            const int kbl = kb - kb0, st = ga % AST;
                            // first use of a loaded chunk: the resident block is in place
                            if (new_b && !(ok = mbar_wait(&S.b_ready[kbl], bc & 1, abort_flag, err))) break;
                            // a stage that needs no zeroing is taken straight from the TMA
                            // barrier; the expert's ragged last k-block comes through the
                            // forwarder
                            if (ragged && kb == ch.nk - 1) {
                                if (!(ok = mbar_wait(&S.a_ready[st], (tail_par >> st) & 1, abort_flag, err))) break;
                                tail_par ^= 1u << st;
                            } else if (!(ok = mbar_wait(&S.a_full[st], (ga / AST) & 1, abort_flag, err))) {
                                break;
                            }
                            tc_fence_after();
                            const uint64_t da = dA0 + (uint64_t)((st * kAStage) >> 4);
                            const uint64_t db = dB0 + (uint64_t)((kbl * kBKb) >> 4);
                            const uint32_t dt = tbase + buf * kSN;
                            // a row-block-outer accumulator sums every chunk of the expert
                            const bool first = to.acc_start(kc) && kb == kb0;
                            if (kb < ch.nk - 1) {   // a full k-block: four MMAs
#pragma unroll
                                for (int kk = 0; kk < 4; ++kk)
                                    mma_ss(dt, da + kk * (2048 >> 4), db + kk * (2048 >> 4), idesc, !(first && kk == 0));
                            } else {
                                const int nks = (min(kSK, cnt - kb * kSK) + 15) / 16;
                                for (int kk = 0; kk < nks; ++kk)
                                    mma_ss(dt, da + kk * (2048 >> 4), db + kk * (2048 >> 4), idesc, !(first && kk == 0));
                            }
                            mma_commit(&S.a_empty[st]);
                        }
                        if (!ok) break;
                        if (to.acc_end(kc)) {
                            mma_commit(&S.acc_full[buf]);
                            ++it;
                        }
                        // the loaded chunk is done with
                        if (to.frees_b(rb)) {
                            mma_commit(&S.b_empty);
                            ++bc;
                        }
                    }
                }
            }
            // every MMA this CTA issued has completed before TMEM is released
            mma_commit(&S.mma_done);
            s_drain(&S.mma_done, 0, err);
        }
        __syncwarp();
    } else if (warp == kFwdWarp) {
        // ---------------- forwarder: filled stage -> MMA, tails zeroed ----------------
        int ga = 0, bc = 0;
        uint32_t tail_par = 0;   // bit st: parity of the next a_tail[st] / a_ready[st] completion
        bool ok = true;
        for (int t = t_lo; t < t_hi && ok;) {
            const Run s = run_at(t, t_hi, nrb, pl.E);
            t += s.rb1 - s.rb0;
            const int cnt = pl.expert_cnt[s.e];
            if (cnt > max_cnt) continue;
            const Chunks ch = chunks_of(cnt);
            const int nb = min(4, (C - s.cb * kSN) / 64);
            // slots of the expert's last k-block; the rest of its last 16-slot group
            // belongs to the next expert and is zeroed in both operands
            const int rem = cnt - (ch.nk - 1) * kSK;
            const bool ragged = ch.nk > 0 && (rem & 15) != 0;
            const TileOrder to{EPI != EPI_SPARSE, ch.n > 1, s.rb0, s.rb1, ch.n};
            for (int i = 0; i < to.n_outer() && ok && ch.n; ++i) {
                for (int j = 0; j < to.n_inner() && ok; ++j) {
                    int rb, kc;
                    to.at(i, j, rb, kc);
                    const int kb0 = kc * ch.per, kb1 = min(ch.nk, kb0 + ch.per);
                    for (int kb = kb0; kb < kb1; ++kb, ++ga) {
                        const int kbl = kb - kb0, st = ga % AST;
                        const bool tail = ragged && kb == ch.nk - 1;
                        if (to.loads_b(rb)) {
                            if (!(ok = warp_wait(&S.b_full[kbl], bc & 1, abort_flag, err))) break;
                            if (tail) {
                                zero_tail(b_res + (size_t)kbl * kBKb, nb, rem, lane);
                                fence_proxy_async();
                            }
                            __syncwarp();
                            if (lane == 0) {
                                mbar_arrive(&S.b_ready[kbl]);
                                // b_ready completes once per chunk: the barriers this chunk
                                // leaves unused get a plain arrive, after b_full[0] showed the
                                // MMA is done with the previous chunk
                                if (kbl == 0)
                                    for (int k = kb1 - kb0; k < kBMaxKb; ++k) mbar_arrive(&S.b_ready[k]);
                            }
                        }
                        // ragged fills only: a_tail says the fill was issued (so the
                        // stage's previous fill has landed and been consumed), and
                        // a_full cannot move past this fill before a_ready lets the
                        // MMA consume it, so both parities are unambiguous
                        if (tail) {
                            if (!(ok = warp_wait(&S.a_tail[st], (tail_par >> st) & 1, abort_flag, err))) break;
                            if (!(ok = warp_wait(&S.a_full[st], (ga / AST) & 1, abort_flag, err))) break;
                            zero_tail(a_ring + (size_t)st * kAStage, 2, rem, lane);
                            fence_proxy_async();
                            __syncwarp();
                            if (lane == 0) mbar_arrive(&S.a_ready[st]);
                            tail_par ^= 1u << st;
                        }
                    }
                    if (to.frees_b(rb)) ++bc;
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 2-17) ----------------
        const int q = warp & 3;                      // TMEM lane quarter
        const int slice = (warp - 2) >> 2;           // columns [64 slice, 64 slice + 64) of the tile
        const int rr = q * 32 + lane;                // row inside the tile
        const uint32_t lane_off = ((uint32_t)(q * 32)) << 16;
        // importance histogram: one 256-bin copy per drain warp in the unused gout stage
        unsigned int *hist_all = reinterpret_cast<unsigned int *>(a_ring + (size_t)(kAStages - 1) * kAStage);
        unsigned int *hw = hist_all + (warp - 2) * kHistBins;
        const int et = tid - 64;   // 0..511 over the drain warps
        if (EPI == EPI_HIST) {
            for (int i = et; i < 16 * kHistBins; i += kEpiThreads) hist_all[i] = 0u;
            named_bar_sync(1, kEpiThreads);
        }
        int it = 0;
        bool ok = true;
        for (int t = t_lo; t < t_hi && ok;) {
            const Run s = run_at(t, t_hi, nrb, pl.E);
            t += s.rb1 - s.rb0;
            const int cnt = pl.expert_cnt[s.e];
            if (cnt > max_cnt) continue;
            const Chunks ch = chunks_of(cnt);
            const int c0 = s.cb * kSN;
            // this warp's 32-column chunks of the block: [j0, j1)
            const int nch = min(8, (C - c0) / 32);
            const int j0 = min(nch, 2 * slice), j1 = min(nch, 2 * slice + 2);
            // importance: an expert without slots has no gradient hook in the reference
            // (it has no tiles either); a threshold below zero means the caller left
            // the expert out: its tiles are drained without counting or emitting
            if (EPI >= EPI_HIST && cnt == 0) continue;
            const bool imp_skip = (EPI == EPI_EMIT && ia.thr[s.e] < 0) ||
                                  (EPI == EPI_HIST && ia.pmask && ia.pval[s.e] < 0);
            if (cnt == 0) {
                // no slots: the gradient is exactly zero
                for (int rb = s.rb0; rb < s.rb1; ++rb) {
                    const int64_t grow = (int64_t)s.e * R + rb * kSM + rr;
                    if (EPI == EPI_DENSE_ABS) {
                        float4 *o = reinterpret_cast<float4 *>(out + grow * C + c0);
                        for (int i = j0 * 8; i < j1 * 8; ++i) o[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                    } else if (j0 < j1) {
                        int q0, q1;
                        uint2 a;
                        slice_start(mask, cbptr, grow, C, ncb, s.cb, slice, a, q0, q1);
                        for (int i = 0; i < __popc(a.x); ++i) out[q0 + i] = 0.0f;
                        for (int i = 0; i < __popc(a.y); ++i) out[q1 + i] = 0.0f;
                    }
                }
                continue;
            }
            const TileOrder to{EPI != EPI_SPARSE, ch.n > 1, s.rb0, s.rb1, ch.n};
            // this row's selection in the warp's two chunks and its first CSR positions
            // in the two halves: loaded one row block ahead, so the loads' latency hides
            // behind a whole tile (sparse mode: chunk outer, row block inner)
            const bool sel = EPI == EPI_SPARSE && j0 < j1;
            SliceRaw nxt = {};
            for (int i = 0; i < to.n_outer() && ok; ++i) {
                for (int jj = 0; jj < to.n_inner(); ++jj) {
                    int rb, kc;
                    to.at(i, jj, rb, kc);
                    if (!to.acc_end(kc)) continue;          // the accumulator still sums chunks
                    if (sel && jj == 0) nxt = slice_load(mask, cbptr, (int64_t)s.e * R + s.rb0 * kSM + rr, C, ncb, s.cb, slice);
                    const int64_t grow = (int64_t)s.e * R + rb * kSM + rr;   // global storage row
                    uint2 mw = make_uint2(0, 0);
                    int p0 = 0, p1 = 0;
                    if (sel) {
                        const SliceRaw cur = nxt;
                        if (rb + 1 < s.rb1) nxt = slice_load(mask, cbptr, grow + kSM, C, ncb, s.cb, slice);
                        slice_decode(cur, slice, mw, p0, p1);
                    }
                    const int buf = it & 1;
                    if (!(ok = warp_wait(&S.acc_full[buf], (it >> 1) & 1, abort_flag, err))) break;
                    tc_fence_after();
                    const uint32_t tb = tbase + lane_off + buf * kSN;
                    if (j0 < j1 && EPI == EPI_SPARSE) {
                        // chunk j holds columns with (c/32) % 2 == j % 2: CSR half j & 1
                        // (j0 is even); one chunk in registers at a time
                        uint32_t va[32];
                        tmem_ld_32x32b_x32(tb + 32 * j0, va);
                        tmem_wait_ld();
                        drain_sparse(va, mw.x, p0, out);
                        tmem_ld_32x32b_x32(tb + 32 * j0 + 32, va);
                        tmem_wait_ld();
                        drain_sparse(va, mw.y, p1, out);
                    } else if (j0 < j1 && EPI >= EPI_HIST && !imp_skip) {
                        const int64_t lrow = (int64_t)rb * kSM + rr;   // row inside the expert
                        const int64_t flat0 = ((int64_t)s.e * R + lrow) * C + c0 + 32 * j0;
#pragma unroll 1
                        for (int h = 0; h < 2; ++h) {
                            uint32_t va[32];
                            tmem_ld_32x32b_x32(tb + 32 * (j0 + h), va);
                            tmem_wait_ld();
                            if (EPI == EPI_HIST) hist_chunk(va, hw, ia.shift, ia.pmask, ia.pmask ? ia.pval[s.e] : 0);
                            else emit_chunk(va, s.e, flat0 + 32 * h, ia.thr[s.e], ia, lane);
                        }
                    } else if (j0 < j1 && EPI == EPI_DENSE_ABS) {
                        uint32_t va[32], vb[32];
                        tmem_ld_32x32b_x32(tb + 32 * j0, va);
                        tmem_ld_32x32b_x32(tb + 32 * j0 + 32, vb);
                        tmem_wait_ld();
                        {
                            float *o = out + grow * C + c0 + 32 * j0;
                            drain_dense(va, o);
                            drain_dense(vb, o + 32);
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(&S.acc_empty[buf]);
                    ++it;
                }
            }
            if (EPI == EPI_HIST) {
                // the run's counts (one expert) into its global histogram; every drain
                // warp gets here, and all take the same decision on a wait that gave up
                ok = named_bar_and(1, kEpiThreads, ok);
                if (!ok) break;
                if (et < kHistBins) {
                    unsigned int sum = 0;
#pragma unroll 4
                    for (int w = 0; w < 16; ++w) {
                        sum += hist_all[w * kHistBins + et];
                        hist_all[w * kHistBins + et] = 0u;
                    }
                    if (sum) atomicAdd(ia.hist + (int64_t)s.e * kHistBins + et, sum);
                }
                named_bar_sync(1, kEpiThreads);
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 s_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// slot-major bf16 matrix [rows, cols] -> boxes of 64 slots x 64 columns, 128-byte swizzle
bool s_tmap(CUtensorMap *m, const void *ptr, int64_t rows, int64_t cols) {
    auto fn = s_encode();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || (cols * 2) % 16) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {64u, (cuuint32_t)kSK};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int s_num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

template <int EPI>
int sddmm_tc_launch(const usaf_route_plan *pl, int R, int C, const __nv_bfloat16 *gout,
                    const __nv_bfloat16 *gin, const uint32_t *mask, const int32_t *cbptr, float *out,
                    cudaStream_t st, const ImpArgs &ia = ImpArgs{}, int max_cnt = INT_MAX) {
    CUtensorMap ta, tb;
    if (!s_tmap(&ta, gout, pl->P_cap, R) || !s_tmap(&tb, gin, pl->P_cap, C)) return USAF_EUNSUPPORTED;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(sddmm_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSSmem) != cudaSuccess)
            return USAF_ECUDA;
        attr = true;
    }
    const int64_t tiles = (int64_t)pl->E * (R / kSM) * ((C + kSN - 1) / kSN);
    if (tiles == 0) return USAF_OK;
    dim3 grid((unsigned)std::min<int64_t>(s_num_sms(), tiles));
    sddmm_tc_kernel<EPI><<<grid, kSThreads, kSSmem, st>>>(ta, tb, *pl, R, C, mask, cbptr, out, ia, max_cnt);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

}  // namespace

bool sddmm_tc_supported(int R, int C) {
    // C % 128: a column block is 128 or 256 columns (whole bitmap words in
    // 16-byte loads)
    return R % kSM == 0 && C % 128 == 0 && s_encode() != nullptr;
}

// compact[c2c[j]] += scale * g[j]   (g already rounded to the activation dtype;
// c2c NULL: the identity map, compact kept in CSR order)
__global__ void sddmm_accumulate(int n, const float *__restrict__ g, const int32_t *__restrict__ c2c,
                                 float scale, float *__restrict__ compact) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
        const int pos = c2c ? c2c[j] : j;
        compact[pos] = __fadd_rn(compact[pos], __fmul_rn(scale, g[j]));
    }
}

// the same when compact is in CSR order (identity map): 16-byte vectors for the
// first n / 4 * 4 entries, the last n % 4 by the first threads
__global__ void sddmm_accumulate_id(int n, const float *__restrict__ g, float scale,
                                    float *__restrict__ compact) {
    const int n4 = n / 4;
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
    float4 *c4 = reinterpret_cast<float4 *>(compact);
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    for (int j = tid; j < n4; j += gridDim.x * blockDim.x) {
        const float4 a = g4[j];
        float4 c = c4[j];
        c.x = __fadd_rn(c.x, __fmul_rn(scale, a.x));
        c.y = __fadd_rn(c.y, __fmul_rn(scale, a.y));
        c.z = __fadd_rn(c.z, __fmul_rn(scale, a.z));
        c.w = __fadd_rn(c.w, __fmul_rn(scale, a.w));
        c4[j] = c;
    }
    if (tid < n - n4 * 4) {
        const int j = n4 * 4 + tid;
        compact[j] = __fadd_rn(compact[j], __fmul_rn(scale, g[j]));
    }
}

int sddmm_stream_sparse(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *gout,
                        const __nv_bfloat16 *gin, int min_cnt, float *scratch, cudaStream_t st);

// g[j] (CSR order) = bf16(D[e][r][c]) for every overlay entry, then
// compact[c2c[j]] += scale * g[j]
int sddmm_tc_sparse(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *gout,
                    const __nv_bfloat16 *gin, const int32_t *c2c, float scale, float *compact,
                    float *scratch, cudaStream_t st) {
    // experts of up to one resident chunk here; larger ones (only possible with
    // more tokens than that, or an unknown token count) in the streaming kernel
    // (sddmm_stream.cu), which sums a tile's slots in one accumulator instead of
    // chunk by chunk
    constexpr int kChunk = kBMaxKb * kSK;
    int rc = sddmm_tc_launch<EPI_SPARSE>(pl, w->R, w->C, gout, gin, w->ov_mask, w->ov_cbptr, scratch, st,
                                         ImpArgs{}, kChunk);
    if (rc == USAF_OK && (pl->T <= 0 || pl->T > kChunk))
        rc = sddmm_stream_sparse(pl, w, gout, gin, kChunk + 1, scratch, st);
    if (rc != USAF_OK) return rc;
    const int n = w->n_ov;
    if (!c2c && !((uintptr_t)scratch & 15) && !((uintptr_t)compact & 15)) {
        const int n4 = n / 4;
        sddmm_accumulate_id<<<std::max(1, std::min((n4 + 255) / 256, 148 * 8)), 256, 0, st>>>(n, scratch, scale,
                                                                                             compact);
    } else {   // a compact map, or an identity map on unaligned buffers
        sddmm_accumulate<<<std::min((n + 255) / 256, 148 * 16), 256, 0, st>>>(n, scratch, c2c, scale, compact);
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

int sddmm_tc_dense_abs(const usaf_route_plan *pl, int R, int C, const __nv_bfloat16 *gout,
                       const __nv_bfloat16 *gin, float *out, cudaStream_t st) {
    return sddmm_tc_launch<EPI_DENSE_ABS>(pl, R, C, gout, gin, nullptr, nullptr, out, st);
}

// importance histogram pass: hist[e][(key >> shift) & 255] += 1 for every key of
// expert e with (key & pmask) == pval[e] (experts without slots are skipped)
int sddmm_tc_key_hist(const usaf_route_plan *pl, int R, int C, const __nv_bfloat16 *gout,
                      const __nv_bfloat16 *gin, int shift, int pmask, const int32_t *pval,
                      unsigned int *hist, cudaStream_t st) {
    ImpArgs ia{};
    ia.shift = shift;
    ia.pmask = pmask;
    ia.pval = pval;
    ia.hist = hist;
    return sddmm_tc_launch<EPI_HIST>(pl, R, C, gout, gin, nullptr, nullptr, nullptr, st, ia);
}

// importance emit pass: coordinates of expert e with key > thr[e] into its
// candidate list (row cand_row[e] of gt_val / gt_idx, k entries a row), those
// with key == thr[e] into its tie list at eq_off[e]; experts with thr < 0 skipped
int sddmm_tc_key_emit(const usaf_route_plan *pl, int R, int C, const __nv_bfloat16 *gout,
                      const __nv_bfloat16 *gin, const int32_t *thr, int64_t k, const int32_t *cand_row,
                      int32_t *n_gt, int32_t *n_eq, float *gt_val, int64_t *gt_idx, const int64_t *eq_off,
                      float *eq_val, int64_t *eq_idx, cudaStream_t st) {
    ImpArgs ia{};
    ia.thr = thr;
    ia.k = k;
    ia.cand_row = cand_row;
    ia.n_gt = n_gt;
    ia.n_eq = n_eq;
    ia.gt_val = gt_val;
    ia.gt_idx = gt_idx;
    ia.eq_off = eq_off;
    ia.eq_val = eq_val;
    ia.eq_idx = eq_idx;
    return sddmm_tc_launch<EPI_EMIT>(pl, R, C, gout, gin, nullptr, nullptr, nullptr, st, ia);
}

// slots above which an expert's gradient is summed over several chunks (the
// importance passes then keep its partial sums in the caller's scratch)
int sddmm_tc_chunk_slots() { return kBMaxKb * kSK; }

}  // namespace usaf
