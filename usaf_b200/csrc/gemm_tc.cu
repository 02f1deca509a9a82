// tcgen05 grouped expert GEMMs over int4 weights (sm_100a).
//
// One CTA computes D[128 weight rows x up to 384 tokens] of one expert:
//   * A (weights) is dequantized on the fly by 4 producer warps: each thread
//     owns one TMEM lane (= one weight row), loads its row's packed int4
//     codes with 128-bit loads (prefetched 3 k-blocks ahead), computes
//     fp16(fp16(q*s)+z) -> bf16 in registers (the reference's rounding),
//     patches trained coordinates from the CSR overlay, and writes the 64-wide
//     k-block straight into TMEM with tcgen05.st -- the dequantized weights
//     never touch shared memory or HBM;
//   * B (tokens of the expert's segment, K-major) arrives in shared memory by
//     TMA with the 128-byte swizzle (plain per-CTA loads, no multicast);
//   * one thread issues tcgen05.mma (kind::f16, M=128, N<=256 for the first
//     256 tokens and N<=128 for the rest, A from TMEM, B from SMEM) into fp32
//     TMEM accumulators; tcgen05.commit
//     frees pipeline stages and finally signals the epilogue;
//   * the epilogue warps read the accumulators (tcgen05.ld), round to bf16,
//     transpose through shared memory and write token rows with 16-byte
//     stores; in gate_up mode the CTA's 128 rows are 64 gate rows and the
//     matching 64 up rows, so SwiGLU is fused here.
// TMEM: columns [0,384) accumulators (3 token sub-tiles), [384,512) four A
// stages of 32 columns (64 bf16 of K per lane).  All waits are bounded.
#include <cudaTypedefs.h>

#include "gemm_tc.cuh"
#include "gemm_tc_dev.cuh"
#include "tc_common.cuh"

namespace usaf {
using namespace tc;
using namespace gemm_dev;

namespace {

constexpr int kStages = 4;
constexpr int kBK = 64;
constexpr int kSub = 128;
constexpr int kMaxSub = 3;
constexpr int kMaxTok = kSub * kMaxSub;          // 384 tokens per CTA
constexpr int kSubBytes = kSub * kBK * 2;        // 16 KB per TMA box
constexpr int kStageBytes = kMaxSub * kSubBytes; // 48 KB per stage
constexpr int kAcol = kMaxTok;                   // first TMEM column of the A stages
constexpr int kThreads = 512;  // warps 0-3 epilogue, 4 TMA + work fetch, 5 MMA (+TMEM alloc), 8-15 dequant
constexpr int kStageLd = 136;                    // epilogue staging row stride (elements)

enum : int { MODE_GATE_UP = 0, MODE_DOWN = 1, MODE_DOWN_BWD = 2, MODE_GU_BWD = 3 };
constexpr int kBoxRows = 32;                     // token rows per TMA box
constexpr int kBoxBytes = kBoxRows * kBK * 2;    // 4 KB
constexpr int kQ = 3;                 // work-item queue depth
constexpr int kQUsers = 13;           // readers of a queue slot: MMA, 8 dequant warps, 4 epilogue warps
constexpr int kMaxOrder = 2048;       // tiles that the longest-first order can hold

struct alignas(8) TcShared {
    uint64_t full_b[kStages];
    uint64_t full_a[kStages];
    uint64_t empty[kStages];
    uint64_t acc;        // accumulators ready (tcgen05.commit)
    uint64_t acc_empty;  // accumulators drained by the epilogue (128 arrivals)
    uint64_t q_full[kQ];   // a work item is in the queue slot
    uint64_t q_empty[kQ];  // every role has read the slot
    int item_q[kQ];        // work item, -1 = no more work
    uint32_t tmem_base;
    int abort_flag;
};

constexpr size_t kStgBytes = (size_t)32 * kStageLd * 2;  // epilogue staging tile
constexpr size_t kSzBytes = (size_t)4 * kBK * 4;          // transposed-mode scale ring
// stages + epilogue staging + scale ring + shared block + tile prefix / counts (E <= 1024)
// + tile order
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + kStgBytes + kSzBytes + sizeof(TcShared) +
                              8 * 1025 + 4 * kMaxOrder + 1024;
static_assert(kSmemBytes <= 232448, "grouped GEMM shared memory above the per-block limit");

// The launch's last CTA returns the work counter pair to zero for the next launch.
__device__ __forceinline__ void sched_exit(int *c) {
    __threadfence();
    if (atomicAdd(c + 1, 1) == (int)gridDim.x - 1) {
        atomicExch(c, 0);
        atomicExch(c + 1, 0);
        __threadfence();
    }
}

// token-count bucket of an expert's tiles (cnt slots in ntt tiles, rounded as in decode_tile)
__device__ __forceinline__ int tile_bucket(int cnt, int ntt) {
    return ((((cnt + ntt - 1) / ntt) + 15) & ~15) >> 4;
}

// next work item from the CTA's queue (one thread): -1 when there is none left
// or a wait gave up
__device__ __forceinline__ int q_take(TcShared &S, int &qi, volatile int *abort_flag, int *err) {
    const int slot = qi % kQ;
    if (!mbar_wait(&S.q_full[slot], (qi / kQ) & 1, abort_flag, err)) return -1;
    const int w = *reinterpret_cast<volatile int *>(&S.item_q[slot]);
    mbar_arrive(&S.q_empty[slot]);
    ++qi;
    return w;
}

// the same for a whole warp (one arrival): -2 when the wait gave up
__device__ __forceinline__ int q_take_warp(TcShared &S, int &qi, volatile int *abort_flag, int *err, int lane) {
    const int slot = qi % kQ;
    const bool ok = mbar_wait(&S.q_full[slot], (qi / kQ) & 1, abort_flag, err);
    if (!__all_sync(0xffffffffu, ok)) return -2;
    const int w = *reinterpret_cast<volatile int *>(&S.item_q[slot]);
    __syncwarp();
    if (lane == 0) mbar_arrive(&S.q_empty[slot]);
    ++qi;
    return w;
}

// MODE_GATE_UP : rows = 64 gate + 64 up storage rows, K = C, SwiGLU epilogue
//                (out0 = gu [P,R], out1 = h [P,R/2])
// MODE_DOWN    : rows = 128 storage rows, K = C           (out0 = y [P,R])
// MODE_DOWN_BWD: rows = 128 storage columns (W^T), K = R, SwiGLU backward
//                epilogue (in1 = gu [P,2C], out0 = dgu [P,2C])
// MODE_GU_BWD  : rows = 128 storage columns (W^T), K = R  (out0 = dx [P,C])
template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmap_b, usaf_route_plan pl, usaf_qweight w,
                   __nv_bfloat16 *__restrict__ out0, __nv_bfloat16 *__restrict__ out1,
                   const __nv_bfloat16 *__restrict__ in1, int nrb) {
    constexpr bool TRANS = MODE >= MODE_DOWN_BWD;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *sbase = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    __nv_bfloat16 *stg = reinterpret_cast<__nv_bfloat16 *>(sbase + (size_t)kStages * kStageBytes);
    uint32_t *sz_ring = reinterpret_cast<uint32_t *>(sbase + (size_t)kStages * kStageBytes + kStgBytes);
    TcShared &S = *reinterpret_cast<TcShared *>(sbase + (size_t)kStages * kStageBytes + kStgBytes + kSzBytes);
    int *tile_off = reinterpret_cast<int *>(&S + 1);         // [E+1]
    int *cnts = tile_off + (pl.E + 1);                        // [E]
    int *order = tile_off + 2 * 1025;                         // [kMaxOrder] tiles, longest first
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int R = w.R, C = w.C, E = pl.E;
    const int K = TRANS ? R : C;
    const int nk = K / kBK;
    int *err = pl.err;

    // ---- per-expert tile prefix (block-wide scan, E <= 1024) ----
    {
        __shared__ int warp_tot[kThreads / 32];
        int c4[4], n4[4], mine = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int e_ = tid * 4 + q;   // 512 threads x 4 >= 1024 experts
            c4[q] = e_ < E ? pl.expert_cnt[e_] : 0;
            n4[q] = (c4[q] + kMaxTok - 1) / kMaxTok;
            mine += n4[q];
        }
        int x = mine;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) warp_tot[warp] = x;
        __syncthreads();
        int run = 0;
        for (int i = 0; i < warp; ++i) run += warp_tot[i];
        run += x - mine;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            int e_ = tid * 4 + q;
            if (e_ < E) { tile_off[e_] = run; cnts[e_] = c4[q]; }
            run += n4[q];
        }
        if (tid == kThreads - 1) tile_off[E] = run;
        if (tid == 0) {
            S.abort_flag = 0;
            for (int st = 0; st < kStages; ++st) {
                mbar_init(&S.full_b[st], 1);
                mbar_init(&S.full_a[st], 8);
                mbar_init(&S.empty[st], 1);
            }
            mbar_init(&S.acc, 1);
            mbar_init(&S.acc_empty, 128);
            for (int i = 0; i < kQ; ++i) {
                mbar_init(&S.q_full[i], 1);
                mbar_init(&S.q_empty[i], kQUsers);
            }
            fence_barrier_init();
        }
    }
    __syncthreads();
    const int n_tiles = tile_off[E];
    const int n_work = n_tiles * nrb;
    if ((int)blockIdx.x >= n_work) {   // whole CTA leaves before any TMEM / async work
        if (tid == 0 && pl.sched) sched_exit(pl.sched + 2 * MODE);
        return;
    }
    volatile int *abort_flag = &S.abort_flag;

    // Work items (tile, row block) are handed out longest tile first: tiles sorted
    // by their token count in buckets of 16 slots, ascending expert inside a
    // bucket.  Every CTA must build the same order (a ticket names an item through
    // it), so the placement is a scan, not shared-memory atomics.
    const bool sorted = n_tiles <= kMaxOrder;
    if (sorted) {
        // bucket = token count / 16, plus the trained coordinates per k-block of the
        // expert's most trained row (column, backward): a row whose coordinates the
        // producer lane walks one by one can make an item take twice as long
        constexpr int kHeavyMax = 40;
        constexpr int kNB = kMaxTok / 16 + kHeavyMax + 1;
        const int32_t *emax = w.n_ov ? (TRANS ? w.ov_emaxT : w.ov_emax) : nullptr;
        __shared__ unsigned char bkt[1024];
        __shared__ int bcnt[kNB], bpos[kNB];
        if (tid < kNB) bcnt[tid] = 0;
        __syncthreads();
        for (int e_ = tid; e_ < E; e_ += kThreads) {
            const int ntt = tile_off[e_ + 1] - tile_off[e_];
            const int heavy = emax ? min(emax[e_] / nk, kHeavyMax) : 0;
            bkt[e_] = ntt ? (unsigned char)(tile_bucket(cnts[e_], ntt) + heavy) : (unsigned char)255;
            if (ntt) atomicAdd(&bcnt[bkt[e_]], ntt);   // integer sums: the same in every CTA
        }
        __syncthreads();
        if (tid == 0) {
            int run = 0;
            for (int b = kNB - 1; b >= 0; --b) {
                bpos[b] = run;
                run += bcnt[b];
            }
        }
        __syncthreads();
        // one warp per bucket: the bucket's experts in ascending order, placed by a
        // warp-wide prefix sum of their tile counts
        for (int b = warp; b < kNB; b += kThreads / 32) {
            int carry = bpos[b];
            for (int e0 = 0; e0 < E; e0 += 32) {
                const int e_ = e0 + lane;
                const int ntt = (e_ < E && bkt[e_] == b) ? tile_off[e_ + 1] - tile_off[e_] : 0;
                int incl = ntt;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                for (int j = 0; j < ntt; ++j) order[carry + incl - ntt + j] = tile_off[e_] + j;
                carry += __shfl_sync(0xffffffffu, incl, 31);
            }
        }
        __syncthreads();
    }
    auto item_tile = [&](int work) { return sorted ? order[work / nrb] : work / nrb; };

    if (warp == 5) tmem_alloc(&S.tmem_base, 512);
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = S.tmem_base;

    if (warp == 4) {
        // ---------------- TMA producer (token rows, 32-row boxes) ----------------
        // It also hands out the work: with plan counters each item goes to the CTA
        // that asks next (longest first), so CTAs finish together whatever the
        // items cost.  The next item is claimed a few k-blocks before this one's
        // loads are all issued -- late enough that a CTA holds no work it is not
        // about to start, early enough that the counter's latency is hidden.
        if (lane == 0) {
            prefetch_tmap(&tmap_b);
            int *ctr = pl.sched ? pl.sched + 2 * MODE : nullptr;
            int fetched = 0;
            auto fetch = [&]() {
                const int t = ctr ? atomicAdd(ctr, 1) : (int)blockIdx.x + fetched * (int)gridDim.x;
                ++fetched;
                return t;
            };
            int g = 0, last_g = -1, qi = 0;
            int next = fetch();
            while (!*abort_flag) {
                const int slot = qi % kQ;
                if (!mbar_wait(&S.q_empty[slot], ((qi / kQ) & 1) ^ 1, abort_flag, err)) break;
                const int work = next < n_work ? next : -1;
                *reinterpret_cast<volatile int *>(&S.item_q[slot]) = work;
                mbar_arrive(&S.q_full[slot]);
                ++qi;
                if (work < 0) break;
                const int fetch_at = max(0, nk - 6);
                int e, t0, ntok;
                decode_tile(tile_off, cnts, E, item_tile(work), e, t0, ntok);
                const int row0 = pl.expert_off[e] + t0;
                const int nbox = (ntok + kBoxRows - 1) / kBoxRows;
                const int rb = work % nrb;
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int st = g % kStages;
                    if (kb == fetch_at) next = fetch();
                    if (!mbar_wait(&S.empty[st], ((g / kStages) & 1) ^ 1, abort_flag, err)) break;
                    mbar_arrive_expect_tx(&S.full_b[st], (uint32_t)(nbox * kBoxBytes + (TRANS ? kBK * 4 : 0)));
                    unsigned char *dst = sbase + (size_t)st * kStageBytes;
                    for (int j = 0; j < nbox; ++j)
                        tma_load_2d(dst + j * kBoxBytes, &tmap_b, &S.full_b[st], kb * kBK, row0 + j * kBoxRows);
                    if (TRANS) {
                        // per-row (scale|zero) words of this k-block for the column group
                        const uint32_t *src = w.szT + ((int64_t)e * (C / w.group_size) +
                                                       (rb * 128) / w.group_size) * R + kb * kBK;
                        bulk_load(sz_ring + st * kBK, src, kBK * 4, &S.full_b[st]);
                    }
                    last_g = g;
                }
            }
            if (*abort_flag) {
                for (int gg = max(0, last_g - kStages + 1); gg <= last_g; ++gg)
                    drain_wait(&S.full_b[gg % kStages], (gg / kStages) & 1, err);
            }
        }
    } else if (warp == 5) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int g = 0, it = 0, qi = 0;
            for (; !*abort_flag; ++it) {
                const int work = q_take(S, qi, abort_flag, err);
                if (work < 0) break;
                int e, t0, ntok;
                decode_tile(tile_off, cnts, E, item_tile(work), e, t0, ntok);
                // tokens [0, 256) in one MMA of N <= 256 (columns 0..255), the rest
                // (tokens 256..383) in a second one (columns 256..383): wide MMAs
                // amortise the per-instruction cost of the A operand read from TMEM
                const int nA = min(2 * kSub, (ntok + 15) & ~15);
                const int n2 = ntok - 2 * kSub;
                const uint32_t idA = idesc_bf16(128, nA);
                const uint32_t id2 = idesc_bf16(128, n2 <= 0 ? 16 : (min(kSub, n2) + 15) & ~15);
                // the epilogue of the previous tile must have drained the accumulators
                if (!mbar_wait(&S.acc_empty, (it & 1) ^ 1, abort_flag, err)) break;
                tc_fence_after();
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int st = g % kStages;
                    const uint32_t par = (g / kStages) & 1;
                    if (!mbar_wait(&S.full_b[st], par, abort_flag, err)) break;
                    if (!mbar_wait(&S.full_a[st], par, abort_flag, err)) break;
                    tc_fence_after();
                    const uint32_t bst = smem_u32(sbase + (size_t)st * kStageBytes);
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {
                        const uint32_t a_t = tbase + kAcol + st * 32 + kk * 8;
                        const uint32_t acc = (kb | kk) != 0;
                        mma_ts(tbase, a_t, smem_desc_sw128(bst + kk * 32), idA, acc);
                        if (n2 > 0) mma_ts(tbase + 2 * kSub, a_t, smem_desc_sw128(bst + 2 * kSubBytes + kk * 32), id2, acc);
                    }
                    mma_commit(&S.empty[st]);
                }
                mma_commit(&S.acc);
            }
        }
    } else if (warp >= 8) {
        // ---------------- dequant producers (warps 8-15) ----------------
        // warp w owns TMEM lane quarter w%4 and K half hf of every 64-wide
        // k-block (columns [hf*32, hf*32+32))
        const int t = tid - 256;                // 0..255
        const int row = t & 127;                // TMEM lane = weight row of the tile
        const int hf = t >> 7;
        const uint32_t lane_off = ((uint32_t)(warp & 3) * 32) << 16;
        const int gs = w.group_size;
        const int kpg = gs / kBK;                      // k-blocks per scale group
        const bool kpg_pow2 = (kpg & (kpg - 1)) == 0;
        const int kshift = __ffs(kpg) - 1;
        const unsigned short *s_ptr = reinterpret_cast<const unsigned short *>(w.s);
        const unsigned short *z_ptr = reinterpret_cast<const unsigned short *>(w.z);
        int g = 0, qi = 0;
        bool ok = true;
        while (ok) {
            const int work = q_take_warp(S, qi, abort_flag, err, lane);
            if (work < 0) break;
            int e, t0, ntok;
            decode_tile(tile_off, cnts, E, item_tile(work), e, t0, ntok);
            const int rb = work % nrb;
            int64_t crow;        // row of q (fwd) or qT (bwd) this lane dequantizes
            int j0 = 0, h0 = 0;  // output column base
            if (MODE == MODE_GATE_UP) {
                const int I = R / 2;
                j0 = rb * 64;
                crow = (int64_t)e * R + (row < 64 ? j0 + row : I + j0 + (row - 64));
            } else if (MODE == MODE_DOWN) {
                h0 = rb * 128;
                crow = (int64_t)e * R + h0 + row;
            } else {
                h0 = rb * 128;   // storage column block
                crow = (int64_t)e * C + h0 + row;
            }
            const uint4 *qrow = reinterpret_cast<const uint4 *>((TRANS ? w.qT : w.qP) + crow * (K / 2)) + hf;
            // scale / zero group of k-block kb: groups run along K and hold gs / 64
            // k-blocks, so it is g0 + kb / kpg (a shift when kpg is a power of two,
            // as for group 128) -- no 64-bit division per k-block
            const int64_t g0 = crow * (int64_t)(K / gs);
            // overlay queue of this lane: next two trained coordinates (K index, bf16 bits)
            const int32_t *ov_ptr = TRANS ? w.colT_ptr : w.row_ptr;
            const int32_t *ov_idx = TRANS ? w.rowT : w.col;
            const float *ov_val = TRANS ? w.valT : w.val;
            int cur = 0, cend = 0, qc0 = 0x7fffffff, qc1 = 0x7fffffff;
            float qv0 = 0.f, qv1 = 0.f;   // raw values: converted where used, so a queue
                                          // refill never waits for its own load
            if (w.n_ov > 0) {
                cur = ov_ptr[crow * 2 + hf];      // this lane's (row, half) segment
                cend = ov_ptr[crow * 2 + hf + 1];
                if (cur < cend) { qc0 = ov_idx[cur]; qv0 = ov_val[cur]; }
                if (cur + 1 < cend) { qc1 = ov_idx[cur + 1]; qv1 = ov_val[cur + 1]; }
            }
            // 3-slot prefetch ring: slot i holds k-block kb with kb % 3 == i; a slot
            // is refilled with kb+3 right after it is consumed (no register moves
            // of in-flight loads, which would wait for them)
            uint4 a0 = make_uint4(0, 0, 0, 0), a1 = a0, a2 = a0;
            // scale and zero stay in separate registers until their use three
            // k-blocks later (combining them at load time would wait for the loads)
            uint2 z0 = make_uint2(0, 0), z1 = z0, z2 = z0;
#define USAF_LOAD(kb_, A_, Z_)                                                                   \
    do {                                                                                         \
        A_ = __ldg(qrow + (kb_) * 2);                                                            \
        if (!TRANS) {                                                                            \
            const int64_t gg = g0 + (kpg_pow2 ? ((kb_) >> kshift) : ((kb_) / kpg));            \
            Z_.x = __ldg(s_ptr + gg);                                                            \
            Z_.y = __ldg(z_ptr + gg);                                                            \
        }                                                                                        \
    } while (0)
            USAF_LOAD(0, a0, z0);
            if (1 < nk) USAF_LOAD(1, a1, z1);
            if (2 < nk) USAF_LOAD(2, a2, z2);
            auto kstep = [&](int kb, uint4 &A, uint2 &Z) {
                const int st = g % kStages;
                const int kh0 = kb * kBK + hf * 32;   // first K index of this lane's half-block
                uint32_t szr[32];
                if (TRANS) {
                    // this k-block's per-row (scale|zero) words arrive with the stage's TMA
                    // (warp-uniform outcome: the warp stores to TMEM together below)
                    const bool w_ok = mbar_wait(&S.full_b[st], (g / kStages) & 1, abort_flag, err);
                    if (!__all_sync(0xffffffffu, w_ok)) { ok = false; return; }
                    const uint32_t *ring = sz_ring + st * kBK + hf * 32;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        uint4 v4 = *reinterpret_cast<const uint4 *>(ring + 4 * i);
                        szr[4 * i] = v4.x; szr[4 * i + 1] = v4.y; szr[4 * i + 2] = v4.z; szr[4 * i + 3] = v4.w;
                    }
                }
                const int rel = qc0 - kh0;
                const bool hit = rel >= 0 && rel < 32;
                const int pj = hit ? (rel >> 1) : 0xFF;
                const uint32_t qb0 = __bfloat16_as_ushort(__float2bfloat16_rn(qv0));
                const uint32_t m2 = qb0 | (qb0 << 16);
                const uint32_t hm = (rel & 1) ? 0xFFFF0000u : 0x0000FFFFu;
                uint32_t r[16];
                dequant16<TRANS>(A, Z.x | (Z.y << 16), szr, pj, m2, hm, r);
                if (kb + 3 < nk) USAF_LOAD(kb + 3, A, Z);   // refill the consumed slot
                if (hit) {
                    // advance the queue; more coordinates in this block take the slow path
                    ++cur;
                    qc0 = qc1; qv0 = qv1;
                    qc1 = 0x7fffffff;
                    if (cur + 1 < cend) { qc1 = ov_idx[cur + 1]; qv1 = ov_val[cur + 1]; }
                    while (qc0 < kh0 + 32) {
                        patch_elem16(r, qc0 - kh0, __bfloat16_as_ushort(__float2bfloat16_rn(qv0)));
                        ++cur;
                        qc0 = qc1; qv0 = qv1;
                        qc1 = 0x7fffffff;
                        if (cur + 1 < cend) { qc1 = ov_idx[cur + 1]; qv1 = ov_val[cur + 1]; }
                    }
                }
                const bool e_ok = mbar_wait(&S.empty[st], ((g / kStages) & 1) ^ 1, abort_flag, err);
                if (!__all_sync(0xffffffffu, e_ok)) { ok = false; return; }
                tc_fence_after();
                tmem_st_32x32b_x16(tbase + lane_off + kAcol + st * 32 + hf * 16, r);
                tmem_wait_st();
                tc_fence_before();
                // one arrival per warp (full_a counts the 8 producer warps)
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.full_a[st]);
                ++g;
            };
            for (int kb = 0; kb < nk && ok; kb += 3) {
                kstep(kb, a0, z0);
                if (kb + 1 < nk && ok) kstep(kb + 1, a1, z1);
                if (kb + 2 < nk && ok) kstep(kb + 2, a2, z2);
            }
#undef USAF_LOAD
            if (!ok) break;
        }
    } else if (warp < 4) {
        // ---------------- epilogue (warps 0-3): overlaps the next tile's dequant ----------------
        const int row = tid;                       // TMEM lane
        const uint32_t lane_off = ((uint32_t)warp * 32) << 16;
        int it = 0, qi = 0;
        for (;; ++it) {
            // one decision for the 128 epilogue threads (see below)
            const int qs = qi % kQ;
            if (!named_bar_and(2, 128, mbar_wait(&S.q_full[qs], (qi / kQ) & 1, abort_flag, err))) break;
            const int work = *reinterpret_cast<volatile int *>(&S.item_q[qs]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.q_empty[qs]);
            ++qi;
            if (work < 0) break;
            int e, t0, ntok;
            decode_tile(tile_off, cnts, E, item_tile(work), e, t0, ntok);
            const int rb = work % nrb;
            const int row0 = pl.expert_off[e] + t0;
            int j0 = 0, h0 = 0;
            if (MODE == MODE_GATE_UP) j0 = rb * 64;
            else h0 = rb * 128;
            // one decision for the 128 epilogue threads: the loop below syncs them on
            // a named barrier, so none may leave it alone
            if (!named_bar_and(2, 128, mbar_wait(&S.acc, it & 1, abort_flag, err))) break;
            tc_fence_after();
            const int gt = row;
            __nv_bfloat16 *stg_g = stg;
            for (int c0 = 0; c0 < ntok; c0 += 32) {
                // MODE_DOWN_BWD: this thread's forward gate/up vectors for the chunk
                // (items gt + 128 q: token j = gt/16 + 8 q, column group gt%16), loaded
                // before the TMEM drain so their latency overlaps it (loading them a
                // chunk earlier measured slower)
                uint4 gpre[4], upre[4];
                if (MODE == MODE_DOWN_BWD) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int j = (gt >> 4) + 8 * q;
                        if (c0 + j < ntok) {
                            const int64_t slot = row0 + c0 + j;
                            const int i0 = h0 + (gt & 15) * 8;
                            gpre[q] = *reinterpret_cast<const uint4 *>(in1 + slot * 2 * C + i0);
                            upre[q] = *reinterpret_cast<const uint4 *>(in1 + slot * 2 * C + C + i0);
                        }
                    }
                }
                uint32_t v[32];
                tmem_ld_32x32b_x32(tbase + lane_off + c0, v);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    stg_g[i * kStageLd + row] = __float2bfloat16_rn(__uint_as_float(v[i]));
                named_bar_sync(1, 128);
                if (MODE == MODE_DOWN || MODE == MODE_GU_BWD) {
                    // four 16-byte items per thread: all loads first, then all stores
                    const int ld = MODE == MODE_DOWN ? R : C;
                    uint4 val[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int item = gt + 128 * q, j = item >> 4, sg = item & 15;
                        val[q] = *reinterpret_cast<const uint4 *>(stg_g + j * kStageLd + sg * 8);
                    }
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int item = gt + 128 * q, j = item >> 4, sg = item & 15;
                        if (c0 + j < ntok)
                            *reinterpret_cast<uint4 *>(out0 + (int64_t)(row0 + c0 + j) * ld + h0 + sg * 8) = val[q];
                    }
                } else if (MODE == MODE_GATE_UP) {
                    const int I = R / 2;
                    for (int item = gt; item < 32 * 8; item += 128) {
                        const int j = item >> 3, sg = item & 7;
                        if (c0 + j < ntok) {
                            const int64_t slot = row0 + c0 + j;
                            uint4 gv = *reinterpret_cast<const uint4 *>(stg_g + j * kStageLd + sg * 8);
                            uint4 uv = *reinterpret_cast<const uint4 *>(stg_g + j * kStageLd + 64 + sg * 8);
                            const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
                            const uint32_t uw[4] = {uv.x, uv.y, uv.z, uv.w};
                            const uint64_t one2 = f2_pack(1.0f, 1.0f);
                            uint32_t h4[4];
#pragma unroll
                            for (int w2 = 0; w2 < 4; ++w2) {
                                // fast exp / divide: silu(g) is rounded to bf16 before the
                                // product, a few fp32 ulps do not survive that rounding
                                const uint64_t g2 = bf2_to_f2(gw[w2]);
                                const uint64_t den2 = f2_add(one2, f2_pack(__expf(-f2_lo(g2)), __expf(-f2_hi(g2))));
                                const uint64_t s2 = f2_pack(__fdividef(f2_lo(g2), f2_lo(den2)),
                                                            __fdividef(f2_hi(g2), f2_hi(den2)));
                                h4[w2] = f2_to_bf2(f2_mul(bf2_to_f2(f2_to_bf2(s2)), bf2_to_f2(uw[w2])));
                            }
                            *reinterpret_cast<uint4 *>(out0 + slot * R + j0 + sg * 8) = gv;
                            *reinterpret_cast<uint4 *>(out0 + slot * R + I + j0 + sg * 8) = uv;
                            *reinterpret_cast<uint4 *>(out1 + slot * I + j0 + sg * 8) = make_uint4(h4[0], h4[1], h4[2], h4[3]);
                        }
                    }
                } else {  // MODE_DOWN_BWD: SwiGLU backward with the forward's gate/up
                    const int I = C;
                    uint4 dv[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int j = (gt >> 4) + 8 * q, sg = gt & 15;
                        dv[q] = *reinterpret_cast<const uint4 *>(stg_g + j * kStageLd + sg * 8);
                    }
                    const uint64_t one2 = f2_pack(1.0f, 1.0f);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int j = (gt >> 4) + 8 * q, sg = gt & 15;
                        const uint32_t dw[4] = {dv[q].x, dv[q].y, dv[q].z, dv[q].w};
                        const uint32_t gw[4] = {gpre[q].x, gpre[q].y, gpre[q].z, gpre[q].w};
                        const uint32_t uw[4] = {upre[q].x, upre[q].y, upre[q].z, upre[q].w};
                        // this item's slot takes the next chunk's vectors, in flight
                        // during the rest of this chunk
                        uint32_t dg4[4], du4[4];
#pragma unroll
                        for (int w2 = 0; w2 < 4; ++w2) {
                            // two elements per packed fp32 operation; fast exp / reciprocal:
                            // the backward products are rounded to bf16, a few fp32 ulps
                            // do not survive that
                            const uint64_t dh2 = bf2_to_f2(dw[w2]), g2 = bf2_to_f2(gw[w2]);
                            const uint64_t u2 = bf2_to_f2(uw[w2]);
                            const uint64_t den2 = f2_add(one2, f2_pack(__expf(-f2_lo(g2)), __expf(-f2_hi(g2))));
                            const uint64_t sig2 = f2_pack(__fdividef(1.0f, f2_lo(den2)), __fdividef(1.0f, f2_hi(den2)));
                            const uint64_t sgr2 = bf2_to_f2(f2_to_bf2(f2_mul(g2, sig2)));
                            const uint64_t dsr2 = bf2_to_f2(f2_to_bf2(f2_mul(dh2, u2)));
                            du4[w2] = f2_to_bf2(f2_mul(dh2, sgr2));
                            const uint64_t tt2 = f2_add(one2, f2_mul(g2, f2_sub(one2, sig2)));
                            dg4[w2] = f2_to_bf2(f2_mul(f2_mul(dsr2, sig2), tt2));
                        }
                        if (c0 + j < ntok) {
                            const int64_t slot = row0 + c0 + j;
                            const int i0 = h0 + sg * 8;
                            *reinterpret_cast<uint4 *>(out0 + slot * 2 * I + i0) = make_uint4(dg4[0], dg4[1], dg4[2], dg4[3]);
                            *reinterpret_cast<uint4 *>(out0 + slot * 2 * I + I + i0) = make_uint4(du4[0], du4[1], du4[2], du4[3]);
                        }
                    }
                }
                named_bar_sync(1, 128);
            }
            tc_fence_before();
            mbar_arrive(&S.acc_empty);
        }
        // accumulators of a tile whose epilogue was skipped must be complete before dealloc
        if (*abort_flag) drain_wait(&S.acc, it & 1, err);
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tbase, 512);
    }
    if (tid == 0 && pl.sched) sched_exit(pl.sched + 2 * MODE);
}

// ---- host: tensor maps ------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// row-major bf16 matrix [rows, cols] -> boxes of 32 rows x 64 cols, 128-byte swizzle
bool make_tmap_rows(CUtensorMap *m, const void *ptr, int64_t rows, int64_t cols) {
    auto fn = encode_fn();
    if (!fn) return false;
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (cols * 2) % 16) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBoxRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides,
                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int num_sms() {
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

template <int MODE>
int launch_tc(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *act,
              __nv_bfloat16 *out0, __nv_bfloat16 *out1, const __nv_bfloat16 *in1, cudaStream_t st) {
    constexpr bool TRANS = MODE >= MODE_DOWN_BWD;
    const int K = TRANS ? w->R : w->C;
    CUtensorMap tm;
    if (!make_tmap_rows(&tm, act, pl->P_cap, K)) return USAF_EUNSUPPORTED;
    static bool attr_set = false;
    if (!attr_set) {
        if (cudaFuncSetAttribute(tc_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSmemBytes) != cudaSuccess)
            return USAF_ECUDA;
        attr_set = true;
    }
    int nrb = MODE == MODE_GATE_UP ? (w->R / 2) / 64 : (MODE == MODE_DOWN ? w->R / 128 : w->C / 128);
    int work_ub = (pl->P_cap / kMaxTok + 1 + pl->E) * nrb;
    dim3 grid(std::min(num_sms(), work_ub));
    tc_gemm_kernel<MODE><<<grid, kThreads, kSmemBytes, st>>>(tm, *pl, *w, out0, out1, in1, nrb);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

bool shape_ok_common(const usaf_qweight *w) {
    return w->E <= 1024 && w->C % kBK == 0 && w->R % kBK == 0 && w->group_size % kBK == 0 &&
           w->C % 32 == 0 && encode_fn() != nullptr;
}

}  // namespace

bool tc_supported_gate_up(const usaf_qweight *w) { return shape_ok_common(w) && w->qP && w->R % 128 == 0; }
bool tc_supported_down(const usaf_qweight *w) { return shape_ok_common(w) && w->qP && w->R % 128 == 0; }
static bool trans_ok(const usaf_qweight *w) {
    return shape_ok_common(w) && w->qT && w->szT && w->C % 128 == 0 && w->group_size % 128 == 0 &&
           (w->n_ov == 0 || (w->colT_ptr && w->rowT && w->valT));
}
bool tc_supported_down_bwd(const usaf_qweight *w) { return trans_ok(w); }
bool tc_supported_gate_up_bwd(const usaf_qweight *w) { return trans_ok(w); }

int tc_gate_up_fwd(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *x_perm,
                   __nv_bfloat16 *gu, __nv_bfloat16 *h, cudaStream_t st) {
    return launch_tc<MODE_GATE_UP>(pl, w, x_perm, gu, h, nullptr, st);
}
int tc_down_fwd(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *h,
                __nv_bfloat16 *y_seg, cudaStream_t st) {
    return launch_tc<MODE_DOWN>(pl, w, h, y_seg, nullptr, nullptr, st);
}
int tc_down_bwd(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *dcur,
                const __nv_bfloat16 *gu, __nv_bfloat16 *dgu, cudaStream_t st) {
    return launch_tc<MODE_DOWN_BWD>(pl, w, dcur, dgu, nullptr, gu, st);
}
int tc_gate_up_bwd(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *dgu,
                   __nv_bfloat16 *dx_seg, cudaStream_t st) {
    return launch_tc<MODE_GU_BWD>(pl, w, dgu, dx_seg, nullptr, nullptr, st);
}

}  // namespace usaf
