// Expert-weight gradients at the selected coordinates for plans whose experts
// hold many slots (usaf_sparse_dw, bf16): the streaming tcgen05 SDDMM.
//
// D_e[r][c] = sum_{s in slots of e} gout[s][r] * gin[s][c] as in sddmm_tc.cu,
// with the same operands, tile (128 storage rows x 256 columns), MN-major
// 128-byte-swizzled TMA boxes and epilogue contract (bf16(D) of every overlay
// entry into a CSR-ordered fp32 vector).  The operand flow differs: every
// stage carries one 64-slot k-block of both operands (gout 128 rows + gin 256
// columns, 48 KB), and a tile sums all of its expert's slots in one TMEM
// accumulator.  This kernel takes the experts above one resident chunk (the
// resident kernel skips them); persistent CTAs walk their tiles round-robin,
// numbered (expert, row block, column block), so at any time the CTAs work on
// neighbouring tiles of the same expert and its gin and gout stay in L2
// however large the expert is.
// The resident kernel of sddmm_tc.cu keeps a 320-slot gin chunk in shared
// memory across row blocks instead, which reads a third of the operand bytes
// for experts of up to 320 slots but would have to cut larger experts into
// chunks (C2 layer, T = 16384, both projections: 1.27 ms here against 2.50 ms
// with 320-slot chunks summed through the output).
//
// Warp 0 issues TMA, warp 1 the MMAs (and owns TMEM), warps 2-5 drain the
// accumulators, warp 6 passes each filled stage on to the MMA after zeroing
// the ragged tail of an expert's last k-block (the slots past the expert's
// end inside its last 16-slot group belong to the next expert); TMEM holds
// two 256-column accumulators so the drain of one tile overlaps the MMAs of
// the next.
#include <cudaTypedefs.h>

#include "tc_common.cuh"

namespace usaf {
using namespace tc;

namespace {

constexpr int kSM = 128;                 // storage rows per tile (MMA M)
constexpr int kSN = 256;                 // columns per tile (MMA N)
constexpr int kSK = 64;                  // slots per k-block
constexpr int kSStages = 4;
constexpr int kSThreads = 224;
constexpr int kBox = kSK * 64 * 2;       // one TMA box: 64 slots x 64 bf16 = 8 KB
constexpr int kAStage = 2 * kBox;        // 128 rows
constexpr int kStage = kAStage + 4 * kBox;   // + 256 columns = 48 KB
constexpr int kRowLd = 33;               // epilogue per-thread row (floats)

constexpr int kStreamMaxE = 1024;

struct alignas(8) SShared {
    uint64_t full[kSStages];
    uint64_t empty[kSStages];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint64_t fixed[kSStages];
    uint64_t mma_done;
    uint32_t tmem_base;
    int abort_flag;
    int n_large;
    int exp[kStreamMaxE];                    // the experts this kernel takes, their slot
    int cnt[kStreamMaxE];                    //   counts and first slots
    int off[kStreamMaxE];
};

constexpr size_t kSSmem = (size_t)kSStages * kStage + (size_t)128 * kRowLd * 4 + sizeof(SShared) + 1024;
static_assert(kSSmem <= 232448, "streaming SDDMM shared memory above the per-block limit");

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

// one work item: a tile (large expert a of the CTA's list, row block rb,
// column block cb); items run column block fastest, so the CTAs that work at
// the same time share the row block's gout rows and the column blocks' gin
__device__ __forceinline__ void item_at(int item, int nrb, int ncb, int &a, int &rb, int &cb) {
    a = item / (nrb * ncb);
    const int r = item - a * nrb * ncb;
    rb = r / ncb;
    cb = r - rb * ncb;
}

__global__ void __launch_bounds__(kSThreads, 1)
    sddmm_stream_kernel(const __grid_constant__ CUtensorMap tm_out, const __grid_constant__ CUtensorMap tm_in,
                        usaf_route_plan pl, int R, int C, int min_cnt, const uint32_t *__restrict__ mask,
                        const int32_t *__restrict__ cbptr, float *__restrict__ out) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *sb = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    float *rows_s = reinterpret_cast<float *>(sb + (size_t)kSStages * kStage);
    SShared &S = *reinterpret_cast<SShared *>(sb + (size_t)kSStages * kStage + (size_t)128 * kRowLd * 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nrb = R / kSM;
    const int ncb = (C + kSN - 1) / kSN;
    int *err = pl.err;
    // the experts of at least min_cnt slots (the others are the resident
    // kernel's), their slot counts and first slots; a CTA without any leaves
    // before it allocates TMEM
    for (int e = tid; e < pl.E; e += kSThreads) {
        S.cnt[e] = pl.expert_cnt[e];
        S.off[e] = pl.expert_off[e];
    }
    __syncthreads();
    if (warp == 0) {
        int n = 0;
        for (int e0 = 0; e0 < pl.E; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < pl.E ? S.cnt[e] : 0, o = e < pl.E ? S.off[e] : 0;
            const bool on = c >= min_cnt;
            const uint32_t m = __ballot_sync(0xffffffffu, on);
            __syncwarp();   // every lane has read its entries before the compaction writes
            if (on) {
                const int a = n + __popc(m & ((1u << lane) - 1));
                S.exp[a] = e;
                S.cnt[a] = c;
                S.off[a] = o;
            }
            n += __popc(m);
            __syncwarp();
        }
        if (lane == 0) {
            S.n_large = n;
            S.abort_flag = 0;
            for (int s = 0; s < kSStages; ++s) {
                mbar_init(&S.full[s], 1);
                mbar_init(&S.empty[s], 1);
                mbar_init(&S.fixed[s], 1);
            }
            for (int b = 0; b < 2; ++b) {
                mbar_init(&S.acc_full[b], 1);
                mbar_init(&S.acc_empty[b], 128);
            }
            mbar_init(&S.mma_done, 1);
            fence_barrier_init();
        }
    }
    __syncthreads();
    const int n_items = S.n_large * nrb * ncb;
    if ((int)blockIdx.x >= n_items) return;   // (uniform over the CTA)
    volatile int *abort_flag = &S.abort_flag;
    if (warp == 1) tmem_alloc(&S.tmem_base, 512);
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = S.tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            prefetch_tmap(&tm_out);
            prefetch_tmap(&tm_in);
            int g = 0, last_g = -1;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
                int a, rb, cb;
                item_at(item, nrb, ncb, a, rb, cb);
                const int cnt = S.cnt[a], row0 = S.off[a];
                const int nk = (cnt + kSK - 1) / kSK;
                const int c0 = cb * kSN;
                const int nb = min(4, (C - c0) / 64);
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int st = g % kSStages;
                    if (!mbar_wait(&S.empty[st], ((g / kSStages) & 1) ^ 1, abort_flag, err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&S.full[st], (uint32_t)((2 + nb) * kBox));
                    unsigned char *dst = sb + (size_t)st * kStage;
                    const int y = row0 + kb * kSK;
                    tma_load_2d(dst, &tm_out, &S.full[st], rb * kSM, y);
                    tma_load_2d(dst + kBox, &tm_out, &S.full[st], rb * kSM + 64, y);
                    for (int j = 0; j < nb; ++j)
                        tma_load_2d(dst + kAStage + j * kBox, &tm_in, &S.full[st], c0 + 64 * j, y);
                    last_g = g;
                }
            }
            if (*abort_flag)
                for (int gg = max(0, last_g - kSStages + 1); gg <= last_g; ++gg)
                    s_drain(&S.full[gg % kSStages], (gg / kSStages) & 1, err);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int g = 0, it = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++it) {
                int a, rb, cb;
                item_at(item, nrb, ncb, a, rb, cb);
                const int cnt = S.cnt[a];
                const int nk = (cnt + kSK - 1) / kSK;
                const int nb = min(4, (C - cb * kSN) / 64);
                const uint32_t idesc = idesc_mn(kSM, nb * 64);
                const int buf = it & 1;
                if (!mbar_wait(&S.acc_empty[buf], ((it >> 1) & 1) ^ 1, abort_flag, err)) { ok = false; break; }
                tc_fence_after();
                for (int kb = 0; kb < nk; ++kb, ++g) {
                    const int st = g % kSStages;
                    const int rem = min(kSK, cnt - kb * kSK);
                    // stages reach the MMA through the fixer warp (fixed[st] completes
                    // once per fill, after any ragged-tail zeroing)
                    if (!mbar_wait(&S.fixed[st], (g / kSStages) & 1, abort_flag, err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a_s = smem_u32(sb + (size_t)st * kStage), b_s = a_s + kAStage;
                    const int nks = (rem + 15) / 16;
                    for (int kk = 0; kk < nks; ++kk)
                        mma_ss(tbase + buf * kSN, desc_mn_sw128(a_s + kk * 2048),
                               desc_mn_sw128(b_s + kk * 2048), idesc, (kb | kk) != 0);
                    mma_commit(&S.empty[st]);
                }
                if (!ok) break;
                mma_commit(&S.acc_full[buf]);
            }
            // every MMA this CTA issued has completed before TMEM is released
            mma_commit(&S.mma_done);
            s_drain(&S.mma_done, 0, err);
        }
        __syncwarp();
    } else if (warp == 6) {
        // ---------------- fixer: forwards every filled stage to the MMA ----------------
        // Slots past the expert's end inside the last 16-slot group of its last
        // k-block belong to the next expert (or lie past the routed slots).  The
        // MMA reads whole 16-slot groups, so those rows are zeroed in every box
        // of the stage first.  Forwarding every fill (not only ragged ones) keeps
        // this warp in step with the stage phases.
        int g = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
            int a, rb, cb;
            item_at(item, nrb, ncb, a, rb, cb);
            const int cnt = S.cnt[a];
            const int nk = (cnt + kSK - 1) / kSK;
            const int rem = cnt - (nk - 1) * kSK;
            const int nb = min(4, (C - cb * kSN) / 64);
            for (int kb = 0; kb < nk; ++kb, ++g) {
                const int st = g % kSStages;
                const uint32_t par = (g / kSStages) & 1;
                if (kb == nk - 1 && (rem % 16)) {
                    ok = mbar_wait(&S.full[st], par, abort_flag, err);
                    ok = __all_sync(0xffffffffu, ok);
                    if (!ok) break;
                    const int r1 = (rem + 15) & ~15;
                    const int per_box = (r1 - rem) * 8;       // 16-byte chunks
                    unsigned char *stage = sb + (size_t)st * kStage;
                    for (int i = lane; i < (2 + nb) * per_box; i += 32) {
                        const int bx = i / per_box, k = i % per_box;
                        *reinterpret_cast<uint4 *>(stage + bx * kBox + rem * 128 + k * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                    fence_proxy_async();
                    __syncwarp();
                } else {
                    int w_ok = 1;
                    if (lane == 0) w_ok = mbar_wait(&S.full[st], par, abort_flag, err);
                    ok = __shfl_sync(0xffffffffu, w_ok, 0) != 0;
                    if (!ok) break;
                }
                if (lane == 0) mbar_arrive(&S.fixed[st]);
            }
        }
    } else if (warp >= 2) {
        // ---------------- epilogue (warps 2-5) ----------------
        const int q = warp & 3;                      // TMEM lane quarter
        const int rr = q * 32 + lane;                // row inside the tile
        const uint32_t lane_off = ((uint32_t)(q * 32)) << 16;
        float *my_row = rows_s + (q * 32 + lane) * kRowLd;
        const int cw = C / 32;                       // bitmap words per storage row
        int it = 0;
        for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
            int a, rb, cb;
            item_at(item, nrb, ncb, a, rb, cb);
            const int64_t grow = (int64_t)S.exp[a] * R + rb * kSM + rr;   // global storage row
            const int c0 = cb * kSN;
            const int nch = min(8, (C - c0) / 32);
            // CSR positions of the row's first entries in this column block (two halves)
            const int2 pp = __ldg(reinterpret_cast<const int2 *>(cbptr + (grow * ncb + cb) * 2));
            int p0 = pp.x, p1 = pp.y;
            uint32_t mw[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) mw[j] = j < nch ? mask[grow * cw + c0 / 32 + j] : 0u;
            const int buf = it & 1;
            if (!mbar_wait(&S.acc_full[buf], (it >> 1) & 1, abort_flag, err)) break;
            tc_fence_after();
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (4 * h >= nch) break;
                uint32_t v[4][32];
                // four 32-column loads in flight, one wait (nch is a multiple of 4)
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    tmem_ld_32x32b_x32(tbase + lane_off + buf * kSN + (4 * h + u) * 32, v[u]);
                tmem_wait_ld();
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int j = 4 * h + u;
                    uint32_t m = mw[j];
                    if (m) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) my_row[i] = __uint_as_float(v[u][i]);
                        // chunk j holds columns with (c/32) % 2 == j % 2: CSR half j&1
                        int p = (j & 1) ? p1 : p0;
                        while (m) {
                            const int b = __ffs(m) - 1;
                            m &= m - 1;
                            out[p++] = round_bf16(my_row[b]);
                        }
                        if (j & 1) p1 = p; else p0 = p;
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&S.acc_empty[buf]);
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

int sddmm_stream_launch(const usaf_route_plan *pl, int R, int C, int min_cnt, const __nv_bfloat16 *gout,
                        const __nv_bfloat16 *gin, const uint32_t *mask, const int32_t *cbptr, float *out,
                        cudaStream_t st) {
    if (pl->E > kStreamMaxE) return USAF_EUNSUPPORTED;
    CUtensorMap ta, tb;
    if (!s_tmap(&ta, gout, pl->P_cap, R) || !s_tmap(&tb, gin, pl->P_cap, C)) return USAF_EUNSUPPORTED;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(sddmm_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kSSmem) != cudaSuccess)
            return USAF_ECUDA;
        attr = true;
    }
    const int64_t tiles = (int64_t)pl->E * (R / kSM) * ((C + kSN - 1) / kSN);
    if (tiles == 0) return USAF_OK;
    dim3 grid((unsigned)std::min<int64_t>(s_num_sms(), tiles));
    sddmm_stream_kernel<<<grid, kSThreads, kSSmem, st>>>(ta, tb, *pl, R, C, min_cnt, mask, cbptr, out);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

}  // namespace

// scratch[j] (CSR order) = bf16(D[e][r][c]) for every overlay entry j of the
// experts with at least min_cnt slots
int sddmm_stream_sparse(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *gout,
                        const __nv_bfloat16 *gin, int min_cnt, float *scratch, cudaStream_t st) {
    return sddmm_stream_launch(pl, w->R, w->C, min_cnt, gout, gin, w->ov_mask, w->ov_cbptr, scratch, st);
}

}  // namespace usaf
