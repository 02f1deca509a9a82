// Dense bf16 GEMM on tcgen05 for the router (logits, dW_r, dX_r).
//
//   P[split][M][N] = sum_{k in split} A[m][k] * B[n][k]      (fp32 partials)
// A [M, K] is row-major bf16 (K contiguous, "K-major"); B is either [N, K]
// (K-major) or [K, N] (N contiguous, "MN-major": the MMA reads it transposed,
// so a row-major activation needs no transpose copy).  Both are staged by TMA
// with the 128-byte swizzle; one thread issues
// tcgen05.mma kind::f16 (A and B from shared memory, M=128, N=128) into a
// TMEM accumulator; 4 epilogue warps drain it to fp32 partials.  A separate
// finalize kernel sums the split-K partials in a fixed order (deterministic)
// and applies the destination's rounding and layout.
#include <cudaTypedefs.h>

#include "tc_common.cuh"

namespace usaf {
using namespace tc;

namespace {

constexpr int kD_BM = 128, kD_BN = 128, kD_BK = 64, kD_Stages = 4, kD_Threads = 192;
constexpr int kD_TileBytes = kD_BM * kD_BK * 2;  // 16 KB per operand per stage

struct alignas(8) DShared {
    uint64_t full[kD_Stages];
    uint64_t empty[kD_Stages];
    uint64_t acc;
    uint32_t tmem_base;
    int abort_flag;
};

constexpr size_t kD_Smem = (size_t)kD_Stages * 2 * kD_TileBytes + sizeof(DShared) + 1024;

__device__ __forceinline__ void d_drain(uint64_t *bar, uint32_t parity, int *err) {
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

// MN-major operand with the 128-byte swizzle: two 64-wide N blocks LBO = 8 KB
// apart (one TMA box each), 8-row K groups SBO = 1 KB apart, version 1
__device__ __forceinline__ uint64_t d_desc_mn_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)(8192 >> 4) << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// grid: (N/128, M/128, splits); each CTA: one 128x128 tile over its K range
template <bool B_MN>
__global__ void __launch_bounds__(kD_Threads, 1)
    dense_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                    int M, int N, int K, int k_per_split, float *__restrict__ part, int64_t ldp,
                    int64_t split_stride, int m_valid, int *err) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *sb = reinterpret_cast<unsigned char *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    DShared &S = *reinterpret_cast<DShared *>(sb + (size_t)kD_Stages * 2 * kD_TileBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * kD_BN, m0 = blockIdx.y * kD_BM;
    const int kbeg = blockIdx.z * k_per_split;
    const int kend = min(K, kbeg + k_per_split);
    const int nk = (kend - kbeg) / kD_BK;
    if (tid == 0) {
        S.abort_flag = 0;
        for (int s = 0; s < kD_Stages; ++s) {
            mbar_init(&S.full[s], 1);
            mbar_init(&S.empty[s], 1);
        }
        mbar_init(&S.acc, 1);
        fence_barrier_init();
    }
    __syncthreads();
    volatile int *abort_flag = &S.abort_flag;
    if (warp == 1) tmem_alloc(&S.tmem_base, 128);
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = S.tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tma_a);
            prefetch_tmap(&tma_b);
            int last = -1;
            for (int kb = 0; kb < nk; ++kb) {
                const int st = kb % kD_Stages;
                if (!mbar_wait(&S.empty[st], ((kb / kD_Stages) & 1) ^ 1, abort_flag, err)) break;
                mbar_arrive_expect_tx(&S.full[st], 2 * kD_TileBytes);
                unsigned char *a_dst = sb + (size_t)st * 2 * kD_TileBytes;
                const int kx = kbeg + kb * kD_BK;
                tma_load_2d(a_dst, &tma_a, &S.full[st], kx, m0);
                if (B_MN) {   // two boxes of 64 K rows x 64 N columns
                    tma_load_2d(a_dst + kD_TileBytes, &tma_b, &S.full[st], n0, kx);
                    tma_load_2d(a_dst + kD_TileBytes + kD_TileBytes / 2, &tma_b, &S.full[st], n0 + 64, kx);
                } else {
                    tma_load_2d(a_dst + kD_TileBytes, &tma_b, &S.full[st], kx, n0);
                }
                last = kb;
            }
            if (*abort_flag)
                for (int kb = max(0, last - kD_Stages + 1); kb <= last; ++kb)
                    d_drain(&S.full[kb % kD_Stages], (kb / kD_Stages) & 1, err);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // bit 16: B transposed (MN-major)
            const uint32_t idesc = idesc_bf16(kD_BM, kD_BN) | (B_MN ? (1u << 16) : 0u);
            for (int kb = 0; kb < nk; ++kb) {
                const int st = kb % kD_Stages;
                if (!mbar_wait(&S.full[st], (kb / kD_Stages) & 1, abort_flag, err)) break;
                tc_fence_after();
                const uint32_t a_s = smem_u32(sb + (size_t)st * 2 * kD_TileBytes);
                const uint32_t b_s = a_s + kD_TileBytes;
#pragma unroll
                for (int kk = 0; kk < kD_BK / 16; ++kk)
                    mma_ss(tbase, smem_desc_sw128(a_s + kk * 32),
                           B_MN ? d_desc_mn_sw128(b_s + kk * 2048) : smem_desc_sw128(b_s + kk * 32), idesc,
                           (kb | kk) != 0);
                mma_commit(&S.empty[st]);
            }
            mma_commit(&S.acc);
        }
    } else {
        // epilogue warps 2..5: warp w reads TMEM lanes 32*(w%4)
        const int q = warp & 3;
        const int row = m0 + q * 32 + lane;
        d_drain(&S.acc, 0, err);
        tc_fence_after();
        float *dst = part + (int64_t)blockIdx.z * split_stride + (int64_t)row * ldp + n0;
        for (int c0 = 0; c0 < kD_BN; c0 += 32) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tbase + ((uint32_t)(q * 32) << 16) + c0, v);
            tmem_wait_ld();
            if (nk > 0 && row < m_valid) {
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4 *>(dst + c0 + i) =
                        make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                    __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
            } else if (row < m_valid) {
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                    *reinterpret_cast<float4 *>(dst + c0 + i) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tbase, 128);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 d_encode() {
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

// bf16 matrix of `rows` x `cols` valid elements, row stride `ld` elements;
// boxes of `box_rows` rows x 64 columns; reads past rows/cols are zero-filled by TMA
bool d_tmap(CUtensorMap *m, const void *ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows = kD_BM) {
    auto fn = d_encode();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 2) % 16 || cols > ld) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
    cuuint32_t box[2] = {(cuuint32_t)kD_BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// B operand tensor map: K-major B [b_rows = N, b_cols = K], or MN-major
// B [b_rows = K, b_cols = N] (boxes of 64 K rows x 64 N columns)
bool d_tmap_b(CUtensorMap *m, const void *ptr, int64_t rows, int64_t cols, int64_t ld, bool b_mn) {
    return b_mn ? d_tmap(m, ptr, rows, cols, ld, 64) : d_tmap(m, ptr, rows, cols, ld);
}

template <bool B_MN>
bool d_attr() {
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(dense_tc_kernel<B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kD_Smem) != cudaSuccess)
            return false;
        attr = true;
    }
    return true;
}

}  // namespace

// P[split][Mp][Np] partials of A * B^T over K in [0, Kp): A has a_rows x a_cols
// valid elements (row stride lda); B has b_rows x b_cols (stride ldb), K-major
// ([N, K]) or, with b_mn, MN-major ([K, N]); Mp, Np multiples of 128, Kp of 64;
// everything outside the valid extents reads as 0.
int dense_tc_partials(const __nv_bfloat16 *A, int a_rows, int a_cols, int lda,
                      const __nv_bfloat16 *B, int b_rows, int b_cols, int ldb, int Mp, int Np,
                      int Kp, int splits, float *part, int *err, cudaStream_t st, bool b_mn) {
    if (Mp % kD_BM || Np % kD_BN || Kp % kD_BK || splits < 1 || !err) return USAF_EUNSUPPORTED;
    int kps = ((Kp / kD_BK + splits - 1) / splits) * kD_BK;
    CUtensorMap ta, tb;
    if (!d_tmap(&ta, A, a_rows, a_cols, lda) || !d_tmap_b(&tb, B, b_rows, b_cols, ldb, b_mn))
        return USAF_EUNSUPPORTED;
    if (!(b_mn ? d_attr<true>() : d_attr<false>())) return USAF_ECUDA;
    dim3 grid(Np / kD_BN, Mp / kD_BM, splits);
    if (b_mn)
        dense_tc_kernel<true><<<grid, kD_Threads, kD_Smem, st>>>(ta, tb, Mp, Np, Kp, kps, part, Np,
                                                                 (int64_t)Mp * Np, Mp, err);
    else
        dense_tc_kernel<false><<<grid, kD_Threads, kD_Smem, st>>>(ta, tb, Mp, Np, Kp, kps, part, Np,
                                                                  (int64_t)Mp * Np, Mp, err);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

// out[m][n] (fp32, row stride ldo) = A * B^T for m < m_valid, n < Np, one K
// split: the product lands in its destination without a partial buffer
// (ldo >= Np, Np a multiple of 128).
int dense_tc_direct(const __nv_bfloat16 *A, int a_rows, int a_cols, int lda, const __nv_bfloat16 *B,
                    int b_rows, int b_cols, int ldb, int Mp, int Np, int Kp, float *out, int64_t ldo,
                    int m_valid, int *err, cudaStream_t st, bool b_mn) {
    if (Mp % kD_BM || Np % kD_BN || Kp % kD_BK || !err || ldo < Np) return USAF_EUNSUPPORTED;
    CUtensorMap ta, tb;
    if (!d_tmap(&ta, A, a_rows, a_cols, lda) || !d_tmap_b(&tb, B, b_rows, b_cols, ldb, b_mn))
        return USAF_EUNSUPPORTED;
    if (!(b_mn ? d_attr<true>() : d_attr<false>())) return USAF_ECUDA;
    dim3 grid(Np / kD_BN, Mp / kD_BM, 1);
    if (b_mn)
        dense_tc_kernel<true><<<grid, kD_Threads, kD_Smem, st>>>(ta, tb, Mp, Np, Kp, Kp, out, ldo, 0, m_valid, err);
    else
        dense_tc_kernel<false><<<grid, kD_Threads, kD_Smem, st>>>(ta, tb, Mp, Np, Kp, Kp, out, ldo, 0, m_valid, err);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

bool dense_tc_available() { return d_encode() != nullptr; }

}  // namespace usaf
