// Expert-weight gradients at the selected coordinates only (SDDMM), and the
// dense per-expert |gradient| used by the importance pass.
//
// The reference materialises the dense per-expert gradient dW_e = gout_e^T gin_e
// (F.linear backward, rounded to the parameter dtype), then gathers the
// active coordinates and index-adds them into compact fp32 vectors
// (usaf/qwen3moe_dml.py:43-56, usaf/moe_loader.py:564-578).  Here only the
// selected coordinates are computed: for coordinate (e, r, c)
//   g = dtype( sum over expert e's slots s of gout[s, r] * gin[s, c] )
// in a fixed slot order (deterministic), then compact[pos] += scale * g.
//
// Work item = (expert, block of 512 storage rows); each thread owns two rows
// and walks their CSR entries.  Token chunks of gin (all columns) and gout
// (the block's rows) are staged transposed in shared memory so every
// coordinate reads contiguous token runs; per-chunk partial sums go to an
// fp32 scratch vector owned one-to-one by coordinates (no atomics).
#include <atomic>
#include "common.cuh"

namespace usaf {

constexpr int kRowsPerBlock = 512;   // storage rows per work item
constexpr int kTC = 32;              // tokens per chunk
constexpr int kThr = 256;

// Stage rows [t0, t0+tn) x columns [c0, c0+ncols) of a row-major [*, ld]
// activation matrix transposed into dst[col][kTC] (token-contiguous rows of
// 64 B for bf16 / 128 B for fp32).  16-byte chunks of each row are XOR
// swizzled by the row index so the transposing stores spread over banks.
template <typename Act>
__device__ __forceinline__ void stage_transposed(const Act *__restrict__ src, int ld, int64_t row0,
                                                 int tn, int c0, int ncols, Act *dst) {
    constexpr int VEC = 16 / sizeof(Act);         // tokens per 16-byte chunk
    constexpr int NCH = kTC / VEC;                // chunks per staged row
    if (sizeof(Act) == 2) {
        // thread item: column pair (c, c+1) x VEC tokens -> two 16-byte chunks
        const int npair = (ncols + 1) / 2;
        for (int it = threadIdx.x; it < npair * NCH; it += kThr) {
            const int cp = it % npair, q = it / npair;
            const int c = 2 * cp;
            uint32_t v[VEC];
#pragma unroll
            for (int u = 0; u < VEC; ++u) {
                const int t = q * VEC + u;
                // ncols is even (checked at launch), so the pair (c, c+1) is in range
                v[u] = t < tn ? *reinterpret_cast<const uint32_t *>(src + (row0 + t) * ld + c0 + c) : 0u;
            }
            uint4 lo, hi;
            uint32_t *pl = reinterpret_cast<uint32_t *>(&lo), *ph = reinterpret_cast<uint32_t *>(&hi);
#pragma unroll
            for (int u = 0; u < VEC / 2; ++u) {
                pl[u] = __byte_perm(v[2 * u], v[2 * u + 1], 0x5410);
                ph[u] = __byte_perm(v[2 * u], v[2 * u + 1], 0x7632);
            }
            const int sw0 = q ^ ((c >> 1) & (NCH - 1));
            *reinterpret_cast<uint4 *>(dst + (size_t)c * kTC + sw0 * VEC) = lo;
            if (c + 1 < ncols) {
                const int sw1 = q ^ (((c + 1) >> 1) & (NCH - 1));
                *reinterpret_cast<uint4 *>(dst + (size_t)(c + 1) * kTC + sw1 * VEC) = hi;
            }
        }
    } else {
        for (int it = threadIdx.x; it < ncols * NCH; it += kThr) {
            const int c = it % ncols, q = it / ncols;
            float4 v;
            float *pv = reinterpret_cast<float *>(&v);
#pragma unroll
            for (int u = 0; u < VEC; ++u) {
                const int t = q * VEC + u;
                pv[u] = t < tn ? to_f(src[(row0 + t) * ld + c0 + c]) : 0.0f;
            }
            const int sw = q ^ ((c >> 1) & (NCH - 1));
            *reinterpret_cast<float4 *>(dst + (size_t)c * kTC + sw * VEC) = v;
        }
    }
}

template <typename Act>
__device__ __forceinline__ void load_staged(const Act *row_base, int c, float (&out)[kTC]) {
    constexpr int VEC = 16 / sizeof(Act);
    constexpr int NCH = kTC / VEC;
#pragma unroll
    for (int q = 0; q < NCH; ++q) {
        const int sw = q ^ ((c >> 1) & (NCH - 1));
        uint4 v = *reinterpret_cast<const uint4 *>(row_base + sw * VEC);
        const uint32_t *pv = reinterpret_cast<const uint32_t *>(&v);
        if (sizeof(Act) == 2) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                out[q * VEC + 2 * u] = __uint_as_float(pv[u] << 16);
                out[q * VEC + 2 * u + 1] = __uint_as_float(pv[u] & 0xFFFF0000u);
            }
        } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) out[q * VEC + u] = __uint_as_float(pv[u]);
        }
    }
}

// Work item = (row block of 512 storage rows, expert).  Per 32-token chunk
// the block stages gin (all C columns) and gout (its 512 columns) transposed
// in shared memory; each thread owns 2 rows and walks their CSR entries,
// dotting 32 staged tokens per entry; per-entry partial sums go to scratch
// (one owner per entry, fixed chunk order -> deterministic).
template <typename Act>
__global__ void __launch_bounds__(kThr) sddmm_kernel(usaf_route_plan pl, usaf_qweight w,
                                                     const Act *__restrict__ gout,
                                                     const Act *__restrict__ gin,
                                                     const int32_t *__restrict__ csr_to_compact,
                                                     float scale, float *__restrict__ compact,
                                                     float *__restrict__ scratch) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Act *ginT = reinterpret_cast<Act *>(smem_raw);               // [C][kTC]
    Act *goutT = ginT + (size_t)w.C * kTC;                       // [kRowsPerBlock][kTC]
    const int e = blockIdx.y;
    const int R = w.R, C = w.C;
    const int cnt = pl.expert_cnt[e];
    if (cnt == 0) return;
    const int64_t seg0 = pl.expert_off[e];
    const int rb0 = blockIdx.x * kRowsPerBlock;
    const int rows_here = min(kRowsPerBlock, R - rb0);
    int jb[2], je[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int rr = threadIdx.x + h * kThr;
        jb[h] = je[h] = 0;
        if (rr < rows_here) {
            jb[h] = w.row_ptr[((int64_t)e * R + rb0 + rr) * 2];       // both half segments
            je[h] = w.row_ptr[((int64_t)e * R + rb0 + rr) * 2 + 2];
        }
    }
    for (int t0 = 0; t0 < cnt; t0 += kTC) {
        const int tn = min(kTC, cnt - t0);
        __syncthreads();
        stage_transposed<Act>(gin, C, seg0 + t0, tn, 0, C, ginT);
        stage_transposed<Act>(gout, R, seg0 + t0, tn, rb0, rows_here, goutT);
        __syncthreads();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            if (jb[h] >= je[h]) continue;
            const int rr = threadIdx.x + h * kThr;
            float a[kTC];
            load_staged<Act>(goutT + (size_t)rr * kTC, rr, a);
            for (int j = jb[h]; j < je[h]; ++j) {
                const int c = w.col[j];
                float b[kTC];
                load_staged<Act>(ginT + (size_t)c * kTC, c, b);
                float d = 0.0f;
#pragma unroll
                for (int t = 0; t < kTC; ++t) d = fmaf(a[t], b[t], d);
                scratch[j] = t0 == 0 ? d : __fadd_rn(scratch[j], d);
            }
        }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        for (int j = jb[h]; j < je[h]; ++j) {
            const int pos = csr_to_compact ? csr_to_compact[j] : j;
            compact[pos] = __fadd_rn(compact[pos], __fmul_rn(scale, round_to<Act>(scratch[j])));
        }
    }
}

// dense |dW_e| for the importance pass: out[e][r][c] = |dtype(sum_s gout[s,r] gin[s,c])|
template <typename Act>
__global__ void __launch_bounds__(256) dense_dw_kernel(usaf_route_plan pl, int R, int C,
                                                       const Act *__restrict__ gout,
                                                       const Act *__restrict__ gin,
                                                       float *__restrict__ out) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const int e = blockIdx.z;
    const int cnt = pl.expert_cnt[e], seg0 = pl.expert_off[e];
    const int r0 = blockIdx.y * 64, c0 = blockIdx.x * 64;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < cnt; k0 += 16) {
        for (int i = threadIdx.x; i < 16 * 64; i += 256) {
            int mm = i & 63, kk = i >> 6;
            int k = k0 + kk;
            As[kk][mm] = (k < cnt && r0 + mm < R) ? to_f(gout[(int64_t)(seg0 + k) * R + r0 + mm]) : 0.0f;
            Bs[kk][mm] = (k < cnt && c0 + mm < C) ? to_f(gin[(int64_t)(seg0 + k) * C + c0 + mm]) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            int rr = r0 + ty * 4 + i, cc = c0 + tx * 4 + j;
            if (rr < R && cc < C) out[((int64_t)e * R + rr) * C + cc] = fabsf(round_to<Act>(acc[i][j]));
        }
}

template <typename Act>
static int sddmm_launch(const usaf_route_plan *pl, const usaf_qweight *w, const Act *gout,
                        const Act *gin, const int32_t *c2c, float scale, float *compact,
                        float *scratch, cudaStream_t st) {
    const size_t bytes = ((size_t)w->C + kRowsPerBlock) * kTC * sizeof(Act);
    if (bytes > 220 * 1024 || (w->C & 1) || (w->R & 1)) return USAF_EUNSUPPORTED;
    if (cudaFuncSetAttribute(sddmm_kernel<Act>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)bytes) != cudaSuccess)
        return USAF_ECUDA;
    dim3 grid(cdiv(w->R, kRowsPerBlock), w->E);
    sddmm_kernel<Act><<<grid, kThr, bytes, st>>>(*pl, *w, gout, gin, c2c, scale, compact, scratch);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

bool sddmm_tc_supported(int R, int C);
int sddmm_tc_sparse(const usaf_route_plan *pl, const usaf_qweight *w, const __nv_bfloat16 *gout,
                    const __nv_bfloat16 *gin, const int32_t *c2c, float scale, float *compact,
                    float *scratch, cudaStream_t st);
int sddmm_tc_dense_abs(const usaf_route_plan *pl, int R, int C, const __nv_bfloat16 *gout,
                       const __nv_bfloat16 *gin, float *out, cudaStream_t st);

}  // namespace usaf

using namespace usaf;

extern "C" int usaf_sparse_dw(const usaf_route_plan *plan, const usaf_qweight *w, const void *gout,
                              const void *gin, int32_t dtype, const int32_t *csr_to_compact,
                              float scale, float *compact, float *scratch, void *stream) {
    USAF_REQUIRE(plan && w && gout && gin && plan->E == w->E);
    if (w->n_ov == 0) return USAF_OK;
    USAF_REQUIRE(compact && scratch && w->row_ptr && w->col);
    cudaStream_t st = as_stream(stream);
    const bool tc = dtype == USAF_BF16 && w->ov_mask && w->ov_cbptr && sddmm_tc_supported(w->R, w->C);
    if (tc && !small_plan(plan))
        return sddmm_tc_sparse(plan, w, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin,
                               csr_to_compact, scale, compact, scratch, st);
    switch (dtype) {
        case USAF_F32: return sddmm_launch<float>(plan, w, (const float *)gout, (const float *)gin, csr_to_compact, scale, compact, scratch, st);
        case USAF_BF16: {
            // a few slots per expert: the CUDA-core kernel, which skips experts without
            // slots (it stages all C columns, so wide projections stay on tensor cores)
            const int rc = sddmm_launch<__nv_bfloat16>(plan, w, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin, csr_to_compact, scale, compact, scratch, st);
            if (rc == USAF_EUNSUPPORTED && tc)
                return sddmm_tc_sparse(plan, w, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin,
                                       csr_to_compact, scale, compact, scratch, st);
            return rc;
        }
        default: return USAF_EINVAL;
    }
}

extern "C" int usaf_expert_dense_dw(const usaf_route_plan *plan, int32_t R, int32_t C,
                                    const void *gout, const void *gin, int32_t dtype, float *out,
                                    void *stream) {
    USAF_REQUIRE(plan && gout && gin && out && R >= 1 && C >= 1);
    cudaStream_t st = as_stream(stream);
    if (dtype == USAF_BF16 && sddmm_tc_supported(R, C))
        return sddmm_tc_dense_abs(plan, R, C, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin, out, st);
    dim3 grid(cdiv(C, 64), cdiv(R, 64), plan->E);
    switch (dtype) {
        case USAF_F32: dense_dw_kernel<float><<<grid, 256, 0, st>>>(*plan, R, C, (const float *)gout, (const float *)gin, out); break;
        case USAF_BF16: dense_dw_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(*plan, R, C, (const __nv_bfloat16 *)gout, (const __nv_bfloat16 *)gin, out); break;
        default: return USAF_EINVAL;
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

// ---- allocation-free variant -------------------------------------------------
// usaf_sparse_dw needs an fp32 scratch vector with one slot per selected
// coordinate.  Some callers cannot allocate device memory when they call in:
// code that runs inside a fixed, pre-reserved memory budget (a serving process
// whose pool is carved up at start-up), or a foreign-language host that only
// hands over buffers it registered earlier and has no binding for cudaMalloc.
// usaf_sparse_dw_noalloc serves them with a scratch array that lives in this
// library's own device memory: a file-scope __device__ array of
// kNoAllocScratchFloats floats (8 MiB), resident on every GPU that loads the
// library until the process exits.
namespace usaf {
constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 21;  // 2,097,152 coordinates
}  // namespace usaf

static __device__ __align__(256) float g_sddmm_noalloc_scratch[usaf::kNoAllocScratchFloats];

// Device address of the scratch array on the current device.  The host-side
// symbol is only a stand-in, so the address is looked up once per device
// (with that device current) and cached.  The cache entries are atomics:
// host threads that make their first call on a device at the same time may
// each look the address up, and they all store the same value.  The cache is
// not refreshed after cudaDeviceReset (the library's module, and with it the
// array, is loaded again at a possibly different address): a process that
// resets a device must not call this entry point on it afterwards.
static float *noalloc_scratch_ptr(int *status) {
    constexpr int kMaxDevices = 64;
    static std::atomic<float *> addr[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *status = USAF_ECUDA;
        return nullptr;
    }
    float *cached = addr[dev].load(std::memory_order_acquire);
    if (!cached) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_sddmm_noalloc_scratch) != cudaSuccess || !p) {
            (void)cudaGetLastError();
            *status = USAF_ECUDA;
            return nullptr;
        }
        cached = static_cast<float *>(p);
        addr[dev].store(cached, std::memory_order_release);
    }
    *status = USAF_OK;
    return cached;
}

extern "C" int usaf_sparse_dw_noalloc(const usaf_route_plan *plan, const usaf_qweight *w,
                                      const void *gout, const void *gin, int32_t dtype,
                                      const int32_t *csr_to_compact, float scale, float *compact,
                                      void *stream) {
    USAF_REQUIRE(plan && w);
    if (w->n_ov > usaf::kNoAllocScratchFloats) return USAF_EUNSUPPORTED;  // beyond the built-in scratch
    int rc = USAF_OK;
    float *scratch = noalloc_scratch_ptr(&rc);
    if (rc != USAF_OK) return rc;
    // every slot the kernel reads is written first (first token chunk stores,
    // later chunks add), so the previous call's contents need no clearing
    return usaf_sparse_dw(plan, w, gout, gin, dtype, csr_to_compact, scale, compact, scratch, stream);
}
