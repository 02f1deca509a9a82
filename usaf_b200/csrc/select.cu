// Top-k selection for the importance / RigL path.
//
// Replaces torch.topk in TopKImportanceStore.add/select
// (usaf/moe_loader.py:607-609, 626) and the np.partition threshold of the
// selectors (usaf/selector.py:6-14).  fp32 scores map to order-preserving
// uint32 keys; an MSB-first radix select (4 passes of 8 bits, block-local
// shared-memory histograms folded into 256 global counters) finds the exact
// k-th largest key; a stable compaction keeps every key above it plus the
// lowest-index elements equal to it; a stable LSD radix sort orders the
// result by descending value (ties in ascending index order).
// All passes are HBM streaming passes over the scores.
#include "common.cuh"

namespace usaf {

__device__ __forceinline__ uint32_t f2key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(u);
}

struct SelState {
    uint32_t prefix, mask;
    long long k_rem;
};

constexpr int kTile = 4096;  // elements per block in compaction / sort passes

struct ScratchLayout {
    size_t state, hist, blk, sort_keys, sort_vals, sort_cnt, scan_part, total;
};

static ScratchLayout layout_for(int64_t n, int64_t k) {
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    ScratchLayout L;
    size_t off = 0;
    int64_t nb = (n + kTile - 1) / kTile;
    int64_t nbk = (k + kTile - 1) / kTile;
    L.state = off; off += al(sizeof(SelState));
    L.hist = off; off += al(256 * sizeof(unsigned long long));
    L.blk = off; off += al((size_t)(nb + 1) * 4 * sizeof(long long));
    L.sort_keys = off; off += al((size_t)k * 2 * sizeof(uint32_t));
    L.sort_vals = off; off += al((size_t)k * 2 * sizeof(int64_t));
    L.sort_cnt = off; off += al((size_t)256 * (nbk + 1) * sizeof(int));
    L.scan_part = off; off += al((size_t)((256 * (nbk + 1)) / 4096 + 2) * sizeof(int));
    L.total = off;
    return L;
}

__global__ void sel_init(SelState *st, unsigned long long *hist, long long k) {
    if (threadIdx.x == 0) { st->prefix = 0; st->mask = 0; st->k_rem = k; }
    hist[threadIdx.x] = 0;
}

__global__ void __launch_bounds__(256) sel_hist(const float *__restrict__ v, int64_t n,
                                                const SelState *__restrict__ st,
                                                unsigned long long *__restrict__ hist, int shift) {
    __shared__ unsigned int h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    uint32_t prefix = st->prefix, mask = st->mask;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        uint32_t key = f2key(v[i]);
        if ((key & mask) == prefix) atomicAdd(&h[(key >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (h[threadIdx.x]) atomicAdd(&hist[threadIdx.x], (unsigned long long)h[threadIdx.x]);
}

// pick the bucket holding the k_rem-th largest among the prefix-matching keys
__global__ void sel_pick(SelState *st, unsigned long long *hist, int shift) {
    __shared__ unsigned long long suf[257];
    int d = threadIdx.x;
    unsigned long long c = hist[d];
    suf[d] = c;
    if (d == 0) suf[256] = 0;
    __syncthreads();
    if (d == 0) {
        for (int b = 254; b >= 0; --b) suf[b] += suf[b + 1];
        long long kr = st->k_rem;
        int bucket = 0;
        for (int b = 255; b >= 0; --b) {
            if ((long long)suf[b] >= kr) { bucket = b; break; }
        }
        st->k_rem = kr - (long long)suf[bucket + 1];
        st->prefix |= (uint32_t)bucket << shift;
        st->mask |= 0xFFu << shift;
    }
    __syncthreads();
    hist[d] = 0;
}

__global__ void write_kth(const SelState *st, float *out) { *out = key2f(st->prefix); }

// ---- stable compaction: keys > thr, then the first k_rem keys == thr ----
__global__ void __launch_bounds__(256) cmp_count(const float *__restrict__ v, int64_t n,
                                                 const SelState *__restrict__ st,
                                                 long long *__restrict__ blk) {
    __shared__ int sg[8], se[8];
    uint32_t thr = st->prefix;
    int64_t base = (int64_t)blockIdx.x * kTile;
    int gt = 0, eq = 0;
    for (int i = threadIdx.x; i < kTile; i += 256) {
        int64_t j = base + i;
        if (j < n) {
            uint32_t key = f2key(v[j]);
            gt += key > thr;
            eq += key == thr;
        }
    }
    for (int o = 16; o; o >>= 1) {
        gt += __shfl_xor_sync(0xffffffffu, gt, o);
        eq += __shfl_xor_sync(0xffffffffu, eq, o);
    }
    if ((threadIdx.x & 31) == 0) { sg[threadIdx.x >> 5] = gt; se[threadIdx.x >> 5] = eq; }
    __syncthreads();
    if (threadIdx.x == 0) {
        long long a = 0, b = 0;
        for (int w = 0; w < 8; ++w) { a += sg[w]; b += se[w]; }
        blk[2 * blockIdx.x] = a;
        blk[2 * blockIdx.x + 1] = b;
    }
}

__global__ void cmp_scan(long long *blk, int64_t nb) {
    // exclusive scans in place; blk[2*nb], blk[2*nb+1] = totals
    if (threadIdx.x == 0) {
        long long a = 0, b = 0;
        for (int64_t i = 0; i < nb; ++i) {
            long long x = blk[2 * i], y = blk[2 * i + 1];
            blk[2 * i] = a;
            blk[2 * i + 1] = b;
            a += x;
            b += y;
        }
        blk[2 * nb] = a;
        blk[2 * nb + 1] = b;
    }
}

__device__ __forceinline__ int block_scan_excl_256(int v, int *warp_tot) {
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[wid] = x;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < wid; ++w) before += warp_tot[w];
    __syncthreads();
    return before + x - v;
}

// per thread: 16 consecutive elements of the block's tile
__global__ void __launch_bounds__(256) cmp_write(const float *__restrict__ v, int64_t n,
                                                 const SelState *__restrict__ st,
                                                 const long long *__restrict__ blk, int64_t nb,
                                                 uint32_t *__restrict__ okey,
                                                 int64_t *__restrict__ opos) {
    __shared__ int wt[8];
    uint32_t thr = st->prefix;
    long long k_rem = st->k_rem;
    long long total_gt = blk[2 * nb];
    int64_t start = (int64_t)blockIdx.x * kTile + threadIdx.x * 16;
    int gt = 0, eq = 0;
    uint32_t keys[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        int64_t j = start + i;
        keys[i] = j < n ? f2key(v[j]) : 0u;
        bool valid = j < n;
        gt += valid && keys[i] > thr;
        eq += valid && keys[i] == thr;
    }
    int gt_off = block_scan_excl_256(gt, wt);
    int eq_off = block_scan_excl_256(eq, wt);
    long long g = blk[2 * blockIdx.x] + gt_off;
    long long q = blk[2 * blockIdx.x + 1] + eq_off;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        int64_t j = start + i;
        if (j >= n) break;
        if (keys[i] > thr) {
            okey[g] = keys[i];
            opos[g] = j;
            ++g;
        } else if (keys[i] == thr) {
            if (q < k_rem) {
                okey[total_gt + q] = keys[i];
                opos[total_gt + q] = j;
            }
            ++q;
        }
    }
}

// ---- stable LSD radix sort by descending key (sorts ~key ascending) ----
__global__ void __launch_bounds__(256) sort_hist(const uint32_t *__restrict__ keys, int64_t n,
                                                 int shift, int *__restrict__ cnt, int64_t nb,
                                                 uint32_t flip) {
    __shared__ int h[256];
    h[threadIdx.x] = 0;
    __syncthreads();
    int64_t base = (int64_t)blockIdx.x * kTile;
    for (int i = threadIdx.x; i < kTile; i += 256) {
        int64_t j = base + i;
        if (j < n) atomicAdd(&h[((keys[j] ^ flip) >> shift) & 0xFF], 1);
    }
    __syncthreads();
    cnt[(int64_t)threadIdx.x * nb + blockIdx.x] = h[threadIdx.x];
}

__global__ void __launch_bounds__(1024) sort_scan(int *cnt, int64_t total) {
    __shared__ int wt[32];
    int carry = 0;
    for (int64_t b0 = 0; b0 < total; b0 += 1024) {
        int64_t i = b0 + threadIdx.x;
        int v = i < total ? cnt[i] : 0;
        int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
        int x = v;
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wt[wid] = x;
        __syncthreads();
        if (wid == 0) {
            int s = wt[lane];
            for (int o = 1; o < 32; o <<= 1) {
                int y = __shfl_up_sync(0xffffffffu, s, o);
                if (lane >= o) s += y;
            }
            wt[lane] = s;
        }
        __syncthreads();
        int before = wid ? wt[wid - 1] : 0;
        if (i < total) cnt[i] = carry + before + x - v;
        int tot = wt[31];
        __syncthreads();
        carry += tot;
    }
}

// Exclusive scan of the digit counts [256][nb] for large sorts: chunk sums,
// a one-block scan of those, then each chunk scanned from its offset (a single
// block walking 256 * nb counts took most of a multi-million-key sort).
constexpr int kScanChunk = 4096;   // counts per block (4 per thread)

__device__ __forceinline__ int block_excl_scan_1024(int v, int *wt, int &total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wt[wid] = x;
    __syncthreads();
    if (wid == 0) {
        int t = wt[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        wt[lane] = t;
    }
    __syncthreads();
    total = wt[31];
    return (wid ? wt[wid - 1] : 0) + x - v;
}

__global__ void __launch_bounds__(1024) scan_chunk_sum(const int *__restrict__ cnt, int64_t total,
                                                       int *__restrict__ part) {
    __shared__ int wt[32];
    const int64_t i0 = (int64_t)blockIdx.x * kScanChunk + threadIdx.x * 4;
    int v = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) v += i0 + j < total ? cnt[i0 + j] : 0;
    int tot;
    block_excl_scan_1024(v, wt, tot);
    if (threadIdx.x == 0) part[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(1024) scan_chunk_apply(int *cnt, int64_t total, const int *__restrict__ part) {
    __shared__ int wt[32];
    const int64_t i0 = (int64_t)blockIdx.x * kScanChunk + threadIdx.x * 4;
    int c[4], v = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        c[j] = i0 + j < total ? cnt[i0 + j] : 0;
        v += c[j];
    }
    int tot;
    int run = block_excl_scan_1024(v, wt, tot) + part[blockIdx.x];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        if (i0 + j < total) cnt[i0 + j] = run;
        run += c[j];
    }
}


static void scan_counts(int *cnt, int64_t total, int *part, cudaStream_t st) {
    if (total <= kScanChunk) {
        sort_scan<<<1, 1024, 0, st>>>(cnt, total);
        return;
    }
    const unsigned nch = (unsigned)((total + kScanChunk - 1) / kScanChunk);
    scan_chunk_sum<<<nch, 1024, 0, st>>>(cnt, total, part);
    sort_scan<<<1, 1024, 0, st>>>(part, nch);
    scan_chunk_apply<<<nch, 1024, 0, st>>>(cnt, total, part);
}

__global__ void __launch_bounds__(256) sort_scatter(const uint32_t *__restrict__ kin,
                                                    const int64_t *__restrict__ vin, int64_t n,
                                                    int shift, const int *__restrict__ cnt,
                                                    int64_t nb, uint32_t *__restrict__ kout,
                                                    int64_t *__restrict__ vout, uint32_t flip) {
    __shared__ int warp_hist[8][256];
    __shared__ int run[256];
    int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    run[threadIdx.x] = cnt[(int64_t)threadIdx.x * nb + blockIdx.x];
    for (int w = 0; w < 8; ++w) warp_hist[w][threadIdx.x] = 0;
    __syncthreads();
    int64_t base = (int64_t)blockIdx.x * kTile;
    for (int r = 0; r < kTile / 256; ++r) {
        int64_t j = base + r * 256 + threadIdx.x;
        bool valid = j < n;
        uint32_t key = valid ? kin[j] : 0u;
        int d = valid ? (int)(((key ^ flip) >> shift) & 0xFF) : 256 + lane;  // invalid lanes never match
        unsigned peers = __match_any_sync(0xffffffffu, d);
        int rank = __popc(peers & ((1u << lane) - 1));
        if (valid && rank == 0) warp_hist[wid][d] = __popc(peers);
        __syncthreads();
        {
            int dd = threadIdx.x;
            int acc = run[dd];
            for (int w = 0; w < 8; ++w) {
                int c = warp_hist[w][dd];
                warp_hist[w][dd] = acc;
                acc += c;
            }
            run[dd] = acc;
        }
        __syncthreads();
        if (valid) {
            int pos = warp_hist[wid][d] + rank;
            kout[pos] = key;
            vout[pos] = vin[j];
        }
        __syncthreads();
        for (int w = 0; w < 8; ++w) warp_hist[w][threadIdx.x] = 0;
        __syncthreads();
    }
}

__global__ void finalize_topk(const uint32_t *__restrict__ keys, const int64_t *__restrict__ pos,
                              int64_t k, const int64_t *__restrict__ idx_map, int64_t idx_base,
                              float *__restrict__ ov, int64_t *__restrict__ oi) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < k;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (ov) ov[i] = key2f(keys[i]);
        int64_t p = pos[i];
        oi[i] = idx_map ? idx_map[p] : idx_base + p;
    }
}

static int radix_select(const float *v, int64_t n, int64_t k, char *scratch, const ScratchLayout &L,
                        cudaStream_t st) {
    SelState *state = reinterpret_cast<SelState *>(scratch + L.state);
    auto *hist = reinterpret_cast<unsigned long long *>(scratch + L.hist);
    sel_init<<<1, 256, 0, st>>>(state, hist, (long long)k);
    unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 8);
    for (int pass = 0; pass < 4; ++pass) {
        int shift = 24 - 8 * pass;
        sel_hist<<<grid, 256, 0, st>>>(v, n, state, hist, shift);
        sel_pick<<<1, 256, 0, st>>>(state, hist, shift);
    }
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

}  // namespace usaf

using namespace usaf;

extern "C" int64_t usaf_topk_scratch_bytes(int64_t n, int64_t k) {
    if (n < 0 || k < 0) return -1;
    return (int64_t)layout_for(n, k).total;
}

extern "C" int usaf_kth_largest(const float *vals, int64_t n, int64_t k, float *out, void *scratch,
                                void *stream) {
    USAF_REQUIRE(vals && out && scratch && n >= 1 && k >= 1 && k <= n);
    ScratchLayout L = layout_for(n, 1);
    cudaStream_t st = as_stream(stream);
    int rc = radix_select(vals, n, k, (char *)scratch, L, st);
    if (rc) return rc;
    write_kth<<<1, 1, 0, st>>>(reinterpret_cast<SelState *>((char *)scratch + L.state), out);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int usaf_topk_desc(const float *vals, int64_t n, int64_t k, const int64_t *idx_map,
                              int64_t idx_base, float *out_vals, int64_t *out_idx, void *scratch,
                              void *stream) {
    USAF_REQUIRE(vals && out_idx && scratch && n >= 1 && k >= 1 && k <= n);
    USAF_REQUIRE(n < (1ll << 31));
    ScratchLayout L = layout_for(n, k);
    char *sc = (char *)scratch;
    cudaStream_t st = as_stream(stream);
    int rc = radix_select(vals, n, k, sc, L, st);
    if (rc) return rc;
    SelState *state = reinterpret_cast<SelState *>(sc + L.state);
    auto *blk = reinterpret_cast<long long *>(sc + L.blk);
    auto *k0 = reinterpret_cast<uint32_t *>(sc + L.sort_keys);
    auto *k1 = k0 + k;
    auto *p0 = reinterpret_cast<int64_t *>(sc + L.sort_vals);
    auto *p1 = p0 + k;
    int64_t nb = (n + kTile - 1) / kTile;
    cmp_count<<<(unsigned)nb, 256, 0, st>>>(vals, n, state, blk);
    cmp_scan<<<1, 32, 0, st>>>(blk, nb);
    cmp_write<<<(unsigned)nb, 256, 0, st>>>(vals, n, state, blk, nb, k0, p0);
    // stable LSD sort of the k survivors by descending key
    int64_t nbk = (k + kTile - 1) / kTile;
    int *cnt = reinterpret_cast<int *>(sc + L.sort_cnt);
    for (int pass = 0; pass < 4; ++pass) {
        int shift = 8 * pass;
        sort_hist<<<(unsigned)nbk, 256, 0, st>>>(k0, k, shift, cnt, nbk, 0xFFFFFFFFu);
        scan_counts(cnt, 256 * nbk, reinterpret_cast<int *>(sc + L.scan_part), st);
        sort_scatter<<<(unsigned)nbk, 256, 0, st>>>(k0, p0, k, shift, cnt, nbk, k1, p1, 0xFFFFFFFFu);
        std::swap(k0, k1);
        std::swap(p0, p1);
    }
    unsigned grid = (unsigned)std::min<int64_t>((k + 255) / 256, 148 * 8);
    finalize_topk<<<grid, 256, 0, st>>>(k0, p0, k, idx_map, idx_base, out_vals, out_idx);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}

extern "C" int64_t usaf_sort_scratch_bytes(int64_t n) {
    if (n < 0) return -1;
    int64_t nb = (n + kTile - 1) / kTile;
    size_t b = ((size_t)n * 2 * (sizeof(uint32_t) + sizeof(int64_t))) + (size_t)256 * (nb + 1) * sizeof(int) + 1024 +
               (size_t)((256 * (nb + 1)) / 4096 + 2) * sizeof(int);
    return (int64_t)b;
}

// Stable LSD radix sort of (uint32 key, int64 payload) pairs, ascending or
// descending by key; equal keys keep their input order.
extern "C" int usaf_sort_u32(const uint32_t *keys_in, const int64_t *vals_in, int64_t n,
                             uint32_t *keys_out, int64_t *vals_out, int32_t descending,
                             void *scratch, void *stream) {
    USAF_REQUIRE(n >= 0 && n < (1ll << 31));
    if (n == 0) return USAF_OK;
    USAF_REQUIRE(keys_in && vals_in && keys_out && vals_out && scratch);
    cudaStream_t st = as_stream(stream);
    char *sc = (char *)scratch;
    uint32_t *k0 = reinterpret_cast<uint32_t *>(sc);
    uint32_t *k1 = k0 + n;
    int64_t *p0 = reinterpret_cast<int64_t *>(sc + (((size_t)n * 2 * sizeof(uint32_t) + 255) & ~(size_t)255));
    int64_t *p1 = p0 + n;
    int *cnt = reinterpret_cast<int *>(p1 + n);
    int64_t nb = (n + kTile - 1) / kTile;
    int *part = cnt + 256 * (nb + 1);
    cudaMemcpyAsync(k0, keys_in, n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(p0, vals_in, n * sizeof(int64_t), cudaMemcpyDeviceToDevice, st);
    uint32_t flip = descending ? 0xFFFFFFFFu : 0u;
    for (int pass = 0; pass < 4; ++pass) {
        int shift = 8 * pass;
        sort_hist<<<(unsigned)nb, 256, 0, st>>>(k0, n, shift, cnt, nb, flip);
        scan_counts(cnt, 256 * nb, part, st);
        sort_scatter<<<(unsigned)nb, 256, 0, st>>>(k0, p0, n, shift, cnt, nb, k1, p1, flip);
        std::swap(k0, k1);
        std::swap(p0, p1);
    }
    cudaMemcpyAsync(keys_out, k0, n * sizeof(uint32_t), cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(vals_out, p0, n * sizeof(int64_t), cudaMemcpyDeviceToDevice, st);
    USAF_CHECK_LAUNCH();
    return USAF_OK;
}
