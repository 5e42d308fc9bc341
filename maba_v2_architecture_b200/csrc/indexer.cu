// DG-Indexer: block pooling (centroids), HCA mean pooling, and fused
// scoring + top-k block selection.
//
// Centroids follow maba_sparse/kernels/common.py:329-350 and
// cpu_indexer.py:16-50: c = 0.5*(sum/block + max) over 64-token blocks, the
// tail block zero-padded (so the mean divides by the full block and the max
// includes 0).
//
// Scoring follows cpu_indexer.py:54-112 (the dispatched CPU path: fp32
// upcast, log1p penalty) and, with decode != 0, the inline decode path of
// maba_sparse/layers/indexer.py:101-112:
//   s[t,n] = sum_d (q[t,d]*scale) * c[n,d]  -  lambda*log1p(qb(t)-n)
// The dot is one sequential fused-multiply-add chain over d (d = 0,1,...),
// the penalty is fl32(fl32(lambda) * fl32(log1p(delta))) from a table
// computed once per call; both rules are mirrored by the CPU oracle so the
// selected indices agree bit for bit.  The score matrix is never
// materialised: each CTA keeps a running top-k per query token in registers
// (one entry per lane, warp bitonic sort + merge) and scans candidate blocks
// from the nearest (largest penalty-free) down, so after the first tile most
// candidates fail the k-th-best threshold and are rejected by one ballot.
#include "common.cuh"

#include <climits>
#include <cmath>

namespace maba {
namespace {

// ---------------------------------------------------------------------------
// pooling
// ---------------------------------------------------------------------------
struct PoolArgs {
    const void* in; void* out;
    int64_t si[3], so[3];
    int64_t L, nblk;
    int D, block;
    int mode;  // 0: centroid 0.5*(mean+max) with zero-padded tail; 1: mean of complete blocks
};

template <typename TI, typename TO, typename ACC>
__global__ void pool_kernel(PoolArgs a) {
    const int64_t n = blockIdx.x;
    const int64_t bi = blockIdx.y;
    const TI* in = static_cast<const TI*>(a.in);
    TO* out = static_cast<TO*>(a.out);
    const int64_t start = n * a.block;
    int64_t end = start + a.block;
    const bool padded = end > a.L;
    if (padded) end = a.L;
    for (int d = threadIdx.x; d < a.D; d += blockDim.x) {
        const TI* p = in + bi * a.si[0] + d * a.si[2];
        ACC sum = ACC(0);
        ACC mx = padded ? ACC(0) : -INFINITY;
        for (int64_t t = start; t < end; ++t) {
            ACC x = load_as<ACC>(p + t * a.si[1]);
            sum += x;
            mx = x > mx ? x : mx;
        }
        ACC mean = sum / ACC(a.block);
        ACC r = a.mode == 0 ? ACC(0.5) * (mean + mx) : mean;
        store_from<TO, ACC>(out + bi * a.so[0] + n * a.so[1] + d * a.so[2], r);
    }
}

// Vectorised form for unit-stride, 16-byte aligned rows of 16- or 32-bit values:
// one thread per (block, 16-byte column group), the block's rows loaded 16 at a
// time (all in flight together) and added in row order, t = start, start + 1, ...
// -- the same fp32 sequence per column as pool_kernel, so the results are identical.
template <typename TI, typename TO>
__global__ void __launch_bounds__(64) pool_vec_kernel(PoolArgs a) {
    constexpr int VEC = 16 / sizeof(TI);
    constexpr int ROWS = 16;
    const int ng = a.D / VEC;
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t bi = blockIdx.y;
    if (g >= a.nblk * ng) return;
    const int64_t n = g / ng;
    const int c0 = (int)(g - n * ng) * VEC;
    const int64_t start = n * a.block;
    int64_t end = start + a.block;
    const bool padded = end > a.L;
    if (padded) end = a.L;
    const TI* p = static_cast<const TI*>(a.in) + bi * a.si[0] + c0;
    float sum[VEC], mx[VEC];
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
        sum[v] = 0.f;
        mx[v] = padded ? 0.f : -INFINITY;
    }
    for (int64_t t = start; t < end; t += ROWS) {
        uint4 buf[ROWS];
#pragma unroll
        for (int i = 0; i < ROWS; ++i)
            if (t + i < end) buf[i] = *reinterpret_cast<const uint4*>(p + (t + i) * a.si[1]);
#pragma unroll
        for (int i = 0; i < ROWS; ++i)
            if (t + i < end) {
                const TI* x = reinterpret_cast<const TI*>(&buf[i]);
#pragma unroll
                for (int v = 0; v < VEC; ++v) {
                    const float xv = Cvt<TI>::to_f(x[v]);
                    sum[v] += xv;
                    mx[v] = xv > mx[v] ? xv : mx[v];
                }
            }
    }
    TO* out = static_cast<TO*>(a.out) + bi * a.so[0] + n * a.so[1];
#pragma unroll
    for (int v = 0; v < VEC; ++v) {
        const float mean = sum[v] / float(a.block);
        const float r = a.mode == 0 ? 0.5f * (mean + mx[v]) : mean;
        store_from<TO, float>(out + (int64_t)(c0 + v) * a.so[2], r);
    }
}

template <typename TI, typename TO>
int launch_pool(PoolArgs& a, int64_t B, cudaStream_t s, const char* what) {
    using ACC = typename std::conditional<sizeof(TI) == 8, double, float>::type;
    if (a.nblk == 0 || B == 0) return MABA_OK;
    if constexpr (sizeof(TI) != 8) {
        constexpr int VEC = 16 / sizeof(TI);
        const bool vec = a.si[2] == 1 && a.D % VEC == 0 && a.si[1] % VEC == 0 && a.si[0] % VEC == 0 &&
                         (reinterpret_cast<uintptr_t>(a.in) & 15) == 0;
        if (vec) {
            const int64_t n = a.nblk * (a.D / VEC);
            pool_vec_kernel<TI, TO><<<dim3((unsigned)ceil_div(n, (int64_t)64), (unsigned)B), 64, 0, s>>>(a);
            return check_launch(what);
        }
    }
    dim3 grid((unsigned)a.nblk, (unsigned)B);
    int threads = a.D >= 128 ? 128 : (a.D >= 64 ? 64 : 32);
    pool_kernel<TI, TO, ACC><<<grid, threads, 0, s>>>(a);
    return check_launch(what);
}

// ---------------------------------------------------------------------------
// top-k helpers
// ---------------------------------------------------------------------------
constexpr unsigned kFull = 0xffffffffu;

template <typename SC>
__device__ __forceinline__ bool better(SC sa, int ia, SC sb, int ib) {
    return sa > sb || (sa == sb && ia < ib);
}

// compare-exchange with the partner lane (lane ^ j); keep_better selects
// which of the two elements this lane retains.
template <typename SC>
__device__ __forceinline__ void cmpx(SC& s, int& i, int j, bool keep_better) {
    SC os = __shfl_xor_sync(kFull, s, j);
    int oi = __shfl_xor_sync(kFull, i, j);
    bool ob = better(os, oi, s, i);
    if (keep_better == ob) {
        s = os;
        i = oi;
    }
}

// bitonic sort of one element per lane into descending order (lane 0 best)
template <typename SC>
__device__ __forceinline__ void warp_sort_desc(SC& s, int& i, int lane) {
#pragma unroll
    for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
        for (int j = k >> 1; j > 0; j >>= 1) {
            const bool desc = (lane & k) == 0;
            const bool lower = (lane & j) == 0;
            cmpx(s, i, j, lower == desc);
        }
    }
}

// list (ls,li) and batch (ns,ni) both sorted descending; leaves the best 32
// of their union in (ls,li), sorted descending.
template <typename SC>
__device__ __forceinline__ void warp_merge(SC& ls, int& li, SC ns, int ni, int lane) {
    SC rs = __shfl_sync(kFull, ns, 31 - lane);
    int ri = __shfl_sync(kFull, ni, 31 - lane);
    if (better(rs, ri, ls, li)) {
        ls = rs;
        li = ri;
    }
#pragma unroll
    for (int j = 16; j > 0; j >>= 1) cmpx(ls, li, j, (lane & j) == 0);
}

// Offer one candidate per lane to the running list; invalid candidates must
// carry the sentinel (-inf, INT_MAX).
template <typename SC>
__device__ __forceinline__ void warp_offer(SC& ls, int& li, SC cs, int ci, int keff, int lane) {
    SC ts = __shfl_sync(kFull, ls, keff - 1);
    int ti = __shfl_sync(kFull, li, keff - 1);
    bool q = better(cs, ci, ts, ti);
    if (__ballot_sync(kFull, q) == 0u) return;
    if (!q) {
        cs = -INFINITY;
        ci = INT_MAX;
    }
    warp_sort_desc(cs, ci, lane);
    // into an empty list (all sentinels) the sorted batch is the merge result
    if (__shfl_sync(kFull, li, 0) == INT_MAX && __shfl_sync(kFull, ls, 0) == -INFINITY) {
        ls = cs;
        li = ci;
        return;
    }
    warp_merge(ls, li, cs, ci, lane);
}

template <typename SC> __device__ __forceinline__ SC fma_sc(SC a, SC b, SC c);
template <> __device__ __forceinline__ float fma_sc<float>(float a, float b, float c) { return fmaf(a, b, c); }
template <> __device__ __forceinline__ double fma_sc<double>(double a, double b, double c) { return fma(a, b, c); }

struct TopkArgs {
    const void* q; const void* c;
    int64_t* idx; void* scores;
    const float* pen;  // penalty table, pen[delta]
    int64_t sq[3], sc[3], si[3], ss[3];
    int64_t L, nb;
    int64_t q_pos0;  // absolute position of query row 0 (prefill)
    const int64_t* pos_dev;  // decode at a device-held position: nb = *pos_dev / block + 1 (<= nb)
    const float* cpref;      // [B][ntiles] prefix max of centroid norms over 64-block tiles (pruning), or null
    int64_t ntiles;
    int vecload;             // q and centroids: unit stride on d, 16-byte aligned rows (16-bit types)
    int D, block, keff, decode;
    float lam_f;             // lambda (the vectorised decode kernel forms the penalty in place)
    float scale_f;
    double scale_d;
};

__global__ void penalty_table_kernel(float* pen, int64_t n, float lam) {
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        // fl32(lambda) * fl32(log1p(delta)), the fp32 arithmetic of cpu_indexer.py:101
        float l = (float)log1p((double)i);
        pen[i] = __fmul_rn(lam, l);
    }
}

// Max centroid norm of each 64-block tile (grid = (ntiles, B), 64 threads).
template <typename T>
__global__ void centroid_tile_norm_kernel(const T* c, int64_t sc0, int64_t sc1, int64_t sc2, int64_t nb, int D,
                                          float* tmax, int64_t ntiles) {
    __shared__ float wmax[2];
    const int64_t b = blockIdx.y, n = (int64_t)blockIdx.x * 64 + threadIdx.x;
    float ss = 0.f;
    if (n < nb)
        for (int d = 0; d < D; ++d) {
            const float x = Cvt<T>::to_f(c[b * sc0 + n * sc1 + d * sc2]);
            ss = fmaf(x, x, ss);
        }
    float m = sqrtf(ss);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) tmax[b * ntiles + blockIdx.x] = fmaxf(wmax[0], wmax[1]);
}

// pref[j] = max(tmax[0..j]) per batch row (grid = B, 256 threads, chunked scan).
__global__ void tile_prefix_max_kernel(const float* tmax, float* pref, int64_t ntiles) {
    __shared__ float part[256];
    const int64_t b = blockIdx.x;
    const int tid = threadIdx.x;
    const int64_t per = (ntiles + 255) / 256, j0 = tid * per;
    float m = 0.f;
    for (int64_t j = j0; j < j0 + per && j < ntiles; ++j) m = fmaxf(m, tmax[b * ntiles + j]);
    part[tid] = m;
    __syncthreads();
    if (tid == 0) {
        float run = 0.f;
        for (int i = 0; i < 256; ++i) {
            const float x = part[i];
            part[i] = run;  // exclusive prefix max
            run = fmaxf(run, x);
        }
    }
    __syncthreads();
    float run = part[tid];
    for (int64_t j = j0; j < j0 + per && j < ntiles; ++j) {
        run = fmaxf(run, tmax[b * ntiles + j]);
        pref[b * ntiles + j] = run;
    }
}

template <typename SC>
__device__ __forceinline__ SC scale_of(const TopkArgs& a);
template <> __device__ __forceinline__ float scale_of<float>(const TopkArgs& a) { return a.scale_f; }
template <> __device__ __forceinline__ double scale_of<double>(const TopkArgs& a) { return a.scale_d; }

__device__ __forceinline__ int64_t query_block(const TopkArgs& a, int64_t t) {
    return a.decode ? (a.nb - 1) : ((a.q_pos0 + t) / a.block);
}

template <typename T, typename SC>
__device__ __forceinline__ void store_score(const TopkArgs& a, int64_t b, int64_t t, int64_t n, SC v) {
    T* sp = static_cast<T*>(a.scores);
    store_from<T, SC>(sp + b * a.ss[0] + t * a.ss[1] + n * a.ss[2], v);
}

// Write the final list of one token: slots [0, nvalid) from the list,
// slots [nvalid, keff) with the lowest unused future block indices.
__device__ __forceinline__ void write_topk_row(const TopkArgs& a, int64_t b, int64_t t, int li, int lane,
                                               int64_t nmax) {
    const int64_t ncand = nmax + 1;
    const int nvalid = (int)(ncand < a.keff ? ncand : a.keff);
    if (lane < a.keff) {
        int64_t v = lane < nvalid ? (int64_t)li : (nmax + 1 + (lane - nvalid));
        a.idx[b * a.si[0] + t * a.si[1] + lane * a.si[2]] = v;
    }
}

// ---------------------------------------------------------------------------
// tile kernel: 64 query tokens x 64 candidate blocks per step (prefill)
// ---------------------------------------------------------------------------
constexpr int kTT = 64;   // tokens per CTA
constexpr int kTN = 64;   // candidates per tile
constexpr int kTopkThreads = 256;

constexpr int kLQ = kTT + 4;  // padded smem rows: 16-byte aligned, conflict-free transposed stores
constexpr int kLC = kTN + 4;

// Loads a [rows x D] tile (rows r0 .. r0+63 of a [.., rows, D] tensor, row stride sr,
// scaled by `scale`) transposed into dst[d * ld + r]; rows at or past `nrows` read 0.
template <typename T, typename SC>
__device__ __forceinline__ void load_tile_t(SC* dst, int ld, const T* base, int64_t sr, int64_t sd, int64_t r0,
                                            int64_t nrows, int D, SC scale, bool vec, int tid) {
    if constexpr (sizeof(T) == 2) {
        if (vec) {
            // one 16-byte row piece per thread; a warp covers 32 consecutive rows of one piece,
            // so the transposed stores hit 32 distinct banks
            for (int e = tid; e < 64 * (D / 8); e += kTopkThreads) {
                const int r = e & 63, ch = e >> 6;
                const int64_t row = r0 + r;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (row < nrows) v = *reinterpret_cast<const uint4*>(base + row * sr + ch * 8);
                const T* x = reinterpret_cast<const T*>(&v);
#pragma unroll
                for (int j = 0; j < 8; ++j) dst[(ch * 8 + j) * ld + r] = load_as<SC>(x + j) * scale;
            }
            return;
        }
    }
    for (int e = tid; e < 64 * D; e += kTopkThreads) {
        const int r = e / D, d = e - (e / D) * D;
        const int64_t row = r0 + r;
        SC x = SC(0);
        if (row < nrows) x = load_as<SC>(base + row * sr + d * sd) * scale;
        dst[d * ld + r] = x;
    }
}

// fp32 scores: three CTAs per SM (80 registers; the warp sort and merge are latency-bound)
template <typename T, typename SC>
__global__ void __launch_bounds__(kTopkThreads, sizeof(SC) == 4 ? 3 : 2) topk_tile_kernel(TopkArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int D = a.D;
    SC* Qs = reinterpret_cast<SC*>(smem_raw);   // [D][kLQ]
    SC* Cs = Qs + (size_t)D * kLQ;              // [D][kLC]
    SC* Ss = Cs + (size_t)D * kLC;              // [kTT][kTN+1]
    const int64_t b = blockIdx.y;
    const int64_t t0 = (int64_t)blockIdx.x * kTT;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const T* q = static_cast<const T*>(a.q);
    const T* c = static_cast<const T*>(a.c);
    const SC scale = scale_of<SC>(a);

    // query block of each of the CTA's tokens, computed once (a 64-bit division), and
    // the last candidate block it may select (-1 for rows past the end); block indices
    // fit in 32 bits, so the per-candidate arithmetic below is 32-bit
    __shared__ int64_t qbs[kTT];
    __shared__ int qb32[kTT], lim32[kTT];
    if (tid < kTT) {
        const int64_t qb = query_block(a, t0 + tid);
        qbs[tid] = qb;
        qb32[tid] = (int)qb;
        lim32[tid] = t0 + tid < a.L ? (int)(qb < a.nb - 1 ? qb : a.nb - 1) : -1;
    }
    load_tile_t<T, SC>(Qs, kLQ, q + b * a.sq[0], a.sq[1], a.sq[2], t0, a.L, D, scale, a.vecload != 0, tid);
    const bool prune = a.cpref != nullptr && a.scores == nullptr;
    // norms of this warp's 8 scaled query rows (for the candidate bound)
    SC qn[8];
    if (prune) {
        __syncthreads();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int tt = warp * 8 + j;
            SC ss = SC(0);
            for (int d = lane; d < D; d += 32) ss += Qs[d * kLQ + tt] * Qs[d * kLQ + tt];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
            qn[j] = sqrt(ss);
        }
    }

    const int64_t tlast = (t0 + kTT - 1 < a.L ? t0 + kTT - 1 : a.L - 1);
    __syncthreads();  // qbs
    int64_t n_hi = qbs[tlast - t0];
    if (n_hi > a.nb - 1) n_hi = a.nb - 1;

    SC ls[8];
    int li[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        ls[j] = -INFINITY;
        li[j] = INT_MAX;
    }

    const int ty = tid >> 4, tx = tid & 15;
    for (int64_t n0 = (n_hi / kTN) * kTN; n0 >= 0; n0 -= kTN) {
        if (prune && n0 < (n_hi / kTN) * kTN) {
            // Every candidate left has index < n0 + kTN, so its score is at most
            // |q| max|c| (prefix max over the tiles left) minus the smallest penalty left.
            // The scan stops when that bound is strictly below every token's current
            // k-th best (ties go to the lower index, so equality must keep scanning).
            const float cm = a.cpref[b * a.ntiles + n0 / kTN];
            bool done = true;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int64_t t = t0 + warp * 8 + j;
                const SC th = __shfl_sync(kFull, ls[j], a.keff - 1);
                if (t < a.L) {
                    const int64_t qb = qbs[warp * 8 + j];
                    const int64_t nhi = n0 + kTN - 1 < qb ? n0 + kTN - 1 : qb;
                    SC bound = qn[j] * (SC)cm * (SC)1.00001 - (SC)a.pen[qb - nhi];
                    bound += (bound < SC(0) ? -bound : bound) * (SC)1e-6 + (SC)1e-30;
                    if (!(bound < th)) done = false;
                }
            }
            if (__syncthreads_and(done)) break;
        }
        __syncthreads();
        load_tile_t<T, SC>(Cs, kLC, c + b * a.sc[0], a.sc[1], a.sc[2], n0, a.nb, D, SC(1), a.vecload != 0, tid);
        __syncthreads();

        SC acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = SC(0);
        for (int d = 0; d < D; ++d) {
            SC qa[4], cb[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) qa[i] = Qs[d * kLQ + 4 * ty + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) cb[j] = Cs[d * kLC + 4 * tx + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fma_sc<SC>(qa[i], cb[j], acc[i][j]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tt = 4 * ty + i;
            const int qb = qb32[tt], lim = lim32[tt];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int nn = 4 * tx + j;
                const int n = (int)n0 + nn;
                SC v = -INFINITY;
                if (n <= lim) v = acc[i][j] - (SC)a.pen[qb - n];
                Ss[tt * (kTN + 1) + nn] = v;
            }
        }
        __syncthreads();

        if (a.scores != nullptr) {
            for (int e = tid; e < kTT * kTN; e += kTopkThreads) {
                const int tt = e / kTN, nn = e - (e / kTN) * kTN;
                const int64_t t = t0 + tt, n = n0 + nn;
                if (t < a.L && n < a.nb) store_score<T, SC>(a, b, t, n, Ss[tt * (kTN + 1) + nn]);
            }
        }

#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int tt = warp * 8 + j;
            const int lim = lim32[tt];
            if (lim >= 0) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    const int nn = half * 32 + lane;
                    const int n = (int)n0 + nn;
                    SC s = -INFINITY;
                    int ci = INT_MAX;
                    if (n <= lim) {
                        s = Ss[tt * (kTN + 1) + nn];
                        ci = n;
                    }
                    warp_offer(ls[j], li[j], s, ci, a.keff, lane);
                }
            }
        }
    }

    // -inf for candidates past the scanned range
    if (a.scores != nullptr) {
        const int64_t nstart = (n_hi / kTN + 1) * kTN;
        for (int tt = warp; tt < kTT; tt += kTopkThreads / 32) {
            const int64_t t = t0 + tt;
            if (t >= a.L) continue;
            for (int64_t n = nstart + lane; n < a.nb; n += 32) store_score<T, SC>(a, b, t, n, SC(-INFINITY));
        }
    }

#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int tt = warp * 8 + j;
        const int64_t t = t0 + tt;
        if (t < a.L) {
            const int64_t qb = query_block(a, t);
            const int64_t nmax = qb < a.nb - 1 ? qb : a.nb - 1;
            write_topk_row(a, b, t, li[j], lane, nmax);
        }
    }
}

// ---------------------------------------------------------------------------
// token kernel: one CTA per query token (decode / single token), 8 warps
// ---------------------------------------------------------------------------
template <typename T, typename SC>
__global__ void __launch_bounds__(kTopkThreads) topk_token_kernel(TopkArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int D = a.D;
    SC* qs = reinterpret_cast<SC*>(smem_raw);          // [D]
    SC* cs_all = qs + D;                                // [8 warps][32][D+1]
    SC* lists_s = cs_all + (size_t)8 * 32 * (D + 1);    // [8][32]
    int* lists_i = reinterpret_cast<int*>(lists_s + 8 * 32);
    const int64_t b = blockIdx.y, t = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const T* q = static_cast<const T*>(a.q);
    const T* c = static_cast<const T*>(a.c);
    const SC scale = scale_of<SC>(a);
    for (int d = tid; d < D; d += kTopkThreads) qs[d] = load_as<SC>(q + b * a.sq[0] + t * a.sq[1] + d * a.sq[2]) * scale;
    __syncthreads();
    const int64_t qb = query_block(a, t);
    const int64_t nmax = qb < a.nb - 1 ? qb : a.nb - 1;
    SC* cs = cs_all + (size_t)warp * 32 * (D + 1);
    SC ls = -INFINITY;
    int li = INT_MAX;
    // chunk g covers candidates (nmax - 32(g+1), nmax - 32g]
    const int64_t nchunks = (nmax + 1 + 31) / 32;
    for (int64_t g = warp; g < nchunks; g += kTopkThreads / 32) {
        const int64_t nbase = nmax - 32 * g - 31;  // lowest candidate of the chunk (may be < 0)
        for (int e = lane; e < 32 * D; e += 32) {
            const int r = e / D, d = e - (e / D) * D;
            const int64_t n = nbase + r;
            SC x = SC(0);
            if (n >= 0) x = load_as<SC>(c + b * a.sc[0] + n * a.sc[1] + d * a.sc[2]);
            cs[r * (D + 1) + d] = x;
        }
        __syncwarp();
        const int64_t n = nbase + lane;
        SC acc = SC(0);
        for (int d = 0; d < D; ++d) acc = fma_sc<SC>(qs[d], cs[lane * (D + 1) + d], acc);
        SC s = -INFINITY;
        int ci = INT_MAX;
        if (n >= 0) {
            s = acc - (SC)a.pen[qb - n];
            ci = (int)n;
            if (a.scores != nullptr) store_score<T, SC>(a, b, t, n, s);
        }
        warp_offer(ls, li, s, ci, a.keff, lane);
        __syncwarp();
    }
    if (a.scores != nullptr) {
        for (int64_t n = nmax + 1 + tid; n < a.nb; n += kTopkThreads) store_score<T, SC>(a, b, t, n, SC(-INFINITY));
    }
    lists_s[warp * 32 + lane] = ls;
    lists_i[warp * 32 + lane] = li;
    __syncthreads();
    if (warp == 0) {
        for (int w = 1; w < kTopkThreads / 32; ++w) {
            SC ns = lists_s[w * 32 + lane];
            int ni = lists_i[w * 32 + lane];
            warp_merge(ls, li, ns, ni, lane);
        }
        write_topk_row(a, b, t, li, lane, nmax);
    }
}

// ---------------------------------------------------------------------------
// generic kernel for top_k > 32: full bitonic sort of one token's candidates
// ---------------------------------------------------------------------------
template <typename T, typename SC>
__global__ void __launch_bounds__(kTopkThreads) topk_sort_kernel(TopkArgs a, int p2) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int D = a.D;
    SC* qs = reinterpret_cast<SC*>(smem_raw);
    SC* ks = qs + D;
    int* ki = reinterpret_cast<int*>(ks + p2);
    const int64_t b = blockIdx.y, t = blockIdx.x;
    const int tid = threadIdx.x;
    const T* q = static_cast<const T*>(a.q);
    const T* c = static_cast<const T*>(a.c);
    const SC scale = scale_of<SC>(a);
    for (int d = tid; d < D; d += kTopkThreads) qs[d] = load_as<SC>(q + b * a.sq[0] + t * a.sq[1] + d * a.sq[2]) * scale;
    __syncthreads();
    const int64_t qb = query_block(a, t);
    const int64_t nmax = qb < a.nb - 1 ? qb : a.nb - 1;
    for (int n = tid; n < p2; n += kTopkThreads) {
        SC s = -INFINITY;
        int ci = INT_MAX;
        if (n <= nmax) {
            SC acc = SC(0);
            const T* cr = c + b * a.sc[0] + (int64_t)n * a.sc[1];
            for (int d = 0; d < D; ++d) acc = fma_sc<SC>(qs[d], load_as<SC>(cr + d * a.sc[2]), acc);
            s = acc - (SC)a.pen[qb - n];
            ci = n;
        }
        if (a.scores != nullptr && n < a.nb) store_score<T, SC>(a, b, t, n, s);
        ks[n] = s;
        ki[n] = ci;
    }
    __syncthreads();
    for (int k = 2; k <= p2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tid; i < p2; i += kTopkThreads) {
                const int pj = i ^ j;
                if (pj > i) {
                    const bool desc = (i & k) == 0;
                    SC s0 = ks[i], s1 = ks[pj];
                    int i0 = ki[i], i1 = ki[pj];
                    const bool second_better = better(s1, i1, s0, i0);
                    if (second_better == desc) {
                        ks[i] = s1; ki[i] = i1;
                        ks[pj] = s0; ki[pj] = i0;
                    }
                }
            }
            __syncthreads();
        }
    }
    const int64_t ncand = nmax + 1;
    const int nvalid = (int)(ncand < a.keff ? ncand : a.keff);
    for (int s = tid; s < a.keff; s += kTopkThreads) {
        int64_t v = s < nvalid ? (int64_t)ki[s] : (nmax + 1 + (s - nvalid));
        a.idx[b * a.si[0] + t * a.si[1] + s * a.si[2]] = v;
    }
}

// ---------------------------------------------------------------------------
// decode split: one token, many candidates -> partial sorted lists per CTA, then
// a warp merge.  The final order is the same total order (score desc, index
// asc) on the same per-candidate scores, so the result equals the token kernel.
// ---------------------------------------------------------------------------
constexpr int kSplitCand = 512;  // candidates per CTA (8 warps x 64)

template <typename T>
__global__ void __launch_bounds__(kTopkThreads) topk_decode_partial_kernel(TopkArgs a, float* part_s, int* part_i,
                                                                           int nsplit) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int D = a.D;
    float* qs = reinterpret_cast<float*>(smem_raw);           // [D]
    float* cs_all = qs + D;                                     // [8][32][D+1]
    float* lists_s = cs_all + (size_t)8 * 32 * (D + 1);         // [8][32]
    int* lists_i = reinterpret_cast<int*>(lists_s + 8 * 32);
    const int split = blockIdx.x;
    const int64_t t = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const T* q = static_cast<const T*>(a.q);
    const T* c = static_cast<const T*>(a.c);
    int64_t nb = a.nb;
    if (a.pos_dev != nullptr) {
        const int64_t v = *a.pos_dev / a.block + 1;
        nb = v < a.nb ? v : a.nb;
    }
    if ((int64_t)split * kSplitCand >= nb) return;  // capacity-sized grid: nothing to score here
    for (int d = tid; d < D; d += kTopkThreads) qs[d] = load_as<float>(q + b * a.sq[0] + t * a.sq[1] + d * a.sq[2]) * a.scale_f;
    __syncthreads();
    const int64_t qb = nb - 1;
    float* cs = cs_all + (size_t)warp * 32 * (D + 1);
    float ls = -INFINITY;
    int li = INT_MAX;
    for (int ch = 0; ch < 2; ++ch) {
        const int64_t nbase = (int64_t)split * kSplitCand + warp * 64 + ch * 32;
        for (int e = lane; e < 32 * D; e += 32) {
            const int r = e / D, d = e - (e / D) * D;
            const int64_t n = nbase + r;
            cs[r * (D + 1) + d] = n < nb ? load_as<float>(c + b * a.sc[0] + n * a.sc[1] + d * a.sc[2]) : 0.f;
        }
        __syncwarp();
        const int64_t n = nbase + lane;
        float sc = -INFINITY;
        int ci = INT_MAX;
        if (n < nb) {
            float acc = 0.f;
            for (int d = 0; d < D; ++d) acc = fmaf(qs[d], cs[lane * (D + 1) + d], acc);
            sc = acc - a.pen[qb - n];
            ci = (int)n;
        }
        warp_offer(ls, li, sc, ci, a.keff, lane);
        __syncwarp();
    }
    lists_s[warp * 32 + lane] = ls;
    lists_i[warp * 32 + lane] = li;
    __syncthreads();
    if (warp == 0) {
        for (int w = 1; w < kTopkThreads / 32; ++w) warp_merge(ls, li, lists_s[w * 32 + lane], lists_i[w * 32 + lane], lane);
        const size_t o = ((size_t)(b * a.L + t) * nsplit + split) * 32 + lane;
        part_s[o] = ls;
        part_i[o] = li;
    }
}


// Vectorised variant for 16-bit centroids with unit-stride, 16-byte-aligned rows
// and d_idx = 8 * DV <= 64: each lane loads its candidate's whole row with DV
// 16-byte loads (both of its candidates' rows issued before any use) and forms
// the score with the same sequential FMA chain over d as the other kernels; the
// eight warp lists are then merged as a tree (3 levels) instead of in sequence.
template <typename T, int DV>
__global__ void __launch_bounds__(kTopkThreads) topk_decode_vec_kernel(TopkArgs a, float* part_s, int* part_i,
                                                                       int nsplit) {
    constexpr int D = DV * 8;
    __shared__ float qs[D];
    __shared__ float lsm[kTopkThreads / 32][32];
    __shared__ int lim[kTopkThreads / 32][32];
    const int split = blockIdx.x;
    const int64_t t = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int64_t nb = a.nb;
    if (a.pos_dev != nullptr) {
        const int64_t v = *a.pos_dev / a.block + 1;
        nb = v < a.nb ? v : a.nb;
    }
    if ((int64_t)split * kSplitCand >= nb) return;
    const T* q = static_cast<const T*>(a.q);
    const T* c = static_cast<const T*>(a.c) + b * a.sc[0];
    for (int d = tid; d < D; d += kTopkThreads) qs[d] = load_as<float>(q + b * a.sq[0] + t * a.sq[1] + d * a.sq[2]) * a.scale_f;
    const int64_t n0 = (int64_t)split * kSplitCand + warp * 64 + lane;
    uint4 r0[DV], r1[DV];
#pragma unroll
    for (int k = 0; k < DV; ++k) {
        r0[k] = n0 < nb ? *reinterpret_cast<const uint4*>(c + n0 * a.sc[1] + k * 8) : make_uint4(0u, 0u, 0u, 0u);
        r1[k] = n0 + 32 < nb ? *reinterpret_cast<const uint4*>(c + (n0 + 32) * a.sc[1] + k * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    const int64_t qb = nb - 1;
    float ls = -INFINITY;
    int li = INT_MAX;
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
        const int64_t n = n0 + 32 * ch;
        float sc = -INFINITY;
        int ci = INT_MAX;
        if (n < nb) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < DV; ++k) {
                const T* e = reinterpret_cast<const T*>(ch == 0 ? &r0[k] : &r1[k]);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc = fmaf(qs[k * 8 + i], Cvt<T>::to_f(e[i]), acc);
            }
            // the penalty table's value, computed in place (penalty_table_kernel's arithmetic)
            sc = acc - __fmul_rn(a.lam_f, (float)log1p((double)(qb - n)));
            ci = (int)n;
        }
        warp_offer(ls, li, sc, ci, a.keff, lane);
    }
    lsm[warp][lane] = ls;
    lim[warp][lane] = li;
    for (int half = kTopkThreads / 64; half > 0; half >>= 1) {
        __syncthreads();
        if (warp < half) {
            warp_merge(ls, li, lsm[warp + half][lane], lim[warp + half][lane], lane);
            lsm[warp][lane] = ls;
            lim[warp][lane] = li;
        }
    }
    if (warp == 0) {
        const size_t o = ((size_t)(b * a.L + t) * nsplit + split) * 32 + lane;
        part_s[o] = ls;
        part_i[o] = li;
    }
}

// Tree merge of the partial lists of one (batch, token) row: warp w first folds
// lists w, w+32, ... in sequence, then the 32 warp lists meet in 5 levels.
__global__ void __launch_bounds__(1024) topk_decode_merge_tree_kernel(TopkArgs a, const float* part_s,
                                                                      const int* part_i, int nsplit, int64_t B) {
    __shared__ float lsm[32][32];
    __shared__ int lim[32][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row = blockIdx.x;
    const int64_t b = row / a.L, t = row - (row / a.L) * a.L;
    int64_t nb = a.nb;
    if (a.pos_dev != nullptr) {
        const int64_t v = *a.pos_dev / a.block + 1;
        nb = v < a.nb ? v : a.nb;
    }
    const int used = (int)((nb + kSplitCand - 1) / kSplitCand);
    const size_t base = (size_t)row * nsplit * 32;
    float ls = -INFINITY;
    int li = INT_MAX;
    for (int sp = warp; sp < used && sp < nsplit; sp += 32)
        warp_merge(ls, li, part_s[base + sp * 32 + lane], part_i[base + sp * 32 + lane], lane);
    lsm[warp][lane] = ls;
    lim[warp][lane] = li;
    for (int half = 16; half > 0; half >>= 1) {
        __syncthreads();
        if (warp < half) {
            warp_merge(ls, li, lsm[warp + half][lane], lim[warp + half][lane], lane);
            lsm[warp][lane] = ls;
            lim[warp][lane] = li;
        }
    }
    if (warp == 0) write_topk_row(a, b, t, li, lane, nb - 1);
    (void)B;
}

// Launches the split decode scan (vectorised partials where the layout allows)
// and the tree merge.
// The vectorised decode kernel applies: 16-bit centroids, unit-stride 16-byte-aligned rows, d <= 64.
bool decode_vec_ok(const TopkArgs& a, int elem_bytes) {
    return elem_bytes == 2 && a.D % 8 == 0 && a.D <= 64 && a.sc[2] == 1 && (a.sc[1] * 2) % 16 == 0 &&
           (a.sc[0] * 2) % 16 == 0 && (reinterpret_cast<uintptr_t>(a.c) & 15u) == 0;
}

template <typename T>
int launch_topk_decode_split(TopkArgs& a, int64_t B, int64_t L, int nsplit, float* ps, int* pi, cudaStream_t s) {
    const bool vec = decode_vec_ok(a, (int)sizeof(T));
    const dim3 grid((unsigned)nsplit, (unsigned)L, (unsigned)B);
    if (vec) {
        switch (a.D / 8) {
            case 1: topk_decode_vec_kernel<T, 1><<<grid, kTopkThreads, 0, s>>>(a, ps, pi, nsplit); break;
            case 2: topk_decode_vec_kernel<T, 2><<<grid, kTopkThreads, 0, s>>>(a, ps, pi, nsplit); break;
            case 3: topk_decode_vec_kernel<T, 3><<<grid, kTopkThreads, 0, s>>>(a, ps, pi, nsplit); break;
            case 4: topk_decode_vec_kernel<T, 4><<<grid, kTopkThreads, 0, s>>>(a, ps, pi, nsplit); break;
            case 5: topk_decode_vec_kernel<T, 5><<<grid, kTopkThreads, 0, s>>>(a, ps, pi, nsplit); break;
            case 6: topk_decode_vec_kernel<T, 6><<<grid, kTopkThreads, 0, s>>>(a, ps, pi, nsplit); break;
            case 7: topk_decode_vec_kernel<T, 7><<<grid, kTopkThreads, 0, s>>>(a, ps, pi, nsplit); break;
            default: topk_decode_vec_kernel<T, 8><<<grid, kTopkThreads, 0, s>>>(a, ps, pi, nsplit); break;
        }
    } else {
        const size_t smem = sizeof(float) * ((size_t)a.D + (size_t)8 * 32 * (a.D + 1) + 8 * 32) + sizeof(int) * 8 * 32;
        auto kern = topk_decode_partial_kernel<T>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, kTopkThreads, smem, s>>>(a, ps, pi, nsplit);
    }
    MABA_TRY(check_launch("index_topk(decode partial)"));
    topk_decode_merge_tree_kernel<<<(unsigned)(B * L), 1024, 0, s>>>(a, ps, pi, nsplit, B);
    return check_launch("index_topk(decode merge)");
}

int64_t decode_split_count(int64_t nb) { return (nb + kSplitCand - 1) / kSplitCand; }

bool decode_split_wanted(const TopkArgs& a, int64_t B, int dtype) {
    return a.decode && dtype != MABA_F64 && a.keff <= 32 && a.nb >= 4 * kSplitCand && B * a.L <= 256 &&
           a.scores == nullptr;
}

template <typename T>
int launch_topk(TopkArgs& a, int64_t B, cudaStream_t s) {
    using SC = typename std::conditional<sizeof(T) == 8, double, float>::type;
    const int D = a.D;
    if (a.keff > 32) {
        int p2 = 1;
        while (p2 < a.nb) p2 <<= 1;
        const size_t smem = sizeof(SC) * (D + p2) + sizeof(int) * p2;
        if (smem > 200 * 1024)
            return set_error(MABA_ERR_UNSUPPORTED, "index_topk: top_k=%d > 32 needs nb <= %d", a.keff,
                             (int)(200 * 1024 / (sizeof(SC) + sizeof(int))));
        auto kern = topk_sort_kernel<T, SC>;
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        dim3 grid((unsigned)a.L, (unsigned)B);
        kern<<<grid, kTopkThreads, smem, s>>>(a, p2);
        return check_launch("index_topk(sort)");
    }
    if (a.decode || a.L < kTT) {
        const size_t smem = sizeof(SC) * (D + (size_t)8 * 32 * (D + 1) + 8 * 32) + sizeof(int) * 8 * 32;
        if (smem > 200 * 1024) return set_error(MABA_ERR_UNSUPPORTED, "index_topk: d_idx=%d too large", D);
        auto kern = topk_token_kernel<T, SC>;
        if (smem > 48 * 1024)
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        dim3 grid((unsigned)a.L, (unsigned)B);
        kern<<<grid, kTopkThreads, smem, s>>>(a);
        return check_launch("index_topk(token)");
    }
    const size_t smem = sizeof(SC) * ((size_t)D * kLQ + (size_t)D * kLC + (size_t)kTT * (kTN + 1));
    if (smem > 200 * 1024) return set_error(MABA_ERR_UNSUPPORTED, "index_topk: d_idx=%d too large", D);
    auto kern = topk_tile_kernel<T, SC>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((unsigned)ceil_div(a.L, kTT), (unsigned)B);
    kern<<<grid, kTopkThreads, smem, s>>>(a);
    return check_launch("index_topk(tile)");
}

int64_t penalty_len(int64_t L, int64_t nb, int32_t block, int decode, int64_t q_pos0 = 0) {
    int64_t n = nb;
    if (!decode && L > 0 && block > 0) {
        int64_t qmax = (q_pos0 + L - 1) / block + 1;
        if (qmax > n) n = qmax;
    }
    return n > 0 ? n : 1;
}

}  // namespace
}  // namespace maba

using namespace maba;

extern "C" int maba_compute_centroids(const maba_tensor* k_idx, const maba_tensor* out, int32_t block_size,
                                      void* stream) {
    if (!present(k_idx) || k_idx->ndim != 3)
        return set_error(MABA_ERR_INVALID, "compute_centroids: k_idx must be 3D [B, L, d_idx]");
    if (block_size <= 0) return set_error(MABA_ERR_INVALID, "compute_centroids: block_size must be positive");
    const int64_t B = k_idx->shape[0], L = k_idx->shape[1], D = k_idx->shape[2];
    const int64_t nb = ceil_div(L, block_size);
    const int64_t so[3] = {B, nb, D};
    MABA_TRY(expect_shape(out, "compute_centroids: out", 3, so));
    MABA_TRY(expect_dtype(out, "compute_centroids: out", k_idx->dtype));
    PoolArgs a{};
    a.in = k_idx->data; a.out = out->data;
    for (int i = 0; i < 3; ++i) { a.si[i] = k_idx->stride[i]; a.so[i] = out->stride[i]; }
    a.L = L; a.nblk = nb; a.D = (int)D; a.block = block_size; a.mode = 0;
    cudaStream_t s = as_stream(stream);
    return MABA_DISPATCH_FLOAT(k_idx->dtype, "compute_centroids", [&] { return launch_pool<T, T>(a, B, s, "compute_centroids"); });
}

extern "C" int maba_hca_pool(const maba_tensor* c_kv, const maba_tensor* out, int32_t r, void* stream) {
    if (!present(c_kv) || c_kv->ndim != 3) return set_error(MABA_ERR_INVALID, "hca_pool: c_kv must be [B, L, d_c]");
    if (r <= 0) return set_error(MABA_ERR_INVALID, "hca_pool: r must be positive");
    const int64_t B = c_kv->shape[0], L = c_kv->shape[1], D = c_kv->shape[2];
    const int64_t nc = L / r;
    const int64_t so[3] = {B, nc, D};
    MABA_TRY(expect_shape(out, "hca_pool: out", 3, so));
    PoolArgs a{};
    a.in = c_kv->data; a.out = out->data;
    for (int i = 0; i < 3; ++i) { a.si[i] = c_kv->stride[i]; a.so[i] = out->stride[i]; }
    a.L = L; a.nblk = nc; a.D = (int)D; a.block = r; a.mode = 1;
    cudaStream_t s = as_stream(stream);
    const int odt = out->dtype;
    return MABA_DISPATCH_FLOAT(c_kv->dtype, "hca_pool", [&] {
        if (odt == MABA_F32) return launch_pool<T, float>(a, B, s, "hca_pool");
        if (odt == c_kv->dtype) return launch_pool<T, T>(a, B, s, "hca_pool");
        return set_error(MABA_ERR_DTYPE, "hca_pool: out dtype must be float32 or c_kv's dtype");
    });
}

// Bytes after the penalty table: the decode split's partial lists, or the
// centroid-norm tables of the pruned tile scan (never both in one call).
static size_t topk_extra_bytes(int64_t B, int64_t L, int64_t nb, int32_t top_k) {
    size_t extra = 0;
    if (B * L <= 256 && nb >= 4 * kSplitCand && top_k <= 32)
        extra = (size_t)B * L * decode_split_count(nb) * 32 * 8;
    const size_t norms = 2 * (size_t)B * ceil_div(nb, (int64_t)kTN) * sizeof(float);
    return extra > norms ? extra : norms;
}

extern "C" size_t maba_index_topk_workspace_size(int64_t B, int64_t L, int64_t nb, int32_t top_k) {
    // penalty table; the block size is not known here, so size for the
    // largest query block any block_size >= 1 could produce is not bounded:
    // callers pass L and nb and the table holds max(nb, L) entries.
    int64_t n = nb > L ? nb : L;
    if (n < 1) n = 1;
    size_t bytes = (size_t)((n * sizeof(float) + 255) / 256 * 256);
    return bytes + topk_extra_bytes(B, L, nb, top_k);
}

static int index_topk_impl(const maba_tensor* q_idx, const maba_tensor* centroids, float lambda_dist,
                           int32_t top_k, int32_t block_size, int32_t decode, int64_t q_pos0,
                           const maba_tensor* idx_out, const maba_tensor* scores_out, void* workspace,
                           size_t workspace_bytes, void* stream) {
    if (!present(q_idx) || !present(centroids) || q_idx->ndim != 3 || centroids->ndim != 3)
        return set_error(MABA_ERR_INVALID, "index_topk: q_idx and centroids must be 3D");
    if (top_k <= 0) return set_error(MABA_ERR_INVALID, "index_topk: top_k must be positive, got %d", top_k);
    if (block_size <= 0) return set_error(MABA_ERR_INVALID, "index_topk: block_size must be positive");
    const int64_t B = q_idx->shape[0], L = q_idx->shape[1], D = q_idx->shape[2];
    const int64_t nb = centroids->shape[1];
    if (centroids->shape[0] != B || centroids->shape[2] != D)
        return set_error(MABA_ERR_INVALID, "index_topk: dimension mismatch between q_idx and centroids");
    MABA_TRY(expect_dtype(centroids, "index_topk: centroids", q_idx->dtype));
    const int64_t keff = top_k < nb ? top_k : nb;
    const int64_t si[3] = {B, L, keff};
    MABA_TRY(expect_shape(idx_out, "index_topk: idx_out", 3, si));
    MABA_TRY(expect_dtype(idx_out, "index_topk: idx_out", MABA_I64));
    if (present(scores_out)) {
        const int64_t ss[3] = {B, L, nb};
        MABA_TRY(expect_shape(scores_out, "index_topk: scores_out", 3, ss));
        MABA_TRY(expect_dtype(scores_out, "index_topk: scores_out", q_idx->dtype));
    }
    if (L == 0 || nb == 0 || B == 0) return MABA_OK;  // caller fills the empty result
    if (nb > INT_MAX / 2) return set_error(MABA_ERR_UNSUPPORTED, "index_topk: nb too large");
    if (q_pos0 < 0) return set_error(MABA_ERR_INVALID, "index_topk: negative query offset");
    const int64_t plen = penalty_len(L, nb, block_size, decode, q_pos0);
    const size_t need = (size_t)plen * sizeof(float);
    if (workspace == nullptr || workspace_bytes < need)
        return set_error(MABA_ERR_WORKSPACE, "index_topk: workspace of %zu bytes required, got %zu", need,
                         workspace_bytes);
    cudaStream_t s = as_stream(stream);
    float* pen = static_cast<float*>(workspace);
    penalty_table_kernel<<<(unsigned)ceil_div(plen, 256), 256, 0, s>>>(pen, plen, lambda_dist);
    MABA_TRY(check_launch("index_topk(penalty)"));

    TopkArgs a{};
    a.q = q_idx->data; a.c = centroids->data;
    a.idx = static_cast<int64_t*>(idx_out->data);
    a.scores = present(scores_out) ? scores_out->data : nullptr;
    a.pen = pen;
    for (int i = 0; i < 3; ++i) {
        a.sq[i] = q_idx->stride[i]; a.sc[i] = centroids->stride[i]; a.si[i] = idx_out->stride[i];
        a.ss[i] = present(scores_out) ? scores_out->stride[i] : 0;
    }
    a.L = L; a.nb = nb; a.D = (int)D; a.block = block_size; a.keff = (int)keff; a.decode = decode ? 1 : 0;
    a.q_pos0 = decode ? 0 : q_pos0;
    a.scale_d = 1.0 / sqrt((double)D);
    a.scale_f = (float)a.scale_d;
    a.lam_f = lambda_dist;
    if (decode_split_wanted(a, B, q_idx->dtype)) {
        const int64_t nsplit = decode_split_count(nb);
        const size_t off = (need + 255) / 256 * 256;
        const size_t part = (size_t)B * L * nsplit * 32;
        if (workspace_bytes >= off + part * 8) {
            float* ps = reinterpret_cast<float*>(static_cast<char*>(workspace) + off);
            int* pi = reinterpret_cast<int*>(ps + part);
            const size_t smem = sizeof(float) * ((size_t)D + (size_t)8 * 32 * (D + 1) + 8 * 32) + sizeof(int) * 8 * 32;
            if (smem <= 200 * 1024) {
                return MABA_DISPATCH_FLOAT(q_idx->dtype, "index_topk", [&] {
                    if constexpr (sizeof(T) == 8) {
                        return launch_topk<T>(a, B, s);
                    } else {
                        return launch_topk_decode_split<T>(a, B, L, (int)nsplit, ps, pi, s);
                    }
                });
            }
        }
    }
    // pruned tile scan: centroid-norm tables after the penalty table
    const int64_t ntiles = ceil_div(nb, (int64_t)kTN);
    const size_t off = (need + 255) / 256 * 256;
    const bool vec_ok = (q_idx->dtype == MABA_BF16 || q_idx->dtype == MABA_F16) && D % 8 == 0 &&
                        q_idx->stride[2] == 1 && centroids->stride[2] == 1 && q_idx->stride[1] % 8 == 0 &&
                        centroids->stride[1] % 8 == 0 && q_idx->stride[0] % 8 == 0 && centroids->stride[0] % 8 == 0 &&
                        (reinterpret_cast<uintptr_t>(q_idx->data) & 15u) == 0 &&
                        (reinterpret_cast<uintptr_t>(centroids->data) & 15u) == 0;
    a.vecload = vec_ok ? 1 : 0;
    if (!decode && !present(scores_out) && L >= kTT && workspace_bytes >= off + 2 * (size_t)B * ntiles * sizeof(float) &&
        q_idx->dtype != MABA_F64) {
        float* tmax = reinterpret_cast<float*>(static_cast<char*>(workspace) + off);
        float* pref = tmax + (size_t)B * ntiles;
        MABA_TRY(MABA_DISPATCH_FLOAT(q_idx->dtype, "index_topk(norms)", [&] {
            centroid_tile_norm_kernel<T><<<dim3((unsigned)ntiles, (unsigned)B), 64, 0, s>>>(
                static_cast<const T*>(centroids->data), centroids->stride[0], centroids->stride[1],
                centroids->stride[2], nb, (int)D, tmax, ntiles);
            return check_launch("index_topk(norms)");
        }));
        tile_prefix_max_kernel<<<(unsigned)B, 256, 0, s>>>(tmax, pref, ntiles);
        MABA_TRY(check_launch("index_topk(prefix max)"));
        a.cpref = pref;
        a.ntiles = ntiles;
    }
    return MABA_DISPATCH_FLOAT(q_idx->dtype, "index_topk", [&] { return launch_topk<T>(a, B, s); });
}

extern "C" int maba_index_topk(const maba_tensor* q_idx, const maba_tensor* centroids, float lambda_dist,
                               int32_t top_k, int32_t block_size, int32_t decode, const maba_tensor* idx_out,
                               const maba_tensor* scores_out, void* workspace, size_t workspace_bytes,
                               void* stream) {
    return index_topk_impl(q_idx, centroids, lambda_dist, top_k, block_size, decode, 0, idx_out, scores_out,
                           workspace, workspace_bytes, stream);
}

extern "C" int maba_index_topk_at(const maba_tensor* q_idx, const maba_tensor* centroids, float lambda_dist,
                                  int32_t top_k, int32_t block_size, int64_t q_pos0, const maba_tensor* idx_out,
                                  const maba_tensor* scores_out, void* workspace, size_t workspace_bytes,
                                  void* stream) {
    return index_topk_impl(q_idx, centroids, lambda_dist, top_k, block_size, 0, q_pos0, idx_out, scores_out,
                           workspace, workspace_bytes, stream);
}

extern "C" size_t maba_index_topk_at_workspace_size(int64_t B, int64_t L, int64_t nb, int32_t top_k, int32_t block_size,
                                                    int64_t q_pos0) {
    const int64_t n = penalty_len(L, nb, block_size > 0 ? block_size : 1, 0, q_pos0 > 0 ? q_pos0 : 0);
    const size_t norms = 2 * (size_t)B * ceil_div(nb, (int64_t)kTN) * sizeof(float);
    (void)top_k;
    return (size_t)((n * sizeof(float) + 255) / 256 * 256) + norms;
}

// ---------------------------------------------------------------------------
// Workspace-free variant (maba_index_topk_noalloc): the scratch of
// index_topk_impl -- the penalty table, then either the pruned scan's centroid
// norm tables or the split decode scan's partial lists, each only when it fits
// behind the table -- lives in a fixed file-scope device array instead of
// caller memory.  The array's device address is looked up once per device and
// kept for the life of the process (not valid across a device reset).
// ---------------------------------------------------------------------------
#include <mutex>

static __device__ __align__(256) float g_noalloc_penalty[MABA_NOALLOC_PENALTY_MAX];

namespace {
std::mutex g_noalloc_mutex;
float* g_noalloc_table[128] = {nullptr};  // device address of g_noalloc_penalty, per device

// Looks the array up once per device (with that device current).  The host
// symbol g_noalloc_penalty is only a stand-in: kernels get the device address.
int noalloc_table(float** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(MABA_ERR_CUDA, "index_topk_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 128) return set_error(MABA_ERR_UNSUPPORTED, "index_topk_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_table[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_penalty);
        if (e != cudaSuccess || p == nullptr)
            return set_error(MABA_ERR_CUDA, "index_topk_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        g_noalloc_table[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_table[dev];
    return MABA_OK;
}
}  // namespace

extern "C" int maba_index_topk_noalloc(const maba_tensor* q_idx, const maba_tensor* centroids, float lambda_dist,
                                       int32_t top_k, int32_t block_size, int32_t decode, const maba_tensor* idx_out,
                                       const maba_tensor* scores_out, void* stream) {
    if (present(q_idx) && present(centroids) && q_idx->ndim == 3 && centroids->ndim == 3 && block_size > 0) {
        const int64_t need = penalty_len(q_idx->shape[1], centroids->shape[1], block_size, decode);
        if (need > MABA_NOALLOC_PENALTY_MAX)
            return set_error(MABA_ERR_UNSUPPORTED,
                             "index_topk_noalloc: needs %lld penalty entries, the fixed scratch holds %d "
                             "(use maba_index_topk with a caller workspace)",
                             (long long)need, MABA_NOALLOC_PENALTY_MAX);
    }
    float* table = nullptr;
    MABA_TRY(noalloc_table(&table));
    return maba_index_topk(q_idx, centroids, lambda_dist, top_k, block_size, decode, idx_out, scores_out, table,
                           sizeof(float) * (size_t)MABA_NOALLOC_PENALTY_MAX, stream);
}

// ---------------------------------------------------------------------------
// Decode at a device-held position (CUDA-graph friendly): cache append + top-k
// ---------------------------------------------------------------------------
namespace maba {
namespace {

struct AppendArgs {
    const void* c_new; const void* k_new;
    void* c; void* kidx; void* cent; void* hca;
    int64_t s_cn[3], s_kn[3], s_c[3], s_k[3], s_ce[3], s_h[3];
    int64_t Lcap, nbcap, nccap;
    int DC, DI, block, r;
    const int64_t* pos_dev;
};

// Writes the new latent / index-key rows at `pos`, refreshes the centroid of
// pos's block (zero-padded tail, as compute_centroids) and, when pos closes an
// r-row group, writes its pooled HCA mean.
template <typename T>
__global__ void decode_append_kernel(AppendArgs a) {
    const int64_t b = blockIdx.x;
    const int64_t pos = *a.pos_dev;
    if (pos < 0 || pos >= a.Lcap) return;
    T* c = static_cast<T*>(a.c);
    T* kidx = static_cast<T*>(a.kidx);
    const T* cn = static_cast<const T*>(a.c_new);
    const T* kn = static_cast<const T*>(a.k_new);
    for (int d = threadIdx.x; d < a.DC; d += blockDim.x)
        c[b * a.s_c[0] + pos * a.s_c[1] + d * a.s_c[2]] = cn[b * a.s_cn[0] + d * a.s_cn[2]];
    for (int d = threadIdx.x; d < a.DI; d += blockDim.x)
        kidx[b * a.s_k[0] + pos * a.s_k[1] + d * a.s_k[2]] = kn[b * a.s_kn[0] + d * a.s_kn[2]];
    __syncthreads();
    const int64_t blk = pos / a.block, start = blk * a.block;
    if (blk < a.nbcap) {
        T* cent = static_cast<T*>(a.cent);
        const bool padded = pos + 1 < start + a.block;
        for (int d = threadIdx.x; d < a.DI; d += blockDim.x) {
            float sum = 0.f, mx = padded ? 0.f : -INFINITY;
            // rows in order (the pooling kernel's fp32 sum); eight loads in flight at a time
            for (int64_t t0 = start; t0 <= pos; t0 += 8) {
                float xs[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    xs[u] = t0 + u <= pos ? load_as<float>(kidx + b * a.s_k[0] + (t0 + u) * a.s_k[1] + d * a.s_k[2]) : 0.f;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (t0 + u > pos) break;
                    sum += xs[u];
                    mx = xs[u] > mx ? xs[u] : mx;
                }
            }
            store_from<T, float>(cent + b * a.s_ce[0] + blk * a.s_ce[1] + d * a.s_ce[2],
                                 0.5f * (sum / float(a.block) + mx));
        }
    }
    if ((pos + 1) % a.r == 0) {
        const int64_t g = (pos + 1) / a.r - 1;
        if (g < a.nccap) {
            T* hca = static_cast<T*>(a.hca);
            for (int d = threadIdx.x; d < a.DC; d += blockDim.x) {
                float sum = 0.f;
                for (int64_t t0 = pos + 1 - a.r; t0 <= pos; t0 += 8) {
                    float xs[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        xs[u] = t0 + u <= pos ? load_as<float>(c + b * a.s_c[0] + (t0 + u) * a.s_c[1] + d * a.s_c[2]) : 0.f;
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        if (t0 + u <= pos) sum += xs[u];
                }
                store_from<T, float>(hca + b * a.s_h[0] + g * a.s_h[1] + d * a.s_h[2], sum / float(a.r));
            }
        }
    }
}

}  // namespace
}  // namespace maba

extern "C" int maba_decode_cache_append(const maba_tensor* c_new, const maba_tensor* k_new, const maba_tensor* c_cache,
                                        const maba_tensor* kidx_cache, const maba_tensor* cent_table,
                                        const maba_tensor* hca_table, const int64_t* pos_dev, int32_t block_size,
                                        int32_t hca_r, void* stream) {
    if (!present(c_cache) || c_cache->ndim != 3 || !present(kidx_cache) || kidx_cache->ndim != 3)
        return set_error(MABA_ERR_INVALID, "decode_cache_append: caches must be [B, Lcap, d]");
    if (pos_dev == nullptr) return set_error(MABA_ERR_INVALID, "decode_cache_append: device position required");
    if (block_size <= 0 || hca_r <= 0) return set_error(MABA_ERR_INVALID, "decode_cache_append: block/r must be positive");
    const int64_t B = c_cache->shape[0], Lcap = c_cache->shape[1], DC = c_cache->shape[2], DI = kidx_cache->shape[2];
    const int64_t scn[3] = {B, 1, DC}, skn[3] = {B, 1, DI}, sk[3] = {B, Lcap, DI};
    MABA_TRY(expect_shape(c_new, "decode_cache_append: c_new", 3, scn));
    MABA_TRY(expect_shape(k_new, "decode_cache_append: k_new", 3, skn));
    MABA_TRY(expect_shape(kidx_cache, "decode_cache_append: kidx_cache", 3, sk));
    const int64_t sce[3] = {B, -1, DI}, sh[3] = {B, -1, DC};
    MABA_TRY(expect_shape(cent_table, "decode_cache_append: cent_table", 3, sce));
    MABA_TRY(expect_shape(hca_table, "decode_cache_append: hca_table", 3, sh));
    const int dt = c_cache->dtype;
    const maba_tensor* all[] = {c_new, k_new, kidx_cache, cent_table, hca_table};
    for (const maba_tensor* t : all) MABA_TRY(expect_dtype(t, "decode_cache_append", dt));
    AppendArgs a{};
    a.c_new = c_new->data; a.k_new = k_new->data; a.c = c_cache->data; a.kidx = kidx_cache->data;
    a.cent = cent_table->data; a.hca = hca_table->data;
    for (int i = 0; i < 3; ++i) {
        a.s_cn[i] = c_new->stride[i]; a.s_kn[i] = k_new->stride[i]; a.s_c[i] = c_cache->stride[i];
        a.s_k[i] = kidx_cache->stride[i]; a.s_ce[i] = cent_table->stride[i]; a.s_h[i] = hca_table->stride[i];
    }
    a.Lcap = Lcap; a.nbcap = cent_table->shape[1]; a.nccap = hca_table->shape[1];
    a.DC = (int)DC; a.DI = (int)DI; a.block = block_size; a.r = hca_r; a.pos_dev = pos_dev;
    cudaStream_t s = as_stream(stream);
    return MABA_DISPATCH_FLOAT(dt, "decode_cache_append", [&] {
        decode_append_kernel<T><<<(unsigned)B, 128, 0, s>>>(a);
        return check_launch("decode_cache_append");
    });
}

extern "C" size_t maba_index_topk_decode_at_workspace_size(int64_t B, int64_t nbcap, int32_t top_k) {
    (void)top_k;
    const size_t pen = (size_t)(((nbcap > 0 ? nbcap : 1) * sizeof(float) + 255) / 256 * 256);
    return pen + (size_t)B * decode_split_count(nbcap) * 32 * 8;
}

extern "C" int maba_index_topk_decode_at(const maba_tensor* q_idx, const maba_tensor* cent_table, float lambda_dist,
                                         int32_t top_k, int32_t block_size, const int64_t* pos_dev,
                                         const maba_tensor* idx_out, void* workspace, size_t workspace_bytes,
                                         void* stream) {
    if (!present(q_idx) || !present(cent_table) || q_idx->ndim != 3 || cent_table->ndim != 3 || q_idx->shape[1] != 1)
        return set_error(MABA_ERR_INVALID, "index_topk_decode_at: q_idx [B,1,d] and cent_table [B,nbcap,d] required");
    if (pos_dev == nullptr) return set_error(MABA_ERR_INVALID, "index_topk_decode_at: device position required");
    if (top_k <= 0 || top_k > 32) return set_error(MABA_ERR_UNSUPPORTED, "index_topk_decode_at: top_k in [1, 32]");
    if (block_size <= 0) return set_error(MABA_ERR_INVALID, "index_topk_decode_at: block_size must be positive");
    const int64_t B = q_idx->shape[0], D = q_idx->shape[2], nbcap = cent_table->shape[1];
    if (cent_table->shape[0] != B || cent_table->shape[2] != D)
        return set_error(MABA_ERR_INVALID, "index_topk_decode_at: dimension mismatch");
    MABA_TRY(expect_dtype(cent_table, "index_topk_decode_at: cent_table", q_idx->dtype));
    if (q_idx->dtype == MABA_F64) return set_error(MABA_ERR_UNSUPPORTED, "index_topk_decode_at: float64");
    const int64_t kout = top_k < nbcap ? top_k : nbcap;
    const int64_t si[3] = {B, 1, kout};
    MABA_TRY(expect_shape(idx_out, "index_topk_decode_at: idx_out", 3, si));
    MABA_TRY(expect_dtype(idx_out, "index_topk_decode_at: idx_out", MABA_I64));
    const size_t need = maba_index_topk_decode_at_workspace_size(B, nbcap, top_k);
    if (workspace == nullptr || workspace_bytes < need)
        return set_error(MABA_ERR_WORKSPACE, "index_topk_decode_at: workspace of %zu bytes required", need);
    cudaStream_t s = as_stream(stream);
    float* pen = static_cast<float*>(workspace);
    const int64_t nsplit = decode_split_count(nbcap);
    const size_t off = (nbcap * sizeof(float) + 255) / 256 * 256;
    float* ps = reinterpret_cast<float*>(static_cast<char*>(workspace) + off);
    int* pi = reinterpret_cast<int*>(ps + (size_t)B * nsplit * 32);
    TopkArgs a{};
    a.q = q_idx->data; a.c = cent_table->data; a.idx = static_cast<int64_t*>(idx_out->data); a.scores = nullptr;
    a.pen = pen;
    for (int i = 0; i < 3; ++i) { a.sq[i] = q_idx->stride[i]; a.sc[i] = cent_table->stride[i]; a.si[i] = idx_out->stride[i]; }
    a.L = 1; a.nb = nbcap; a.D = (int)D; a.block = block_size; a.keff = (int)kout; a.decode = 1;
    a.scale_d = 1.0 / sqrt((double)D); a.scale_f = (float)a.scale_d;
    a.lam_f = lambda_dist; a.pos_dev = pos_dev;
    const size_t smem = sizeof(float) * ((size_t)D + (size_t)8 * 32 * (D + 1) + 8 * 32) + sizeof(int) * 8 * 32;
    if (smem > 200 * 1024) return set_error(MABA_ERR_UNSUPPORTED, "index_topk_decode_at: d_idx too large");
    // the vectorised kernel forms the penalties itself; the other one reads the table
    if (!decode_vec_ok(a, q_idx->dtype == MABA_F32 ? 4 : 2)) {
        penalty_table_kernel<<<(unsigned)ceil_div(nbcap, 256), 256, 0, s>>>(pen, nbcap, lambda_dist);
        MABA_TRY(check_launch("index_topk_decode_at(penalty)"));
    }
    return MABA_DISPATCH_FLOAT(q_idx->dtype, "index_topk_decode_at", [&] {
        if constexpr (sizeof(T) == 8) {
            return set_error(MABA_ERR_UNSUPPORTED, "index_topk_decode_at: float64");
        } else {
            return launch_topk_decode_split<T>(a, B, 1, (int)nsplit, ps, pi, s);
        }
    });
}
