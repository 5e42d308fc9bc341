// Split-K MABA-SA attention for single-token decode (Lq == 1).
//
// Same math as sa_attention.cu (maba_sparse/layers/sparse_attention.py:79-219,
// 274-275; the decode gathers of :84-93 and :129-143), organised for one query
// token against a long latent cache: the keys of the three streams are cut into
// splits (local: sinks + window; sparse: groups of selected blocks; HCA: ranges
// of the pooled table, 16,384 rows at a 1M context), one CTA per split computes
// per head a partial online softmax (max, sum, sum p*c over d_c) into the
// workspace, and a combine kernel merges the partials of each stream, adds the
// HCA cumulative-mean path for pos < r-1, and applies the gate softmax.
// Every CTA reads only its keys once for all heads (the latent rows are shared
// by the heads), so the HBM traffic is the decode minimum: window + selected
// blocks + pooled table.
#include "sa_attention.cuh"
#include "mma_util.cuh"

namespace maba {
namespace {

constexpr int KT = 32;           // keys per smem tile (generic kernel)
constexpr int SPLIT_KEYS = 128;  // keys per split (every stream)
constexpr int MAXH = 16;
constexpr int MAXDC = 256;

struct DecodePlan {
    int n_local, n_sparse, n_hca;  // splits per stream
    int blocks_per_split;          // sparse: selected blocks per split
    int64_t nhca;                  // pooled keys visible to the query
    int64_t lo, nsink_extra, nlocal;
    __host__ __device__ int total() const { return n_local + n_sparse + n_hca; }
};

// Plan for a query at position Lkv-1 (Lkv = the visible cache length).
__host__ __device__ inline DecodePlan make_plan(const SaArgs& a, int64_t Lkv) {
    DecodePlan p;
    const int64_t pos = Lkv - 1;
    p.lo = pos - a.window + 1 > 0 ? pos - a.window + 1 : 0;
    const int64_t nsink = a.n_sinks < Lkv ? a.n_sinks : Lkv;
    p.nsink_extra = nsink < p.lo ? nsink : p.lo;
    p.nlocal = p.nsink_extra + (pos - p.lo + 1);
    // a fixed count (independent of the position), so that a capacity-sized launch and the
    // combine agree on which splits hold which stream; splits past the stream's keys are empty
    p.n_local = (int)((a.window + a.n_sinks + SPLIT_KEYS - 1) / SPLIT_KEYS);
    p.blocks_per_split = SPLIT_KEYS / a.block > 0 ? SPLIT_KEYS / a.block : 1;
    p.n_sparse = (a.K + p.blocks_per_split - 1) / p.blocks_per_split;
    p.nhca = 0;
    if (pos >= a.hca_r - 1) {
        p.nhca = (pos + 1) / a.hca_r;
        if (p.nhca > a.NC) p.nhca = a.NC;
    }
    p.n_hca = (int)((p.nhca + SPLIT_KEYS - 1) / SPLIT_KEYS);
    return p;
}

// partial record per (b, split, head): m, l, o[DC]
__device__ __forceinline__ float* part_ptr(float* ws, int64_t b, int split, int h, int nsplit, int H, int DC) {
    return ws + (((size_t)b * nsplit + split) * H + h) * (size_t)(DC + 2);
}

__device__ __forceinline__ int64_t visible_len(const SaArgs& a) { return a.pos_dev ? *a.pos_dev + 1 : a.Lkv; }

template <typename T>
__global__ void sa_decode_partial_kernel_t(SaArgs a, float* ws, int nsplit) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int DC = a.DC, H = a.H;
    int64_t* rows = reinterpret_cast<int64_t*>(smem_raw);
    int* kvalid = reinterpret_cast<int*>(smem_raw + KT * sizeof(int64_t));
    float* qs = reinterpret_cast<float*>(smem_raw + KT * (sizeof(int64_t) + sizeof(int)));  // [H][DC]
    float* ks = qs + H * DC;                                                                // [KT][DC+1]
    const int split = blockIdx.x;
    const int64_t b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = blockDim.x >> 5;
    const int64_t Lkv = visible_len(a);
    const DecodePlan p = make_plan(a, Lkv);
    if (split >= p.total()) return;  // capacity-sized grid: HCA splits past the visible table
    const int64_t pos = Lkv - 1;
    const int64_t nb_kv = (Lkv + a.block - 1) / a.block;
    const T* qh = static_cast<const T*>(a.qhat);
    const T* ckv = static_cast<const T*>(a.ckv);
    const T* hca = static_cast<const T*>(a.hca);

    int stream;
    int64_t k0, k1;
    if (split < p.n_local) {
        stream = 0;
        k0 = (int64_t)split * SPLIT_KEYS;
        k1 = k0 + SPLIT_KEYS < p.nlocal ? k0 + SPLIT_KEYS : p.nlocal;
    } else if (split < p.n_local + p.n_sparse) {
        stream = 1;
        const int s = split - p.n_local;
        k0 = (int64_t)s * p.blocks_per_split * a.block;
        k1 = k0 + (int64_t)p.blocks_per_split * a.block;
        const int64_t kmax = (int64_t)a.K * a.block;
        if (k1 > kmax) k1 = kmax;
    } else {
        stream = 2;
        const int s = split - p.n_local - p.n_sparse;
        k0 = (int64_t)s * SPLIT_KEYS;
        k1 = k0 + SPLIT_KEYS < p.nhca ? k0 + SPLIT_KEYS : p.nhca;
    }

    for (int e = tid; e < H * DC; e += blockDim.x) {
        const int h = e / DC, d = e - (e / DC) * DC;
        qs[e] = load_as<float>(qh + b * a.sq[0] + h * a.sq[2] + d * a.sq[3]);
    }
    constexpr int NPL = MAXDC / 32;
    float m_run = -INFINITY, l_run = 0.f, o_run[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) o_run[i] = 0.f;
    const int h = warp;  // one warp per head (blockDim = 32*H)

    for (int64_t n0 = k0; n0 < k1; n0 += KT) {
        __syncthreads();
        if (tid < KT) {
            const int64_t n = n0 + tid;
            int64_t row = -1;
            if (n < k1) {
                if (stream == 0) {
                    row = n < p.nsink_extra ? n : p.lo + (n - p.nsink_extra);
                } else if (stream == 1) {
                    const int64_t slot = n / a.block, off = n - (n / a.block) * a.block;
                    const int64_t blk = a.top_idx[b * a.st[0] + slot * a.st[2]];
                    const int64_t tok = blk * a.block + off;
                    if (blk >= 0 && blk < nb_kv && tok < Lkv && tok <= pos) row = tok;
                } else {
                    row = n;
                }
            }
            rows[tid] = row;
            kvalid[tid] = row >= 0;
        }
        __syncthreads();
        for (int e = tid; e < KT * DC; e += blockDim.x) {
            const int r = e / DC, d = e - (e / DC) * DC;
            const int64_t row = rows[r];
            float x = 0.f;
            if (row >= 0) {
                x = stream == 2 ? load_as<float>(hca + b * a.sh[0] + row * a.sh[1] + d * a.sh[2])
                                : load_as<float>(ckv + b * a.sc[0] + row * a.sc[1] + d * a.sc[2]);
            }
            ks[r * (DC + 1) + d] = x;
        }
        __syncthreads();
        if (h < H) {
            const float* qr = qs + h * DC;
            const float* kr = ks + lane * (DC + 1);
            float s = 0.f;
            for (int d = 0; d < DC; ++d) s = fmaf(qr[d], kr[d], s);
            if (!kvalid[lane]) s = -INFINITY;
            float mt = s;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            const float mn = fmaxf(m_run, mt);
            if (mn != -INFINITY) {
                const float corr = __expf(m_run - mn);
                const float pr = s == -INFINITY ? 0.f : __expf(s - mn);
                float ps = pr;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
                l_run = l_run * corr + ps;
                m_run = mn;
#pragma unroll
                for (int i = 0; i < NPL; ++i) o_run[i] *= corr;
                for (int j = 0; j < KT; ++j) {
                    const float pj = __shfl_sync(0xffffffffu, pr, j);
                    if (pj != 0.f) {
                        const float* kj = ks + j * (DC + 1);
#pragma unroll
                        for (int i = 0; i < NPL; ++i) {
                            const int d = lane + 32 * i;
                            if (d < DC) o_run[i] = fmaf(pj, kj[d], o_run[i]);
                        }
                    }
                }
            }
        }
    }
    (void)nwarps;
    if (h < H) {
        float* pp = part_ptr(ws, b, split, h, nsplit, H, DC);
        if (lane == 0) {
            pp[0] = m_run;
            pp[1] = l_run;
        }
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int d = lane + 32 * i;
            if (d < DC) pp[2 + d] = o_run[i];
        }
    }
}

template <typename T>
__global__ void sa_decode_combine_kernel(SaArgs a, const float* ws, int nsplit) {
    const int DC = a.DC, H = a.H;
    const int64_t b = blockIdx.x;
    const int lane = threadIdx.x & 31, h = threadIdx.x >> 5;
    if (h >= H) return;
    const int64_t Lkv = visible_len(a);
    const DecodePlan p = make_plan(a, Lkv);
    const int64_t pos = Lkv - 1;
    constexpr int NPL = MAXDC / 32;
    float res[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) res[i] = 0.f;
    const T* gp = static_cast<const T*>(a.gate);
    const T* gr = a.gate4d ? gp + b * a.sg[0] + h * a.sg[1] : gp + b * a.sg[0];
    const int64_t gs = a.gate4d ? a.sg[3] : a.sg[2];
    float g0 = load_as<float>(gr), g1 = load_as<float>(gr + gs), g2 = load_as<float>(gr + 2 * gs);
    const float mg = fmaxf(g0, fmaxf(g1, g2));
    const float e0 = expf(g0 - mg), e1 = expf(g1 - mg), e2 = expf(g2 - mg);
    const float gsum = e0 + e1 + e2;
    const float gate[3] = {e0 / gsum, e1 / gsum, e2 / gsum};
    const int first[3] = {0, p.n_local, p.n_local + p.n_sparse};
    const int cnt[3] = {p.n_local, p.n_sparse, p.n_hca};
    for (int s = 0; s < 3; ++s) {
        if (s == 2 && pos < a.hca_r - 1) {
            // cumulative mean of the latent prefix (sparse_attention.py:189-199)
            const T* ckv = static_cast<const T*>(a.ckv) + b * a.sc[0];
#pragma unroll
            for (int i = 0; i < NPL; ++i) {
                const int d = lane + 32 * i;
                if (d < DC) {
                    float acc = 0.f;
                    for (int64_t j = 0; j <= pos; ++j) acc += load_as<float>(ckv + j * a.sc[1] + d * a.sc[2]);
                    res[i] += gate[2] * (acc / float(pos + 1));
                }
            }
            continue;
        }
        float M = -INFINITY;
        for (int k = 0; k < cnt[s]; ++k) M = fmaxf(M, part_ptr(const_cast<float*>(ws), b, first[s] + k, h, nsplit, H, DC)[0]);
        if (M == -INFINITY) continue;
        float Lsum = 0.f, O[NPL];
#pragma unroll
        for (int i = 0; i < NPL; ++i) O[i] = 0.f;
        for (int k = 0; k < cnt[s]; ++k) {
            const float* pp = part_ptr(const_cast<float*>(ws), b, first[s] + k, h, nsplit, H, DC);
            if (pp[0] == -INFINITY) continue;
            const float f = __expf(pp[0] - M);
            Lsum += f * pp[1];
#pragma unroll
            for (int i = 0; i < NPL; ++i) {
                const int d = lane + 32 * i;
                if (d < DC) O[i] += f * pp[2 + d];
            }
        }
        if (Lsum > 0.f) {
            const float w = gate[s] / Lsum;
#pragma unroll
            for (int i = 0; i < NPL; ++i) res[i] += w * O[i];
        }
    }
    T* out = static_cast<T*>(a.out);
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
        const int d = lane + 32 * i;
        if (d < DC) store_from<T, float>(out + b * a.so[0] + h * a.so[2] + d * a.so[3], res[i]);
    }
}

// ---------------------------------------------------------------------------
// 16-bit tensor-core split kernel: one split of up to SPLIT_KEYS keys per CTA,
// 4 warps of 32 keys each.  The split's latent (or pooled) rows are gathered
// into shared memory with 16-byte loads, all issued before the first use; the
// heads are the 16 rows of the mma.sync tiles (zero rows past H):
//   S = Qhat K^T (16 x 32 per warp, K = d_c), masked, softmax numerator in fp32,
//   P (16-bit) -> shared, O = P V (16 x d_c per warp);
// the four warps' (max, sum, O) are merged through shared memory into one
// partial record per head.  Rows are padded by 8 elements, so the ldmatrix
// reads of 8 rows hit 8 different bank groups.
// ---------------------------------------------------------------------------
constexpr int kMmaWarps = 4;
constexpr int kMmaDC = 128;
constexpr int kMmaLD = kMmaDC + 8;
constexpr int kPLD = 32 + 8;

template <typename T>
__global__ void __launch_bounds__(32 * kMmaWarps) sa_decode_mma_kernel(SaArgs a, float* ws, int nsplit) {
    constexpr int DC = kMmaDC, LD = kMmaLD, CPR = DC / 8;
    constexpr int NTHR = 32 * kMmaWarps;
    constexpr int MAXL = SPLIT_KEYS * CPR / NTHR;  // 16 chunks per thread
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* ks = reinterpret_cast<T*>(smem_raw);                           // [SPLIT_KEYS][LD]; later the O merge area
    T* qs = ks + SPLIT_KEYS * LD;                                     // [16][LD]
    T* ps = qs + 16 * LD;                                             // [warps][16][kPLD]
    float* mw = reinterpret_cast<float*>(ps + kMmaWarps * 16 * kPLD);  // [warps][16]
    float* lw = mw + kMmaWarps * 16;                                  // [warps][16]
    int64_t* rows = reinterpret_cast<int64_t*>(lw + kMmaWarps * 16);  // [SPLIT_KEYS]
    const int H = a.H;
    const int split = blockIdx.x;
    const int64_t b = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t Lkv = visible_len(a);
    const DecodePlan p = make_plan(a, Lkv);
    if (split >= p.total()) return;
    const int64_t pos = Lkv - 1;
    const int64_t nb_kv = (Lkv + a.block - 1) / a.block;
    int stream;
    int64_t k0, k1;
    if (split < p.n_local) {
        stream = 0;
        k0 = (int64_t)split * SPLIT_KEYS;
        k1 = k0 + SPLIT_KEYS < p.nlocal ? k0 + SPLIT_KEYS : p.nlocal;
    } else if (split < p.n_local + p.n_sparse) {
        stream = 1;
        k0 = (int64_t)(split - p.n_local) * p.blocks_per_split * a.block;
        k1 = k0 + (int64_t)p.blocks_per_split * a.block;
        const int64_t kmax = (int64_t)a.K * a.block;
        if (k1 > kmax) k1 = kmax;
    } else {
        stream = 2;
        k0 = (int64_t)(split - p.n_local - p.n_sparse) * SPLIT_KEYS;
        k1 = k0 + SPLIT_KEYS < p.nhca ? k0 + SPLIT_KEYS : p.nhca;
    }
    const int nk = k1 > k0 ? (int)(k1 - k0) : 0;
    // key row of split key i (-1: none); the sparse stream reads its block from the top-k list
    auto row_of = [&](int i) -> int64_t {
        if (i >= nk) return -1;
        const int64_t n = k0 + i;
        if (stream == 0) return n < p.nsink_extra ? n : p.lo + (n - p.nsink_extra);
        if (stream == 1) {
            const int64_t slot = n / a.block, off = n - slot * a.block;
            const int64_t blk = a.top_idx[b * a.st[0] + slot * a.st[2]];
            const int64_t tok = blk * a.block + off;
            return (blk >= 0 && blk < nb_kv && tok <= pos) ? tok : -1;
        }
        return n;
    };
    // keys and queries in one round of loads: this thread's 16-byte key chunks (chunk e of
    // the tile is key e / CPR, columns (e % CPR) * 8) and its query elements
    {
        const T* base = stream == 2 ? static_cast<const T*>(a.hca) + b * a.sh[0] : static_cast<const T*>(a.ckv) + b * a.sc[0];
        const int64_t rs = stream == 2 ? a.sh[1] : a.sc[1];
        uint4 v[MAXL];
#pragma unroll
        for (int j = 0; j < MAXL; ++j) {
            const int e = tid + j * NTHR;
            const int64_t row = row_of(e / CPR);
            if ((e % CPR) == 0) rows[e / CPR] = row;
            v[j] = row >= 0 ? *reinterpret_cast<const uint4*>(base + row * rs + (e % CPR) * 8) : make_uint4(0u, 0u, 0u, 0u);
        }
        const T* qh = static_cast<const T*>(a.qhat);
        const bool qvec = a.sq[3] == 1 && (a.sq[2] % 8) == 0 && (a.sq[0] % 8) == 0 &&
                          (reinterpret_cast<uintptr_t>(qh) & 15u) == 0;
        if (qvec) {
            for (int e = tid; e < 16 * CPR; e += NTHR) {
                const int r = e / CPR, c = e - r * CPR;
                const uint4 q = r < H ? *reinterpret_cast<const uint4*>(qh + b * a.sq[0] + r * a.sq[2] + c * 8)
                                      : make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(qs + r * LD + c * 8) = q;
            }
        } else {
            for (int e = tid; e < 16 * DC; e += NTHR) {
                const int r = e / DC, d = e - r * DC;
                qs[r * LD + d] = r < H ? qh[b * a.sq[0] + r * a.sq[2] + d * a.sq[3]] : Cvt<T>::from_f(0.f);
            }
        }
#pragma unroll
        for (int j = 0; j < MAXL; ++j) {
            const int e = tid + j * NTHR;
            *reinterpret_cast<uint4*>(ks + (e / CPR) * LD + (e % CPR) * 8) = v[j];
        }
    }
    __syncthreads();
    // ---- scores of this warp's 32 keys
    const T* kw = ks + warp * 32 * LD;
    float sacc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c) sacc[n][c] = 0.f;
    warp_mma<T, false, false, 4>(sacc, qs, LD, kw, LD, DC, lane);
    const int g = lane >> 2, t2 = (lane & 3) * 2;
    float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const int key = warp * 32 + n * 8 + t2 + c;
            const bool ok = key < nk && rows[key] >= 0;
            if (!ok) {
                sacc[n][c] = -INFINITY;
                sacc[n][c + 2] = -INFINITY;
            }
            m0 = fmaxf(m0, sacc[n][c]);
            m1 = fmaxf(m1, sacc[n][c + 2]);
        }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    float l0 = 0.f, l1 = 0.f;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            const float p0 = sacc[n][c] == -INFINITY ? 0.f : __expf(sacc[n][c] - m0);
            const float p1 = sacc[n][c + 2] == -INFINITY ? 0.f : __expf(sacc[n][c + 2] - m1);
            sacc[n][c] = p0;
            sacc[n][c + 2] = p1;
            l0 += p0;
            l1 += p1;
        }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, o);
        l1 += __shfl_xor_sync(0xffffffffu, l1, o);
    }
    T* pw = ps + warp * 16 * kPLD;
    store_acc16<T, 4>(pw, kPLD, sacc, lane);
    if ((lane & 3) == 0) {
        mw[warp * 16 + g] = m0;
        mw[warp * 16 + g + 8] = m1;
        lw[warp * 16 + g] = l0;
        lw[warp * 16 + g + 8] = l1;
    }
    __syncwarp();
    // ---- O = P V for this warp's keys
    float oacc[DC / 8][4];
#pragma unroll
    for (int n = 0; n < DC / 8; ++n)
#pragma unroll
        for (int c = 0; c < 4; ++c) oacc[n][c] = 0.f;
    warp_mma<T, false, true, DC / 8>(oacc, pw, kPLD, kw, LD, 32, lane);
    __syncthreads();  // every warp is done with the key tile: reuse it for the O merge
    float* om = reinterpret_cast<float*>(ks);  // [warps][16][DC]
#pragma unroll
    for (int n = 0; n < DC / 8; ++n) {
        float* r0 = om + (warp * 16 + g) * DC + n * 8 + t2;
        float* r1 = om + (warp * 16 + g + 8) * DC + n * 8 + t2;
        r0[0] = oacc[n][0];
        r0[1] = oacc[n][1];
        r1[0] = oacc[n][2];
        r1[1] = oacc[n][3];
    }
    __syncthreads();
    for (int e = tid; e < H * DC; e += NTHR) {
        const int h = e / DC, d = e - h * DC;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kMmaWarps; ++w) M = fmaxf(M, mw[w * 16 + h]);
        float L = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kMmaWarps; ++w) {
                const float mwv = mw[w * 16 + h];
                const float f = mwv == -INFINITY ? 0.f : __expf(mwv - M);
                L = fmaf(f, lw[w * 16 + h], L);
                O = fmaf(f, om[(w * 16 + h) * DC + d], O);
            }
        }
        float* pp = part_ptr(ws, b, split, h, nsplit, H, DC);
        if (d == 0) {
            pp[0] = M;
            pp[1] = L;
        }
        pp[2 + d] = O;
    }
}

// Combine of the partial records: one CTA per (head, 32-dimension slice, batch
// row), 8 warps, lane = dimension.  Per stream the maximum of the partial maxima
// is found first (every warp reads all of them, 32 at a time), so the weighted
// sums over the splits (warp w: splits w, w+8, ...) have no dependence between
// iterations and their loads overlap; the warps' sums meet in shared memory and
// the three streams are superposed with the gate softmax (and the HCA cumulative
// mean for pos < r-1).
constexpr int kCombWarps = 8;

template <typename T>
__global__ void __launch_bounds__(32 * kCombWarps) sa_decode_combine2_kernel(SaArgs a, const float* ws, int nsplit) {
    const int DC = a.DC, H = a.H;
    const int h = blockIdx.x;
    const int d = blockIdx.y * 32 + (threadIdx.x & 31);
    const int64_t b = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __shared__ float wl[kCombWarps], wo[kCombWarps][32];
    const int64_t Lkv = visible_len(a);
    const DecodePlan p = make_plan(a, Lkv);
    const int64_t pos = Lkv - 1;
    const T* gp = static_cast<const T*>(a.gate);
    const T* gr = a.gate4d ? gp + b * a.sg[0] + h * a.sg[1] : gp + b * a.sg[0];
    const int64_t gs = a.gate4d ? a.sg[3] : a.sg[2];
    const float g0 = load_as<float>(gr), g1 = load_as<float>(gr + gs), g2 = load_as<float>(gr + 2 * gs);
    const float mg = fmaxf(g0, fmaxf(g1, g2));
    const float e0 = expf(g0 - mg), e1 = expf(g1 - mg), e2 = expf(g2 - mg);
    const float gsum = e0 + e1 + e2;
    const float gate[3] = {e0 / gsum, e1 / gsum, e2 / gsum};
    const int first[3] = {0, p.n_local, p.n_local + p.n_sparse};
    const int cnt[3] = {p.n_local, p.n_sparse, p.n_hca};
    const size_t rec = DC + 2;
    const float* base = ws + ((size_t)b * nsplit * H + h) * rec;  // record of split k: base + k * H * rec
    const size_t kstride = (size_t)H * rec;
    float res = 0.f;
    for (int s = 0; s < 3; ++s) {
        if (s == 2 && pos < a.hca_r - 1) {
            // cumulative mean of the latent prefix (sparse_attention.py:189-199)
            if (warp == 0 && d < DC) {
                const T* ckv = static_cast<const T*>(a.ckv) + b * a.sc[0];
                float acc = 0.f;
                for (int64_t j = 0; j <= pos; ++j) acc += load_as<float>(ckv + j * a.sc[1] + d * a.sc[2]);
                res += gate[2] * (acc / float(pos + 1));
            }
            continue;
        }
        const float* sb = base + (size_t)first[s] * kstride;
        float M = -INFINITY;
        for (int k = lane; k < cnt[s]; k += 32) M = fmaxf(M, sb[k * kstride]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        if (M == -INFINITY) continue;  // the same in every warp
        float L = 0.f, O = 0.f;
#pragma unroll 8
        for (int k = warp; k < cnt[s]; k += kCombWarps) {
            const float* pp = sb + k * kstride;
            const float mk = pp[0];
            const float f = mk == -INFINITY ? 0.f : __expf(mk - M);
            L = fmaf(f, pp[1], L);
            if (d < DC) O = fmaf(f, pp[2 + d], O);
        }
        __syncthreads();
        if (lane == 0) wl[warp] = L;
        wo[warp][lane] = O;
        __syncthreads();
        if (warp == 0) {
            float LL = 0.f, OO = 0.f;
#pragma unroll
            for (int w = 0; w < kCombWarps; ++w) {
                LL += wl[w];
                OO += wo[w][lane];
            }
            if (LL > 0.f) res += gate[s] * OO / LL;
        }
    }
    if (warp == 0 && d < DC) store_from<T, float>(static_cast<T*>(a.out) + b * a.so[0] + h * a.so[2] + d * a.so[3], res);
}

bool tile_path_ok(const SaArgs& a, int es) {
    if (es != 2 || a.DC != kMmaDC || a.H > 16) return false;
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (a.sc[2] != 1 || (a.sc[1] * es) % 16 || (a.sc[0] * es) % 16 || !al(a.ckv)) return false;
    if (a.hca != nullptr && (a.sh[2] != 1 || (a.sh[1] * es) % 16 || (a.sh[0] * es) % 16 || !al(a.hca))) return false;
    return true;
}

// Splits of the launch: exact for a host-known length, capacity-sized (every
// split the largest visible table could need) for a device-held position.
int decode_splits(const SaArgs& a) {
    if (a.pos_dev == nullptr) return make_plan(a, a.Lkv).total();
    DecodePlan p = make_plan(a, a.Lkv);  // a.Lkv = cache capacity
    const int64_t ncap = a.NC;
    p.n_hca = (int)((ncap + SPLIT_KEYS - 1) / SPLIT_KEYS);
    return p.n_local + p.n_sparse + p.n_hca;
}

template <typename T>
int launch_decode(SaArgs& a, int64_t B, cudaStream_t s) {
    const int nsplit = decode_splits(a);
    const size_t need = (size_t)B * nsplit * a.H * (a.DC + 2) * sizeof(float);
    if (a.workspace == nullptr || a.workspace_bytes < need)
        return set_error(MABA_ERR_WORKSPACE, "sa_attention(decode): workspace of %zu bytes required, got %zu", need,
                         a.workspace_bytes);
    float* ws = static_cast<float*>(a.workspace);
    bool done = false;
    if constexpr (sizeof(T) == 2) {
        if (tile_path_ok(a, (int)sizeof(T))) {
            const size_t smem = sizeof(T) * ((size_t)SPLIT_KEYS * kMmaLD + 16 * kMmaLD + kMmaWarps * 16 * kPLD) +
                                sizeof(float) * 2 * kMmaWarps * 16 + sizeof(int64_t) * SPLIT_KEYS;
            auto kern = sa_decode_mma_kernel<T>;
            if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            kern<<<dim3((unsigned)nsplit, (unsigned)B), 32 * kMmaWarps, smem, s>>>(a, ws, nsplit);
            done = true;
        }
    }
    if (!done) {
        const size_t smem = KT * (sizeof(int64_t) + sizeof(int)) + sizeof(float) * ((size_t)a.H * a.DC + (size_t)KT * (a.DC + 1));
        auto k1 = sa_decode_partial_kernel_t<T>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        k1<<<dim3((unsigned)nsplit, (unsigned)B), 32 * a.H, smem, s>>>(a, ws, nsplit);
    }
    MABA_TRY(check_launch("sa_attention(decode partial)"));
    sa_decode_combine2_kernel<T><<<dim3((unsigned)a.H, (unsigned)ceil_div(a.DC, 32), (unsigned)B), 32 * kCombWarps, 0,
                                   s>>>(a, ws, nsplit);
    return check_launch("sa_attention(decode combine)");
}

}  // namespace

bool sa_attention_decode_supported(const SaArgs& a) {
    return a.Lq == 1 && a.H <= MAXH && a.DC <= MAXDC && a.Lkv > 0;
}

size_t sa_attention_decode_workspace(int64_t B, int64_t Lq, int64_t Lkv, int64_t H, int64_t DC, int64_t K,
                                     int32_t block, int32_t window, int32_t n_sinks, int32_t hca_r) {
    if (Lq != 1 || Lkv <= 0 || block <= 0 || hca_r <= 0) return 0;
    SaArgs a{};
    a.Lq = 1; a.Lkv = Lkv; a.NC = Lkv / hca_r; a.H = (int)H; a.DC = (int)DC; a.K = (int)K;
    a.window = window; a.n_sinks = n_sinks; a.block = block; a.hca_r = hca_r;
    return (size_t)B * decode_splits(a) * H * (DC + 2) * sizeof(float);
}

size_t sa_attention_decode_at_workspace(int64_t B, int64_t Lcap, int64_t NCcap, int64_t H, int64_t DC, int64_t K,
                                        int32_t block, int32_t window, int32_t n_sinks, int32_t hca_r) {
    SaArgs a{};
    a.Lq = 1; a.Lkv = Lcap; a.NC = NCcap; a.H = (int)H; a.DC = (int)DC; a.K = (int)K;
    a.window = window; a.n_sinks = n_sinks; a.block = block; a.hca_r = hca_r;
    int64_t one = 0;
    a.pos_dev = &one;  // any non-null: capacity-sized plan
    return (size_t)B * decode_splits(a) * H * (DC + 2) * sizeof(float);
}

int sa_attention_decode(SaArgs& a, int64_t B, int dtype, cudaStream_t s) {
    return MABA_DISPATCH_FLOAT(dtype, "sa_attention(decode)", [&] {
        if constexpr (sizeof(T) == 8) return set_error(MABA_ERR_UNSUPPORTED, "sa_attention(decode): float64");
        else return launch_decode<T>(a, B, s);
    });
}

}  // namespace maba
