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

namespace maba {
namespace {

constexpr int KT = 32;           // keys per smem tile
constexpr int SPLIT_KEYS = 256;  // keys per split (HCA / sparse)
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
    p.n_local = 1;
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
        stream = 0; k0 = 0; k1 = p.nlocal;
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
    const size_t smem = KT * (sizeof(int64_t) + sizeof(int)) + sizeof(float) * ((size_t)a.H * a.DC + (size_t)KT * (a.DC + 1));
    auto k1 = sa_decode_partial_kernel_t<T>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k1<<<dim3((unsigned)nsplit, (unsigned)B), 32 * a.H, smem, s>>>(a, ws, nsplit);
    MABA_TRY(check_launch("sa_attention(decode partial)"));
    sa_decode_combine_kernel<T><<<(unsigned)B, 32 * a.H, 0, s>>>(a, ws, nsplit);
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
