// MABA-SA three-stream attention in the latent (MLA-absorbed) space.
//
// Reference math, maba_sparse/layers/sparse_attention.py:
//   local  (:79-105)  softmax over keys j <= pos with pos-j < window or j < n_sinks
//   sparse (:107-171) softmax over the tokens of the selected blocks that are <= pos
//   hca    (:173-219) pos < r-1: v_up(mean(c[0..pos]));  otherwise softmax over the
//                     pooled complete blocks j with (j+1)r-1 <= pos
//   superposition (:274-275, common.py:406-438): softmax(gate) weighted sum.
// Keys are K_h = W_uk,h c and values V_h = W_uv,h c; with qhat_h = scale*W_uk,h^T q_h
// the scores are qhat_h . c and every stream output is W_uv,h (sum_j p_j c_j), so all
// streams (and their gate-weighted sum) are computed on the shared d_c latent rows
// and the caller applies W_uv once.  A stream with no valid key contributes 0
// (the reference's nan_to_num of an all -inf softmax).
//
// This file holds the exact CUDA-core kernel (fp32 math for fp32/fp16/bf16,
// fp64 for fp64): one CTA per query token, one warp per head, keys streamed in
// tiles of 32 latent rows through shared memory with an online softmax per
// (stream, head).  The tensor-core path for 16-bit inputs is sa_attention_mma.cu.
#include "common.cuh"
#include "sa_attention.cuh"

namespace maba {
namespace {

constexpr int KT = 32;  // keys per tile

template <typename ACC>
__device__ __forceinline__ ACC warp_max(ACC v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ACC x = __shfl_xor_sync(0xffffffffu, v, o);
        v = x > v ? x : v;
    }
    return v;
}
template <typename ACC>
__device__ __forceinline__ ACC warp_sum(ACC v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

template <typename T, typename ACC, int DCMAX>
__global__ void sa_attention_simt_kernel(SaArgs a) {
    constexpr int NPL = DCMAX / 32;  // latent dims per lane
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int DC = a.DC, H = a.H;
    int64_t* rows = reinterpret_cast<int64_t*>(smem_raw);            // [KT] latent row per tile slot
    int* kvalid = reinterpret_cast<int*>(smem_raw + KT * sizeof(int64_t));
    ACC* qs = reinterpret_cast<ACC*>(smem_raw + KT * (sizeof(int64_t) + sizeof(int)));  // [H][DC]
    ACC* ks = qs + (size_t)H * DC;                                     // [KT][DC+1]

    const int64_t t = blockIdx.x, b = blockIdx.y;
    const int64_t pos = a.Lkv - a.Lq + t;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nwarps = blockDim.x >> 5;
    const T* qh = static_cast<const T*>(a.qhat);
    const T* ckv = static_cast<const T*>(a.ckv);
    const T* hca = static_cast<const T*>(a.hca);
    const int64_t* tix = a.top_idx;

    for (int e = tid; e < H * DC; e += blockDim.x) {
        const int h = e / DC, d = e - (e / DC) * DC;
        qs[e] = load_as<ACC>(qh + b * a.sq[0] + t * a.sq[1] + h * a.sq[2] + d * a.sq[3]);
    }

    // gate weights for the heads of this warp (computed when needed)
    ACC res[2][NPL];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int m = 0; m < NPL; ++m) res[hh][m] = 0;

    const int64_t nb_kv = (a.Lkv + a.block - 1) / a.block;
    const int64_t lo = pos - a.window + 1 > 0 ? pos - a.window + 1 : 0;
    const int64_t nsink = a.n_sinks < a.Lkv ? a.n_sinks : a.Lkv;
    const int64_t nsink_extra = nsink < lo ? nsink : lo;  // sinks outside the window
    const int64_t nlocal = nsink_extra + (pos - lo + 1);
    const int64_t nsparse = (int64_t)a.K * a.block;
    const bool hca_early = pos < a.hca_r - 1;
    int64_t nhca = 0;
    if (!hca_early) {
        nhca = (pos + 1) / a.hca_r;
        if (nhca > a.NC) nhca = a.NC;
    }

    for (int stream = 0; stream < 3; ++stream) {
        int64_t nkeys = stream == 0 ? nlocal : (stream == 1 ? nsparse : (hca_early ? 0 : nhca));
        ACC m_run[2], l_run[2], o_run[2][NPL];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            m_run[hh] = -INFINITY;
            l_run[hh] = 0;
#pragma unroll
            for (int mm = 0; mm < NPL; ++mm) o_run[hh][mm] = 0;
        }
        for (int64_t n0 = 0; n0 < nkeys; n0 += KT) {
            __syncthreads();
            // key row of each tile slot
            if (tid < KT) {
                const int64_t n = n0 + tid;
                int64_t row = -1;
                if (n < nkeys) {
                    if (stream == 0) {
                        row = n < nsink_extra ? n : lo + (n - nsink_extra);
                    } else if (stream == 1) {
                        const int64_t slot = n / a.block, off = n - (n / a.block) * a.block;
                        const int64_t blk = tix[b * a.st[0] + t * a.st[1] + slot * a.st[2]];
                        const int64_t tok = blk * a.block + off;
                        if (blk >= 0 && blk < nb_kv && tok < a.Lkv && tok <= pos) row = tok;
                    } else {
                        row = n;
                    }
                }
                kvalid[tid] = row >= 0 ? 1 : 0;
                rows[tid] = row;
            }
            __syncthreads();
            for (int e = tid; e < KT * DC; e += blockDim.x) {
                const int r = e / DC, d = e - (e / DC) * DC;
                const int64_t row = rows[r];
                ACC x = 0;
                if (row >= 0) {
                    if (stream == 2) x = load_as<ACC>(hca + b * a.sh[0] + row * a.sh[1] + d * a.sh[2]);
                    else x = load_as<ACC>(ckv + b * a.sc[0] + row * a.sc[1] + d * a.sc[2]);
                }
                ks[r * (DC + 1) + d] = x;
            }
            __syncthreads();
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int h = warp + hh * nwarps;
                if (h >= H) continue;
                const ACC* qr = qs + (size_t)h * DC;
                const ACC* kr = ks + (size_t)lane * (DC + 1);
                ACC s = 0;
                for (int d = 0; d < DC; ++d) s += qr[d] * kr[d];
                if (!kvalid[lane]) s = -INFINITY;
                const ACC mt = warp_max(s);
                const ACC mnew = mt > m_run[hh] ? mt : m_run[hh];
                if (mnew == -INFINITY) continue;  // nothing valid yet
                const ACC corr = exp_acc<ACC>(m_run[hh] - mnew);
                const ACC p = s == -INFINITY ? ACC(0) : exp_acc<ACC>(s - mnew);
                l_run[hh] = l_run[hh] * corr + warp_sum(p);
                m_run[hh] = mnew;
#pragma unroll
                for (int mm = 0; mm < NPL; ++mm) o_run[hh][mm] *= corr;
                for (int j = 0; j < KT; ++j) {
                    const ACC pj = __shfl_sync(0xffffffffu, p, j);
                    if (pj != ACC(0)) {
                        const ACC* kj = ks + (size_t)j * (DC + 1);
#pragma unroll
                        for (int mm = 0; mm < NPL; ++mm) {
                            const int d = lane + 32 * mm;
                            if (d < DC) o_run[hh][mm] += pj * kj[d];
                        }
                    }
                }
            }
        }
        // fold this stream into the gate-weighted result
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int h = warp + hh * nwarps;
            if (h >= H) continue;
            const T* gp = static_cast<const T*>(a.gate);
            const T* gr = a.gate4d ? gp + b * a.sg[0] + h * a.sg[1] + t * a.sg[2] : gp + b * a.sg[0] + t * a.sg[1];
            const int64_t gs = a.gate4d ? a.sg[3] : a.sg[2];
            ACC g0 = load_as<ACC>(gr), g1 = load_as<ACC>(gr + gs), g2 = load_as<ACC>(gr + 2 * gs);
            ACC mg = g0 > g1 ? g0 : g1;
            mg = mg > g2 ? mg : g2;
            ACC e0 = exp_acc<ACC>(g0 - mg), e1 = exp_acc<ACC>(g1 - mg), e2 = exp_acc<ACC>(g2 - mg);
            const ACC gsel = (stream == 0 ? e0 : (stream == 1 ? e1 : e2)) / (e0 + e1 + e2);
            if (stream == 2 && hca_early) {
                // mean of the latent prefix c[0..pos]
#pragma unroll
                for (int mm = 0; mm < NPL; ++mm) {
                    const int d = lane + 32 * mm;
                    if (d < DC) {
                        ACC s = 0;
                        for (int64_t j = 0; j <= pos; ++j) s += load_as<ACC>(ckv + b * a.sc[0] + j * a.sc[1] + d * a.sc[2]);
                        res[hh][mm] += gsel * (s / ACC(pos + 1));
                    }
                }
            } else if (l_run[hh] > ACC(0)) {
                const ACC inv = ACC(1) / l_run[hh];
#pragma unroll
                for (int mm = 0; mm < NPL; ++mm) res[hh][mm] += gsel * (o_run[hh][mm] * inv);
            }
        }
    }
    T* out = static_cast<T*>(a.out);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int h = warp + hh * nwarps;
        if (h >= H) continue;
#pragma unroll
        for (int mm = 0; mm < NPL; ++mm) {
            const int d = lane + 32 * mm;
            if (d < DC) store_from<T, ACC>(out + b * a.so[0] + t * a.so[1] + h * a.so[2] + d * a.so[3], res[hh][mm]);
        }
    }
}

template <typename T>
int launch_simt(SaArgs& a, int64_t B, cudaStream_t s) {
    using ACC = typename std::conditional<sizeof(T) == 8, double, float>::type;
    if (a.H > 32) return set_error(MABA_ERR_UNSUPPORTED, "sa_attention: n_heads=%d > 32", a.H);
    if (a.DC > 256) return set_error(MABA_ERR_UNSUPPORTED, "sa_attention: d_c=%d > 256", a.DC);
    const int nwarps = a.H < 16 ? a.H : 16;
    const size_t smem = sizeof(ACC) * ((size_t)a.H * a.DC + (size_t)KT * (a.DC + 1)) +
                        KT * (sizeof(int64_t) + sizeof(int));
    dim3 grid((unsigned)a.Lq, (unsigned)B);
    if (a.DC <= 128) {
        auto kern = sa_attention_simt_kernel<T, ACC, 128>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, 32 * nwarps, smem, s>>>(a);
    } else {
        auto kern = sa_attention_simt_kernel<T, ACC, 256>;
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, 32 * nwarps, smem, s>>>(a);
    }
    return check_launch("sa_attention(simt)");
}

}  // namespace

int sa_attention_simt(SaArgs& a, int64_t B, int dtype, cudaStream_t s) {
    return MABA_DISPATCH_FLOAT(dtype, "sa_attention", [&] { return launch_simt<T>(a, B, s); });
}

}  // namespace maba

using namespace maba;

extern "C" size_t maba_sa_attention_workspace_size(int32_t dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t H,
                                                   int64_t d_c, int64_t K, int32_t window, int32_t n_sinks,
                                                   int32_t block_size, int32_t hca_r) {
    return sa_attention_workspace_bytes(dtype, B, Lq, Lkv, H, d_c, K, block_size, window, n_sinks, hca_r);
}

extern "C" int maba_sa_attention(const maba_tensor* qhat, const maba_tensor* c_kv, const maba_tensor* hca,
                                 const maba_tensor* top_idx, const maba_tensor* gate, const maba_tensor* out,
                                 int32_t window, int32_t n_sinks, int32_t block_size, int32_t hca_r, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    if (!present(qhat) || qhat->ndim != 4)
        return set_error(MABA_ERR_INVALID, "sa_attention: qhat must be [B, Lq, H, d_c]");
    const int64_t B = qhat->shape[0], Lq = qhat->shape[1], H = qhat->shape[2], DC = qhat->shape[3];
    if (!present(c_kv) || c_kv->ndim != 3) return set_error(MABA_ERR_INVALID, "sa_attention: c_kv must be [B, Lkv, d_c]");
    const int64_t Lkv = c_kv->shape[1];
    if (c_kv->shape[0] != B || c_kv->shape[2] != DC)
        return set_error(MABA_ERR_INVALID, "sa_attention: c_kv shape mismatch");
    if (Lkv < Lq) return set_error(MABA_ERR_INVALID, "sa_attention: Lkv (%lld) < Lq (%lld)", (long long)Lkv, (long long)Lq);
    if (window <= 0 || n_sinks < 0 || block_size <= 0 || hca_r <= 0)
        return set_error(MABA_ERR_INVALID, "sa_attention: window/block/hca_r must be positive");
    const int64_t NC = Lkv / hca_r;
    if (NC > 0) {
        const int64_t sh[3] = {B, NC, DC};
        MABA_TRY(expect_shape(hca, "sa_attention: hca", 3, sh));
        MABA_TRY(expect_dtype(hca, "sa_attention: hca", qhat->dtype));
    }
    if (!present(top_idx) || top_idx->ndim != 3 || top_idx->shape[0] != B || top_idx->shape[1] != Lq)
        return set_error(MABA_ERR_INVALID, "sa_attention: top_idx must be [B, Lq, K]");
    MABA_TRY(expect_dtype(top_idx, "sa_attention: top_idx", MABA_I64));
    const int64_t K = top_idx->shape[2];
    if (!present(gate)) return set_error(MABA_ERR_INVALID, "sa_attention: gate is required");
    MABA_TRY(expect_dtype(gate, "sa_attention: gate", qhat->dtype));
    int gate4d = 0;
    if (gate->ndim == 3) {
        const int64_t g3[3] = {B, Lq, 3};
        MABA_TRY(expect_shape(gate, "sa_attention: gate", 3, g3));
    } else if (gate->ndim == 4) {
        const int64_t g4[4] = {B, H, Lq, 3};
        MABA_TRY(expect_shape(gate, "sa_attention: gate", 4, g4));
        gate4d = 1;
    } else {
        return set_error(MABA_ERR_INVALID, "sa_attention: gate must be 3D or 4D");
    }
    const int64_t so[4] = {B, Lq, H, DC};
    MABA_TRY(expect_shape(out, "sa_attention: out", 4, so));
    MABA_TRY(expect_dtype(out, "sa_attention: out", qhat->dtype));
    MABA_TRY(expect_dtype(c_kv, "sa_attention: c_kv", qhat->dtype));

    SaArgs a{};
    a.qhat = qhat->data; a.ckv = c_kv->data; a.hca = NC > 0 ? hca->data : nullptr;
    a.top_idx = static_cast<const int64_t*>(top_idx->data);
    a.gate = gate->data; a.out = out->data;
    for (int i = 0; i < 4; ++i) { a.sq[i] = qhat->stride[i]; a.so[i] = out->stride[i]; a.sg[i] = i < gate->ndim ? gate->stride[i] : 0; }
    for (int i = 0; i < 3; ++i) {
        a.sc[i] = c_kv->stride[i]; a.st[i] = top_idx->stride[i]; a.sh[i] = NC > 0 ? hca->stride[i] : 0;
    }
    a.Lq = Lq; a.Lkv = Lkv; a.NC = NC; a.H = (int)H; a.DC = (int)DC; a.K = (int)K;
    a.window = window; a.n_sinks = n_sinks; a.block = block_size; a.hca_r = hca_r; a.gate4d = gate4d;
    a.workspace = workspace; a.workspace_bytes = workspace_bytes;
    if (B == 0 || Lq == 0) return MABA_OK;
    return sa_attention_dispatch(a, B, qhat->dtype, as_stream(stream));
}

extern "C" size_t maba_sa_attention_decode_at_workspace_size(int64_t B, int64_t Lcap, int64_t NCcap, int64_t H,
                                                             int64_t d_c, int64_t K, int32_t window, int32_t n_sinks,
                                                             int32_t block_size, int32_t hca_r) {
    return sa_attention_decode_at_workspace(B, Lcap, NCcap, H, d_c, K, block_size, window, n_sinks, hca_r);
}

extern "C" int maba_sa_attention_decode_at(const maba_tensor* qhat, const maba_tensor* c_cache,
                                           const maba_tensor* hca_table, const maba_tensor* top_idx,
                                           const maba_tensor* gate, const maba_tensor* out, const int64_t* pos_dev,
                                           int32_t window, int32_t n_sinks, int32_t block_size, int32_t hca_r,
                                           void* workspace, size_t workspace_bytes, void* stream) {
    if (pos_dev == nullptr) return set_error(MABA_ERR_INVALID, "sa_attention_decode_at: device position required");
    if (!present(qhat) || qhat->ndim != 4 || qhat->shape[1] != 1)
        return set_error(MABA_ERR_INVALID, "sa_attention_decode_at: qhat must be [B, 1, H, d_c]");
    if (!present(c_cache) || c_cache->ndim != 3 || !present(hca_table) || hca_table->ndim != 3)
        return set_error(MABA_ERR_INVALID, "sa_attention_decode_at: c_cache / hca_table must be 3D");
    const int64_t B = qhat->shape[0], H = qhat->shape[2], DC = qhat->shape[3];
    if (c_cache->shape[0] != B || c_cache->shape[2] != DC || hca_table->shape[0] != B || hca_table->shape[2] != DC)
        return set_error(MABA_ERR_INVALID, "sa_attention_decode_at: shape mismatch");
    if (!present(top_idx) || top_idx->ndim != 3 || top_idx->shape[0] != B || top_idx->shape[1] != 1)
        return set_error(MABA_ERR_INVALID, "sa_attention_decode_at: top_idx must be [B, 1, K]");
    if (H > 16 || DC > 256) return set_error(MABA_ERR_UNSUPPORTED, "sa_attention_decode_at: H <= 16, d_c <= 256");
    const int dt = qhat->dtype;
    if (dt == MABA_F64) return set_error(MABA_ERR_UNSUPPORTED, "sa_attention_decode_at: float64");
    MABA_TRY(expect_dtype(c_cache, "sa_attention_decode_at: c_cache", dt));
    MABA_TRY(expect_dtype(hca_table, "sa_attention_decode_at: hca_table", dt));
    MABA_TRY(expect_dtype(gate, "sa_attention_decode_at: gate", dt));
    MABA_TRY(expect_dtype(top_idx, "sa_attention_decode_at: top_idx", MABA_I64));
    const int64_t so[4] = {B, 1, H, DC};
    MABA_TRY(expect_shape(out, "sa_attention_decode_at: out", 4, so));
    MABA_TRY(expect_dtype(out, "sa_attention_decode_at: out", dt));
    int gate4d = gate->ndim == 4 ? 1 : 0;
    SaArgs a{};
    a.qhat = qhat->data; a.ckv = c_cache->data; a.hca = hca_table->data;
    a.top_idx = static_cast<const int64_t*>(top_idx->data); a.gate = gate->data; a.out = out->data;
    for (int i = 0; i < 4; ++i) { a.sq[i] = qhat->stride[i]; a.so[i] = out->stride[i]; a.sg[i] = i < gate->ndim ? gate->stride[i] : 0; }
    for (int i = 0; i < 3; ++i) { a.sc[i] = c_cache->stride[i]; a.st[i] = top_idx->stride[i]; a.sh[i] = hca_table->stride[i]; }
    a.Lq = 1; a.Lkv = c_cache->shape[1]; a.NC = hca_table->shape[1]; a.H = (int)H; a.DC = (int)DC;
    a.K = (int)top_idx->shape[2]; a.window = window; a.n_sinks = n_sinks; a.block = block_size; a.hca_r = hca_r;
    a.gate4d = gate4d; a.workspace = workspace; a.workspace_bytes = workspace_bytes; a.pos_dev = pos_dev;
    if (window <= 0 || n_sinks < 0 || block_size <= 0 || hca_r <= 0)
        return set_error(MABA_ERR_INVALID, "sa_attention_decode_at: window/block/hca_r must be positive");
    return sa_attention_decode(a, B, dt, as_stream(stream));
}
