// Model-level kernels of the inference engine: the parts of a Maba block and of
// the model head that surround the hot-path ops.
//
// Prefill (token-batched, many rows):
//   maba_rmsnorm_residual -- x += sigmoid(res_gate) * y, then h = RMSNorm(x) * w
//                            (maba_sparse/model.py:18-26 RMSNorm, :107-108 and
//                            :126-127 the gated residuals), one warp per row;
//   maba_swiglu           -- silu(gate) * up of the fused gate|up projection
//                            (model.py:28-37 SwiGLUFFN).
// Decode (a handful of rows, weight-streaming GEMVs with fused prologues and
// epilogues, one launch per step of the block):
//   maba_decode_gemv      -- out = W h (+ bias), with h = RMSNorm(x) * w, a gathered
//                            embedding row or a plain vector, and the result
//                            stored, added to the residual stream with its gate,
//                            turned into the DGDA features (conv with history +
//                            SiLU, gates), into SwiGLU products, or into logits
//                            with their argmax.
//   maba_decode_dgda_state -- k L2-norm + one recurrence step per (batch, head,
//                            group of 16 state columns).
// The decode kernels are launched with programmatic dependent launch: each one
// loads what does not depend on its predecessor (its weights, its state slice)
// before waiting for it, so in a captured decode step the weight streams of
// consecutive kernels overlap.
//
// A GEMV CTA owns 16 weight rows (a warp two of them).  It copies the rows into
// shared memory with cp.async before the programmatic-dependency wait, together
// with the rows' epilogue weights (bias, residual gate, conv taps); after the wait
// it issues the epilogue's dependent loads (residual row, conv history), builds
// the NB (<= 8) input vectors in shared memory (every CTA recomputes the input
// normalisation, a few KB), and multiplies 16-byte weight chunks with them.
#include "common.cuh"
#include "activations.cuh"
#include "pdl.cuh"

namespace maba {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kRowsPerWarp = 2;
constexpr int kRowsPerCta = kGemvWarps * kRowsPerWarp;

enum Prologue { PRO_NORM = 0, PRO_GATHER = 1, PRO_VEC = 2 };
enum Epilogue { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_DGDA = 2, EPI_SWIGLU = 3, EPI_LOGITS = 4 };

// One recurrence step: k L2-norm, S' = a*S + k (w*v - (b*k)^T (a*S)), o = q^T S'.
// The columns of S evolve independently (delta_j and o_j only involve column j),
// so one CTA owns a group of 16 columns of one (batch, head) for all dk rows:
// thread (ty, tx) holds rows ty, ty+16, ... of column tx, and the two sums over
// rows go through shared memory.
constexpr int kStateCols = 16;
constexpr int kStateThreads = 256;

struct StateArgs {
    const float* feats; int64_t ldf;  // [B, 4*H*dk + 2*H*dv] decode features
    float* state;                     // [B, H, dk, dv]
    float* o; int64_t ldo;            // [B, H*dv]
    int B, H, dk, dv;
    int off_q, off_k, off_v, off_a, off_b, off_w;
    float eps;
    int nblocks;                      // H * ceil(dv / kStateCols) * B
};

struct GemvArgs {
    const void* w;            // [rows, K] weight (dtype TW), row stride ldw
    int64_t ldw;
    int N;                    // outputs (SwiGLU: I, reading gate rows [0,I) and up rows [I,2I))
    int K;
    int B;
    int pro, epi;
    // prologue
    const float* x; int64_t ldx;            // PRO_NORM: residual stream [B, K] fp32
    const void* norm_w; float eps;           // PRO_NORM: RMSNorm weight [K] (TW)
    const int64_t* ids; const void* emb; int64_t lde;  // PRO_GATHER: emb[ids[b]] rows (TW)
    const void* vec; int64_t ldv; int vec_f32;          // PRO_VEC: [B, K] (fp32 or TW)
    // epilogue
    void* out; int64_t ldo; int out_f32;     // EPI_STORE / EPI_DGDA / EPI_SWIGLU / EPI_LOGITS output
    const float* bias;                       // EPI_STORE: optional [N] fp32
    float* xres; int64_t ldr; const float* gate;  // EPI_RESIDUAL: x[b][n] += gate[n] * y
    const void* taps; int ktaps;             // EPI_DGDA: [nconv, ktaps] conv taps (TW)
    float* hist; int64_t ldh;                // EPI_DGDA: [B, nconv, ktaps-1] fp32 conv history (updated)
    int nconv, a_end;                        // EPI_DGDA: rows [0,nconv) conv, [nconv,a_end) alpha, the rest gates
    unsigned long long* keys;                // EPI_LOGITS: per-b argmax keys (zero before the first call)
    unsigned int* ticket;                    // EPI_LOGITS: CTA counter (zero before the first call)
    int64_t* ids_out; int64_t* pos_dev;      // EPI_LOGITS: argmax ids [B]; position advanced by 1 (optional)
    int nblocks;                             // CTA-blocks of the launch (or phase)
    // EPI_DGDA with st_tickets: the last CTA of each head's rows runs the head's recurrence step
    StateArgs st;                            // st.feats = out
    unsigned int* st_tickets;                // [H] CTA counters (zero before the first call; left zeroed)
    int st_per_head;                         // CTAs whose rows belong to one head: (4 dk + 2 dv) / 16
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

// 8 weights from shared memory (16 bytes for 16-bit types, 32 for float32)
template <typename T>
__device__ __forceinline__ void load_chunk8_smem(const T* p, float* v);
template <>
__device__ __forceinline__ void load_chunk8_smem<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
template <>
__device__ __forceinline__ void load_chunk8_smem<__half>(const __half* p, float* v) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
        v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
    }
}
template <>
__device__ __forceinline__ void load_chunk8_smem<float>(const float* p, float* v) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    const float4 y = *reinterpret_cast<const float4*>(p + 4);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
}

// (value desc, index asc) as one unsigned key: larger key = better
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    unsigned int u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)idx);
}

// Head of stacked DGDA row r (sections q | k | v | alpha | erase | write).
__device__ __forceinline__ int dgda_head_of_row(const StateArgs& a, int r) {
    const int cqk = a.H * a.dk, cv = a.H * a.dv;
    if (r < 2 * cqk) return (r % cqk) / a.dk;
    r -= 2 * cqk;
    if (r < cv) return r / a.dv;
    r -= cv;
    if (r < 2 * cqk) return (r % cqk) / a.dk;
    return (r - 2 * cqk) / a.dv;
}

// One recurrence step of (batch b, head h) by a whole 256-thread CTA (dk, dv <= 64):
// k L2-norm, S' = a*S + k (w*v - (b*k)^T (a*S)), o = q^T S'.  Thread (rg, j) holds rows
// rg, rg + 4, ... of column j; the two sums over rows go through shared memory.  The
// features were written by other CTAs of this launch: they are read through L2.
__device__ __forceinline__ void state_step_cta(const StateArgs& a, int b, int h) {
    __shared__ float vq[64], vk[64], va[64], vb[64];
    __shared__ float red4[4][64];
    __shared__ float knorm_s;
    const int tid = threadIdx.x, j = tid & 63, rg = tid >> 6;
    const int dk = a.dk, dv = a.dv;
    const bool colv = j < dv;
    float* S = a.state + ((int64_t)b * a.H + h) * dk * dv;
    const float* f = a.feats + (int64_t)b * a.ldf;
    float sd[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int i = rg + 4 * r;
        sd[r] = (i < dk && colv) ? S[(int64_t)i * dv + j] : 0.f;
    }
    if (tid < dk) {
        vq[tid] = __ldcg(f + a.off_q + h * dk + tid);
        vk[tid] = __ldcg(f + a.off_k + h * dk + tid);
        va[tid] = expf(__ldcg(f + a.off_a + h * dk + tid));
        vb[tid] = __ldcg(f + a.off_b + h * dk + tid);
    }
    const float wv = colv ? __ldcg(f + a.off_w + h * dv + j) * __ldcg(f + a.off_v + h * dv + j) : 0.f;
    __syncthreads();
    if (tid < 32) {
        float ss = 0.f;
        for (int i = tid; i < dk; i += 32) ss = fmaf(vk[i], vk[i], ss);
        for (int o2 = 16; o2 > 0; o2 >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o2);
        if (tid == 0) knorm_s = 1.f / (sqrtf(ss) + a.eps);
    }
    __syncthreads();
    const float kn = knorm_s;
    float dp = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int i = rg + 4 * r;
        if (i < dk) {
            sd[r] *= va[i];
            dp = fmaf(vb[i] * (vk[i] * kn), sd[r], dp);
        }
    }
    red4[rg][j] = dp;
    __syncthreads();
    const float delta = wv - ((red4[0][j] + red4[1][j]) + (red4[2][j] + red4[3][j]));
    __syncthreads();
    float op = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
        const int i = rg + 4 * r;
        if (i < dk && colv) {
            const float s2 = fmaf(vk[i] * kn, delta, sd[r]);
            S[(int64_t)i * dv + j] = s2;
            op = fmaf(vq[i], s2, op);
        }
    }
    red4[rg][j] = op;
    __syncthreads();
    if (rg == 0 && colv) a.o[(int64_t)b * a.ldo + h * dv + j] = (red4[0][j] + red4[1][j]) + (red4[2][j] + red4[3][j]);
    __syncthreads();
}

// One CTA-block of a decode GEMV: block `blk` of the launch's a.nblocks.  `wait` runs
// between the weight prefetch and the first read of data an earlier kernel wrote
// (the programmatic-dependency wait).
template <typename TW, int NB, bool MIX, class Wait>
__device__ __forceinline__ void gemv_body(const GemvArgs& a, int blk, float* hs, Wait wait) {
    __shared__ float red[kGemvWarps][NB];
    __shared__ unsigned long long best[kGemvWarps][NB];
    __shared__ unsigned int last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K;
    const bool swiglu = a.epi == EPI_SWIGLU;
    // ---- the CTA's weight rows into shared memory by cp.async: the weights do not depend
    // on the previous kernel, so the copies run under its tail.  Shared row rr belongs to
    // warp rr >> 1: (SwiGLU) the gate row o and the up row N + o of output o; else two
    // consecutive rows.
    TW* wsm = reinterpret_cast<TW*>(hs + NB * K);  // [kRowsPerCta][K], after the input vectors
    const int c16 = K * (int)sizeof(TW) / 16;       // 16-byte chunks per row
    const int half = kRowsPerCta / 2;
    for (int e = tid; e < kRowsPerCta * c16; e += kGemvThreads) {
        const int rr = e / c16, c = e - rr * c16;
        const int o = blk * half + (rr >> 1);
        const int row = swiglu ? ((rr & 1) ? a.N + o : o) : blk * kRowsPerCta + rr;
        const bool lv = swiglu ? o < a.N : row < a.N;
        if (lv)
            cp_async16(reinterpret_cast<char*>(wsm + (size_t)rr * K) + c * 16,
                       reinterpret_cast<const char*>(static_cast<const TW*>(a.w) + (int64_t)row * a.ldw) + c * 16);
    }
    cp_async_commit();
    const int on = swiglu ? blk * half + warp : -1;  // SwiGLU output of this warp
    int rows[2];
    rows[0] = swiglu ? on : blk * kRowsPerCta + warp * kRowsPerWarp;
    rows[1] = swiglu ? a.N + on : rows[0] + 1;
    const bool live0 = swiglu ? on < a.N : rows[0] < a.N;
    const bool live1 = swiglu ? on < a.N : rows[1] < a.N;
    // ---- epilogue weights of the warp's rows (bias, residual gate or conv taps), also
    // independent of the previous kernel
    float ew[2][8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int j = 0; j < 8; ++j) ew[r][j] = 0.f;
        const bool lv = r == 0 ? live0 : live1;
        const int n = rows[r];
        if (!lv) continue;
        if (a.epi == EPI_STORE && a.bias) ew[r][0] = a.bias[n];
        else if (a.epi == EPI_RESIDUAL) ew[r][0] = a.gate[n];
        else if (a.epi == EPI_DGDA && n < a.nconv) {
            // history taps in slots 0..ktaps-2, the current token's tap in slot 7
            const TW* tp = static_cast<const TW*>(a.taps) + (int64_t)n * a.ktaps;
#pragma unroll
            for (int j = 0; j < 7; ++j)
                if (j < a.ktaps - 1) ew[r][j] = Cvt<TW>::to_f(tp[j]);
            ew[r][7] = Cvt<TW>::to_f(tp[a.ktaps - 1]);
        }
    }
    // the RMSNorm weight (a weight: loaded before the wait as well), K <= 8 * kGemvThreads
    constexpr int kNormPer = 8;
    float nwv[kNormPer];
#pragma unroll
    for (int j = 0; j < kNormPer; ++j) {
        const int k = tid + j * kGemvThreads;
        nwv[j] = (a.pro == PRO_NORM && k < K) ? Cvt<TW>::to_f(static_cast<const TW*>(a.norm_w)[k]) : 0.f;
    }
    wait();
    __syncthreads();
    // ---- the epilogue's inputs written by earlier kernels (lane b: batch row b), in flight
    // during the prologue and the products
    float ev[2][8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int j = 0; j < 8; ++j) ev[r][j] = 0.f;
        const bool lv = r == 0 ? live0 : live1;
        const int n = rows[r];
        if (!lv || lane >= a.B) continue;
        if (a.epi == EPI_RESIDUAL) ev[r][0] = a.xres[lane * a.ldr + n];
        else if (a.epi == EPI_DGDA && n < a.nconv) {
            const float* h = a.hist + lane * a.ldh + (int64_t)n * (a.ktaps - 1);
#pragma unroll
            for (int j = 0; j < 7; ++j)
                if (j < a.ktaps - 1) ev[r][j] = h[j];
        }
    }
    // ---- prologue: the NB input vectors in shared memory (fp32)
    if (a.pro == PRO_NORM) {
        for (int b = 0; b < NB; ++b) {
            float ss = 0.f;
            if (b < a.B)
                for (int k = tid; k < K; k += kGemvThreads) {
                    const float v = a.x[b * a.ldx + k];
                    hs[b * K + k] = v;
                    ss = fmaf(v, v, ss);
                }
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red[warp][b] = ss;
        }
        __syncthreads();
        for (int b = 0; b < NB; ++b) {
            float ss = 0.f;
#pragma unroll
            for (int w = 0; w < kGemvWarps; ++w) ss += red[w][b];
            const float r = rsqrtf(ss / (float)K + a.eps);
#pragma unroll
            for (int j = 0; j < kNormPer; ++j) {
                const int k = tid + j * kGemvThreads;
                if (k < K) hs[b * K + k] = b < a.B ? hs[b * K + k] * r * nwv[j] : 0.f;
            }
        }
    } else if (a.pro == PRO_GATHER) {
        const TW* e = static_cast<const TW*>(a.emb);
        for (int b = 0; b < NB; ++b) {
            const int64_t row = b < a.B ? a.ids[b] : 0;
            for (int k = tid; k < K; k += kGemvThreads) hs[b * K + k] = b < a.B ? Cvt<TW>::to_f(e[row * a.lde + k]) : 0.f;
        }
    } else {
        for (int b = 0; b < NB; ++b)
            for (int k = tid; k < K; k += kGemvThreads) {
                float v = 0.f;
                if (b < a.B)
                    v = a.vec_f32 ? static_cast<const float*>(a.vec)[b * a.ldv + k]
                                  : Cvt<TW>::to_f(static_cast<const TW*>(a.vec)[b * a.ldv + k]);
                hs[b * K + k] = v;
            }
    }
    cp_async_wait_all();
    __syncthreads();

    float acc[2][NB];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b) acc[r][b] = 0.f;
    const TW* w0 = wsm + (size_t)(2 * warp) * K;
    const TW* w1 = w0 + K;
    const int nch = K / 8;
    for (int c = lane; c < nch; c += 32) {
        float v0[8], v1[8];
        if (live0) load_chunk8_smem<TW>(w0 + c * 8, v0);
        if (live1) load_chunk8_smem<TW>(w1 + c * 8, v1);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const float4 h0 = *reinterpret_cast<const float4*>(hs + b * K + c * 8);
            const float4 h1 = *reinterpret_cast<const float4*>(hs + b * K + c * 8 + 4);
            const float hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
            if (live0)
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[0][b] = fmaf(v0[i], hv[i], acc[0][b]);
            if (live1)
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[1][b] = fmaf(v1[i], hv[i], acc[1][b]);
        }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int b = 0; b < NB; ++b)
            for (int o = 16; o > 0; o >>= 1) acc[r][b] += __shfl_xor_sync(0xffffffffu, acc[r][b], o);

    // ---- epilogue: lane b (< B) handles batch row b
    unsigned long long mykey[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) mykey[b] = 0ull;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        if (lane != b || b >= a.B) continue;
        if (swiglu) {
            if (live0) {
                const float y = silu_f(acc[0][b]) * acc[1][b];
                if (a.out_f32) static_cast<float*>(a.out)[b * a.ldo + on] = y;
                else static_cast<TW*>(a.out)[b * a.ldo + on] = Cvt<TW>::from_f(y);
            }
            continue;
        }
        // one output row: n, its value y, its epilogue weights tw and dependent inputs hv
        auto row_out = [&](int n, float y, const float (&tw)[8], const float (&hv)[8]) {
            if (a.epi == EPI_STORE) {
                if (a.bias) y += tw[0];
                if (a.out_f32) static_cast<float*>(a.out)[b * a.ldo + n] = y;
                else static_cast<TW*>(a.out)[b * a.ldo + n] = Cvt<TW>::from_f(y);
            } else if (a.epi == EPI_RESIDUAL) {
                a.xres[b * a.ldr + n] = fmaf(tw[0], y, hv[0]);
            } else if (a.epi == EPI_DGDA) {
                float f;
                if (n < a.nconv) {
                    // causal conv over the history (oldest first) and this token, then SiLU
                    float* h = a.hist + b * a.ldh + (int64_t)n * (a.ktaps - 1);
                    float cv = tw[7] * y;
#pragma unroll
                    for (int j = 0; j < 7; ++j)
                        if (j < a.ktaps - 1) cv = fmaf(tw[j], hv[j], cv);
#pragma unroll
                    for (int j = 0; j < 6; ++j)
                        if (j + 1 < a.ktaps - 1) h[j] = hv[j + 1];
                    if (a.ktaps > 1) h[a.ktaps - 2] = y;
                    f = silu_f(cv);
                } else if (n < a.a_end) {
                    f = neg_softplus_clamped(y);
                } else {
                    f = sigmoid_f(y);
                }
                static_cast<float*>(a.out)[b * a.ldo + n] = f;
            } else {  // EPI_LOGITS
                static_cast<float*>(a.out)[b * a.ldo + n] = y;
                const unsigned long long k = argmax_key(y, n);
                mykey[b] = k > mykey[b] ? k : mykey[b];
            }
        };
        if (live0) row_out(rows[0], acc[0][b], ew[0], ev[0]);
        if (live1) row_out(rows[1], acc[1][b], ew[1], ev[1]);
    }
    if constexpr (MIX) {
        // the head's last CTA (its rows are one head's slice of one section) runs the step
        const int h = dgda_head_of_row(a.st, blk * kRowsPerCta);
        __threadfence();
        __syncthreads();
        if (tid == 0) last = atomicAdd(a.st_tickets + h, 1u) == (unsigned)a.st_per_head - 1 ? 1u : 0u;
        __syncthreads();
        if (!last) return;
        __threadfence();
        for (int b = 0; b < a.B; ++b) state_step_cta(a.st, b, h);
        if (tid == 0) a.st_tickets[h] = 0u;
        return;
    }
    if (a.epi != EPI_LOGITS) return;
    // ---- argmax: warp -> CTA -> global key, the last CTA publishes the ids
#pragma unroll
    for (int b = 0; b < NB; ++b) {
        const unsigned long long k = __shfl_sync(0xffffffffu, mykey[b], b);
        if (lane == 0) best[warp][b] = k;
    }
    __syncthreads();
    if (tid < NB && tid < a.B) {
        unsigned long long k = 0ull;
#pragma unroll
        for (int w = 0; w < kGemvWarps; ++w) k = best[w][tid] > k ? best[w][tid] : k;
        atomicMax(a.keys + tid, k);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(a.ticket, 1u) == (unsigned)a.nblocks - 1 ? 1u : 0u;
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid < a.B) {
        const unsigned long long k = atomicExch(a.keys + tid, 0ull);
        a.ids_out[tid] = (int64_t)(0xFFFFFFFFu - (unsigned int)(k & 0xFFFFFFFFull));
    }
    if (tid == 0) {
        *a.ticket = 0u;
        if (a.pos_dev) *a.pos_dev += 1;
    }
}

// MIX: the DGDA mixer form (EPI_DGDA with the recurrence step in each head's last CTA).
// The plain 16-bit form for up to two batch rows is held to 64 registers, so four CTAs fit
// per SM and the CTAs of the next GEMVs in the chain find room to start their weight copies
// early (2.8 % per decode step at B = 1); wider batches keep three, float32 weights two.
template <typename TW, int NB, bool MIX>
__global__ void __launch_bounds__(kGemvThreads, (MIX || sizeof(TW) == 4) ? 2 : (NB <= 2 ? 4 : 3)) gemv_kernel(GemvArgs a) {
    extern __shared__ float hs[];  // [NB][K] input vectors, then the CTA's weight rows
    griddep_launch_dependents();
    gemv_body<TW, NB, MIX>(a, blockIdx.x, hs, [] { griddep_wait(); });
}

template <class Wait>
__device__ __forceinline__ void state_body(const StateArgs& a, int blk, Wait wait) {
    const int ncg = (a.dv + kStateCols - 1) / kStateCols;
    const int h = blk % a.H, j0 = (blk / a.H) % ncg * kStateCols, b = blk / (a.H * ncg);
    const float* feats = a.feats;
    const int64_t ldf = a.ldf;
    float* state = a.state;
    float* o = a.o;
    const int64_t ldo = a.ldo;
    const int H = a.H, dk = a.dk, dv = a.dv;
    const int off_q = a.off_q, off_k = a.off_k, off_v = a.off_v, off_a = a.off_a, off_b = a.off_b, off_w = a.off_w;
    const float eps = a.eps;
    const int tid = threadIdx.x, tx = tid % kStateCols, ty = tid / kStateCols;
    constexpr int RY = kStateThreads / kStateCols;  // 16 row groups
    __shared__ float sq[64], sk[64], sa[64], sbk[64];
    __shared__ float red[RY][kStateCols + 1];
    __shared__ float knorm;
    float* S = state + ((int64_t)b * H + h) * dk * dv;
    const int j = j0 + tx;
    const bool colv = j < dv;
    // the state is read after the wait: its last writer (this layer's step before) is only
    // known to be complete once every kernel before this one is.  Before the wait its lines
    // are only asked into L2 (a prefetch moves no data into this SM, so it cannot be stale).
    if (tx == 0)
        for (int r = ty; r < dk; r += RY) asm volatile("prefetch.global.L2 [%0];" ::"l"(S + (int64_t)r * dv + j0));
    wait();
    __syncthreads();
    float sd[64 / RY];
#pragma unroll
    for (int r = 0; r < 64 / RY; ++r) {
        const int i = ty + RY * r;
        sd[r] = (i < dk && colv) ? S[(int64_t)i * dv + j] : 0.f;
    }
    const float* f = feats + (int64_t)b * ldf;
    if (tid < dk) {
        sq[tid] = f[off_q + h * dk + tid];
        sk[tid] = f[off_k + h * dk + tid];
        sa[tid] = expf(f[off_a + h * dk + tid]);
        sbk[tid] = f[off_b + h * dk + tid];
    }
    __syncthreads();
    if (tid < 32) {
        float ss = 0.f;
        for (int i = tid; i < dk; i += 32) ss = fmaf(sk[i], sk[i], ss);
        for (int o2 = 16; o2 > 0; o2 >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o2);
        if (tid == 0) knorm = 1.f / (sqrtf(ss) + eps);
    }
    __syncthreads();
    float dp = 0.f;
#pragma unroll
    for (int r = 0; r < 64 / RY; ++r) {
        const int i = ty + RY * r;
        if (i < dk) {
            sd[r] *= sa[i];
            dp = fmaf(sbk[i] * (sk[i] * knorm), sd[r], dp);
        }
    }
    red[ty][tx] = dp;
    __syncthreads();
    float delta = 0.f;
    if (colv) {
        float tot = 0.f;
#pragma unroll
        for (int y = 0; y < RY; ++y) tot += red[y][tx];
        delta = f[off_w + h * dv + j] * f[off_v + h * dv + j] - tot;
    }
    __syncthreads();
    float op = 0.f;
#pragma unroll
    for (int r = 0; r < 64 / RY; ++r) {
        const int i = ty + RY * r;
        if (i < dk && colv) {
            const float s2 = fmaf(sk[i] * knorm, delta, sd[r]);
            S[(int64_t)i * dv + j] = s2;
            op = fmaf(sq[i], s2, op);
        }
    }
    red[ty][tx] = op;
    __syncthreads();
    if (ty == 0 && colv) {
        float tot = 0.f;
#pragma unroll
        for (int y = 0; y < RY; ++y) tot += red[y][tx];
        o[(int64_t)b * ldo + h * dv + j] = tot;
    }
    __syncthreads();  // shared arrays are reused by the next body in a persistent launch
}

__global__ void __launch_bounds__(kStateThreads) dgda_state_kernel(StateArgs a) {
    griddep_launch_dependents();
    state_body(a, blockIdx.x, [] { griddep_wait(); });
}



// prefill: x += gate * y (optional), h = x * rsqrt(mean(x^2) + eps) * w; one warp per row.
// Rows of D = 128 * NV elements (and unit column strides) take the vector path: every lane
// holds 4 consecutive elements of NV 128-element slices, all loads issued at once.
template <typename T> __device__ __forceinline__ void store4(T* p, float a, float b, float c, float d) {
    p[0] = Cvt<T>::from_f(a);
    p[1] = Cvt<T>::from_f(b);
    p[2] = Cvt<T>::from_f(c);
    p[3] = Cvt<T>::from_f(d);
}
template <> __device__ __forceinline__ void store4<float>(float* p, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
template <> __device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p, float a, float b, float c, float d) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p) = u;
}
template <> __device__ __forceinline__ void store4<__half>(__half* p, float a, float b, float c, float d) {
    __half2 lo = __floats2half2_rn(a, b), hi = __floats2half2_rn(c, d);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&lo);
    u.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(p) = u;
}
template <typename T> __device__ __forceinline__ float4 load4(const T* p) {
    return make_float4(Cvt<T>::to_f(p[0]), Cvt<T>::to_f(p[1]), Cvt<T>::to_f(p[2]), Cvt<T>::to_f(p[3]));
}
template <> __device__ __forceinline__ float4 load4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <> __device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
template <> __device__ __forceinline__ float4 load4<__half>(const __half* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
}

template <typename TO, typename TY, int NV>
__global__ void rmsnorm_residual_vec_kernel(float* x, int64_t ldx, const TY* y, int64_t ldy, const float* gate,
                                            const TO* w, float eps, TO* h, int64_t ldh, int64_t N) {
    constexpr int D = 128 * NV;
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= N) return;
    float* xr = x + row * ldx;
    float4 v[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = *reinterpret_cast<const float4*>(xr + j * 128 + lane * 4);
    if (y != nullptr) {
        float4 yv[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) yv[j] = load4<TY>(y + row * ldy + j * 128 + lane * 4);
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const float4 g = *reinterpret_cast<const float4*>(gate + j * 128 + lane * 4);
            v[j].x = fmaf(g.x, yv[j].x, v[j].x);
            v[j].y = fmaf(g.y, yv[j].y, v[j].y);
            v[j].z = fmaf(g.z, yv[j].z, v[j].z);
            v[j].w = fmaf(g.w, yv[j].w, v[j].w);
            *reinterpret_cast<float4*>(xr + j * 128 + lane * 4) = v[j];
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / (float)D + eps);
    if (h == nullptr) return;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
        const float4 wv = load4<TO>(w + j * 128 + lane * 4);
        store4<TO>(h + row * ldh + j * 128 + lane * 4, v[j].x * r * wv.x, v[j].y * r * wv.y, v[j].z * r * wv.z,
                   v[j].w * r * wv.w);
    }
}

template <typename TO, typename TY>
__global__ void rmsnorm_residual_kernel(float* x, int64_t ldx, const TY* y, int64_t ldy, const float* gate,
                                        const TO* w, float eps, TO* h, int64_t ldh, int64_t N, int D) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= N) return;
    float* xr = x + row * ldx;
    float ss = 0.f;
    for (int k = lane; k < D; k += 32) {
        float v = xr[k];
        if (y != nullptr) {
            v += gate[k] * Cvt<TY>::to_f(y[row * ldy + k]);
            xr[k] = v;
        }
        ss = fmaf(v, v, ss);
    }
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / (float)D + eps);
    if (h == nullptr) return;
    for (int k = lane; k < D; k += 32) h[row * ldh + k] = Cvt<TO>::from_f(xr[k] * r * Cvt<TO>::to_f(w[k]));
}

// silu(gate) * up, 8 outputs per thread (16-byte loads and stores where I % 8 == 0)
template <typename T>
__global__ void swiglu_vec_kernel(const T* u, int64_t ldu, T* out, int64_t ldo, int64_t N, int I) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int per_row = I / 8;
    if (i >= N * per_row) return;
    const int64_t row = i / per_row;
    const int c = (int)(i - row * per_row) * 8;
    const uint4 gu = *reinterpret_cast<const uint4*>(u + row * ldu + c);
    const uint4 uu = *reinterpret_cast<const uint4*>(u + row * ldu + I + c);
    const T* g8 = reinterpret_cast<const T*>(&gu);
    const T* u8 = reinterpret_cast<const T*>(&uu);
    uint4 o;
    T* o8 = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int k = 0; k < 8; ++k) o8[k] = Cvt<T>::from_f(silu_f(Cvt<T>::to_f(g8[k])) * Cvt<T>::to_f(u8[k]));
    *reinterpret_cast<uint4*>(out + row * ldo + c) = o;
}

template <typename T>
__global__ void swiglu_kernel(const T* u, int64_t ldu, T* out, int64_t ldo, int64_t N, int I) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= N * I) return;
    const int64_t row = i / I;
    const int c = (int)(i % I);
    const float g = Cvt<T>::to_f(u[row * ldu + c]);
    const float v = Cvt<T>::to_f(u[row * ldu + I + c]);
    out[row * ldo + c] = Cvt<T>::from_f(silu_f(g) * v);
}

template <typename TO, typename TY>
void launch_rmsnorm(bool vec, int nv, unsigned grid, cudaStream_t s, float* x, int64_t ldx, const TY* y, int64_t ldy,
                    const float* gate, const TO* w, float eps, TO* h, int64_t ldh, int64_t N, int D) {
    if (!vec) {
        rmsnorm_residual_kernel<TO, TY><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N, D);
        return;
    }
    switch (nv) {
        case 1: rmsnorm_residual_vec_kernel<TO, TY, 1><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N); break;
        case 2: rmsnorm_residual_vec_kernel<TO, TY, 2><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N); break;
        case 3: rmsnorm_residual_vec_kernel<TO, TY, 3><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N); break;
        case 4: rmsnorm_residual_vec_kernel<TO, TY, 4><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N); break;
        case 5: rmsnorm_residual_vec_kernel<TO, TY, 5><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N); break;
        case 6: rmsnorm_residual_vec_kernel<TO, TY, 6><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N); break;
        case 7: rmsnorm_residual_vec_kernel<TO, TY, 7><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N); break;
        default: rmsnorm_residual_vec_kernel<TO, TY, 8><<<grid, 256, 0, s>>>(x, ldx, y, ldy, gate, w, eps, h, ldh, N); break;
    }
}

int wdtype_ok(int dt) { return dt == MABA_F32 || dt == MABA_BF16 || dt == MABA_F16; }

template <typename TW>
int launch_gemv(GemvArgs& a, cudaStream_t s) {
    const int outs = a.epi == EPI_SWIGLU ? a.N : a.N;
    const int per_cta = a.epi == EPI_SWIGLU ? kRowsPerCta / 2 : kRowsPerCta;
    const unsigned grid = (unsigned)ceil_div(outs, per_cta);
    int nb = a.B <= 1 ? 1 : a.B <= 2 ? 2 : a.B <= 4 ? 4 : 8;
    // input vectors [nb][K] fp32, then the CTA's weight rows [kRowsPerCta][K]
    const size_t smem = sizeof(float) * (size_t)nb * a.K + sizeof(TW) * (size_t)kRowsPerCta * a.K;
    if (smem > 200 * 1024) return set_error(MABA_ERR_UNSUPPORTED, "decode_gemv: B x K too large for shared memory");
    a.nblocks = (int)grid;
    auto go = [&](auto kern) {
        if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        MABA_TRY(launch_pdl(kern, dim3(grid), dim3(kGemvThreads), smem, s, a));
        return check_launch("decode_gemv");
    };
    const bool mix = a.st_tickets != nullptr;
    switch (nb) {
        case 1: return mix ? go(gemv_kernel<TW, 1, true>) : go(gemv_kernel<TW, 1, false>);
        case 2: return mix ? go(gemv_kernel<TW, 2, true>) : go(gemv_kernel<TW, 2, false>);
        case 4: return mix ? go(gemv_kernel<TW, 4, true>) : go(gemv_kernel<TW, 4, false>);
        default: return mix ? go(gemv_kernel<TW, 8, true>) : go(gemv_kernel<TW, 8, false>);
    }
}

bool row_vec_ok(const maba_tensor* t) {
    const int es = t->dtype == MABA_F32 ? 4 : 2;
    return t->stride[1] == 1 && (t->stride[0] * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(t->data) & 15u) == 0;
}

}  // namespace
}  // namespace maba

using namespace maba;

// ---------------------------------------------------------------------------
// prefill helpers
// ---------------------------------------------------------------------------
extern "C" int maba_rmsnorm_residual(const maba_tensor* x, const maba_tensor* y, const maba_tensor* gate,
                                     const maba_tensor* weight, float eps, const maba_tensor* h_out, void* stream) {
    if (!present(x) || x->ndim != 2 || x->dtype != MABA_F32 || x->stride[1] != 1)
        return set_error(MABA_ERR_INVALID, "rmsnorm_residual: x must be a float32 [N, D] tensor with unit column stride");
    const int64_t N = x->shape[0], D = x->shape[1];
    const bool has_y = present(y);
    if (has_y) {
        const int64_t sy[2] = {N, D};
        MABA_TRY(expect_shape(y, "rmsnorm_residual: y", 2, sy));
        const int64_t sg[1] = {D};
        MABA_TRY(expect_shape(gate, "rmsnorm_residual: gate", 1, sg));
        MABA_TRY(expect_dtype(gate, "rmsnorm_residual: gate", MABA_F32));
        if (y->stride[1] != 1 || gate->stride[0] != 1)
            return set_error(MABA_ERR_INVALID, "rmsnorm_residual: unit column strides required");
    }
    const bool has_h = present(h_out);
    int odt = MABA_F32;
    if (has_h) {
        const int64_t sh[2] = {N, D};
        MABA_TRY(expect_shape(h_out, "rmsnorm_residual: h_out", 2, sh));
        const int64_t sw[1] = {D};
        MABA_TRY(expect_shape(weight, "rmsnorm_residual: weight", 1, sw));
        MABA_TRY(expect_dtype(weight, "rmsnorm_residual: weight", h_out->dtype));
        if (h_out->stride[1] != 1 || weight->stride[0] != 1)
            return set_error(MABA_ERR_INVALID, "rmsnorm_residual: unit column strides required");
        odt = h_out->dtype;
    }
    if (has_y && y->dtype != odt && y->dtype != MABA_F32)
        return set_error(MABA_ERR_DTYPE, "rmsnorm_residual: y must be float32 or the output dtype");
    if (N == 0) return MABA_OK;
    cudaStream_t s = as_stream(stream);
    const unsigned grid = (unsigned)ceil_div(N, 8);
    float* xp = static_cast<float*>(x->data);
    const float* gp = has_y ? static_cast<const float*>(gate->data) : nullptr;
    const int64_t ldy = has_y ? y->stride[0] : 0, ldh = has_h ? h_out->stride[0] : 0;
    return MABA_DISPATCH_FLOAT(odt, "rmsnorm_residual", [&] {
        if constexpr (sizeof(T) == 8) {
            return set_error(MABA_ERR_DTYPE, "rmsnorm_residual: float64");
        } else {
            const T* wp = has_h ? static_cast<const T*>(weight->data) : nullptr;
            T* hp = has_h ? static_cast<T*>(h_out->data) : nullptr;
            const bool yf = has_y && y->dtype == MABA_F32 && odt != MABA_F32;
            const bool vec = D % 128 == 0 && D / 128 <= 8 && x->stride[0] % 4 == 0 && (!has_y || y->stride[0] % 4 == 0) &&
                             (!has_h || h_out->stride[0] % 4 == 0) && (reinterpret_cast<uintptr_t>(xp) & 15u) == 0;
            auto go = [&](auto ty_tag) {
                using TY = decltype(ty_tag);
                launch_rmsnorm<T, TY>(vec, (int)(D / 128), grid, s, xp, x->stride[0],
                                      has_y ? static_cast<const TY*>(y->data) : nullptr, ldy, gp, wp, eps, hp, ldh, N,
                                      (int)D);
            };
            if (yf) go(float{});
            else go(T{});
            return check_launch("rmsnorm_residual");
        }
    });
}

extern "C" int maba_swiglu(const maba_tensor* u, const maba_tensor* out, void* stream) {
    if (!present(u) || u->ndim != 2 || u->shape[1] % 2 != 0 || u->stride[1] != 1)
        return set_error(MABA_ERR_INVALID, "swiglu: u must be [N, 2I] with unit column stride");
    const int64_t N = u->shape[0], I = u->shape[1] / 2;
    const int64_t so[2] = {N, I};
    MABA_TRY(expect_shape(out, "swiglu: out", 2, so));
    MABA_TRY(expect_dtype(out, "swiglu: out", u->dtype));
    if (out->stride[1] != 1) return set_error(MABA_ERR_INVALID, "swiglu: unit column stride required");
    if (N == 0 || I == 0) return MABA_OK;
    cudaStream_t s = as_stream(stream);
    return MABA_DISPATCH_FLOAT(u->dtype, "swiglu", [&] {
        if constexpr (sizeof(T) == 8) {
            return set_error(MABA_ERR_DTYPE, "swiglu: float64");
        } else {
            const bool vec = sizeof(T) == 2 && I % 8 == 0 && u->stride[0] % 8 == 0 && out->stride[0] % 8 == 0 &&
                             (reinterpret_cast<uintptr_t>(u->data) & 15u) == 0 &&
                             (reinterpret_cast<uintptr_t>(out->data) & 15u) == 0;
            if (vec)
                swiglu_vec_kernel<T><<<(unsigned)ceil_div(N * (I / 8), 256), 256, 0, s>>>(
                    static_cast<const T*>(u->data), u->stride[0], static_cast<T*>(out->data), out->stride[0], N, (int)I);
            else
                swiglu_kernel<T><<<(unsigned)ceil_div(N * I, 256), 256, 0, s>>>(
                    static_cast<const T*>(u->data), u->stride[0], static_cast<T*>(out->data), out->stride[0], N, (int)I);
            return check_launch("swiglu");
        }
    });
}

// ---------------------------------------------------------------------------
// decode GEMV with fused prologue / epilogue
// ---------------------------------------------------------------------------
extern "C" size_t maba_decode_gemv_workspace_size(int64_t B) { return (size_t)(B > 0 ? B : 1) * 8 + 16; }

namespace maba {
namespace {
// Validates one decode GEMV and fills its kernel arguments (nblocks included).
int build_gemv(GemvArgs& a, int& dt_out, const maba_tensor* w, int32_t prologue, const maba_tensor* x,
               const maba_tensor* aux, float eps, const maba_tensor* ids, int32_t epilogue, const maba_tensor* out,
               const maba_tensor* bias, const maba_tensor* gate, const maba_tensor* taps, const maba_tensor* hist,
               int32_t n_conv, int32_t alpha_end, const maba_tensor* ids_out, int64_t* pos_dev, void* workspace,
               size_t workspace_bytes) {
    const maba_tensor* norm_w = aux;
    if (!present(w) || w->ndim != 2 || !wdtype_ok(w->dtype))
        return set_error(MABA_ERR_INVALID, "decode_gemv: w must be a [rows, K] float32 / float16 / bfloat16 weight");
    if (!row_vec_ok(w) || w->shape[1] % 8 != 0)
        return set_error(MABA_ERR_UNSUPPORTED, "decode_gemv: w rows must be contiguous, 16-byte aligned, K %% 8 == 0");
    const int dt = w->dtype;
    dt_out = dt;
    const int64_t rows = w->shape[0], K = w->shape[1];
    a = GemvArgs{};
    a.w = w->data; a.ldw = w->stride[0]; a.K = (int)K; a.pro = prologue; a.epi = epilogue;
    a.N = (int)(epilogue == EPI_SWIGLU ? rows / 2 : rows);
    if (epilogue == EPI_SWIGLU && rows % 2 != 0) return set_error(MABA_ERR_INVALID, "decode_gemv: SwiGLU needs 2I rows");
    int64_t B = -1;
    if (prologue == PRO_NORM || prologue == PRO_VEC) {
        if (!present(x) || x->ndim != 2 || x->shape[1] != K || x->stride[1] != 1)
            return set_error(MABA_ERR_INVALID, "decode_gemv: x must be [B, K] with unit column stride");
        B = x->shape[0];
        if (prologue == PRO_NORM) {
            if (K > 8 * kGemvThreads) return set_error(MABA_ERR_UNSUPPORTED, "decode_gemv: RMSNorm prologue K <= 2048");
            MABA_TRY(expect_dtype(x, "decode_gemv: x", MABA_F32));
            const int64_t sn[1] = {K};
            MABA_TRY(expect_shape(norm_w, "decode_gemv: norm_w", 1, sn));
            MABA_TRY(expect_dtype(norm_w, "decode_gemv: norm_w", dt));
            a.x = static_cast<const float*>(x->data); a.ldx = x->stride[0]; a.norm_w = norm_w->data; a.eps = eps;
        } else {
            if (x->dtype != MABA_F32 && x->dtype != dt)
                return set_error(MABA_ERR_DTYPE, "decode_gemv: vector must be float32 or the weight dtype");
            a.vec = x->data; a.ldv = x->stride[0]; a.vec_f32 = x->dtype == MABA_F32;
        }
    } else if (prologue == PRO_GATHER) {
        if (!present(ids) || ids->ndim != 1 || ids->dtype != MABA_I64 || ids->stride[0] != 1)
            return set_error(MABA_ERR_INVALID, "decode_gemv: ids must be a contiguous int64 [B] tensor");
        if (!present(norm_w) || norm_w->ndim != 2 || norm_w->shape[1] != K || norm_w->stride[1] != 1)
            return set_error(MABA_ERR_INVALID, "decode_gemv: the embedding table (aux) must be [V, K]");
        MABA_TRY(expect_dtype(norm_w, "decode_gemv: embedding", dt));
        B = ids->shape[0];
        a.ids = static_cast<const int64_t*>(ids->data); a.emb = norm_w->data; a.lde = norm_w->stride[0];
    } else {
        return set_error(MABA_ERR_INVALID, "decode_gemv: unknown prologue %d", prologue);
    }
    if (B <= 0 || B > 8) return set_error(MABA_ERR_UNSUPPORTED, "decode_gemv: batch 1..8");
    a.B = (int)B;
    if (!present(out) || out->ndim != 2 || out->shape[0] != B || out->stride[1] != 1)
        return set_error(MABA_ERR_INVALID, "decode_gemv: out must be [B, N] with unit column stride");
    a.out = out->data; a.ldo = out->stride[0]; a.out_f32 = out->dtype == MABA_F32;
    if (out->dtype != MABA_F32 && out->dtype != dt)
        return set_error(MABA_ERR_DTYPE, "decode_gemv: out must be float32 or the weight dtype");
    switch (epilogue) {
        case EPI_STORE:
            if (out->shape[1] != a.N) return set_error(MABA_ERR_INVALID, "decode_gemv: out must have one column per row");
            if (present(bias)) {
                if (bias->ndim != 1 || bias->shape[0] != a.N || bias->dtype != MABA_F32 || bias->stride[0] != 1)
                    return set_error(MABA_ERR_INVALID, "decode_gemv: bias must be a contiguous float32 [N]");
                a.bias = static_cast<const float*>(bias->data);
            }
            break;
        case EPI_RESIDUAL:
            if (out->shape[1] != a.N || out->dtype != MABA_F32)
                return set_error(MABA_ERR_INVALID, "decode_gemv: the residual stream (out) must be float32 [B, N]");
            if (!present(gate) || gate->ndim != 1 || gate->shape[0] != a.N || gate->dtype != MABA_F32 || gate->stride[0] != 1)
                return set_error(MABA_ERR_INVALID, "decode_gemv: gate must be a contiguous float32 [N]");
            a.xres = static_cast<float*>(out->data); a.ldr = out->stride[0]; a.gate = static_cast<const float*>(gate->data);
            break;
        case EPI_DGDA: {
            if (out->shape[1] != a.N || out->dtype != MABA_F32)
                return set_error(MABA_ERR_INVALID, "decode_gemv: the DGDA features (out) must be float32 [B, N]");
            if (n_conv < 0 || n_conv > alpha_end || alpha_end > a.N)
                return set_error(MABA_ERR_INVALID, "decode_gemv: bad DGDA section bounds");
            if (!present(taps) || taps->ndim != 2 || taps->shape[0] != n_conv || taps->stride[1] != 1 ||
                taps->stride[0] != taps->shape[1] || taps->dtype != dt)
                return set_error(MABA_ERR_INVALID, "decode_gemv: taps must be a contiguous [n_conv, K] weight");
            const int kt = (int)taps->shape[1];
            if (kt < 1 || kt > 8) return set_error(MABA_ERR_UNSUPPORTED, "decode_gemv: conv kernel size 1..8");
            const int64_t shh[3] = {B, n_conv, kt - 1};
            MABA_TRY(expect_shape(hist, "decode_gemv: hist", 3, shh));
            MABA_TRY(expect_dtype(hist, "decode_gemv: hist", MABA_F32));
            if (hist->stride[2] != 1 || hist->stride[1] != kt - 1)
                return set_error(MABA_ERR_INVALID, "decode_gemv: hist rows must be contiguous");
            a.taps = taps->data; a.ktaps = kt; a.hist = static_cast<float*>(hist->data); a.ldh = hist->stride[0];
            a.nconv = n_conv; a.a_end = alpha_end;
            break;
        }
        case EPI_SWIGLU:
            if (out->shape[1] != a.N) return set_error(MABA_ERR_INVALID, "decode_gemv: SwiGLU out must be [B, I]");
            break;
        case EPI_LOGITS: {
            if (out->shape[1] != a.N || out->dtype != MABA_F32)
                return set_error(MABA_ERR_INVALID, "decode_gemv: logits (out) must be float32 [B, V]");
            if (!present(ids_out) || ids_out->ndim != 1 || ids_out->shape[0] != B || ids_out->dtype != MABA_I64 ||
                ids_out->stride[0] != 1)
                return set_error(MABA_ERR_INVALID, "decode_gemv: ids_out must be a contiguous int64 [B]");
            const size_t need = maba_decode_gemv_workspace_size(B);
            if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 7u))
                return set_error(MABA_ERR_WORKSPACE, "decode_gemv: zeroed, 8-byte aligned workspace of %zu bytes required",
                                 need);
            a.keys = static_cast<unsigned long long*>(workspace);
            a.ticket = reinterpret_cast<unsigned int*>(static_cast<char*>(workspace) + (size_t)B * 8);
            a.ids_out = static_cast<int64_t*>(ids_out->data);
            a.pos_dev = pos_dev;
            break;
        }
        default:
            return set_error(MABA_ERR_INVALID, "decode_gemv: unknown epilogue %d", epilogue);
    }
    const int per_cta = a.epi == EPI_SWIGLU ? kRowsPerCta / 2 : kRowsPerCta;
    a.nblocks = (int)ceil_div(a.N, per_cta);
    return MABA_OK;
}

int build_state(StateArgs& sa, const maba_tensor* feats, const maba_tensor* state, const maba_tensor* o_out,
                int32_t n_heads, float eps) {
    if (!present(feats) || feats->ndim != 2 || feats->dtype != MABA_F32 || feats->stride[1] != 1)
        return set_error(MABA_ERR_INVALID, "decode_dgda_state: feats must be float32 [B, 4*H*dk + 2*H*dv]");
    if (!present(state) || state->ndim != 4 || state->dtype != MABA_F32)
        return set_error(MABA_ERR_INVALID, "decode_dgda_state: state must be float32 [B, H, dk, dv]");
    const int64_t B = state->shape[0], H = state->shape[1], dk = state->shape[2], dv = state->shape[3];
    if (H != n_heads || feats->shape[0] != B || feats->shape[1] != 4 * H * dk + 2 * H * dv)
        return set_error(MABA_ERR_INVALID, "decode_dgda_state: feats / state shapes disagree");
    if (state->stride[3] != 1 || state->stride[2] != dv || state->stride[1] != dk * dv || state->stride[0] != H * dk * dv)
        return set_error(MABA_ERR_INVALID, "decode_dgda_state: state must be contiguous");
    if (dk > 64 || dk <= 0 || dv <= 0)
        return set_error(MABA_ERR_UNSUPPORTED, "decode_dgda_state: dk <= 64");
    const int64_t so[2] = {B, H * dv};
    MABA_TRY(expect_shape(o_out, "decode_dgda_state: o_out", 2, so));
    MABA_TRY(expect_dtype(o_out, "decode_dgda_state: o_out", MABA_F32));
    if (o_out->stride[1] != 1) return set_error(MABA_ERR_INVALID, "decode_dgda_state: o_out unit column stride");
    const int cqk = (int)(H * dk), cv = (int)(H * dv);
    sa = StateArgs{};
    sa.feats = static_cast<const float*>(feats->data); sa.ldf = feats->stride[0];
    sa.state = static_cast<float*>(state->data); sa.o = static_cast<float*>(o_out->data); sa.ldo = o_out->stride[0];
    sa.B = (int)B; sa.H = (int)H; sa.dk = (int)dk; sa.dv = (int)dv;
    sa.off_q = 0; sa.off_k = cqk; sa.off_v = 2 * cqk; sa.off_a = 2 * cqk + cv; sa.off_b = 3 * cqk + cv; sa.off_w = 4 * cqk + cv;
    sa.eps = eps;
    sa.nblocks = (int)(H * ceil_div(dv, kStateCols) * B);
    return MABA_OK;
}

}  // namespace
}  // namespace maba

extern "C" int maba_decode_gemv(const maba_tensor* w, int32_t prologue, const maba_tensor* x,
                                const maba_tensor* aux, float eps, const maba_tensor* ids, int32_t epilogue,
                                const maba_tensor* out, const maba_tensor* bias, const maba_tensor* gate,
                                const maba_tensor* taps, const maba_tensor* hist, int32_t n_conv, int32_t alpha_end,
                                const maba_tensor* ids_out, int64_t* pos_dev, void* workspace,
                                size_t workspace_bytes, void* stream) {
    GemvArgs a;
    int dt = 0;
    MABA_TRY(build_gemv(a, dt, w, prologue, x, aux, eps, ids, epilogue, out, bias, gate, taps, hist, n_conv,
                        alpha_end, ids_out, pos_dev, workspace, workspace_bytes));
    cudaStream_t s = as_stream(stream);
    switch (dt) {
        case MABA_F32: return launch_gemv<float>(a, s);
        case MABA_F16: return launch_gemv<__half>(a, s);
        default: return launch_gemv<__nv_bfloat16>(a, s);
    }
}

extern "C" size_t maba_decode_dgda_mix_workspace_size(int32_t n_heads) {
    return (size_t)(n_heads > 0 ? n_heads : 1) * 4 + 16;
}

extern "C" int maba_decode_dgda_mix(const maba_tensor* w, const maba_tensor* x, const maba_tensor* norm_w, float eps,
                                    const maba_tensor* taps, const maba_tensor* hist, const maba_tensor* feats,
                                    const maba_tensor* state, const maba_tensor* o_out, int32_t n_heads, float k_eps,
                                    void* workspace, size_t workspace_bytes, void* stream) {
    using namespace maba;
    if (!present(state) || state->ndim != 4)
        return set_error(MABA_ERR_INVALID, "decode_dgda_mix: state must be float32 [B, H, dk, dv]");
    const int64_t H = state->shape[1], dk = state->shape[2], dv = state->shape[3];
    if (dk % 16 != 0 || dv % 16 != 0 || dk > 64 || dv > 64)
        return set_error(MABA_ERR_UNSUPPORTED, "decode_dgda_mix: head dims must be multiples of 16, at most 64");
    const int cqk = (int)(H * dk), cv = (int)(H * dv);
    if (!present(w) || w->ndim != 2 || w->shape[0] != 4 * (int64_t)cqk + 2 * cv)
        return set_error(MABA_ERR_INVALID, "decode_dgda_mix: w must hold the 4*H*dk + 2*H*dv stacked rows");
    GemvArgs a;
    int dt = 0;
    MABA_TRY(build_gemv(a, dt, w, PRO_NORM, x, norm_w, eps, nullptr, EPI_DGDA, feats, nullptr, nullptr, taps, hist,
                        2 * cqk + cv, 3 * cqk + cv, nullptr, nullptr, nullptr, 0));
    MABA_TRY(build_state(a.st, feats, state, o_out, n_heads, k_eps));
    if (a.st.B != a.B) return set_error(MABA_ERR_INVALID, "decode_dgda_mix: x and state batches differ");
    if (workspace == nullptr || workspace_bytes < maba_decode_dgda_mix_workspace_size(n_heads) ||
        (reinterpret_cast<uintptr_t>(workspace) & 3u))
        return set_error(MABA_ERR_WORKSPACE, "decode_dgda_mix: zeroed, 4-byte aligned workspace of %zu bytes required",
                         maba_decode_dgda_mix_workspace_size(n_heads));
    a.st_tickets = static_cast<unsigned int*>(workspace);
    a.st_per_head = (int)((4 * dk + 2 * dv) / kRowsPerCta);
    cudaStream_t s = as_stream(stream);
    switch (dt) {
        case MABA_F32: return launch_gemv<float>(a, s);
        case MABA_F16: return launch_gemv<__half>(a, s);
        default: return launch_gemv<__nv_bfloat16>(a, s);
    }
}

extern "C" int maba_decode_dgda_state(const maba_tensor* feats, const maba_tensor* state, const maba_tensor* o_out,
                                      int32_t n_heads, float eps, void* stream) {
    StateArgs sa;
    MABA_TRY(build_state(sa, feats, state, o_out, n_heads, eps));
    MABA_TRY(launch_pdl(dgda_state_kernel, dim3((unsigned)sa.nblocks), dim3(kStateThreads), 0, as_stream(stream), sa));
    return check_launch("decode_dgda_state");
}
