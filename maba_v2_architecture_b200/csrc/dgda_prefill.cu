// DGDA chunked prefill (gated delta rule with per-channel decay).
//
// Recurrence (maba_sparse/kernels/common.py:256-265):
//   Sd = diag(alpha_t) S;  delta = w_t*v_t - (b_t*k_t)^T Sd;  S = Sd + k_t delta^T;  o_t = q_t^T S
// Chunked WY/UT form (maba_sparse/kernels/cpu_dgda.py:101-146), per chunk of C
// tokens with G = cumsum(log alpha) over the chunk:
//   L[i,j] = sum_d (b k)_i[d] k_j[d] e^{G_i[d]-G_j[d]}   (j < i)
//   A[i,j] = sum_d q_i[d]     k_j[d] e^{G_i[d]-G_j[d]}   (j <= i)
//   (I+L) [W | U] = [(b k) e^{G} | w v]                 (exact blocked solve)
//   V' = U - W S;   o = (q e^{G}) S + A V';   S <- e^{G_end} S + (k e^{G_end-G})^T V'
// The solve is exact (16x16 diagonal inverses by forward substitution plus
// block back-substitution): the Neumann series of cpu_dgda.py:110-114 diverges
// for large inputs (reference tests/test_dgda_stress.py:169-190).
//
// Parallelism.  Columns of S evolve independently, chunks of one (b,h) are a
// serial chain.  When B*H alone cannot fill the GPU the sequence is cut into
// segments: pass 1 runs every segment from the augmented state [0 | I] and
// records its affine transition S_end = P S_start + R (P is dk x dk); a small
// combine pass chains the transitions; pass 2 reruns each segment from its
// true starting state and writes the outputs.  This is the same affine-chain
// that splits a sequence across GPUs.
//
// This file holds the CUDA-core (FFMA) chunk kernel -- exact fp32 compute for
// fp32 inputs, fp64 for fp64 inputs, head dims up to 64 -- the segment combine
// kernel and the launcher; 16-bit inputs run the tensor-core chunk kernel of
// dgda_prefill_mma.cu.
#include "dgda_prefill.cuh"

#include <cstdlib>

namespace maba {
namespace {

constexpr int NT = 256;   // threads per CTA
constexpr int DP = 64;    // padded head dim
constexpr int SUB = 16;   // diagonal block of the triangular solve



template <typename ACC> __device__ __forceinline__ ACC fast_exp(ACC x);
template <> __device__ __forceinline__ float fast_exp<float>(float x) { return __expf(x); }
template <> __device__ __forceinline__ double fast_exp<double>(double x) { return exp(x); }

template <typename ACC, int C, int MODE>
struct Smem {
    static constexpr int RS = DP + 1;
    static constexpr int XRS = 2 * DP + 1;
    static constexpr int NCOL = MODE == 1 ? 2 * DP : DP;
    static constexpr int VRS = NCOL + 1;
    static constexpr int NB = C / SUB;
    static constexpr size_t kQ = 0;
    static constexpr size_t kK = kQ + (size_t)C * RS;
    static constexpr size_t kB = kK + (size_t)C * RS;
    static constexpr size_t kG = kB + (size_t)C * RS;
    static constexpr size_t kX = kG + (size_t)C * RS;
    static constexpr size_t kL = kX + (size_t)C * XRS;
    static constexpr size_t kA = kL + (size_t)C * (C + 1);
    static constexpr size_t kS = kA + (size_t)C * (C + 1);
    static constexpr size_t kV = kS + (size_t)DP * NCOL;
    static constexpr size_t kVsz = ((size_t)C * VRS > (size_t)SUB * XRS) ? (size_t)C * VRS : (size_t)SUB * XRS;
    static constexpr size_t kT = kV + kVsz;
    static constexpr size_t kD = kT + (size_t)NB * SUB * (SUB + 1);
    static constexpr size_t kTotal = kD + DP;
    static constexpr size_t bytes = kTotal * sizeof(ACC);
};

// MODE 0: single pass from initial_state; MODE 1: transition pass from [0|I];
// MODE 2: output pass of one segment from its combined starting state.
template <typename T, typename TS, typename ACC, int C, int MODE>
__global__ void __launch_bounds__(NT, 1) dgda_chunk_kernel(PrefillArgs a) {
    using SM = Smem<ACC, C, MODE>;
    constexpr int RS = SM::RS, XRS = SM::XRS, NCOL = SM::NCOL, VRS = SM::VRS, NB = SM::NB;
    constexpr int RPT = C / 16;          // rows per thread in the state phase
    constexpr int CPT = NCOL / 16;       // columns per thread in the state phase
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ACC* sm = reinterpret_cast<ACC*>(smem_raw);
    ACC* Qs = sm + SM::kQ;
    ACC* Ks = sm + SM::kK;
    ACC* Bs = sm + SM::kB;
    ACC* Gs = sm + SM::kG;
    ACC* Xs = sm + SM::kX;
    ACC* Ls = sm + SM::kL;
    ACC* As = sm + SM::kA;
    ACC* Ss = sm + SM::kS;
    ACC* Vt = sm + SM::kV;
    ACC* Tb = sm + SM::kT;
    ACC* dend = sm + SM::kD;

    const int tid = threadIdx.x;
    const int bh = blockIdx.x;
    const int seg = blockIdx.y;
    const int64_t bi = bh / a.H, hi = bh % a.H;
    const int dk = a.dk, dv = a.dv;

    const T* q = static_cast<const T*>(a.q);
    const T* k = static_cast<const T*>(a.k);
    const T* v = static_cast<const T*>(a.v);
    const T* bb = static_cast<const T*>(a.b);
    const T* w = static_cast<const T*>(a.w);
    const T* al = static_cast<const T*>(a.alpha);
    const T* lal = static_cast<const T*>(a.log_alpha);

    // ---- initial state ----------------------------------------------------
    for (int e = tid; e < DP * NCOL; e += NT) {
        const int d = e / NCOL, c = e - (e / NCOL) * NCOL;
        ACC s = ACC(0);
        if (MODE == 0) {
            if (a.init != nullptr && d < dk && c < dv)
                s = load_as<ACC>(static_cast<const TS*>(a.init) + bi * a.si[0] + hi * a.si[1] +
                                 (int64_t)d * a.si[2] + (int64_t)c * a.si[3]);
        } else if (MODE == 1) {
            s = (c >= DP && c - DP == d) ? ACC(1) : ACC(0);
        } else {
            s = (ACC)a.ws_start[(((size_t)bh * a.nseg + seg) * DP + d) * DP + c];
        }
        Ss[d * NCOL + c] = s;
    }

    const int64_t t_begin = (int64_t)seg * a.seg_len;
    int64_t t_end = t_begin + a.seg_len;
    if (t_end > a.L) t_end = a.L;

    for (int64_t c0 = t_begin; c0 < t_end; c0 += C) {
        __syncthreads();
        // ---- load the chunk (zero rows past the end, zero padded channels) ----
        for (int e = tid; e < C * DP; e += NT) {
            const int r = e / DP, d = e - (e / DP) * DP;
            const int64_t t = c0 + r;
            ACC qv = 0, kv = 0, bv = 0, gv = 0, wvv = 0;
            if (t < t_end) {
                if (d < dk) {
                    qv = load_as<ACC>(q + bi * a.sq[0] + hi * a.sq[1] + t * a.sq[2] + d * a.sq[3]);
                    kv = load_as<ACC>(k + bi * a.sk[0] + hi * a.sk[1] + t * a.sk[2] + d * a.sk[3]);
                    bv = load_as<ACC>(bb + bi * a.sb[0] + hi * a.sb[1] + t * a.sb[2] + d * a.sb[3]);
                    if (lal != nullptr) {
                        gv = load_as<ACC>(lal + bi * a.sla[0] + hi * a.sla[1] + t * a.sla[2] + d * a.sla[3]);
                        gv = gv < ACC(-46) ? ACC(-46) : (gv > ACC(0) ? ACC(0) : gv);
                    } else {
                        ACC x = load_as<ACC>(al + bi * a.sa[0] + hi * a.sa[1] + t * a.sa[2] + d * a.sa[3]);
                        x = x < ACC(1e-20) ? ACC(1e-20) : (x > ACC(1) ? ACC(1) : x);
                        gv = log_acc<ACC>(x);
                    }
                }
                if (d < dv) {
                    ACC vv = load_as<ACC>(v + bi * a.sv[0] + hi * a.sv[1] + t * a.sv[2] + d * a.sv[3]);
                    ACC ww = load_as<ACC>(w + bi * a.sw[0] + hi * a.sw[1] + t * a.sw[2] + d * a.sw[3]);
                    wvv = ww * vv;
                }
            }
            Qs[r * RS + d] = qv;
            Ks[r * RS + d] = kv;
            Bs[r * RS + d] = bv * kv;
            Gs[r * RS + d] = gv;
            Xs[r * XRS + DP + d] = wvv;
        }
        __syncthreads();
        // ---- cumulative log decay per channel (sequential, as torch.cumsum) ----
        if (tid < DP) {
            ACC run = 0;
            for (int r = 0; r < C; ++r) {
                run += Gs[r * RS + tid];
                Gs[r * RS + tid] = run;
            }
        }
        __syncthreads();
        // ---- A and L with explicit per-channel decay --------------------------
        {
            constexpr int TPR = NT / (C / 2);   // threads per row pair
            const int rp = tid / TPR, sub = tid - (tid / TPR) * TPR;
            const int iA = rp, iB = C - 1 - rp;
            for (int p = sub; p < C + 1; p += TPR) {
                int i, j;
                if (p <= iA) { i = iA; j = p; } else { i = iB; j = p - iA - 1; }
                ACC av = 0, lv = 0;
                const ACC* gi = Gs + i * RS;
                const ACC* gj = Gs + j * RS;
                const ACC* qi = Qs + i * RS;
                const ACC* bki = Bs + i * RS;
                const ACC* kj = Ks + j * RS;
                for (int d = 0; d < dk; ++d) {
                    const ACC kd = kj[d] * fast_exp<ACC>(gi[d] - gj[d]);
                    av += qi[d] * kd;
                    lv += bki[d] * kd;
                }
                As[i * (C + 1) + j] = av;
                Ls[i * (C + 1) + j] = i > j ? lv : ACC(0);
            }
        }
        __syncthreads();
        // ---- decayed operands; diagonal-block inverses ------------------------
        for (int e = tid; e < C * DP; e += NT) {
            const int r = e / DP, d = e - (e / DP) * DP;
            const ACC g = Gs[r * RS + d];
            const ACC ge = Gs[(C - 1) * RS + d];
            const ACC eg = fast_exp<ACC>(g);
            Xs[r * XRS + d] = Bs[r * RS + d] * eg;          // (b k) e^{G}
            Qs[r * RS + d] = Qs[r * RS + d] * eg;           // q e^{G}
            Ks[r * RS + d] = Ks[r * RS + d] * fast_exp<ACC>(ge - g);  // k e^{G_end - G}
            if (r == 0) dend[d] = fast_exp<ACC>(ge);
        }
        if (tid < NB * SUB) {
            const int blk = tid / SUB, c = tid - (tid / SUB) * SUB;
            ACC* T_ = Tb + blk * SUB * (SUB + 1);
            const ACC* Lb = Ls + (blk * SUB) * (C + 1) + blk * SUB;
            for (int r = 0; r < c; ++r) T_[r * (SUB + 1) + c] = 0;
            T_[c * (SUB + 1) + c] = 1;
            for (int r = c + 1; r < SUB; ++r) {
                ACC s = 0;
                for (int m = c; m < r; ++m) s += Lb[r * (C + 1) + m] * T_[m * (SUB + 1) + c];
                T_[r * (SUB + 1) + c] = -s;
            }
        }
        __syncthreads();
        // ---- blocked forward substitution: (I+L) X = RHS, in place in Xs -------
        {
            constexpr int NX = 2 * DP;
            ACC* Rt = Vt;  // [SUB][XRS] temporary
            for (int I = 0; I < NB; ++I) {
                for (int e = tid; e < SUB * NX; e += NT) {
                    const int r = e / NX, c = e - (e / NX) * NX;
                    const int row = I * SUB + r;
                    ACC s = Xs[row * XRS + c];
                    const ACC* lr = Ls + row * (C + 1);
                    for (int j = 0; j < I * SUB; ++j) s -= lr[j] * Xs[j * XRS + c];
                    Rt[r * XRS + c] = s;
                }
                __syncthreads();
                const ACC* T_ = Tb + I * SUB * (SUB + 1);
                for (int e = tid; e < SUB * NX; e += NT) {
                    const int r = e / NX, c = e - (e / NX) * NX;
                    ACC s = 0;
                    for (int m = 0; m <= r; ++m) s += T_[r * (SUB + 1) + m] * Rt[m * XRS + c];
                    Xs[(I * SUB + r) * XRS + c] = s;
                }
                __syncthreads();
            }
        }
        // ---- state phase ---------------------------------------------------------
        const int tr = tid >> 4, tc = tid & 15;
        ACC accq[RPT][DP / 16];
        {
            ACC accv[RPT][CPT];
#pragma unroll
            for (int m = 0; m < RPT; ++m) {
#pragma unroll
                for (int kk = 0; kk < CPT; ++kk) accv[m][kk] = 0;
#pragma unroll
                for (int kk = 0; kk < DP / 16; ++kk) accq[m][kk] = 0;
            }
            for (int d = 0; d < dk; ++d) {
                ACC s[CPT];
#pragma unroll
                for (int kk = 0; kk < CPT; ++kk) s[kk] = Ss[d * NCOL + tc + 16 * kk];
#pragma unroll
                for (int m = 0; m < RPT; ++m) {
                    const int i = tr + 16 * m;
                    const ACC wv = Xs[i * XRS + d];
#pragma unroll
                    for (int kk = 0; kk < CPT; ++kk) accv[m][kk] += wv * s[kk];
                    if (MODE != 1) {
                        const ACC qt = Qs[i * RS + d];
#pragma unroll
                        for (int kk = 0; kk < DP / 16; ++kk) accq[m][kk] += qt * s[kk];
                    }
                }
            }
#pragma unroll
            for (int m = 0; m < RPT; ++m) {
                const int i = tr + 16 * m;
#pragma unroll
                for (int kk = 0; kk < CPT; ++kk) {
                    const int c = tc + 16 * kk;
                    const ACC u = c < DP ? Xs[i * XRS + DP + c] : ACC(0);
                    Vt[i * VRS + c] = u - accv[m][kk];
                }
            }
        }
        __syncthreads();
        if (MODE != 1) {
            T* o = static_cast<T*>(a.out);
#pragma unroll
            for (int m = 0; m < RPT; ++m) {
                const int i = tr + 16 * m;
                const int64_t t = c0 + i;
                const ACC* ar = As + i * (C + 1);
#pragma unroll
                for (int kk = 0; kk < DP / 16; ++kk) {
                    const int c = tc + 16 * kk;
                    ACC s = accq[m][kk];
                    for (int j = 0; j <= i; ++j) s += ar[j] * Vt[j * VRS + c];
                    if (t < t_end && c < dv)
                        store_from<T, ACC>(o + bi * a.so[0] + hi * a.so[1] + t * a.so[2] + (int64_t)c * a.so[3], s);
                }
            }
        }
        {
            ACC acc[DP / 16][CPT];
#pragma unroll
            for (int m = 0; m < DP / 16; ++m) {
                const int d = tr + 16 * m;
#pragma unroll
                for (int kk = 0; kk < CPT; ++kk) acc[m][kk] = dend[d] * Ss[d * NCOL + tc + 16 * kk];
            }
            for (int i = 0; i < C; ++i) {
                ACC vv[CPT];
#pragma unroll
                for (int kk = 0; kk < CPT; ++kk) vv[kk] = Vt[i * VRS + tc + 16 * kk];
#pragma unroll
                for (int m = 0; m < DP / 16; ++m) {
                    const ACC kt = Ks[i * RS + tr + 16 * m];
#pragma unroll
                    for (int kk = 0; kk < CPT; ++kk) acc[m][kk] += kt * vv[kk];
                }
            }
#pragma unroll
            for (int m = 0; m < DP / 16; ++m) {
                const int d = tr + 16 * m;
#pragma unroll
                for (int kk = 0; kk < CPT; ++kk) Ss[d * NCOL + tc + 16 * kk] = acc[m][kk];
            }
        }
    }
    __syncthreads();
    // ---- results ---------------------------------------------------------------
    if (MODE == 1) {
        float* dst = a.ws_trans + ((size_t)bh * a.nseg + seg) * DP * (2 * DP);
        for (int e = tid; e < DP * NCOL; e += NT) dst[e] = (float)Ss[e];
    } else if (MODE == 0 || seg == a.nseg - 1) {
        TS* f = static_cast<TS*>(a.fin);
        for (int e = tid; e < DP * NCOL; e += NT) {
            const int d = e / NCOL, c = e - (e / NCOL) * NCOL;
            if (d < dk && c < dv)
                store_from<TS, ACC>(f + bi * a.sf[0] + hi * a.sf[1] + (int64_t)d * a.sf[2] + (int64_t)c * a.sf[3],
                                    Ss[e]);
        }
    }
}

// Chains the segment transitions: start[0] = S0, start[s+1] = P_s start[s] + R_s.
// One CTA per (b,h).  P is kept in a padded tile (row stride 65: the rows a warp
// reads at one column fall in distinct banks); the next segment's P and R are
// loaded into registers while the current product runs.
template <typename TS>
__global__ void __launch_bounds__(NT) dgda_combine_kernel(PrefillArgs a) {
    __shared__ float S[DP * DP];
    __shared__ float Pm[DP * (DP + 1)];
    const int tid = threadIdx.x;
    const int bh = blockIdx.x;
    const int64_t bi = bh / a.H, hi = bh % a.H;
    for (int e = tid; e < DP * DP; e += NT) {
        const int d = e / DP, c = e - (e / DP) * DP;
        float s = 0.f;
        if (a.init != nullptr && d < a.dk && c < a.dv)
            s = load_as<float>(static_cast<const TS*>(a.init) + bi * a.si[0] + hi * a.si[1] + (int64_t)d * a.si[2] +
                               (int64_t)c * a.si[3]);
        S[e] = s;
    }
    const int tr = tid >> 4, tc = tid & 15;
    const float* trans = a.ws_trans + (size_t)bh * a.nseg * DP * (2 * DP);
    // this thread's share of a transition: 16 elements of P (4 float4) and its 16 outputs' R
    float4 pp[4];
    float rr[4][4];
    auto fetch = [&](int sg) {
        const float* src = trans + (size_t)sg * DP * (2 * DP);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int q = (tid * 4 + j) * 4;  // element of the 64x64 P
            const int d = q >> 6, e = q & 63;
            pp[j] = *reinterpret_cast<const float4*>(src + d * (2 * DP) + DP + e);
        }
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) rr[m][kk] = src[(tr + 16 * m) * (2 * DP) + tc + 16 * kk];
    };
    auto stash = [&]() {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int q = (tid * 4 + j) * 4;
            const int d = q >> 6, e = q & 63;
            float* dst = Pm + d * (DP + 1) + e;
            dst[0] = pp[j].x;
            dst[1] = pp[j].y;
            dst[2] = pp[j].z;
            dst[3] = pp[j].w;
        }
    };
    if (a.nseg > 1) {
        fetch(0);
        stash();
    }
    for (int sg = 0; sg < a.nseg; ++sg) {
        __syncthreads();
        float* dst = a.ws_start + ((size_t)bh * a.nseg + sg) * DP * DP;
        for (int e = tid * 4; e < DP * DP; e += NT * 4)
            *reinterpret_cast<float4*>(dst + e) = *reinterpret_cast<const float4*>(S + e);
        if (sg == a.nseg - 1) break;
        float acc[4][4];
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) acc[m][kk] = rr[m][kk];
        if (sg + 2 < a.nseg) fetch(sg + 1);  // next P, R in flight during the product
        for (int e = 0; e < DP; ++e) {
            float sv[4];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) sv[kk] = S[e * DP + tc + 16 * kk];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const float p = Pm[(tr + 16 * m) * (DP + 1) + e];  // P[d][e]
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) acc[m][kk] = fmaf(p, sv[kk], acc[m][kk]);
            }
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) S[(tr + 16 * m) * DP + tc + 16 * kk] = acc[m][kk];
        if (sg + 2 < a.nseg) stash();
    }
}

// Starting state of every segment (chunk-parallel path) by the chain
// start[0] = S0 (or 0), start[s+1] = P_s start[s] + R_s over the segment
// transitions [R_s | P_s].  The columns of the state evolve independently, so one
// (b,h)'s chain is split over 64 / CH_COLS CTAs (grid = (B*H, 64 / CH_COLS)), each
// carrying CH_COLS columns: a step is a 64 x 64 x CH_COLS product.  Thread layout:
// row tid & 63, columns 4 (tid >> 6) .. + 3 of the CTA's slice.  P_s sits in a padded
// tile (row stride 65: a warp's 32 rows at one column fall in distinct banks); the
// next segment's P and R are loaded into registers while the current step runs.
constexpr int CH_COLS = 8;
constexpr int CH_NT = 64 * CH_COLS / 4;

template <typename TS>
__global__ void __launch_bounds__(CH_NT) dgda_chain_starts_kernel(PrefillArgs a, const float* trans) {
    __shared__ float Pm[2][DP * (DP + 1)];
    __shared__ __align__(16) float Sx[DP * CH_COLS];
    const int tid = threadIdx.x;
    const int bh = blockIdx.x, cb = blockIdx.y * CH_COLS;
    const int64_t bi = bh / a.H, hi = bh % a.H;
    const int row = tid & 63, c4 = (tid >> 6) * 4;  // this thread's state entries: (row, cb + c4 .. + 3)
    const float* tr = trans + (size_t)bh * a.nseg * DP * 2 * DP;
    constexpr int PF = DP * DP / 4 / CH_NT;  // float4 of P per thread
    float4 pre[PF];
    float4 rpre;
    auto load = [&](int sg) {
        const float* T = tr + (size_t)sg * DP * 2 * DP;
#pragma unroll
        for (int i = 0; i < PF; ++i) {
            const int f = tid + CH_NT * i, r = f >> 4, c = (f & 15) * 4;
            pre[i] = *reinterpret_cast<const float4*>(T + r * 2 * DP + DP + c);
        }
        rpre = *reinterpret_cast<const float4*>(T + row * 2 * DP + cb + c4);
    };
    auto stage = [&](int buf) {
#pragma unroll
        for (int i = 0; i < PF; ++i) {
            const int f = tid + CH_NT * i, r = f >> 4, c = (f & 15) * 4;
            float* d = &Pm[buf][r * (DP + 1) + c];
            d[0] = pre[i].x;
            d[1] = pre[i].y;
            d[2] = pre[i].z;
            d[3] = pre[i].w;
        }
    };
    float st[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = cb + c4 + j;
        float v = 0.f;
        if (a.init != nullptr && row < a.dk && c < a.dv)
            v = load_as<float>(static_cast<const TS*>(a.init) + bi * a.si[0] + hi * a.si[1] + (int64_t)row * a.si[2] +
                               (int64_t)c * a.si[3]);
        st[j] = v;
    }
    if (a.nseg > 1) {
        load(0);
        stage(0);
    }
    float4 rcur = rpre;
    for (int sg = 0; sg < a.nseg; ++sg) {
        float* dst = a.ws_start + ((size_t)bh * a.nseg + sg) * DP * DP + (size_t)row * DP + cb + c4;
        *reinterpret_cast<float4*>(dst) = make_float4(st[0], st[1], st[2], st[3]);
        if (sg + 1 >= a.nseg) break;
        *reinterpret_cast<float4*>(&Sx[row * CH_COLS + c4]) = make_float4(st[0], st[1], st[2], st[3]);
        if (sg + 2 < a.nseg) load(sg + 1);
        __syncthreads();  // P_sg staged, the state slice in Sx
        const float* P = Pm[sg & 1] + row * (DP + 1);
        float acc[4] = {rcur.x, rcur.y, rcur.z, rcur.w};
#pragma unroll 16
        for (int k = 0; k < DP; ++k) {
            const float p = P[k];
            const float4 x = *reinterpret_cast<const float4*>(&Sx[k * CH_COLS + c4]);
            acc[0] = fmaf(p, x.x, acc[0]);
            acc[1] = fmaf(p, x.y, acc[1]);
            acc[2] = fmaf(p, x.z, acc[2]);
            acc[3] = fmaf(p, x.w, acc[3]);
        }
        if (sg + 2 < a.nseg) {
            stage((sg + 1) & 1);
            rcur = rpre;
        }
        __syncthreads();  // every read of Sx and of Pm[sg & 1] is done
#pragma unroll
        for (int j = 0; j < 4; ++j) st[j] = acc[j];
    }
}

// Composes the per-segment transitions of one (b,h) into the transition of the
// whole range: X = [R | P] starts at [0 | I]; X <- P_s X + [R_s | 0].
__global__ void __launch_bounds__(NT) dgda_compose_kernel(const float* ws_trans, float* out, int nseg, int64_t out_bh_stride) {
    __shared__ float X[DP * 2 * DP];
    __shared__ float Pm[DP * DP];
    const int tid = threadIdx.x;
    const int bh = blockIdx.x;
    for (int e = tid; e < DP * 2 * DP; e += NT) {
        const int d = e / (2 * DP), c = e - (e / (2 * DP)) * (2 * DP);
        X[e] = (c >= DP && c - DP == d) ? 1.f : 0.f;
    }
    const int tr = tid >> 4, tc = tid & 15;
    for (int sg = 0; sg < nseg; ++sg) {
        const float* T = ws_trans + ((size_t)bh * nseg + sg) * DP * 2 * DP;
        __syncthreads();
        for (int e = tid; e < DP * DP; e += NT) Pm[e] = T[(e / DP) * 2 * DP + DP + (e % DP)];
        __syncthreads();
        float acc[4][8];
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
                const int d = tr + 16 * m, c = tc + 16 * kk;
                acc[m][kk] = c < DP ? T[d * 2 * DP + c] : 0.f;  // + [R_s | 0]
            }
        for (int e = 0; e < DP; ++e) {
            float xv[8];
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) xv[kk] = X[e * 2 * DP + tc + 16 * kk];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                const float p = Pm[(tr + 16 * m) * DP + e];
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) acc[m][kk] += p * xv[kk];
            }
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) X[(tr + 16 * m) * 2 * DP + tc + 16 * kk] = acc[m][kk];
    }
    __syncthreads();
    for (int e = tid; e < DP * 2 * DP; e += NT) out[(size_t)bh * out_bh_stride + e] = X[e];
}

int choose_segments(int dtype, int64_t BH, int64_t L) {
    if (dtype == MABA_F64) return 1;
    const int64_t nchunks = ceil_div(L, 64);
    const int64_t sms = sm_count();
    if (BH >= sms || nchunks < 12) return 1;
    // one CTA per SM (shared-memory bound): segments pay ~2.5x the work, so use
    // them only to fill a single wave, and only when that is >= 3 segments
    int64_t nseg = sms / BH;
    if (nseg > nchunks / 4) nseg = nchunks / 4;
    if (nseg > 64) nseg = 64;
    return nseg < 3 ? 1 : (int)nseg;
}

// Chunk-parallel path (16-bit inputs): chunk records for a window of `win`
// chunks (the sequence is processed in windows so the records stay within a
// fixed budget), `nseg` scan segments per window, and the fp32 state carried
// between windows.
struct ChunkPlan {
    int64_t nch, win, nwin;
    int nseg;
    size_t rec_bytes, bytes;
};

constexpr size_t kChunkWsBudget = size_t(2) << 30;

// MABA_DGDA_WINDOW_CHUNKS (> 0) caps the window length in chunks; it exists so
// the multi-window path can be exercised on short sequences.
int64_t window_cap() {
    const char* e = getenv("MABA_DGDA_WINDOW_CHUNKS");
    if (e == nullptr) return 0;
    const long long v = atoll(e);
    return v > 0 ? (int64_t)v : 0;
}

ChunkPlan chunk_plan(int64_t BH, int64_t L) {
    ChunkPlan p{};
    p.nch = ceil_div(L, 64);
    int64_t win = (int64_t)(kChunkWsBudget / ((size_t)BH * CHUNK_REC));
    if (win < 64) win = 64;
    const int64_t cap = window_cap();
    if (cap > 0 && win > cap) win = cap;
    if (win > p.nch) win = p.nch;
    p.win = win > 0 ? win : 1;
    p.nwin = ceil_div(p.nch, p.win);
    const int64_t sms = sm_count();
    int64_t nseg = BH >= sms ? 1 : (2 * sms) / BH;  // two scan CTAs per SM
    if (nseg > p.win / 8) nseg = p.win / 8;
    if (nseg > 32) nseg = 32;
    p.nseg = nseg < 2 ? 1 : (int)nseg;
    p.rec_bytes = (size_t)BH * p.win * CHUNK_REC;
    // records, transitions, segment starts, the carried state
    p.bytes = p.rec_bytes + (size_t)BH * p.nseg * (DP * 2 * DP + DP * DP) * sizeof(float) +
              (size_t)BH * DP * DP * sizeof(float);
    return p;
}

template <typename K>
int set_smem(K kern, size_t bytes) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return set_error(MABA_ERR_CUDA, "dgda_prefill: smem attribute: %s", cudaGetErrorString(e));
    return MABA_OK;
}

// Chunk-parallel prefill (16-bit): per window, the preparation pass over all
// chunks and the segmented state scan (which writes the outputs).
template <typename T>
int launch_chunked(const PrefillArgs& a0, int64_t BH, const ChunkPlan& p, int dtype, int sdtype, cudaStream_t s,
                   void* ws) {
    unsigned char* base = static_cast<unsigned char*>(ws);
    float* trans = reinterpret_cast<float*>(base + p.rec_bytes);
    float* start = trans + (size_t)BH * p.nseg * DP * 2 * DP;
    float* carry = start + (size_t)BH * p.nseg * DP * DP;  // fp32 [B][H][64][64] between windows
    for (int64_t w = 0; w < p.nwin; ++w) {
        PrefillArgs a = a0;
        const int64_t t0 = w * p.win * 64;
        const int64_t len = (a0.L - t0) < p.win * 64 ? (a0.L - t0) : p.win * 64;
        auto shift = [&](const void* ptr, const int64_t* st) -> const void* {
            return ptr ? static_cast<const void*>(static_cast<const T*>(ptr) + t0 * st[2]) : nullptr;
        };
        a.q = shift(a0.q, a0.sq); a.k = shift(a0.k, a0.sk); a.v = shift(a0.v, a0.sv);
        a.alpha = shift(a0.alpha, a0.sa); a.log_alpha = shift(a0.log_alpha, a0.sla);
        a.b = shift(a0.b, a0.sb); a.w = shift(a0.w, a0.sw);
        a.out = static_cast<T*>(a0.out) + t0 * a0.so[2];
        a.L = len;
        a.nch = ceil_div(len, 64);
        a.ws_chunk = base;
        const int64_t carry_st[4] = {(int64_t)a0.H * DP * DP, DP * DP, DP, 1};
        if (w > 0) {
            a.init = carry;
            for (int i = 0; i < 4; ++i) a.si[i] = carry_st[i];
        }
        if (w + 1 < p.nwin) {
            a.fin = carry;
            for (int i = 0; i < 4; ++i) a.sf[i] = carry_st[i];
        }
        MABA_TRY(dgda_prep_launch(a, BH, dtype, s));
        const int64_t seg_chunks = ceil_div(a.nch, (int64_t)p.nseg);
        a.seg_len = seg_chunks * 64;
        a.nseg = (int)ceil_div(a.nch, seg_chunks);
        if (a.nseg <= 1) {
            a.nseg = 1;
            MABA_TRY(dgda_scan_launch(a, dim3((unsigned)BH, 1), 0, dtype, sdtype, s));
        } else {
            a.ws_trans = trans;
            a.ws_start = start;
            const dim3 grid((unsigned)BH, (unsigned)a.nseg);
            MABA_TRY(dgda_scan_launch(a, grid, 1, dtype, sdtype, s));
            // starting state of every segment: the transition chain, each (b,h)'s
            // state columns split over 64 / CH_COLS CTAs
            const dim3 cgrid((unsigned)BH, (unsigned)(DP / CH_COLS));
            if (sdtype == MABA_F32) dgda_chain_starts_kernel<float><<<cgrid, CH_NT, 0, s>>>(a, trans);
            else dgda_chain_starts_kernel<T><<<cgrid, CH_NT, 0, s>>>(a, trans);
            MABA_TRY(check_launch("dgda_prefill(segment starts)"));
            MABA_TRY(dgda_scan_launch(a, grid, 2, dtype, sdtype, s));
        }
    }
    return MABA_OK;
}

template <typename T, typename TS>
int launch_prefill(PrefillArgs& a, int64_t B, int dtype, int sdtype, cudaStream_t s, void* ws, size_t ws_bytes) {
    using ACC = typename std::conditional<sizeof(T) == 8, double, float>::type;
    constexpr int C = sizeof(T) == 8 ? 32 : 64;
    constexpr bool k16 = sizeof(T) == 2;  // 16-bit inputs: tensor-core chunk kernels
    const int64_t BH = B * a.H;
    if (BH == 0) return MABA_OK;
    if constexpr (k16) {
        // chunk-parallel path when the caller's workspace holds its plan (windows
        // after the first carry an fp32 state, so they need an fp32 state dtype)
        if (a.L >= 2 * 64 && a.vec8) {
            const ChunkPlan p = chunk_plan(BH, a.L);
            if (ws != nullptr && ws_bytes >= p.bytes && (p.nwin == 1 || sdtype == MABA_F32))
                return launch_chunked<T>(a, BH, p, dtype, sdtype, s, ws);
        }
    }
    const int nseg = choose_segments(dtype, BH, a.L);
    if (nseg <= 1) {
        a.nseg = 1;
        a.seg_len = a.L > 0 ? a.L : 1;
        if (k16) return dgda_mma_launch(a, dim3((unsigned)BH, 1), 0, dtype, sdtype, s);
        auto kern = dgda_chunk_kernel<T, TS, ACC, C, 0>;
        MABA_TRY(set_smem(kern, Smem<ACC, C, 0>::bytes));
        kern<<<dim3((unsigned)BH, 1), NT, Smem<ACC, C, 0>::bytes, s>>>(a);
        return check_launch("dgda_prefill");
    }
    if constexpr (sizeof(T) == 8) {
        return set_error(MABA_ERR_UNSUPPORTED, "dgda_prefill: segmented fp64 path not built");
    } else {
        const int64_t nchunks = ceil_div(a.L, C);
        a.nseg = nseg;
        a.seg_len = ceil_div(nchunks, nseg) * C;
        a.nseg = (int)ceil_div(a.L, a.seg_len);
        const size_t need = (size_t)BH * a.nseg * (DP * 2 * DP + DP * DP) * sizeof(float);
        if (ws == nullptr || ws_bytes < need)
            return set_error(MABA_ERR_WORKSPACE, "dgda_prefill: workspace of %zu bytes required, got %zu", need, ws_bytes);
        a.ws_trans = static_cast<float*>(ws);
        a.ws_start = a.ws_trans + (size_t)BH * a.nseg * DP * 2 * DP;
        const dim3 grid((unsigned)BH, (unsigned)a.nseg);
        if (k16) {
            MABA_TRY(dgda_mma_launch(a, grid, 1, dtype, sdtype, s));
        } else {
            auto k1 = dgda_chunk_kernel<T, TS, ACC, C, 1>;
            MABA_TRY(set_smem(k1, Smem<ACC, C, 1>::bytes));
            k1<<<grid, NT, Smem<ACC, C, 1>::bytes, s>>>(a);
            MABA_TRY(check_launch("dgda_prefill(transition)"));
        }
        dgda_combine_kernel<TS><<<(unsigned)BH, NT, 0, s>>>(a);
        MABA_TRY(check_launch("dgda_prefill(combine)"));
        if (k16) return dgda_mma_launch(a, grid, 2, dtype, sdtype, s);
        auto k2 = dgda_chunk_kernel<T, TS, ACC, C, 2>;
        MABA_TRY(set_smem(k2, Smem<ACC, C, 2>::bytes));
        k2<<<grid, NT, Smem<ACC, C, 2>::bytes, s>>>(a);
        return check_launch("dgda_prefill(apply)");
    }
}

bool vec8_ok(const maba_tensor* t) {
    if (!present(t)) return true;
    if (t->stride[3] != 1 || (t->stride[2] % 8) || (t->stride[1] % 8) || (t->stride[0] % 8)) return false;
    return (reinterpret_cast<uintptr_t>(t->data) & 15u) == 0;
}

}  // namespace
}  // namespace maba

using namespace maba;

extern "C" size_t maba_dgda_prefill_workspace_size(int32_t dtype, int64_t B, int64_t H, int64_t L, int64_t dk,
                                                   int64_t dv) {
    (void)dk; (void)dv;
    const int64_t BH = B * H;
    size_t need = 0;
    const int nseg0 = choose_segments(dtype, BH, L);
    if (nseg0 > 1) {
        const int64_t nchunks = ceil_div(L, 64);
        const int64_t seg_len = ceil_div(nchunks, nseg0) * 64;
        const int64_t nseg = ceil_div(L, seg_len);
        need = (size_t)BH * nseg * (DP * 2 * DP + DP * DP) * sizeof(float);
    }
    if ((dtype == MABA_BF16 || dtype == MABA_F16) && BH > 0 && L >= 2 * 64) {
        const size_t c = chunk_plan(BH, L).bytes;
        if (c > need) need = c;
    }
    return need;
}

extern "C" int maba_dgda_prefill(const maba_tensor* q, const maba_tensor* k, const maba_tensor* v,
                                 const maba_tensor* alpha, const maba_tensor* log_alpha, const maba_tensor* b,
                                 const maba_tensor* w, const maba_tensor* initial_state, const maba_tensor* out,
                                 const maba_tensor* final_state, int32_t chunk_size, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    (void)chunk_size;
    if (!present(q) || q->ndim != 4) return set_error(MABA_ERR_INVALID, "dgda_prefill: q must be 4D [B, H, L, dk]");
    const int64_t B = q->shape[0], H = q->shape[1], L = q->shape[2], dk = q->shape[3];
    if (!present(v) || v->ndim != 4) return set_error(MABA_ERR_INVALID, "dgda_prefill: v must be 4D [B, H, L, dv]");
    const int64_t dv = v->shape[3];
    const int64_t s_k[4] = {B, H, L, dk}, s_v[4] = {B, H, L, dv}, s_s[4] = {B, H, dk, dv};
    MABA_TRY(expect_shape(k, "dgda_prefill: k", 4, s_k));
    MABA_TRY(expect_shape(v, "dgda_prefill: v", 4, s_v));
    MABA_TRY(expect_shape(b, "dgda_prefill: b", 4, s_k));
    MABA_TRY(expect_shape(w, "dgda_prefill: w", 4, s_v));
    MABA_TRY(expect_shape(out, "dgda_prefill: out", 4, s_v));
    MABA_TRY(expect_shape(final_state, "dgda_prefill: final_state", 4, s_s));
    if (!present(alpha) && !present(log_alpha))
        return set_error(MABA_ERR_INVALID, "dgda_prefill: either alpha or log_alpha must be provided");
    if (present(alpha)) MABA_TRY(expect_shape(alpha, "dgda_prefill: alpha", 4, s_k));
    if (present(log_alpha)) MABA_TRY(expect_shape(log_alpha, "dgda_prefill: log_alpha", 4, s_k));
    if (present(initial_state)) MABA_TRY(expect_shape(initial_state, "dgda_prefill: initial_state", 4, s_s));
    const int dt = q->dtype;
    const maba_tensor* same[] = {k, v, b, w, out};
    const char* names[] = {"k", "v", "b", "w", "out"};
    for (int i = 0; i < 5; ++i)
        if (same[i]->dtype != dt)
            return set_error(MABA_ERR_DTYPE, "dgda_prefill: %s dtype %s differs from q (%s)", names[i],
                             dtype_name(same[i]->dtype), dtype_name(dt));
    if (present(alpha) && alpha->dtype != dt) return set_error(MABA_ERR_DTYPE, "dgda_prefill: alpha dtype mismatch");
    if (present(log_alpha) && log_alpha->dtype != dt)
        return set_error(MABA_ERR_DTYPE, "dgda_prefill: log_alpha dtype mismatch");
    const int sdt = final_state->dtype;
    if (present(initial_state) && initial_state->dtype != sdt)
        return set_error(MABA_ERR_DTYPE, "dgda_prefill: initial_state and final_state dtypes differ");
    if (sdt != dt && sdt != MABA_F32)
        return set_error(MABA_ERR_DTYPE, "dgda_prefill: state dtype must be q's dtype or float32");
    if (dk > DP || dv > DP || dk <= 0 || dv <= 0)
        return set_error(MABA_ERR_UNSUPPORTED, "dgda_prefill: head dims dk=%lld dv=%lld outside [1, %d]",
                         (long long)dk, (long long)dv, DP);

    PrefillArgs a{};
    a.q = q->data; a.k = k->data; a.v = v->data;
    a.alpha = present(alpha) ? alpha->data : nullptr;
    a.log_alpha = present(log_alpha) ? log_alpha->data : nullptr;
    a.b = b->data; a.w = w->data;
    a.init = present(initial_state) ? initial_state->data : nullptr;
    a.out = out->data; a.fin = final_state->data;
    for (int i = 0; i < 4; ++i) {
        a.sq[i] = q->stride[i]; a.sk[i] = k->stride[i]; a.sv[i] = v->stride[i];
        a.sa[i] = present(alpha) ? alpha->stride[i] : 0;
        a.sla[i] = present(log_alpha) ? log_alpha->stride[i] : 0;
        a.sb[i] = b->stride[i]; a.sw[i] = w->stride[i];
        a.si[i] = present(initial_state) ? initial_state->stride[i] : 0;
        a.so[i] = out->stride[i]; a.sf[i] = final_state->stride[i];
    }
    a.L = L; a.H = (int)H; a.dk = (int)dk; a.dv = (int)dv;
    a.vec8 = (dk == DP && dv == DP && vec8_ok(q) && vec8_ok(k) && vec8_ok(v) && vec8_ok(b) && vec8_ok(w) &&
              vec8_ok(log_alpha) && (present(log_alpha) || vec8_ok(alpha))) ? 1 : 0;
    cudaStream_t s = as_stream(stream);
    switch (dt) {
        case MABA_F32: return launch_prefill<float, float>(a, B, dt, sdt, s, workspace, workspace_bytes);
        case MABA_F64:
            if (sdt != MABA_F64) return set_error(MABA_ERR_DTYPE, "dgda_prefill: float64 needs a float64 state");
            return launch_prefill<double, double>(a, B, dt, sdt, s, workspace, workspace_bytes);
        case MABA_F16:
            return sdt == MABA_F32 ? launch_prefill<__half, float>(a, B, dt, sdt, s, workspace, workspace_bytes)
                                   : launch_prefill<__half, __half>(a, B, dt, sdt, s, workspace, workspace_bytes);
        case MABA_BF16:
            return sdt == MABA_F32 ? launch_prefill<__nv_bfloat16, float>(a, B, dt, sdt, s, workspace, workspace_bytes)
                                   : launch_prefill<__nv_bfloat16, __nv_bfloat16>(a, B, dt, sdt, s, workspace, workspace_bytes);
        default: return set_error(MABA_ERR_DTYPE, "dgda_prefill: unsupported dtype %s", dtype_name(dt));
    }
}

extern "C" size_t maba_dgda_transition_workspace_size(int32_t dtype, int64_t B, int64_t H, int64_t L) {
    const int64_t BH = B * H;
    int nseg = choose_segments(dtype, BH, L);
    if (nseg < 1) nseg = 1;
    const int64_t nchunks = ceil_div(L > 0 ? L : 1, 64);
    const int64_t seg_len = ceil_div(nchunks, nseg) * 64;
    const int64_t ns = ceil_div(L > 0 ? L : 1, seg_len);
    return (size_t)BH * ns * DP * 2 * DP * sizeof(float);
}

extern "C" int maba_dgda_transition(const maba_tensor* q, const maba_tensor* k, const maba_tensor* v,
                                    const maba_tensor* alpha, const maba_tensor* log_alpha, const maba_tensor* b,
                                    const maba_tensor* w, const maba_tensor* trans_out, void* workspace,
                                    size_t workspace_bytes, void* stream) {
    if (!present(q) || q->ndim != 4 || !present(v) || v->ndim != 4)
        return set_error(MABA_ERR_INVALID, "dgda_transition: q, v must be 4D [B, H, L, d]");
    const int64_t B = q->shape[0], H = q->shape[1], L = q->shape[2], dk = q->shape[3], dv = v->shape[3];
    const int64_t s_k[4] = {B, H, L, dk}, s_v[4] = {B, H, L, dv}, s_t[4] = {B, H, DP, 2 * DP};
    MABA_TRY(expect_shape(k, "dgda_transition: k", 4, s_k));
    MABA_TRY(expect_shape(b, "dgda_transition: b", 4, s_k));
    MABA_TRY(expect_shape(w, "dgda_transition: w", 4, s_v));
    MABA_TRY(expect_shape(trans_out, "dgda_transition: trans_out", 4, s_t));
    MABA_TRY(expect_dtype(trans_out, "dgda_transition: trans_out", MABA_F32));
    if (!present(alpha) && !present(log_alpha))
        return set_error(MABA_ERR_INVALID, "dgda_transition: either alpha or log_alpha must be provided");
    if (dk > DP || dv > DP) return set_error(MABA_ERR_UNSUPPORTED, "dgda_transition: head dims <= %d", DP);
    const int64_t tst[4] = {H * DP * 2 * DP, DP * 2 * DP, 2 * DP, 1};
    for (int i = 0; i < 4; ++i)
        if (trans_out->stride[i] != tst[i]) return set_error(MABA_ERR_INVALID, "dgda_transition: trans_out must be contiguous");
    const int dt = q->dtype;
    if (dt != MABA_F32 && dt != MABA_F16 && dt != MABA_BF16)
        return set_error(MABA_ERR_DTYPE, "dgda_transition: float32 / float16 / bfloat16 inputs");
    const size_t need = maba_dgda_transition_workspace_size(dt, B, H, L);
    if (workspace == nullptr || workspace_bytes < need)
        return set_error(MABA_ERR_WORKSPACE, "dgda_transition: workspace of %zu bytes required", need);
    PrefillArgs a{};
    a.q = q->data; a.k = k->data; a.v = v->data;
    a.alpha = present(alpha) ? alpha->data : nullptr;
    a.log_alpha = present(log_alpha) ? log_alpha->data : nullptr;
    a.b = b->data; a.w = w->data; a.init = nullptr; a.out = nullptr; a.fin = nullptr;
    for (int i = 0; i < 4; ++i) {
        a.sq[i] = q->stride[i]; a.sk[i] = k->stride[i]; a.sv[i] = v->stride[i];
        a.sa[i] = present(alpha) ? alpha->stride[i] : 0;
        a.sla[i] = present(log_alpha) ? log_alpha->stride[i] : 0;
        a.sb[i] = b->stride[i]; a.sw[i] = w->stride[i];
    }
    a.L = L; a.H = (int)H; a.dk = (int)dk; a.dv = (int)dv;
    a.vec8 = (dk == DP && dv == DP && vec8_ok(q) && vec8_ok(k) && vec8_ok(v) && vec8_ok(b) && vec8_ok(w) &&
              vec8_ok(log_alpha) && (present(log_alpha) || vec8_ok(alpha))) ? 1 : 0;
    const int64_t BH = B * H;
    int nseg = choose_segments(dt, BH, L);
    if (nseg < 1) nseg = 1;
    const int64_t nchunks = ceil_div(L > 0 ? L : 1, 64);
    a.seg_len = ceil_div(nchunks, nseg) * 64;
    a.nseg = (int)ceil_div(L > 0 ? L : 1, a.seg_len);
    a.ws_trans = static_cast<float*>(workspace);
    cudaStream_t s = as_stream(stream);
    const dim3 grid((unsigned)BH, (unsigned)a.nseg);
    if (dt == MABA_F32) {
        auto k1 = dgda_chunk_kernel<float, float, float, 64, 1>;
        MABA_TRY(set_smem(k1, Smem<float, 64, 1>::bytes));
        k1<<<grid, NT, Smem<float, 64, 1>::bytes, s>>>(a);
        MABA_TRY(check_launch("dgda_transition"));
    } else {
        MABA_TRY(dgda_mma_launch(a, grid, 1, dt, MABA_F32, s));
    }
    dgda_compose_kernel<<<(unsigned)BH, NT, 0, s>>>(a.ws_trans, static_cast<float*>(trans_out->data), a.nseg,
                                                   DP * 2 * DP);
    return check_launch("dgda_transition(compose)");
}
