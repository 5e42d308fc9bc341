// Tensor-core DGDA chunk kernel for 16-bit inputs (bf16 / fp16), dk, dv <= 64.
//
// Same recurrence and chunked WY/UT form as dgda_prefill.cu (reference
// maba_sparse/kernels/common.py:256-265 and cpu_dgda.py:101-146), chunk of 64,
// with every chunk contraction on mma.sync.m16n8k16 (16-bit operands, fp32
// accumulation) fed by ldmatrix from padded shared-memory tiles:
//
//   A, L off-diagonal 16x16 blocks  -- factorised decay: for query sub-block I with
//        reference r_I = G[16I-1], exp(G_i - G_j) = exp(G_i - r_I) exp(r_I - G_j),
//        both factors <= 1 (G is non-increasing), so the products are tensor-core
//        GEMMs of pre-scaled operands with no overflow;
//   A, L diagonal 16x16 blocks      -- the same factorisation around the block's first
//        row when the block's decay spread is <= 80 (bf16; 8 for fp16) in every
//        channel (the factors stay inside the 16-bit range), else explicit
//        per-element decay (fp32);
//   T = (I + L)^{-1}                -- 16x16 diagonal inverses by forward substitution
//        (fp32) plus block back-substitution on the tensor cores (exact solve);
//   per chunk state chain           -- R = w v - (b k e^G) S;  V' = T R;
//        o = (q e^G) S + A V';  S <- e^{G_end} S + (k e^{G_end - G})^T V'.
// The state S lives in fp32 accumulator registers across chunks (a 16-bit copy
// in shared memory feeds the next chunk's MMAs).  Segment passes (mode 1/2) and
// the combine kernel are shared with the CUDA-core path.
#include "dgda_prefill.cuh"
#include "mma_util.cuh"

namespace maba {
namespace {

constexpr int C = 64;     // chunk
constexpr int D = 64;     // padded head dim
constexpr int NTH = 256;  // 8 warps
constexpr int NB = 4;     // 16-row sub-blocks per chunk
constexpr int LB = 72;    // 16-bit row stride of 64-wide tiles (144 B: conflict-free ldmatrix)
constexpr int LF = 68;    // fp32 row stride
constexpr int LT = 24;    // 16-bit row stride of the 16x16 diagonal inverses

template <int NCOL>
struct MS {
    static constexpr int LN = NCOL + 8;
    static constexpr size_t G = 0;                              // fp32 [C][LF] cumulative log decay
    static constexpr size_t BK = G + (size_t)C * LF * 4;        // fp32 [C][LF] b*k
    static constexpr size_t WV = BK + (size_t)C * LF * 4;       // fp32 [C][LF] w*v
    static constexpr size_t LD = WV + (size_t)C * LF * 4;       // fp32 [NB][16][17] diagonal blocks of L
    static constexpr size_t DEND = LD + (size_t)NB * 16 * 17 * 4;  // fp32 [D] exp(G_end)
    static constexpr size_t TD = DEND + (size_t)D * 4;          // 16-bit [NB][16][LT] diagonal inverses
    static constexpr size_t QR = TD + (size_t)NB * 16 * LT * 2; // 16-bit [C][LB] q
    static constexpr size_t KR = QR + (size_t)C * LB * 2;       // k
    static constexpr size_t QT = KR + (size_t)C * LB * 2;       // q e^G
    static constexpr size_t BT = QT + (size_t)C * LB * 2;       // (b k) e^G
    static constexpr size_t KT = BT + (size_t)C * LB * 2;       // k e^{G_end - G}
    static constexpr size_t AM = KT + (size_t)C * LB * 2;       // A (lower, incl. diagonal)
    static constexpr size_t LM = AM + (size_t)C * LB * 2;       // L (strictly lower)
    static constexpr size_t SB = LM + (size_t)C * LB * 2;       // [D][LN] 16-bit copy of the state
    static constexpr size_t TM = SB + (size_t)D * LN * 2;       // [C][LB] T = (I+L)^-1
    static constexpr size_t VP = TM + (size_t)C * LB * 2;       // [C][LN] V'
    static constexpr size_t RB = VP + (size_t)C * LN * 2;       // [C][LN] R
    static constexpr size_t QD = RB + (size_t)C * LN * 2;       // [C][LB] q e^{G - G_blockstart}
    static constexpr size_t BD = QD + (size_t)C * LB * 2;       // [C][LB] (b k) e^{G - G_blockstart}
    static constexpr size_t KD = BD + (size_t)C * LB * 2;       // [C][LB] k e^{G_blockstart - G}
    static constexpr size_t FLG = KD + (size_t)C * LB * 2;      // int [NB]: block decay too steep to factorise
    static constexpr size_t TOTAL = FLG + 16;
    // decay-factor operands of the off-diagonal blocks alias TM.. during the A/L phase
    static constexpr size_t QH = TM;                            // [48][LB]
    static constexpr size_t BH = QH + (size_t)48 * LB * 2;      // [48][LB]
    static constexpr size_t KH = BH + (size_t)48 * LB * 2;      // [96][LB]: I=1 rows 0..15, I=2 16..47, I=3 48..95
    static_assert(KH + (size_t)96 * LB * 2 <= QD, "off-diagonal scratch must fit");
};

__device__ __forceinline__ int kh_off(int I) { return I == 1 ? 0 : (I == 2 ? 16 : 48); }

template <typename T>
__device__ __forceinline__ float f32(T x) { return Cvt<T>::to_f(x); }

template <typename T, typename TS, int MODE>
__global__ void __launch_bounds__(NTH, 1) dgda_mma_kernel(PrefillArgs a) {
    constexpr int NCOL = MODE == 1 ? 2 * D : D;
    using S_ = MS<NCOL>;
    constexpr int LN = S_::LN;
    constexpr int NTW = NCOL / 16;  // n8 tiles per warp: warp tile = 16 rows x NCOL/2 columns
    extern __shared__ __align__(16) unsigned char sm[];
    float* Gs = reinterpret_cast<float*>(sm + S_::G);
    float* BKs = reinterpret_cast<float*>(sm + S_::BK);
    float* WVs = reinterpret_cast<float*>(sm + S_::WV);
    float* LDs = reinterpret_cast<float*>(sm + S_::LD);
    float* dend = reinterpret_cast<float*>(sm + S_::DEND);
    T* TDs = reinterpret_cast<T*>(sm + S_::TD);
    T* QR = reinterpret_cast<T*>(sm + S_::QR);
    T* KR = reinterpret_cast<T*>(sm + S_::KR);
    T* QTs = reinterpret_cast<T*>(sm + S_::QT);
    T* BTs = reinterpret_cast<T*>(sm + S_::BT);
    T* KTs = reinterpret_cast<T*>(sm + S_::KT);
    T* AM = reinterpret_cast<T*>(sm + S_::AM);
    T* LM = reinterpret_cast<T*>(sm + S_::LM);
    T* SB = reinterpret_cast<T*>(sm + S_::SB);
    T* TM = reinterpret_cast<T*>(sm + S_::TM);
    T* VP = reinterpret_cast<T*>(sm + S_::VP);
    T* RB = reinterpret_cast<T*>(sm + S_::RB);
    T* QH = reinterpret_cast<T*>(sm + S_::QH);
    T* BHs = reinterpret_cast<T*>(sm + S_::BH);
    T* KH = reinterpret_cast<T*>(sm + S_::KH);
    T* QD = reinterpret_cast<T*>(sm + S_::QD);
    T* BDs = reinterpret_cast<T*>(sm + S_::BD);
    T* KD = reinterpret_cast<T*>(sm + S_::KD);
    int* flags = reinterpret_cast<int*>(sm + S_::FLG);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x, seg = blockIdx.y;
    const int64_t bi = bh / a.H, hi = bh % a.H;
    const int dk = a.dk, dv = a.dv;
    const int wr = (warp & 3) * 16;           // warp rows in [64 x NCOL] products
    const int wc = (warp >> 2) * (NCOL / 2);  // warp columns
    const int fr = lane >> 2, fc = (lane & 3) * 2;

    const T* q = static_cast<const T*>(a.q) + bi * a.sq[0] + hi * a.sq[1];
    const T* k = static_cast<const T*>(a.k) + bi * a.sk[0] + hi * a.sk[1];
    const T* v = static_cast<const T*>(a.v) + bi * a.sv[0] + hi * a.sv[1];
    const T* bb = static_cast<const T*>(a.b) + bi * a.sb[0] + hi * a.sb[1];
    const T* w = static_cast<const T*>(a.w) + bi * a.sw[0] + hi * a.sw[1];
    const T* lal = a.log_alpha ? static_cast<const T*>(a.log_alpha) + bi * a.sla[0] + hi * a.sla[1] : nullptr;
    const T* al = a.alpha ? static_cast<const T*>(a.alpha) + bi * a.sa[0] + hi * a.sa[1] : nullptr;

    // ---- initial state in accumulator registers --------------------------------
    float sacc[NTW][4];
#pragma unroll
    for (int n = 0; n < NTW; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = wr + fr + (e >> 1) * 8;
            const int c = wc + n * 8 + fc + (e & 1);
            float s = 0.f;
            if (MODE == 0) {
                if (a.init != nullptr && d < dk && c < dv)
                    s = load_as<float>(static_cast<const TS*>(a.init) + bi * a.si[0] + hi * a.si[1] +
                                       (int64_t)d * a.si[2] + (int64_t)c * a.si[3]);
            } else if (MODE == 1) {
                s = (c >= D && c - D == d) ? 1.f : 0.f;
            } else {
                s = a.ws_start[(((size_t)bh * a.nseg + seg) * D + d) * D + c];
            }
            sacc[n][e] = s;
            SB[d * LN + c] = to16<T>(s);
        }

    const int64_t t_begin = (int64_t)seg * a.seg_len;
    int64_t t_end = t_begin + a.seg_len;
    if (t_end > a.L) t_end = a.L;

    for (int64_t c0 = t_begin; c0 < t_end; c0 += C) {
        __syncthreads();
        // ---------------- load the chunk -----------------------------------------
        if (a.vec8) {
            for (int e = tid; e < C * (D / 8); e += NTH) {
                const int r = e >> 3, d0 = (e & 7) * 8;
                const int64_t t = c0 + r;
                const bool ok = t < t_end;
                uint4 qv = make_uint4(0, 0, 0, 0), kv = qv, bv = qv, gv = qv, vv = qv, wv = qv;
                if (ok) {
                    qv = *reinterpret_cast<const uint4*>(q + t * a.sq[2] + d0);
                    kv = *reinterpret_cast<const uint4*>(k + t * a.sk[2] + d0);
                    bv = *reinterpret_cast<const uint4*>(bb + t * a.sb[2] + d0);
                    gv = lal ? *reinterpret_cast<const uint4*>(lal + t * a.sla[2] + d0)
                             : *reinterpret_cast<const uint4*>(al + t * a.sa[2] + d0);
                    vv = *reinterpret_cast<const uint4*>(v + t * a.sv[2] + d0);
                    wv = *reinterpret_cast<const uint4*>(w + t * a.sw[2] + d0);
                }
                *reinterpret_cast<uint4*>(QR + r * LB + d0) = qv;
                *reinterpret_cast<uint4*>(KR + r * LB + d0) = kv;
                const T* kx = reinterpret_cast<const T*>(&kv);
                const T* bx = reinterpret_cast<const T*>(&bv);
                const T* gx = reinterpret_cast<const T*>(&gv);
                const T* vx = reinterpret_cast<const T*>(&vv);
                const T* wx = reinterpret_cast<const T*>(&wv);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float g = 0.f;
                    if (ok) {
                        if (lal) {
                            g = fminf(fmaxf(f32(gx[j]), -46.f), 0.f);
                        } else {
                            g = logf(fminf(fmaxf(f32(gx[j]), 1e-20f), 1.f));
                        }
                    }
                    Gs[r * LF + d0 + j] = g;
                    BKs[r * LF + d0 + j] = f32(bx[j]) * f32(kx[j]);
                    WVs[r * LF + d0 + j] = f32(wx[j]) * f32(vx[j]);
                }
            }
        } else {
            for (int e = tid; e < C * D; e += NTH) {
                const int r = e >> 6, d = e & 63;
                const int64_t t = c0 + r;
                float qv = 0.f, kv = 0.f, bv = 0.f, g = 0.f, wvv = 0.f;
                if (t < t_end) {
                    if (d < dk) {
                        qv = f32(q[t * a.sq[2] + d * a.sq[3]]);
                        kv = f32(k[t * a.sk[2] + d * a.sk[3]]);
                        bv = f32(bb[t * a.sb[2] + d * a.sb[3]]);
                        if (lal) g = fminf(fmaxf(f32(lal[t * a.sla[2] + d * a.sla[3]]), -46.f), 0.f);
                        else g = logf(fminf(fmaxf(f32(al[t * a.sa[2] + d * a.sa[3]]), 1e-20f), 1.f));
                    }
                    if (d < dv) wvv = f32(w[t * a.sw[2] + d * a.sw[3]]) * f32(v[t * a.sv[2] + d * a.sv[3]]);
                }
                QR[r * LB + d] = to16<T>(qv);
                KR[r * LB + d] = to16<T>(kv);
                BKs[r * LF + d] = bv * kv;
                Gs[r * LF + d] = g;
                WVs[r * LF + d] = wvv;
            }
        }
        __syncthreads();
        // ---------------- cumulative log decay per channel -------------------------
        if (tid < D) {
            float run = 0.f;
            for (int r = 0; r < C; ++r) {
                run += Gs[r * LF + tid];
                Gs[r * LF + tid] = run;
            }
        }
        if (tid < NB) flags[tid] = 0;
        __syncthreads();
        // ---------------- decayed operands, factor operands -----------------------
        for (int e = tid; e < C * D; e += NTH) {
            const int r = e >> 6, d = e & 63;
            const float g = Gs[r * LF + d];
            const float ge = Gs[(C - 1) * LF + d];
            const float qv = f32(QR[r * LB + d]), kv = f32(KR[r * LB + d]), bk = BKs[r * LF + d];
            const float eg = __expf(g);
            QTs[r * LB + d] = to16<T>(qv * eg);
            BTs[r * LB + d] = to16<T>(bk * eg);
            KTs[r * LB + d] = to16<T>(kv * __expf(ge - g));
            if (r == 0) dend[d] = __expf(ge);
            if (r >= 16) {
                const int I = r >> 4;
                const float f = __expf(g - Gs[(16 * I - 1) * LF + d]);
                QH[(r - 16) * LB + d] = to16<T>(qv * f);
                BHs[(r - 16) * LB + d] = to16<T>(bk * f);
            }
            const float g0 = Gs[(r & ~15) * LF + d];  // first row of this row's 16-block
            const float fd = __expf(g - g0);           // <= 1
            QD[r * LB + d] = to16<T>(qv * fd);
            BDs[r * LB + d] = to16<T>(bk * fd);
            KD[r * LB + d] = to16<T>(kv * __expf(g0 - g));  // >= 1, bounded when the block is flat enough
            // factor range: bf16 keeps e^80 (8-bit exponent), fp16 tops out near 6.5e4
            constexpr float kFlat = std::is_same<T, __half>::value ? 8.f : 80.f;
            if ((r & 15) == 15 && g0 - g > kFlat) atomicOr(&flags[r >> 4], 1);
        }
        for (int e = tid; e < 96 * D; e += NTH) {
            const int row = e >> 6, d = e & 63;
            const int I = row < 16 ? 1 : (row < 48 ? 2 : 3);
            const int j = row - kh_off(I);
            const float ref = Gs[(16 * I - 1) * LF + d];
            KH[row * LB + d] = to16<T>(f32(KR[j * LB + d]) * __expf(ref - Gs[j * LF + d]));
        }
        for (int e = tid; e < C * C; e += NTH) {  // strictly-upper off-diagonal blocks
            const int i = e >> 6, j = e & 63;
            if ((j >> 4) > (i >> 4)) {
                AM[i * LB + j] = to16<T>(0.f);
                LM[i * LB + j] = to16<T>(0.f);
            }
        }
        __syncthreads();
        // ---------------- A / L blocks: off-diagonal and factorisable diagonal on the tensor cores ----
        {
            // diagonal block blk, A (warp even) or L (warp odd): one 16x16 product per warp
            const int blk = warp >> 1;
            const bool isL = warp & 1;
            if (!flags[blk]) {
                float acc[2][4] = {};
                warp_mma<T, false, false, 2>(acc, (isL ? BDs : QD) + (16 * blk) * LB, LB, KD + (16 * blk) * LB, LB, D,
                                             lane);
#pragma unroll
                for (int n = 0; n < 2; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int ii = fr + (e >> 1) * 8, jj = n * 8 + fc + (e & 1);
                        const float x = isL ? (jj < ii ? acc[n][e] : 0.f) : (jj <= ii ? acc[n][e] : 0.f);
                        const int i = blk * 16 + ii, j = blk * 16 + jj;
                        if (isL) {
                            LM[i * LB + j] = to16<T>(x);
                            LDs[(blk * 16 + ii) * 17 + jj] = x;
                        } else {
                            AM[i * LB + j] = to16<T>(x);
                        }
                    }
            }
        }
        for (int p = tid; p < NB * 256; p += NTH) {  // steep blocks: explicit per-element decay
            const int blk = p >> 8, ii = (p >> 4) & 15, jj = p & 15;
            if (!flags[blk]) continue;
            const int i = blk * 16 + ii, j = blk * 16 + jj;
            float av = 0.f, lv = 0.f;
            if (jj <= ii) {
                const float* gi = Gs + i * LF;
                const float* gj = Gs + j * LF;
                const float* bki = BKs + i * LF;
                for (int d = 0; d < dk; ++d) {
                    const float kd = f32(KR[j * LB + d]) * __expf(gi[d] - gj[d]);
                    av = fmaf(f32(QR[i * LB + d]), kd, av);
                    lv = fmaf(bki[d], kd, lv);
                }
            }
            if (jj >= ii) lv = 0.f;
            AM[i * LB + j] = to16<T>(av);
            LM[i * LB + j] = to16<T>(lv);
            LDs[(blk * 16 + ii) * 17 + jj] = lv;
        }
        for (int tile = warp; tile < 12; tile += 8) {
            // I=1: tiles 0,1; I=2: 2..5; I=3: 6..11; within I: first I tiles give A, next I give L
            const int I = tile < 2 ? 1 : (tile < 6 ? 2 : 3);
            const int t_in = tile - (I == 1 ? 0 : (I == 2 ? 2 : 6));
            const bool isL = t_in >= I;
            const int n16 = isL ? t_in - I : t_in;  // 16-key column tile within [0, 16I)
            float acc[2][4] = {};
            const T* Ap = (isL ? BHs : QH) + (16 * (I - 1)) * LB;
            const T* Bp = KH + (kh_off(I) + 16 * n16) * LB;
            warp_mma<T, false, false, 2>(acc, Ap, LB, Bp, LB, D, lane);
            store_acc16<T, 2>((isL ? LM : AM) + (16 * I) * LB + 16 * n16, LB, acc, lane);
        }
        __syncthreads();
        if (tid < 64) {
            const int blk = tid >> 4, c = tid & 15;
            float tcol[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) tcol[r] = r == c ? 1.f : 0.f;
#pragma unroll
            for (int r = 1; r < 16; ++r) {
                if (r > c) {
                    float s = 0.f;
                    for (int m = c; m < r; ++m) s = fmaf(LDs[(blk * 16 + r) * 17 + m], tcol[m], s);
                    tcol[r] = -s;
                }
            }
#pragma unroll
            for (int r = 0; r < 16; ++r) TDs[(blk * 16 + r) * LT + c] = to16<T>(tcol[r]);
        }
        __syncthreads();
        // ---------------- T = (I + L)^{-1} by blocks ------------------------------------
        for (int e = tid; e < 16 * C; e += NTH) {
            const int r = e >> 6, c = e & 63;
            TM[r * LB + c] = c < 16 ? TDs[r * LT + c] : to16<T>(0.f);
        }
        __syncthreads();
        for (int I = 1; I < NB; ++I) {
            // M = L[I, <I] T[<I, <I]  (16 x 16I), one 16-column tile per warp
            if (warp < I) {
                float acc[2][4] = {};
                warp_mma<T, false, true, 2>(acc, LM + (16 * I) * LB, LB, TM + 16 * warp, LB, 16 * I, lane);
                store_acc16<T, 2>(RB + 16 * warp, LB, acc, lane);
            }
            __syncthreads();
            if (warp < I) {  // T[I, <I] = -T_II M
                float acc[2][4] = {};
                warp_mma<T, false, true, 2>(acc, TDs + (16 * I) * LT, LT, RB + 16 * warp, LB, 16, lane);
#pragma unroll
                for (int n = 0; n < 2; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[n][e] = -acc[n][e];
                store_acc16<T, 2>(TM + (16 * I) * LB + 16 * warp, LB, acc, lane);
            }
            for (int e = tid; e < 16 * (C - 16 * I); e += NTH) {
                const int r = e / (C - 16 * I), c = 16 * I + e % (C - 16 * I);
                TM[(16 * I + r) * LB + c] = c < 16 * I + 16 ? TDs[(16 * I + r) * LT + (c - 16 * I)] : to16<T>(0.f);
            }
            __syncthreads();
        }
        // ---------------- state chain ---------------------------------------------------
        float racc[NTW][4] = {};
        float qacc[NTW][4] = {};
        warp_mma<T, false, true, NTW>(racc, BTs + wr * LB, LB, SB + wc, LN, D, lane);
        if (MODE != 1) warp_mma<T, false, true, NTW>(qacc, QTs + wr * LB, LB, SB + wc, LN, D, lane);
#pragma unroll
        for (int n = 0; n < NTW; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = wr + fr + (e >> 1) * 8;
                const int c = wc + n * 8 + fc + (e & 1);
                const float u = c < D ? WVs[r * LF + c] : 0.f;
                racc[n][e] = u - racc[n][e];
            }
        store_acc16<T, NTW>(RB + wr * LN + wc, LN, racc, lane);
        __syncthreads();
        {
            float vacc[NTW][4] = {};
            warp_mma<T, false, true, NTW>(vacc, TM + wr * LB, LB, RB + wc, LN, C, lane);
            store_acc16<T, NTW>(VP + wr * LN + wc, LN, vacc, lane);
        }
        __syncthreads();
        if (MODE != 1) {
            warp_mma<T, false, true, NTW>(qacc, AM + wr * LB, LB, VP + wc, LN, C, lane);
            T* o = static_cast<T*>(a.out);
#pragma unroll
            for (int n = 0; n < NTW; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int r = wr + fr + (e >> 1) * 8;
                    const int c = wc + n * 8 + fc + (e & 1);
                    const int64_t t = c0 + r;
                    if (t < t_end && c < dv)
                        o[bi * a.so[0] + hi * a.so[1] + t * a.so[2] + (int64_t)c * a.so[3]] = to16<T>(qacc[n][e]);
                }
        }
#pragma unroll
        for (int n = 0; n < NTW; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) sacc[n][e] *= dend[wr + fr + (e >> 1) * 8];
        warp_mma<T, true, true, NTW>(sacc, KTs + wr, LB, VP + wc, LN, C, lane);
        store_acc16<T, NTW>(SB + wr * LN + wc, LN, sacc, lane);
    }
    __syncthreads();
    // ---------------- results -----------------------------------------------------------
#pragma unroll
    for (int n = 0; n < NTW; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = wr + fr + (e >> 1) * 8;
            const int c = wc + n * 8 + fc + (e & 1);
            if (MODE == 1) {
                a.ws_trans[(((size_t)bh * a.nseg + seg) * D + d) * (2 * D) + c] = sacc[n][e];
            } else if (MODE == 0 || seg == a.nseg - 1) {
                if (d < dk && c < dv)
                    store_from<TS, float>(static_cast<TS*>(a.fin) + bi * a.sf[0] + hi * a.sf[1] + (int64_t)d * a.sf[2] +
                                              (int64_t)c * a.sf[3],
                                          sacc[n][e]);
            }
        }
}

template <typename T, typename TS, int MODE>
int launch_one(const PrefillArgs& a, dim3 grid, cudaStream_t s) {
    constexpr size_t smem = MS<MODE == 1 ? 2 * D : D>::TOTAL;
    auto kern = dgda_mma_kernel<T, TS, MODE>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(MABA_ERR_CUDA, "dgda_prefill(mma): %s", cudaGetErrorString(e));
    kern<<<grid, NTH, smem, s>>>(a);
    return check_launch("dgda_prefill(mma)");
}

template <typename T, typename TS>
int launch_mode(const PrefillArgs& a, dim3 grid, int mode, cudaStream_t s) {
    switch (mode) {
        case 0: return launch_one<T, TS, 0>(a, grid, s);
        case 1: return launch_one<T, TS, 1>(a, grid, s);
        default: return launch_one<T, TS, 2>(a, grid, s);
    }
}

}  // namespace

size_t dgda_mma_smem_bytes(int mode) { return mode == 1 ? MS<2 * D>::TOTAL : MS<D>::TOTAL; }

int dgda_mma_launch(const PrefillArgs& a, dim3 grid, int mode, int dtype, int state_dtype, cudaStream_t s) {
    if (dtype == MABA_BF16)
        return state_dtype == MABA_F32 ? launch_mode<__nv_bfloat16, float>(a, grid, mode, s)
                                       : launch_mode<__nv_bfloat16, __nv_bfloat16>(a, grid, mode, s);
    if (dtype == MABA_F16)
        return state_dtype == MABA_F32 ? launch_mode<__half, float>(a, grid, mode, s)
                                       : launch_mode<__half, __half>(a, grid, mode, s);
    return set_error(MABA_ERR_DTYPE, "dgda_prefill(mma): 16-bit inputs only");
}

}  // namespace maba
