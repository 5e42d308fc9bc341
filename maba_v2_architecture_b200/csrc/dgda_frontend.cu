// DGDA front end: everything the DGDA layer computes between its projections and
// the recurrence, in one pass over the projected features.
//
// Reference (maba_sparse/layers/dgda.py): the causal depthwise conv (kernel
// K = 4) with history and SiLU on q, k and v (_apply_conv :103-122, called at
// :186-190 and :254-258), the gates b = sigmoid(gate_erase x), w = sigmoid(
// gate_write x), log alpha = max(-softplus(gate_alpha x), -14) (:192-197,
// :260-264), and the per-head L2 normalisation k / (||k|| + eps) (:207, :270).
//
// Layout: every operand is a [B, L, C] view (any strides; C = H * d), the six
// projected inputs typically being column ranges of one fused projection
// output.  One thread owns 8 consecutive channels of one section and a run of
// RUN consecutive tokens: it keeps the last K-1 conv inputs in registers, so
// each input row is read once; threads of one token run cover all six sections
// in channel order, so a warp's loads of a row are contiguous.  The head norm
// of k is a shuffle reduction over the d/8 lanes of a head (d/8 a power of two
// <= 32, so a head never straddles a warp).
#include "common.cuh"
#include "activations.cuh"

namespace maba {
namespace {

constexpr int kVec = 8;       // channels per thread
constexpr int kRun = 8;       // tokens per thread
constexpr int kMaxTaps = 8;   // conv kernel size limit
constexpr int kFeThreads = 256;

struct FeSection {
    const void* x;            // projected input [B, L, C]
    void* out;                // feature output [B, L, C]
    int64_t sx[3], so[3];
};

struct FeArgs {
    FeSection sec[6];         // q, k, v, alpha, erase (b), write (w)
    const void* conv[3];      // [C, K] taps of q, k, v
    int64_t sconv[3][2];
    const void* hist[3];      // [B, C, K-1] conv inputs before token 0 (nullptr: zeros)
    int64_t sh[3][3];
    int64_t B, L;
    int C[6];                 // channels per section (q, k, alpha, erase: H*dk; v, write: H*dv)
    int groups[6];            // C / 8
    int gbase[7];             // prefix sums of groups: thread index of each section inside a token run
    int per_run;              // threads per token run: gbase[6] rounded up to a warp
    int K;                    // conv taps
    int hw;                   // lanes per head of the k section (dk / 8)
    float eps;
    int hist_f32;             // history stored as float32 (else the feature dtype)
};

template <typename T>
__device__ __forceinline__ void load8(const T* p, int64_t stride, float* v) {
#pragma unroll
    for (int i = 0; i < kVec; ++i) v[i] = Cvt<T>::to_f(p[i * stride]);
}

template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, int64_t stride, float* v) {
    if (stride == 1 && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < kVec; ++i) v[i] = __bfloat162float(p[i * stride]);
    }
}

template <typename T>
__device__ __forceinline__ void store8(T* p, int64_t stride, const float* v) {
#pragma unroll
    for (int i = 0; i < kVec; ++i) p[i * stride] = Cvt<T>::from_f(v[i]);
}

template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* p, int64_t stride, const float* v) {
    if (stride == 1 && (reinterpret_cast<uintptr_t>(p) & 15u) == 0) {
        uint4 u;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        *reinterpret_cast<uint4*>(p) = u;
    } else {
#pragma unroll
        for (int i = 0; i < kVec; ++i) p[i * stride] = __float2bfloat16_rn(v[i]);
    }
}


template <typename T, int K>
__global__ void __launch_bounds__(kFeThreads) dgda_frontend_kernel(FeArgs a, int64_t nruns) {
    const int per_run = a.per_run;
    const int64_t gid = (int64_t)blockIdx.x * kFeThreads + threadIdx.x;
    const int64_t total = a.B * nruns * per_run;
    const int64_t gg = gid < total ? gid : 0;
    const int slot = (int)(gg % per_run);
    const bool live = gid < total && slot < a.gbase[6];
    const int64_t run = (gg / per_run) % nruns;
    const int64_t b = gg / ((int64_t)per_run * nruns);
    int s = 0;
#pragma unroll
    for (int i = 1; i < 6; ++i) s += slot >= a.gbase[i] ? 1 : 0;
    const int g = slot - a.gbase[s];
    const int c0 = g * kVec;
    const FeSection& sec = a.sec[s];
    const T* x = static_cast<const T*>(sec.x) + b * sec.sx[0] + (int64_t)c0 * sec.sx[2];
    T* out = static_cast<T*>(sec.out) + b * sec.so[0] + (int64_t)c0 * sec.so[2];
    const int64_t t0 = run * kRun;
    const bool conv = s < 3;

    // conv taps of these 8 channels and the K-1 inputs before t0
    float w[K][kVec];
    float win[K][kVec];  // win[j] = input at t0 - (K-1) + j, j < K-1
    if (conv && live) {
        const T* cw = static_cast<const T*>(a.conv[s]);
#pragma unroll
        for (int j = 0; j < K; ++j)
#pragma unroll
            for (int i = 0; i < kVec; ++i)
                w[j][i] = Cvt<T>::to_f(cw[(int64_t)(c0 + i) * a.sconv[s][0] + j * a.sconv[s][1]]);
#pragma unroll
        for (int j = 0; j < K - 1; ++j) {
            const int64_t t = t0 - (K - 1) + j;
            if (t >= 0) {
                load8<T>(x + t * sec.sx[1], sec.sx[2], win[j]);
            } else if (a.hist[s] != nullptr) {
                const int64_t hj = (K - 1) + t;  // column of the history (oldest first)
                const int64_t base = b * a.sh[s][0] + hj * a.sh[s][2];
#pragma unroll
                for (int i = 0; i < kVec; ++i) {
                    const int64_t off = base + (int64_t)(c0 + i) * a.sh[s][1];
                    win[j][i] = a.hist_f32 ? static_cast<const float*>(a.hist[s])[off]
                                           : Cvt<T>::to_f(static_cast<const T*>(a.hist[s])[off]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < kVec; ++i) win[j][i] = 0.f;
            }
        }
    }
#pragma unroll 1
    for (int r = 0; r < kRun; ++r) {
        const int64_t t = t0 + r;
        const bool ok = live && t < a.L;
        float v[kVec];
        if (ok) load8<T>(x + t * sec.sx[1], sec.sx[2], v);
        float y[kVec];
        if (conv) {
#pragma unroll
            for (int i = 0; i < kVec; ++i) {
                float acc = 0.f;
#pragma unroll
                for (int j = 0; j < K - 1; ++j) acc = fmaf(w[j][i], win[j][i], acc);
                acc = fmaf(w[K - 1][i], ok ? v[i] : 0.f, acc);
                y[i] = silu_f(acc);
            }
#pragma unroll
            for (int j = 0; j + 1 < K - 1; ++j)
#pragma unroll
                for (int i = 0; i < kVec; ++i) win[j][i] = win[j + 1][i];
            if constexpr (K > 1)
#pragma unroll
                for (int i = 0; i < kVec; ++i) win[K - 2][i] = ok ? v[i] : 0.f;
        } else if (s == 3) {
#pragma unroll
            for (int i = 0; i < kVec; ++i) y[i] = ok ? neg_softplus_clamped(v[i]) : 0.f;
        } else {
#pragma unroll
            for (int i = 0; i < kVec; ++i) y[i] = ok ? sigmoid_f(v[i]) : 0.f;
        }
        // per-head L2 norm of k: every lane takes part in the shuffles
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kVec; ++i) ss = fmaf(y[i], y[i], ss);
        for (int o = a.hw >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (s == 1) {
            const float inv = 1.f / (sqrtf(ss) + a.eps);
#pragma unroll
            for (int i = 0; i < kVec; ++i) y[i] *= inv;
        }
        if (ok) store8<T>(out + t * sec.so[1], sec.so[2], y);
    }
}

// Tiled variant for sections of a multiple of 128 channels (heads of dk <= 128
// lanes x 8 channels): one CTA owns 128 tokens x 128 channels of one section.  The
// tile's input rows and the K-1 rows before it (or the conv history) are staged in
// shared memory with 16-byte loads, all in flight at once, together with the 128
// channels' taps; thread (token group, channel group of 8) then forms its outputs
// from shared memory, so the loads of a token's neighbours cost no extra DRAM
// traffic and every thread has its whole input staged before it computes (eight
// 16-byte loads in flight per thread).
constexpr int kTileTok = 128;
constexpr int kTileCh = 128;

// 8 16-bit values <-> a 16-byte word, in registers (no addressable temporaries)
template <typename T> __device__ __forceinline__ void unpack8_bits(const uint4& u, float* v);
template <> __device__ __forceinline__ void unpack8_bits<__nv_bfloat16>(const uint4& u, float* v) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
template <> __device__ __forceinline__ void unpack8_bits<__half>(const uint4& u, float* v) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
        v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
    }
}
template <typename T> __device__ __forceinline__ uint32_t pack2_bits(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2_bits<__nv_bfloat16>(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
template <> __device__ __forceinline__ uint32_t pack2_bits<__half>(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}

template <typename T, int K>
__global__ void __launch_bounds__(256, 4) dgda_frontend_tile_kernel(FeArgs a, int64_t ntt, int nct) {
    constexpr int ROWS = kTileTok + K - 1;
    constexpr int LDS = kTileCh + 8;  // padded row (16-bit elements)
    __shared__ __align__(16) T xs[ROWS][LDS];
    __shared__ float taps[kTileCh][K];
    const int tid = threadIdx.x;
    int64_t blk = blockIdx.x;
    const int ct = (int)(blk % nct);  // 128-channel chunk over the six sections
    blk /= nct;
    const int64_t tt = blk % ntt;
    const int64_t b = blk / ntt;
    // section of this chunk (sections are multiples of 128 channels)
    int s = 0, cbase = ct * kTileCh;
#pragma unroll
    for (int i = 0; i < 5; ++i)
        if (cbase >= a.C[s]) { cbase -= a.C[s]; ++s; }
    const FeSection& sec = a.sec[s];
    const T* x = static_cast<const T*>(sec.x) + b * sec.sx[0] + (int64_t)cbase * sec.sx[2];
    const int64_t t0 = tt * kTileTok;
    const bool conv = s < 3;
    // stage rows t0-(K-1) .. t0+31: 16 chunks of 8 channels per row
    for (int e = tid; e < ROWS * 16; e += 256) {
        const int r = e >> 4, c8 = (e & 15) * 8;
        const int64_t t = t0 - (K - 1) + r;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (t >= 0 && t < a.L) {
            v = *reinterpret_cast<const uint4*>(x + t * sec.sx[1] + c8);
        } else if (t < 0 && conv && a.hist[s] != nullptr) {
            T* h8 = reinterpret_cast<T*>(&v);
            const int64_t hj = (K - 1) + t;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int64_t off = b * a.sh[s][0] + (int64_t)(cbase + c8 + i) * a.sh[s][1] + hj * a.sh[s][2];
                const float hv = a.hist_f32 ? static_cast<const float*>(a.hist[s])[off]
                                            : Cvt<T>::to_f(static_cast<const T*>(a.hist[s])[off]);
                h8[i] = Cvt<T>::from_f(hv);
            }
        }
        *reinterpret_cast<uint4*>(&xs[r][c8]) = v;
    }
    if (conv) {
        const T* cw = static_cast<const T*>(a.conv[s]);
        for (int e = tid; e < kTileCh * K; e += 256) {
            const int c = e / K, j = e - (e / K) * K;
            taps[c][j] = Cvt<T>::to_f(cw[(int64_t)(cbase + c) * a.sconv[s][0] + j * a.sconv[s][1]]);
        }
    }
    __syncthreads();
    const int g = tid & 15;          // channel group (8 channels)
    const int tp = tid >> 4;         // token group 0..15 (kTileTok / 16 consecutive tokens)
    T* out = static_cast<T*>(sec.out) + b * sec.so[0] + (int64_t)(cbase + g * 8) * sec.so[2];
    float w[kVec][K];
    if (conv)
#pragma unroll
        for (int i = 0; i < kVec; ++i)
#pragma unroll
            for (int j = 0; j < K; ++j) w[i][j] = taps[g * 8 + i][j];
    constexpr int TPT = kTileTok / 16;  // tokens per thread
#pragma unroll 2
    for (int u = 0; u < TPT; ++u) {
        const int r = tp * TPT + u;  // token t0 + r, staged at row r + K - 1
        const int64_t t = t0 + r;
        float y[kVec];
        if (conv) {
            float acc[kVec];
#pragma unroll
            for (int i = 0; i < kVec; ++i) acc[i] = 0.f;
#pragma unroll
            for (int j = 0; j < K; ++j) {
                float e[kVec];
                unpack8_bits<T>(*reinterpret_cast<const uint4*>(&xs[r + j][g * 8]), e);
#pragma unroll
                for (int i = 0; i < kVec; ++i) acc[i] = fmaf(w[i][j], e[i], acc[i]);
            }
#pragma unroll
            for (int i = 0; i < kVec; ++i) y[i] = silu_f(acc[i]);
        } else {
            float e[kVec];
            unpack8_bits<T>(*reinterpret_cast<const uint4*>(&xs[r + K - 1][g * 8]), e);
#pragma unroll
            for (int i = 0; i < kVec; ++i) y[i] = s == 3 ? neg_softplus_clamped(e[i]) : sigmoid_f(e[i]);
        }
        if (s == 1) {  // per-head L2 norm of k (the section is the same for the whole CTA)
            float ss = 0.f;
#pragma unroll
            for (int i = 0; i < kVec; ++i) ss = fmaf(y[i], y[i], ss);
            for (int o = a.hw >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv = 1.f / (sqrtf(ss) + a.eps);
#pragma unroll
            for (int i = 0; i < kVec; ++i) y[i] *= inv;
        }
        if (t < a.L) {
            T* op = out + t * sec.so[1];
            if (sec.so[2] == 1 && (reinterpret_cast<uintptr_t>(op) & 15u) == 0)
                *reinterpret_cast<uint4*>(op) = make_uint4(pack2_bits<T>(y[0], y[1]), pack2_bits<T>(y[2], y[3]),
                                                           pack2_bits<T>(y[4], y[5]), pack2_bits<T>(y[6], y[7]));
            else
                store8<T>(op, sec.so[2], y);
        }
    }
}

// Persistent double-buffered form of the tiled kernel: each CTA walks the tiles
// blockIdx.x, blockIdx.x + gridDim.x, ... and copies the next tile's input rows (and
// its conv taps) into the other shared-memory stage with cp.async while it computes
// the current one, so the loads of one tile run under the conv and gates of the
// previous.  Rows before token 0 are zero-filled by the copy and then overwritten
// from the conv history; rows past the end are zero-filled.  Needs 16-byte aligned
// contiguous taps ([C, K] rows of K 16-bit values) and K <= 8.
__device__ __forceinline__ void fe_cp16(void* dst, const void* src, bool valid) {
    // cp.async with a source size of 0 writes zeros (the source is not read)
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
                 "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void fe_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void fe_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

template <typename T, int K>
__global__ void __launch_bounds__(256, 3) dgda_frontend_pipe_kernel(FeArgs a, int64_t ntt, int nct, int64_t ntiles) {
    constexpr int ROWS = kTileTok + K - 1;
    constexpr int LDS = kTileCh + 8;  // padded row (16-bit elements)
    constexpr int TAPB = kTileCh * K * 2;  // bytes of one tile's taps (multiple of 16: K even or 128 channels)
    extern __shared__ __align__(16) unsigned char fe_sm[];
    T* xs0 = reinterpret_cast<T*>(fe_sm);                                  // [2][ROWS][LDS]
    T* tp0 = reinterpret_cast<T*>(fe_sm + 2 * (size_t)ROWS * LDS * 2);     // [2][kTileCh * K]
    const int tid = threadIdx.x;
    const int g = tid & 15;   // channel group (8 channels)
    const int tp = tid >> 4;  // token group
    constexpr int TPT = kTileTok / 16;

    struct Tile { int64_t b, t0; int s, cbase; };
    auto decode = [&](int64_t blk) {
        Tile tl;
        const int ct = (int)(blk % nct);
        blk /= nct;
        tl.t0 = (blk % ntt) * kTileTok;
        tl.b = blk / ntt;
        tl.s = 0;
        tl.cbase = ct * kTileCh;
#pragma unroll
        for (int i = 0; i < 5; ++i)
            if (tl.cbase >= a.C[tl.s]) { tl.cbase -= a.C[tl.s]; ++tl.s; }
        return tl;
    };
    auto issue = [&](int64_t blk, int stage) {
        const Tile tl = decode(blk);
        const FeSection& sec = a.sec[tl.s];
        const T* x = static_cast<const T*>(sec.x) + tl.b * sec.sx[0] + (int64_t)tl.cbase * sec.sx[2];
        T* xs = xs0 + (size_t)stage * ROWS * LDS;
        for (int e = tid; e < ROWS * 16; e += 256) {
            const int r = e >> 4, c8 = (e & 15) * 8;
            const int64_t t = tl.t0 - (K - 1) + r;
            const bool ok = t >= 0 && t < a.L;
            fe_cp16(xs + r * LDS + c8, ok ? static_cast<const void*>(x + t * sec.sx[1] + c8) : static_cast<const void*>(x), ok);
        }
        if (tl.s < 3 && tid < TAPB / 16) {
            const T* cw = static_cast<const T*>(a.conv[tl.s]) + (int64_t)tl.cbase * K;
            fe_cp16(reinterpret_cast<unsigned char*>(tp0 + (size_t)stage * kTileCh * K) + tid * 16,
                    reinterpret_cast<const unsigned char*>(cw) + tid * 16, true);
        }
        fe_commit();
    };

    int64_t blk = blockIdx.x;
    if (blk < ntiles) issue(blk, 0);
    for (int k = 0; blk < ntiles; ++k, blk += gridDim.x) {
        const int stage = k & 1;
        const int64_t nxt = blk + gridDim.x;
        if (nxt < ntiles) {
            issue(nxt, stage ^ 1);
            fe_wait<1>();
        } else {
            fe_wait<0>();
        }
        __syncthreads();
        const Tile tl = decode(blk);
        const FeSection& sec = a.sec[tl.s];
        const bool conv = tl.s < 3;
        T* xs = xs0 + (size_t)stage * ROWS * LDS;
        if (conv && tl.t0 == 0 && a.hist[tl.s] != nullptr) {
            // the K-1 rows before token 0 come from the conv history
            for (int e = tid; e < (K - 1) * kTileCh; e += 256) {
                const int r = e / kTileCh, c = e - r * kTileCh;
                const int64_t hj = r;  // history column (oldest first) = staged row r
                const int64_t off = tl.b * a.sh[tl.s][0] + (int64_t)(tl.cbase + c) * a.sh[tl.s][1] + hj * a.sh[tl.s][2];
                const float hv = a.hist_f32 ? static_cast<const float*>(a.hist[tl.s])[off]
                                            : Cvt<T>::to_f(static_cast<const T*>(a.hist[tl.s])[off]);
                xs[r * LDS + c] = Cvt<T>::from_f(hv);
            }
            __syncthreads();
        }
        T* out = static_cast<T*>(sec.out) + tl.b * sec.so[0] + (int64_t)(tl.cbase + g * 8) * sec.so[2];
        float w[kVec][K];
        if (conv) {
            const T* tps = tp0 + (size_t)stage * kTileCh * K;
#pragma unroll
            for (int i = 0; i < kVec; ++i)
#pragma unroll
                for (int j = 0; j < K; ++j) w[i][j] = Cvt<T>::to_f(tps[(g * 8 + i) * K + j]);
        }
#pragma unroll 2
        for (int u = 0; u < TPT; ++u) {
            const int r = tp * TPT + u;  // token t0 + r, staged at row r + K - 1
            const int64_t t = tl.t0 + r;
            float y[kVec];
            if (conv) {
                float acc[kVec];
#pragma unroll
                for (int i = 0; i < kVec; ++i) acc[i] = 0.f;
#pragma unroll
                for (int j = 0; j < K; ++j) {
                    float e[kVec];
                    unpack8_bits<T>(*reinterpret_cast<const uint4*>(xs + (r + j) * LDS + g * 8), e);
#pragma unroll
                    for (int i = 0; i < kVec; ++i) acc[i] = fmaf(w[i][j], e[i], acc[i]);
                }
#pragma unroll
                for (int i = 0; i < kVec; ++i) y[i] = silu_f(acc[i]);
            } else {
                float e[kVec];
                unpack8_bits<T>(*reinterpret_cast<const uint4*>(xs + (r + K - 1) * LDS + g * 8), e);
#pragma unroll
                for (int i = 0; i < kVec; ++i) y[i] = tl.s == 3 ? neg_softplus_clamped(e[i]) : sigmoid_f(e[i]);
            }
            if (tl.s == 1) {  // per-head L2 norm of k
                float ss = 0.f;
#pragma unroll
                for (int i = 0; i < kVec; ++i) ss = fmaf(y[i], y[i], ss);
                for (int o = a.hw >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                const float inv = 1.f / (sqrtf(ss) + a.eps);
#pragma unroll
                for (int i = 0; i < kVec; ++i) y[i] *= inv;
            }
            if (t < a.L) {
                T* op = out + t * sec.so[1];
                if (sec.so[2] == 1 && (reinterpret_cast<uintptr_t>(op) & 15u) == 0)
                    *reinterpret_cast<uint4*>(op) = make_uint4(pack2_bits<T>(y[0], y[1]), pack2_bits<T>(y[2], y[3]),
                                                               pack2_bits<T>(y[4], y[5]), pack2_bits<T>(y[6], y[7]));
                else
                    store8<T>(op, sec.so[2], y);
            }
        }
        __syncthreads();  // every read of this stage is done before the next copy into it
    }
}

// new conv history [B, C, K-1]: the last K-1 inputs of [history | x]
template <typename T, typename TH>
__global__ void dgda_frontend_hist_kernel(FeArgs a, void* nq, void* nk, void* nv, int64_t snh0, int64_t snh1,
                                          int64_t snh2, int64_t snh3, int64_t snh4, int64_t snh5, int64_t snh6,
                                          int64_t snh7, int64_t snh8) {
    const int64_t sn[3][3] = {{snh0, snh1, snh2}, {snh3, snh4, snh5}, {snh6, snh7, snh8}};
    void* dst[3] = {nq, nk, nv};
    const int K1 = a.K - 1;
    const int64_t per_b = (int64_t)(a.C[0] + a.C[1] + a.C[2]) * K1;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.B * per_b) return;
    const int64_t b = i / per_b;
    int64_t rem = i % per_b;
    int s = 0;
    while (s < 2 && rem >= (int64_t)a.C[s] * K1) { rem -= (int64_t)a.C[s] * K1; ++s; }
    if (dst[s] == nullptr) return;
    const int64_t c = rem / K1;
    const int j = (int)(rem % K1);
    const int64_t t = a.L - K1 + j;  // time index of history column j
    float v = 0.f;
    if (t >= 0) {
        const FeSection& sec = a.sec[s];
        v = Cvt<T>::to_f(static_cast<const T*>(sec.x)[b * sec.sx[0] + t * sec.sx[1] + c * sec.sx[2]]);
    } else if (a.hist[s] != nullptr) {
        const int64_t off = b * a.sh[s][0] + c * a.sh[s][1] + (K1 + t) * a.sh[s][2];
        v = a.hist_f32 ? static_cast<const float*>(a.hist[s])[off] : Cvt<T>::to_f(static_cast<const T*>(a.hist[s])[off]);
    }
    static_cast<TH*>(dst[s])[b * sn[s][0] + c * sn[s][1] + j * sn[s][2]] = Cvt<TH>::from_f(v);
}

}  // namespace
}  // namespace maba

using namespace maba;

extern "C" int maba_dgda_frontend(const maba_tensor* proj, const maba_tensor* conv_w, const maba_tensor* hist,
                                  const maba_tensor* out, const maba_tensor* new_hist, int32_t n_heads, float eps,
                                  void* stream) {
    if (proj == nullptr || conv_w == nullptr || out == nullptr)
        return set_error(MABA_ERR_INVALID, "dgda_frontend: proj[6], conv_w[3] and out[6] are required");
    if (n_heads <= 0) return set_error(MABA_ERR_INVALID, "dgda_frontend: n_heads must be positive");
    for (int s = 0; s < 6; ++s)
        if (!present(&proj[s]) || proj[s].ndim != 3)
            return set_error(MABA_ERR_INVALID, "dgda_frontend: proj[%d] must be [B, L, C]", s);
    const int dt = proj[0].dtype;
    if (dt != MABA_F32 && dt != MABA_BF16 && dt != MABA_F16)
        return set_error(MABA_ERR_DTYPE, "dgda_frontend: float32 / float16 / bfloat16 features only");
    const int64_t B = proj[0].shape[0], L = proj[0].shape[1];
    FeArgs a{};
    a.B = B; a.L = L; a.eps = eps;
    for (int s = 0; s < 6; ++s) {
        const int64_t C = proj[s].shape[2];
        const int64_t sp[3] = {B, L, C};
        MABA_TRY(expect_shape(&proj[s], "dgda_frontend: proj", 3, sp));
        MABA_TRY(expect_dtype(&proj[s], "dgda_frontend: proj", dt));
        MABA_TRY(expect_shape(&out[s], "dgda_frontend: out", 3, sp));
        MABA_TRY(expect_dtype(&out[s], "dgda_frontend: out", dt));
        if (C <= 0 || C % kVec != 0 || C % n_heads != 0)
            return set_error(MABA_ERR_UNSUPPORTED, "dgda_frontend: channels (%lld) must be a multiple of 8 and of the "
                             "head count", (long long)C);
        a.C[s] = (int)C;
        a.groups[s] = (int)(C / kVec);
        a.sec[s].x = proj[s].data; a.sec[s].out = out[s].data;
        for (int i = 0; i < 3; ++i) { a.sec[s].sx[i] = proj[s].stride[i]; a.sec[s].so[i] = out[s].stride[i]; }
    }
    // q, k, alpha, erase share H*dk channels; v and write share H*dv
    if (a.C[1] != a.C[0] || a.C[3] != a.C[0] || a.C[4] != a.C[0] || a.C[5] != a.C[2])
        return set_error(MABA_ERR_INVALID, "dgda_frontend: q/k/alpha/erase and v/write channel counts must agree");
    const int dk = a.C[1] / n_heads;
    a.hw = dk / kVec;
    if (dk % kVec != 0 || a.hw > 32 || (a.hw & (a.hw - 1)) != 0)
        return set_error(MABA_ERR_UNSUPPORTED, "dgda_frontend: dk = %d must be 8 x a power of two <= 256", dk);
    a.gbase[0] = 0;
    for (int s = 0; s < 6; ++s) a.gbase[s + 1] = a.gbase[s] + a.groups[s];
    // whole warps per token run: a head's lanes of the k section then never straddle a warp
    a.per_run = (a.gbase[6] + 31) / 32 * 32;
    int K = -1;
    for (int s = 0; s < 3; ++s) {
        if (!present(&conv_w[s]) || conv_w[s].ndim != 2 || conv_w[s].shape[0] != a.C[s])
            return set_error(MABA_ERR_INVALID, "dgda_frontend: conv_w[%d] must be [C, K]", s);
        MABA_TRY(expect_dtype(&conv_w[s], "dgda_frontend: conv_w", dt));
        if (K < 0) K = (int)conv_w[s].shape[1];
        if (conv_w[s].shape[1] != K) return set_error(MABA_ERR_INVALID, "dgda_frontend: conv kernel sizes differ");
        a.conv[s] = conv_w[s].data;
        a.sconv[s][0] = conv_w[s].stride[0]; a.sconv[s][1] = conv_w[s].stride[1];
    }
    if (K < 1 || K > kMaxTaps) return set_error(MABA_ERR_UNSUPPORTED, "dgda_frontend: conv kernel size 1..%d", kMaxTaps);
    a.K = K;
    int hdt = -1;
    for (int s = 0; s < 3; ++s) {
        const maba_tensor* hs[2] = {hist != nullptr ? &hist[s] : nullptr, new_hist != nullptr ? &new_hist[s] : nullptr};
        for (const maba_tensor* h : hs) {
            if (!present(h)) continue;
            const int64_t sh[3] = {B, a.C[s], K - 1};
            MABA_TRY(expect_shape(h, "dgda_frontend: conv history", 3, sh));
            if (h->dtype != dt && h->dtype != MABA_F32)
                return set_error(MABA_ERR_DTYPE, "dgda_frontend: conv history must be float32 or the feature dtype");
            if (hdt < 0) hdt = h->dtype;
            if (h->dtype != hdt) return set_error(MABA_ERR_DTYPE, "dgda_frontend: conv histories differ in dtype");
        }
        a.hist[s] = (hist != nullptr && present(&hist[s])) ? hist[s].data : nullptr;
        for (int i = 0; i < 3; ++i) a.sh[s][i] = a.hist[s] ? hist[s].stride[i] : 0;
    }
    a.hist_f32 = (hdt == MABA_F32 && dt != MABA_F32) ? 1 : 0;
    if (B == 0 || L == 0) return MABA_OK;
    cudaStream_t st = as_stream(stream);
    const int64_t nruns = ceil_div(L, kRun);
    bool tiled = dt != MABA_F32 && a.hw <= 16;
    for (int sct = 0; sct < 6; ++sct)
        tiled = tiled && a.C[sct] % kTileCh == 0 && proj[sct].stride[2] == 1 && proj[sct].stride[1] % 8 == 0 &&
                proj[sct].stride[0] % 8 == 0 && (reinterpret_cast<uintptr_t>(proj[sct].data) & 15u) == 0;
    bool piped = tiled && K >= 1 && K <= 8;
    for (int sct = 0; sct < 3; ++sct)
        piped = piped && a.sconv[sct][1] == 1 && a.sconv[sct][0] == K &&
                (reinterpret_cast<uintptr_t>(a.conv[sct]) & 15u) == 0;
    if (piped) {
        const int64_t ntt = ceil_div(L, kTileTok);
        const int nct = (a.C[0] + a.C[1] + a.C[2] + a.C[3] + a.C[4] + a.C[5]) / kTileCh;
        const int64_t ntiles = B * ntt * nct;
        const size_t smem = 2 * (size_t)(kTileTok + K - 1) * (kTileCh + 8) * 2 + 2 * (size_t)kTileCh * K * 2;
        const int64_t cap = (int64_t)sm_count() * 3;
        const unsigned pgrid = (unsigned)(ntiles < cap ? ntiles : cap);
        MABA_TRY(MABA_DISPATCH_FLOAT(dt, "dgda_frontend", [&] {
            if constexpr (sizeof(T) != 2) {
                return set_error(MABA_ERR_DTYPE, "dgda_frontend: tiled path is 16-bit");
            } else {
                auto go = [&](auto kern) {
                    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                    kern<<<pgrid, 256, smem, st>>>(a, ntt, nct, ntiles);
                    return check_launch("dgda_frontend(pipe)");
                };
                switch (K) {
                    case 1: return go(dgda_frontend_pipe_kernel<T, 1>);
                    case 2: return go(dgda_frontend_pipe_kernel<T, 2>);
                    case 3: return go(dgda_frontend_pipe_kernel<T, 3>);
                    case 4: return go(dgda_frontend_pipe_kernel<T, 4>);
                    case 5: return go(dgda_frontend_pipe_kernel<T, 5>);
                    case 6: return go(dgda_frontend_pipe_kernel<T, 6>);
                    case 7: return go(dgda_frontend_pipe_kernel<T, 7>);
                    default: return go(dgda_frontend_pipe_kernel<T, 8>);
                }
            }
        }));
    } else if (tiled) {
        const int64_t ntt = ceil_div(L, kTileTok);
        const int nct = (a.C[0] + a.C[1] + a.C[2] + a.C[3] + a.C[4] + a.C[5]) / kTileCh;
        const unsigned tgrid = (unsigned)(B * ntt * nct);
        MABA_TRY(MABA_DISPATCH_FLOAT(dt, "dgda_frontend", [&] {
            if constexpr (sizeof(T) != 2) {
                return set_error(MABA_ERR_DTYPE, "dgda_frontend: tiled path is 16-bit");
            } else {
                switch (K) {
                    case 1: dgda_frontend_tile_kernel<T, 1><<<tgrid, 256, 0, st>>>(a, ntt, nct); break;
                    case 2: dgda_frontend_tile_kernel<T, 2><<<tgrid, 256, 0, st>>>(a, ntt, nct); break;
                    case 3: dgda_frontend_tile_kernel<T, 3><<<tgrid, 256, 0, st>>>(a, ntt, nct); break;
                    case 4: dgda_frontend_tile_kernel<T, 4><<<tgrid, 256, 0, st>>>(a, ntt, nct); break;
                    case 5: dgda_frontend_tile_kernel<T, 5><<<tgrid, 256, 0, st>>>(a, ntt, nct); break;
                    case 6: dgda_frontend_tile_kernel<T, 6><<<tgrid, 256, 0, st>>>(a, ntt, nct); break;
                    case 7: dgda_frontend_tile_kernel<T, 7><<<tgrid, 256, 0, st>>>(a, ntt, nct); break;
                    default: dgda_frontend_tile_kernel<T, 8><<<tgrid, 256, 0, st>>>(a, ntt, nct); break;
                }
                return check_launch("dgda_frontend(tile)");
            }
        }));
    }
    const int64_t threads = tiled ? 0 : B * nruns * a.per_run;
    const unsigned grid = (unsigned)ceil_div(threads, kFeThreads);
    if (!tiled) MABA_TRY(MABA_DISPATCH_FLOAT(dt, "dgda_frontend", [&] {
        if constexpr (sizeof(T) == 8) {
            return set_error(MABA_ERR_DTYPE, "dgda_frontend: float64");
        } else {
            switch (K) {
                case 1: dgda_frontend_kernel<T, 1><<<grid, kFeThreads, 0, st>>>(a, nruns); break;
                case 2: dgda_frontend_kernel<T, 2><<<grid, kFeThreads, 0, st>>>(a, nruns); break;
                case 3: dgda_frontend_kernel<T, 3><<<grid, kFeThreads, 0, st>>>(a, nruns); break;
                case 4: dgda_frontend_kernel<T, 4><<<grid, kFeThreads, 0, st>>>(a, nruns); break;
                case 5: dgda_frontend_kernel<T, 5><<<grid, kFeThreads, 0, st>>>(a, nruns); break;
                case 6: dgda_frontend_kernel<T, 6><<<grid, kFeThreads, 0, st>>>(a, nruns); break;
                case 7: dgda_frontend_kernel<T, 7><<<grid, kFeThreads, 0, st>>>(a, nruns); break;
                default: dgda_frontend_kernel<T, 8><<<grid, kFeThreads, 0, st>>>(a, nruns); break;
            }
            return check_launch("dgda_frontend");
        }
    }));
    if (new_hist == nullptr || K == 1) return MABA_OK;
    void* nh[3];
    int64_t sn[9] = {0};
    bool any = false;
    for (int s = 0; s < 3; ++s) {
        nh[s] = present(&new_hist[s]) ? new_hist[s].data : nullptr;
        any = any || nh[s] != nullptr;
        for (int i = 0; i < 3; ++i) sn[3 * s + i] = nh[s] ? new_hist[s].stride[i] : 0;
    }
    if (!any) return MABA_OK;
    const int64_t n = B * (int64_t)(a.C[0] + a.C[1] + a.C[2]) * (K - 1);
    const bool f32h = hdt == MABA_F32;
    return MABA_DISPATCH_FLOAT(dt, "dgda_frontend(history)", [&] {
        if constexpr (sizeof(T) == 8) {
            return set_error(MABA_ERR_DTYPE, "dgda_frontend: float64");
        } else {
            if (f32h)
                dgda_frontend_hist_kernel<T, float><<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(
                    a, nh[0], nh[1], nh[2], sn[0], sn[1], sn[2], sn[3], sn[4], sn[5], sn[6], sn[7], sn[8]);
            else
                dgda_frontend_hist_kernel<T, T><<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(
                    a, nh[0], nh[1], nh[2], sn[0], sn[1], sn[2], sn[3], sn[4], sn[5], sn[6], sn[7], sn[8]);
            return check_launch("dgda_frontend(history)");
        }
    });
}
