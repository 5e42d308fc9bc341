// Chunk-parallel DGDA prefill for 16-bit inputs: the preparation pass (per-chunk
// WY/UT records) and the state scan, which also writes the outputs.
//
// Same recurrence as dgda_prefill_mma.cu (reference maba_sparse/kernels/
// common.py:256-265, chunked form cpu_dgda.py:101-146) with the per-chunk WY/UT
// quantities precomputed in parallel over all chunks (record: dgda_prefill.cuh):
//   S' = e^{G_end} S + (k e^{G_end-G})^T (U - W S) = e^{G_end} S + N - M S
//   o  = (q e^G) S + A (U - W S)                   = QW S + AU
// so the sequential part per chunk is one 64x64x64 product for the state and one
// for the chunk's outputs.  The decay term e^{G_end} S stays in fp32; only the
// correction M S, the increment N and the output product pass through 16-bit
// operands, as in the single-pass kernel.
//
// Scan (grid = (B*H, segments), 8 warps): the next chunk's record tiles are
// fetched by cp.async while the current products run; the state is held in fp32
// accumulator registers, with a double-buffered 16-bit copy in shared memory
// that feeds both products.  Modes: 0 -- one segment from the initial state;
// 1 -- the affine transition [R | P] of each segment (the augmented state starts
// at [0 | I]: X' = e^{G_end} X + [N | 0] - M X; no outputs); 2 -- each segment
// from its start state.
#include "dgda_prefill.cuh"
#include "mma_util.cuh"

#include <type_traits>

namespace maba {
namespace {

constexpr int C = 64;
constexpr int D = 64;
constexpr int NTH = 256;
constexpr int LB = 72;  // padded 16-bit row (144 B): conflict-free ldmatrix

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem_addr(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

// 64x64 16-bit tile of a chunk record -> padded shared tile (all threads)
template <typename T>
__device__ __forceinline__ void fetch_tile(T* dst, const unsigned char* src, int tid) {
    for (int e = tid; e < 64 * 8; e += NTH) {
        const int r = e >> 3, c8 = (e & 7) * 8;
        cp_async16(dst + r * LB + c8, src + (size_t)(r * 64 + c8) * 2);
    }
}

template <int NCOL, bool OUT>
struct ScanSmem {
    static constexpr int LN = NCOL + 8;
    static constexpr size_t TILE = (size_t)C * LB * 2;
    static constexpr size_t QW = 2 * TILE + 64 * 4, AU = QW + TILE;  // output operands (OUT)
    static constexpr size_t REC = QW + (OUT ? 2 * TILE : 0);        // M, N, dend[, QW, AU]
    static constexpr size_t SB = 2 * REC;                          // 2 x [D][LN] 16-bit state
    static constexpr size_t SBSZ = (size_t)D * LN * 2;
    static constexpr size_t TOTAL = SB + 2 * SBSZ;
};

template <typename T, typename TS, int MODE>
__global__ void __launch_bounds__(NTH, 2) dgda_scan_kernel(PrefillArgs a) {
    constexpr int NCOL = MODE == 1 ? 2 * D : D;
    constexpr bool OUT = MODE != 1;  // modes 0 and 2 produce the chunk outputs
    using SM = ScanSmem<NCOL, OUT>;
    constexpr int LN = SM::LN;
    constexpr int NTW = NCOL / 16;
    extern __shared__ __align__(16) unsigned char sm[];
    T* SB = reinterpret_cast<T*>(sm + SM::SB);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x, seg = blockIdx.y;
    const int64_t bi = bh / a.H, hi = bh % a.H;
    const int dk = a.dk, dv = a.dv;
    const int wr = (warp & 3) * 16;
    const int wc = (warp >> 2) * (NCOL / 2);
    const int fr = lane >> 2, fc = (lane & 3) * 2;

    const int64_t c_begin = MODE == 0 ? 0 : (int64_t)seg * (a.seg_len / C);
    int64_t c_end = MODE == 0 ? a.nch : c_begin + a.seg_len / C;
    if (c_end > a.nch) c_end = a.nch;
    const unsigned char* recs = a.ws_chunk + (size_t)bh * a.nch * CHUNK_REC;
    using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
    T* out = OUT ? static_cast<T*>(a.out) + bi * a.so[0] + hi * a.so[1] : nullptr;
    // paired (4-byte) output stores: unit column stride, even dv, 4-byte aligned rows
    const bool pair_out = OUT && a.so[3] == 1 && (dv & 1) == 0 &&
                          ((reinterpret_cast<uintptr_t>(out) | (uintptr_t)(a.so[2] * 2)) & 3) == 0;

    auto fetch = [&](int64_t c, int buf) {
        unsigned char* base = sm + buf * SM::REC;
        const unsigned char* r = recs + (size_t)c * CHUNK_REC;
        fetch_tile<T>(reinterpret_cast<T*>(base), r + CH_M, tid);
        fetch_tile<T>(reinterpret_cast<T*>(base + SM::TILE), r + CH_N, tid);
        if (tid < 16) cp_async16(base + 2 * SM::TILE + tid * 16, r + CH_DEND + tid * 16);
        if (OUT) {
            fetch_tile<T>(reinterpret_cast<T*>(base + SM::QW), r + CH_QW, tid);
            fetch_tile<T>(reinterpret_cast<T*>(base + SM::AU), r + CH_AU, tid);
        }
        cp_async_commit();
    };
    if (c_begin < c_end) fetch(c_begin, 0);

    // ---- starting state ----------------------------------------------------
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

    int buf = 0;
    for (int64_t c = c_begin; c < c_end; ++c, buf ^= 1) {
        cp_async_wait_all();
        __syncthreads();  // this chunk's record and the current state copy are visible
        if (c + 1 < c_end) fetch(c + 1, buf ^ 1);
        const T* Mt = reinterpret_cast<const T*>(sm + buf * SM::REC);
        const T* Nt = reinterpret_cast<const T*>(sm + buf * SM::REC + SM::TILE);
        const float* dend = reinterpret_cast<const float*>(sm + buf * SM::REC + 2 * SM::TILE);
        const T* Sc = SB + buf * (SM::SBSZ / 2);        // state at the chunk start (16-bit)
        T* Sn = SB + (buf ^ 1) * (SM::SBSZ / 2);        // state after the chunk
        // S' = e^{G_end} S + [N | 0] - M S
        float macc[NTW][4] = {};
        warp_mma<T, false, true, NTW>(macc, Mt + wr * LB, LB, Sc + wc, LN, D, lane);
#pragma unroll
        for (int n = 0; n < NTW; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = wr + fr + (e >> 1) * 8;
                const int col = wc + n * 8 + fc + (e & 1);
                const float nv = col < D ? Cvt<T>::to_f(Nt[r * LB + col]) : 0.f;
                sacc[n][e] = fmaf(sacc[n][e], dend[r], nv - macc[n][e]);
            }
        store_acc16<T, NTW>(Sn + wr * LN + wc, LN, sacc, lane);
        if constexpr (OUT) {
            // the chunk's outputs from its start state: o = QW S + AU
            const T* QWt = reinterpret_cast<const T*>(sm + buf * SM::REC + SM::QW);
            const T* AUt = reinterpret_cast<const T*>(sm + buf * SM::REC + SM::AU);
            float qacc[NTW][4] = {};
            warp_mma<T, false, true, NTW>(qacc, QWt + wr * LB, LB, Sc + wc, LN, D, lane);
            const int64_t t0 = c * C;
#pragma unroll
            for (int n = 0; n < NTW; ++n)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int r = wr + fr + h * 8;
                    const int col = wc + n * 8 + fc;
                    const int64_t t = t0 + r;
                    if (t >= a.L) continue;
                    const float o0 = qacc[n][2 * h] + Cvt<T>::to_f(AUt[r * LB + col]);
                    const float o1 = qacc[n][2 * h + 1] + Cvt<T>::to_f(AUt[r * LB + col + 1]);
                    T* dst = out + t * a.so[2] + (int64_t)col * a.so[3];
                    if (pair_out) {
                        if (col < dv) {
                            T2 v2;
                            v2.x = to16<T>(o0);
                            v2.y = to16<T>(o1);
                            *reinterpret_cast<T2*>(dst) = v2;
                        }
                    } else {
                        if (col < dv) dst[0] = to16<T>(o0);
                        if (col + 1 < dv) dst[a.so[3]] = to16<T>(o1);
                    }
                }
        }
    }
    cp_async_wait_all();
    // ---- results -------------------------------------------------------------
#pragma unroll
    for (int n = 0; n < NTW; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = wr + fr + (e >> 1) * 8;
            const int col = wc + n * 8 + fc + (e & 1);
            if (MODE == 1) {
                a.ws_trans[(((size_t)bh * a.nseg + seg) * D + d) * (2 * D) + col] = sacc[n][e];
            } else if (MODE == 0 || seg == a.nseg - 1) {
                if (d < dk && col < dv)
                    store_from<TS, float>(static_cast<TS*>(a.fin) + bi * a.sf[0] + hi * a.sf[1] + (int64_t)d * a.sf[2] +
                                              (int64_t)col * a.sf[3],
                                          sacc[n][e]);
            }
        }
}

// ---------------------------------------------------------------------------
// Preparation pass: one CTA per (b*h, chunk), two CTAs per SM.
// Warp w owns rows 8w .. 8w+7, lane l owns columns 2l, 2l+1: each thread loads
// its 8 x 2 slice of every input (coalesced 128-byte rows, all loads in flight
// at once), prefix-sums the log-decays in registers (group totals exchanged
// through shared memory), and produces every decayed operand of its slice
// directly -- nothing fp32 of size C x D is staged in shared memory.
//   QT = q e^G, KT = k e^{G_end - G}            -> registers (packed pairs) until the epilogue
//   BT = (b k) e^G, WV = w v                    -> shared (operands of W, U)
//   QD, BD, KD (diagonal factors around the block's first row), QH, BH, KH
//   (off-diagonal factors around the end of the previous block)  -> shared
// then A, L (tensor cores; per-element decay for blocks too steep to factor,
// recomputed exactly from the log-decays), T = (I + L)^{-1} (16x16 diagonal
// inverses + block back-substitution), W = T BT, U = T WV -> chunk record.
namespace prep {
constexpr int LT = 24;                      // row stride of the 16x16 diagonal inverses
constexpr size_t TILE = (size_t)C * LB * 2; // 9216
constexpr size_t BT = 0, WV = TILE, AM = 2 * TILE, LM = 3 * TILE;
constexpr size_t LD = 4 * TILE;                         // fp32 [4][16][17] diagonal blocks of L
constexpr size_t TD = LD + 4 * 16 * 17 * 4;             // 16-bit [4][16][LT] diagonal inverses
constexpr size_t DEND = TD + 4 * 16 * LT * 2;           // fp32 [64]
constexpr size_t TOT = DEND + 64 * 4;                   // fp32 [8][64] group totals + [4][64] block starts
constexpr size_t FLG = TOT + 12 * 64 * 4;               // int [4]
constexpr size_t R1 = FLG + 16;                         // A/L operand region (dead after A/L)
constexpr size_t QD = R1, BD = QD + TILE, KD = BD + TILE;
constexpr size_t QH = KD + TILE;                        // [48][LB]
constexpr size_t BH = QH + (size_t)48 * LB * 2;         // [48][LB]
constexpr size_t KH = BH + (size_t)48 * LB * 2;         // [96][LB]
constexpr size_t TOTAL = KH + (size_t)96 * LB * 2;
// aliases of the dead A/L region during the solve and the epilogue
constexpr size_t TM = R1, SCR = R1 + TILE;
constexpr size_t EP_KT = SCR + (size_t)16 * LB * 2, EP_QT = EP_KT + TILE, EP_W = EP_QT + TILE, EP_U = EP_W + TILE;
static_assert(EP_U + TILE <= TOTAL, "epilogue tiles fit in the A/L region");
static_assert(TOTAL <= 113 * 1024, "two CTAs per SM");
}  // namespace prep

__device__ __forceinline__ int kh_off(int I) { return I == 1 ? 0 : (I == 2 ? 16 : 48); }

template <typename T>
__device__ __forceinline__ float lg(const PrefillArgs& a, const T* lal, const T* al, int64_t t, int d) {
    if (lal) return fminf(fmaxf(Cvt<T>::to_f(lal[t * a.sla[2] + d * a.sla[3]]), -46.f), 0.f);
    return logf(fminf(fmaxf(Cvt<T>::to_f(al[t * a.sa[2] + d * a.sa[3]]), 1e-20f), 1.f));
}

template <typename T>
__global__ void __launch_bounds__(NTH, 2) dgda_prep_kernel(PrefillArgs a) {
    using namespace prep;
    extern __shared__ __align__(16) unsigned char sm[];
    T* BTs = reinterpret_cast<T*>(sm + BT);
    T* WVs = reinterpret_cast<T*>(sm + WV);
    T* AMs = reinterpret_cast<T*>(sm + AM);
    T* LMs = reinterpret_cast<T*>(sm + LM);
    float* LDs = reinterpret_cast<float*>(sm + LD);
    T* TDs = reinterpret_cast<T*>(sm + TD);
    float* dend = reinterpret_cast<float*>(sm + DEND);
    float* tot = reinterpret_cast<float*>(sm + TOT);
    int* flags = reinterpret_cast<int*>(sm + FLG);
    T* QDs = reinterpret_cast<T*>(sm + QD);
    T* BDs = reinterpret_cast<T*>(sm + BD);
    T* KDs = reinterpret_cast<T*>(sm + KD);
    T* QHs = reinterpret_cast<T*>(sm + QH);
    T* BHs = reinterpret_cast<T*>(sm + BH);
    T* KHs = reinterpret_cast<T*>(sm + KH);
    T* TMs = reinterpret_cast<T*>(sm + TM);
    T* SCRs = reinterpret_cast<T*>(sm + SCR);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int bh = blockIdx.x;
    const int64_t chunk = blockIdx.y;
    const int64_t bi = bh / a.H, hi = bh % a.H;
    const int dk = a.dk, dv = a.dv;
    const int fr = lane >> 2, fc = (lane & 3) * 2;
    const int64_t t0 = chunk * C;
    unsigned char* rec = a.ws_chunk + ((size_t)bh * a.nch + chunk) * CHUNK_REC;

    const T* q = static_cast<const T*>(a.q) + bi * a.sq[0] + hi * a.sq[1];
    const T* k = static_cast<const T*>(a.k) + bi * a.sk[0] + hi * a.sk[1];
    const T* v = static_cast<const T*>(a.v) + bi * a.sv[0] + hi * a.sv[1];
    const T* bb = static_cast<const T*>(a.b) + bi * a.sb[0] + hi * a.sb[1];
    const T* w = static_cast<const T*>(a.w) + bi * a.sw[0] + hi * a.sw[1];
    const T* lal = a.log_alpha ? static_cast<const T*>(a.log_alpha) + bi * a.sla[0] + hi * a.sla[1] : nullptr;
    const T* al = a.alpha ? static_cast<const T*>(a.alpha) + bi * a.sa[0] + hi * a.sa[1] : nullptr;

    // the next wave's inputs into L2: one line prefetch per 128-byte row segment of
    // each of the six operands (rows are 16-byte aligned, a.vec8)
    if (a.pf_ahead > 0) {
        const int64_t nxt = (int64_t)blockIdx.y * gridDim.x + blockIdx.x + a.pf_ahead;
        const int64_t pc = nxt / gridDim.x;
        if (pc < a.nch) {
            const int64_t pbh = nxt - pc * gridDim.x, pb = pbh / a.H, ph = pbh % a.H;
            for (int e = tid; e < 6 * C; e += NTH) {
                const int op = e / C;
                const int64_t t = pc * C + (e - op * C);
                if (t >= a.L) continue;
                const T* src;
                int n;
                switch (op) {
                    case 0: src = static_cast<const T*>(a.q) + pb * a.sq[0] + ph * a.sq[1] + t * a.sq[2]; n = dk; break;
                    case 1: src = static_cast<const T*>(a.k) + pb * a.sk[0] + ph * a.sk[1] + t * a.sk[2]; n = dk; break;
                    case 2: src = static_cast<const T*>(a.b) + pb * a.sb[0] + ph * a.sb[1] + t * a.sb[2]; n = dk; break;
                    case 3: src = static_cast<const T*>(a.v) + pb * a.sv[0] + ph * a.sv[1] + t * a.sv[2]; n = dv; break;
                    case 4: src = static_cast<const T*>(a.w) + pb * a.sw[0] + ph * a.sw[1] + t * a.sw[2]; n = dv; break;
                    default:
                        src = a.log_alpha
                                  ? static_cast<const T*>(a.log_alpha) + pb * a.sla[0] + ph * a.sla[1] + t * a.sla[2]
                                  : static_cast<const T*>(a.alpha) + pb * a.sa[0] + ph * a.sa[1] + t * a.sa[2];
                        n = dk;
                }
                for (int o = 0; o < n; o += 64)  // 64 16-bit values = one 128-byte line
                    asm volatile("prefetch.global.L2 [%0];" ::"l"(src + o));
            }
        }
    }

    // ---------------- log-decays of this thread's 8 x 2 slice ------------------------
    // warp rg owns rows 8 rg .. 8 rg + 7 (half of block blk = rg / 2); lane owns columns
    // d0, d0 + 1: every load / store of a row is one coalesced 128-byte access per warp
    const int rg = warp, blk = rg >> 1, d0 = 2 * lane;
    using T2 = typename std::conditional<std::is_same<T, __half>::value, __half2, __nv_bfloat162>::type;
    // raw pairs of 16-bit values (converted at use).  Every load is unconditional
    // (this path requires unit-stride, 16-byte aligned rows, a.vec8): rows past
    // the end re-read the last row and are zeroed below, so all 48 loads of the
    // thread are in flight together.
    auto fx = [](T2 v2) { return Cvt<T>::to_f(v2.x); };
    auto fy = [](T2 v2) { return Cvt<T>::to_f(v2.y); };
    const T* gsrc = lal ? lal : al;
    const int64_t* gst = lal ? a.sla : a.sa;
    T2 gr[8], qv[8], kv[8], bv[8], wv[8], vv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int64_t t = t0 + 8 * rg + i;
        t = t < a.L ? t : a.L - 1;
        gr[i] = *reinterpret_cast<const T2*>(gsrc + t * gst[2] + d0);
        qv[i] = *reinterpret_cast<const T2*>(q + t * a.sq[2] + d0);
        kv[i] = *reinterpret_cast<const T2*>(k + t * a.sk[2] + d0);
        bv[i] = *reinterpret_cast<const T2*>(bb + t * a.sb[2] + d0);
        wv[i] = *reinterpret_cast<const T2*>(w + t * a.sw[2] + d0);
        vv[i] = *reinterpret_cast<const T2*>(v + t * a.sv[2] + d0);
    }
    float G0[8], G1[8];  // log-decay of columns d0, d0 + 1
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const bool ok = t0 + 8 * rg + i < a.L;
        float x0 = fx(gr[i]), x1 = fy(gr[i]);
        if (lal) {
            x0 = fminf(fmaxf(x0, -46.f), 0.f);
            x1 = fminf(fmaxf(x1, -46.f), 0.f);
        } else {
            x0 = logf(fminf(fmaxf(x0, 1e-20f), 1.f));
            x1 = logf(fminf(fmaxf(x1, 1e-20f), 1.f));
        }
        G0[i] = ok ? x0 : 0.f;
        G1[i] = ok ? x1 : 0.f;
        if (!ok) {  // rows past the end contribute nothing
            const T z = to16<T>(0.f);
            qv[i].x = qv[i].y = kv[i].x = kv[i].y = bv[i].x = bv[i].y = z;
            wv[i].x = wv[i].y = vv[i].x = vv[i].y = z;
        }
    }
#pragma unroll
    for (int i = 1; i < 8; ++i) {
        G0[i] += G0[i - 1];
        G1[i] += G1[i - 1];
    }
    float* gtot = tot;               // [8][64] group totals
    float* gfirst = tot + 8 * 64;    // [4][64] log-decay at each block's first row
    gtot[rg * 64 + d0] = G0[7];
    gtot[rg * 64 + d0 + 1] = G1[7];
    if (tid < 4) flags[tid] = 0;
    __syncthreads();
    float off0 = 0.f, off1 = 0.f;
    float bend0[4], bend1[4];  // cumulative log-decay at the end of each 16-row block
    {
        float r0 = 0.f, r1 = 0.f;
#pragma unroll
        for (int g2 = 0; g2 < 8; ++g2) {
            if (g2 == rg) {
                off0 = r0;
                off1 = r1;
            }
            r0 += gtot[g2 * 64 + d0];
            r1 += gtot[g2 * 64 + d0 + 1];
            if (g2 & 1) {
                bend0[g2 >> 1] = r0;
                bend1[g2 >> 1] = r1;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        G0[i] += off0;
        G1[i] += off1;
    }
    if (!(rg & 1)) {
        gfirst[blk * 64 + d0] = G0[0];
        gfirst[blk * 64 + d0 + 1] = G1[0];
    }
    if (blk == 3 && (rg & 1)) {
        dend[d0] = __expf(bend0[3]);
        dend[d0 + 1] = __expf(bend1[3]);
    }
    __syncthreads();
    const float g00 = gfirst[blk * 64 + d0], g01 = gfirst[blk * 64 + d0 + 1];
    constexpr float kFlat = std::is_same<T, __half>::value ? 8.f : 80.f;
    if ((rg & 1) && (g00 - G0[7] > kFlat || g01 - G1[7] > kFlat)) atomicOr(&flags[blk], 1);
    const float ge0 = bend0[3], ge1 = bend1[3];
    const float pr0 = blk == 0 ? 0.f : (blk == 1 ? bend0[0] : (blk == 2 ? bend0[1] : bend0[2]));
    const float pr1 = blk == 0 ? 0.f : (blk == 1 ? bend1[0] : (blk == 2 ? bend1[1] : bend1[2]));

    // ---------------- decayed operands ----------------------------------------------
    // QT and KT stay in registers (packed 16-bit pairs) until the epilogue stages them
    uint32_t qtp[8], ktp[8];
    auto pk2 = [](float x, float y) {
        T2 v2;
        v2.x = to16<T>(x);
        v2.y = to16<T>(y);
        return *reinterpret_cast<uint32_t*>(&v2);
    };
    auto st2 = [](T* p, float x, float y) {
        T2 v2;
        v2.x = to16<T>(x);
        v2.y = to16<T>(y);
        *reinterpret_cast<T2*>(p) = v2;
    };
    // Every factor is built from the block-relative decay f = e^{G - g0} (<= 1) and
    // its reciprocal (<= e^80 on blocks flat enough to factor; steep blocks take
    // the per-element path for A and L), times per-column constants:
    //   e^G = e^{g0} f,  e^{G_end - G} = e^{G_end - g0} / f,  e^{G - G_prev_end} =
    //   e^{g0 - G_prev_end} f,  e^{G_end(I-1) - G} = e^{G_end(I-1) - g0} / f.
    const float cg0 = __expf(g00), cg1 = __expf(g01);
    const float ce0 = __expf(ge0 - g00), ce1 = __expf(ge1 - g01);
    const float cp0 = __expf(g00 - pr0), cp1 = __expf(g01 - pr1);
    float ck0[3], ck1[3];
#pragma unroll
    for (int I = 1; I < 4; ++I) {
        ck0[I - 1] = __expf(bend0[I - 1] - g00);
        ck1[I - 1] = __expf(bend1[I - 1] - g01);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = 8 * rg + i;
        const float q0 = fx(qv[i]), q1 = fy(qv[i]), k0 = fx(kv[i]), k1 = fy(kv[i]);
        const float bk0 = fx(bv[i]) * k0, bk1 = fy(bv[i]) * k1;
        const float f0 = __expf(G0[i] - g00), f1 = __expf(G1[i] - g01);  // <= 1
        const float r0 = __fdividef(1.f, f0), r1 = __fdividef(1.f, f1);
        const float e0 = cg0 * f0, e1 = cg1 * f1;
        qtp[i] = pk2(q0 * e0, q1 * e1);
        ktp[i] = pk2(k0 * (ce0 * r0), k1 * (ce1 * r1));
        st2(BTs + r * LB + d0, bk0 * e0, bk1 * e1);
        st2(WVs + r * LB + d0, fx(wv[i]) * fx(vv[i]), fy(wv[i]) * fy(vv[i]));
        st2(QDs + r * LB + d0, q0 * f0, q1 * f1);
        st2(BDs + r * LB + d0, bk0 * f0, bk1 * f1);
        st2(KDs + r * LB + d0, k0 * r0, k1 * r1);
        if (blk >= 1) {
            const float h0 = cp0 * f0, h1 = cp1 * f1;
            st2(QHs + (r - 16) * LB + d0, q0 * h0, q1 * h1);
            st2(BHs + (r - 16) * LB + d0, bk0 * h0, bk1 * h1);
        }
#pragma unroll
        for (int I = 1; I < 4; ++I)
            if (I > blk) st2(KHs + (kh_off(I) + r) * LB + d0, k0 * (ck0[I - 1] * r0), k1 * (ck1[I - 1] * r1));
    }
    // strictly-upper off-diagonal 16x16 blocks of A and L are zero: 6 blocks x 16 rows
    // x two 16-byte pieces per matrix
    for (int e = tid; e < 2 * 6 * 16 * 2; e += NTH) {
        const int mat = e / 192, r = e - mat * 192;
        const int blkid = r >> 5, row16 = (r >> 1) & 15, half = r & 1;
        // block (I, J) with J > I, enumerated (0,1) (0,2) (0,3) (1,2) (1,3) (2,3)
        const int I = blkid < 3 ? 0 : (blkid < 5 ? 1 : 2);
        const int J = blkid < 3 ? blkid + 1 : (blkid < 5 ? blkid - 1 : 3);
        T* base = (mat ? LMs : AMs) + (16 * I + row16) * LB + 16 * J + 8 * half;
        *reinterpret_cast<uint4*>(base) = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    // ---------------- A / L blocks -------------------------------------------------------
    {
        const int db = warp >> 1;
        const bool isL = warp & 1;
        if (!flags[db]) {
            float acc[2][4] = {};
            warp_mma<T, false, false, 2>(acc, (isL ? BDs : QDs) + (16 * db) * LB, LB, KDs + (16 * db) * LB, LB, D,
                                         lane);
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int ii = fr + (e >> 1) * 8, jj = n * 8 + fc + (e & 1);
                    const float x = isL ? (jj < ii ? acc[n][e] : 0.f) : (jj <= ii ? acc[n][e] : 0.f);
                    const int i = db * 16 + ii, j = db * 16 + jj;
                    if (isL) {
                        LMs[i * LB + j] = to16<T>(x);
                        LDs[(db * 16 + ii) * 17 + jj] = x;
                    } else {
                        AMs[i * LB + j] = to16<T>(x);
                    }
                }
        }
    }
    for (int p = tid; p < 4 * 256; p += NTH) {  // steep blocks: per-element decay, exact from the log-decays
        const int db = p >> 8, ii = (p >> 4) & 15, jj = p & 15;
        if (!flags[db]) continue;
        const int i = db * 16 + ii, j = db * 16 + jj;
        float av = 0.f, lv = 0.f;
        if (jj <= ii && t0 + i < a.L) {
            const int64_t ti = t0 + i, tj = t0 + j;
            for (int dd = 0; dd < dk; ++dd) {
                float sg = 0.f;  // sum of the log-decays over (j, i]
                for (int64_t tt = tj + 1; tt <= ti; ++tt) sg += lg<T>(a, lal, al, tt, dd);
                const float kd = Cvt<T>::to_f(k[tj * a.sk[2] + dd * a.sk[3]]) * __expf(sg);
                av = fmaf(Cvt<T>::to_f(q[ti * a.sq[2] + dd * a.sq[3]]), kd, av);
                lv = fmaf(Cvt<T>::to_f(bb[ti * a.sb[2] + dd * a.sb[3]]) * Cvt<T>::to_f(k[ti * a.sk[2] + dd * a.sk[3]]),
                          kd, lv);
            }
        }
        if (jj >= ii) lv = 0.f;
        AMs[i * LB + j] = to16<T>(av);
        LMs[i * LB + j] = to16<T>(lv);
        LDs[(db * 16 + ii) * 17 + jj] = lv;
    }
    __syncthreads();
    // ---------------- 16x16 diagonal inverses of (I + L) (fp32) --------------------------
    // Warps 0-1 (they need only the diagonal blocks of L): column c of block db by
    // forward substitution in column (axpy) order -- once tcol[m] is final, every later
    // row takes -L[r][m] tcol[m], one FMA per step on the dependency chain, the loads
    // of L independent of it.
    if (warp < 2) {  // tid < 64
        const int db = tid >> 4, c = tid & 15;
        const float* Lb = LDs + db * 16 * 17;
        float tcol[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) tcol[r] = r == c ? 1.f : 0.f;
#pragma unroll
        for (int m = 0; m < 15; ++m) {
            if (m >= c) {
                const float tm = tcol[m];
#pragma unroll
                for (int r = m + 1; r < 16; ++r) tcol[r] = fmaf(-Lb[r * 17 + m], tm, tcol[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < 16; ++r) TDs[(db * 16 + r) * LT + c] = to16<T>(tcol[r]);
    } else {
        // meanwhile warps 2-7: the off-diagonal 16x16 tiles of A and L
        for (int tile = warp - 2; tile < 12; tile += 6) {
            // off-diagonal 16x16 tiles: I=1: tiles 0,1; I=2: 2..5; I=3: 6..11 (first I give A, next I give L)
            const int I = tile < 2 ? 1 : (tile < 6 ? 2 : 3);
            const int t_in = tile - (I == 1 ? 0 : (I == 2 ? 2 : 6));
            const bool isL = t_in >= I;
            const int n16 = isL ? t_in - I : t_in;
            float acc[2][4] = {};
            const T* Ap = (isL ? BHs : QHs) + (16 * (I - 1)) * LB;
            const T* Bp = KHs + (kh_off(I) + 16 * n16) * LB;
            warp_mma<T, false, false, 2>(acc, Ap, LB, Bp, LB, D, lane);
            store_acc16<T, 2>((isL ? LMs : AMs) + (16 * I) * LB + 16 * n16, LB, acc, lane);
        }
    }
    __syncthreads();
    // ---------------- T = (I + L)^{-1} by blocks --------------------------------------
    for (int e = tid; e < 16 * C; e += NTH) {
        const int r = e >> 6, c = e & 63;
        TMs[r * LB + c] = c < 16 ? TDs[r * LT + c] : to16<T>(0.f);
    }
    __syncthreads();
    for (int I = 1; I < 4; ++I) {
        if (warp < I) {  // M = L[I, <I] T[<I, <I]
            float acc[2][4] = {};
            warp_mma<T, false, true, 2>(acc, LMs + (16 * I) * LB, LB, TMs + 16 * warp, LB, 16 * I, lane);
            store_acc16<T, 2>(SCRs + 16 * warp, LB, acc, lane);
        }
        __syncthreads();
        if (warp < I) {  // T[I, <I] = -T_II M
            float acc[2][4] = {};
            warp_mma<T, false, true, 2>(acc, TDs + (16 * I) * LT, LT, SCRs + 16 * warp, LB, 16, lane);
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[n][e] = -acc[n][e];
            store_acc16<T, 2>(TMs + (16 * I) * LB + 16 * warp, LB, acc, lane);
        }
        for (int e = tid; e < 16 * (C - 16 * I); e += NTH) {
            const int r = e / (C - 16 * I), c = 16 * I + e % (C - 16 * I);
            TMs[(16 * I + r) * LB + c] = c < 16 * I + 16 ? TDs[(16 * I + r) * LT + (c - 16 * I)] : to16<T>(0.f);
        }
        __syncthreads();
    }
    // ---------------- W = T BT, U = T WV; M, N, QW, AU -> chunk record --------------------
    {
        constexpr int NTW = D / 16;
        const int wr = (warp & 3) * 16, wc = (warp >> 2) * (D / 2);
        T* KTs = reinterpret_cast<T*>(sm + EP_KT);
        T* QTs = reinterpret_cast<T*>(sm + EP_QT);
        T* W16 = reinterpret_cast<T*>(sm + EP_W);
        T* U16 = reinterpret_cast<T*>(sm + EP_U);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            *reinterpret_cast<uint32_t*>(KTs + (8 * rg + i) * LB + d0) = ktp[i];
            *reinterpret_cast<uint32_t*>(QTs + (8 * rg + i) * LB + d0) = qtp[i];
        }
        {
            float wacc[NTW][4] = {};
            float uacc[NTW][4] = {};
            warp_mma<T, false, true, NTW>(wacc, TMs + wr * LB, LB, BTs + wc, LB, C, lane);
            warp_mma<T, false, true, NTW>(uacc, TMs + wr * LB, LB, WVs + wc, LB, C, lane);
            store_acc16<T, NTW>(W16 + wr * LB + wc, LB, wacc, lane);
            store_acc16<T, NTW>(U16 + wr * LB + wc, LB, uacc, lane);
        }
        __syncthreads();  // W, U, KT, QT in shared memory
        auto put = [&](size_t off, const float (&acc)[NTW][4], const T* sub) {
            T* g = reinterpret_cast<T*>(rec + off);
#pragma unroll
            for (int n = 0; n < NTW; ++n)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int r = wr + fr + h * 8, c = wc + n * 8 + fc;
                    float x0 = acc[n][2 * h], x1 = acc[n][2 * h + 1];
                    if (sub != nullptr) {
                        x0 = Cvt<T>::to_f(sub[r * LB + c]) - x0;
                        x1 = Cvt<T>::to_f(sub[r * LB + c + 1]) - x1;
                    }
                    T p2[2] = {to16<T>(x0), to16<T>(x1)};
                    *reinterpret_cast<uint32_t*>(g + r * 64 + c) = *reinterpret_cast<uint32_t*>(p2);
                }
        };
        {
            float macc[NTW][4] = {};
            float nacc[NTW][4] = {};
            warp_mma<T, true, true, NTW>(macc, KTs + wr, LB, W16 + wc, LB, C, lane);  // KT^T W
            warp_mma<T, true, true, NTW>(nacc, KTs + wr, LB, U16 + wc, LB, C, lane);  // KT^T U
            put(CH_M, macc, nullptr);
            put(CH_N, nacc, nullptr);
        }
        {
            float qacc[NTW][4] = {};
            float aacc[NTW][4] = {};
            warp_mma<T, false, true, NTW>(qacc, AMs + wr * LB, LB, W16 + wc, LB, C, lane);  // A W
            warp_mma<T, false, true, NTW>(aacc, AMs + wr * LB, LB, U16 + wc, LB, C, lane);  // A U
            put(CH_QW, qacc, QTs);  // QT - A W
            put(CH_AU, aacc, nullptr);
        }
    }
    if (tid < D) reinterpret_cast<float*>(rec + CH_DEND)[tid] = dend[tid];
}

template <typename K>
int smem_attr(K kern, size_t bytes) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return set_error(MABA_ERR_CUDA, "dgda_prefill(chunked): %s", cudaGetErrorString(e));
    return MABA_OK;
}

template <typename T, typename TS, int MODE>
int scan_one(const PrefillArgs& a, dim3 grid, cudaStream_t s) {
    constexpr size_t smem = ScanSmem<MODE == 1 ? 2 * D : D, MODE != 1>::TOTAL;
    auto kern = dgda_scan_kernel<T, TS, MODE>;
    MABA_TRY(smem_attr(kern, smem));
    kern<<<grid, NTH, smem, s>>>(a);
    return check_launch("dgda_prefill(scan)");
}

template <typename T, typename TS>
int scan_mode(const PrefillArgs& a, dim3 grid, int mode, cudaStream_t s) {
    switch (mode) {
        case 0: return scan_one<T, TS, 0>(a, grid, s);
        case 1: return scan_one<T, TS, 1>(a, grid, s);
        default: return scan_one<T, TS, 2>(a, grid, s);
    }
}

template <typename T>
int prep_one(const PrefillArgs& a, int64_t BH, cudaStream_t s) {
    auto kern = dgda_prep_kernel<T>;
    MABA_TRY(smem_attr(kern, prep::TOTAL));
    PrefillArgs b = a;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NTH, prep::TOTAL) != cudaSuccess) {
        (void)cudaGetLastError();
        per_sm = 0;
    }
    b.pf_ahead = (int64_t)per_sm * sm_count();
    kern<<<dim3((unsigned)BH, (unsigned)a.nch), NTH, prep::TOTAL, s>>>(b);
    return check_launch("dgda_prefill(prep)");
}

}  // namespace

int dgda_scan_launch(const PrefillArgs& a, dim3 grid, int mode, int dtype, int state_dtype, cudaStream_t s) {
    if (dtype == MABA_BF16)
        return state_dtype == MABA_F32 ? scan_mode<__nv_bfloat16, float>(a, grid, mode, s)
                                       : scan_mode<__nv_bfloat16, __nv_bfloat16>(a, grid, mode, s);
    if (dtype == MABA_F16)
        return state_dtype == MABA_F32 ? scan_mode<__half, float>(a, grid, mode, s)
                                       : scan_mode<__half, __half>(a, grid, mode, s);
    return set_error(MABA_ERR_DTYPE, "dgda_prefill(chunked): 16-bit inputs only");
}

int dgda_prep_launch(const PrefillArgs& a, int64_t BH, int dtype, cudaStream_t s) {
    if (dtype == MABA_BF16) return prep_one<__nv_bfloat16>(a, BH, s);
    if (dtype == MABA_F16) return prep_one<__half>(a, BH, s);
    return set_error(MABA_ERR_DTYPE, "dgda_prefill(chunked): 16-bit inputs only");
}

}  // namespace maba
