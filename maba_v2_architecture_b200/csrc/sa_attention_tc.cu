// MABA-SA attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA),
// 16-bit inputs, latent dim 128, block size 64.
//
// Same math as sa_attention.cu / sa_attention_mma.cu (maba_sparse/layers/
// sparse_attention.py:79-219 and 274-275 in the MLA-absorbed latent space):
// three streams (window + sinks, the selected blocks, the pooled HCA rows),
// one softmax per stream and row, superposed by the softmax of the gate.
//
// One CTA per 64 query tokens; it runs the heads two at a time (128 MMA rows,
// row m = 2 t + h) over one tile schedule built once per CTA.  The tiles of
// all head pairs form one sequence g = hp * n_tiles + j, so every pipeline
// barrier's phases simply count g.  12 warps in three warpgroups:
//  * warps 0..7: softmax and epilogue, two groups of four (warp w handles TMEM
//    lane quarter w & 3, one thread per MMA row); group w >> 2 owns the tiles
//    g with g & 1 == group and S buffer `group`.  Per tile: load S from TMEM,
//    release the S buffer, exponentials against the row's reference maximum,
//    P (16-bit) into shared-memory buffer g & 3 (128-byte swizzled rows, the A
//    operand of PV), arrive.  Per head pair: the gate-weighted sum of the
//    three streams' O / l;
//  * warp 8: TMA producer -- the Q tile of each head pair into one of two
//    buffers (box 64 x 2 heads x 64 tokens, two 64-wide halves of d_c), every
//    latent key tile into a 4-stage ring (box 64 rows x 64 columns, twice);
//    all with 128-byte swizzle;
//  * warp 9: allocates the 512 TMEM columns and issues S = Q K^T (M=128,
//    N=64, K=128; K-major A and B) into the owning group's S buffer, two
//    tiles ahead of the softmax;
//  * warp 10: issues O_s += P V (M=128, N=128, K=64; A = P from shared
//    memory, B = the same key tile read MN-major) into the TMEM accumulator of
//    the tile's stream; its commits free the key stage and the P buffer;
//  * warp 11: idle (completes the warpgroup that lends registers).
// TMEM: S buffers in columns [0,128), O of stream s in [128+128s, 256+128s).
// The bound-referenced instantiation (EXACT = false) needs no running
// maximum: see the comment above the softmax code; the running-maximum one
// (EXACT = true) serves fp16 and the CTAs the first pass listed.
// The sparse stream runs over the union of the blocks the 64 tokens selected
// (bitmap + popcount ranks + 64-bit token masks), as in the mma kernel.
//
// Every mbarrier wait is bounded: a wait that runs out raises a shared abort
// flag, all roles leave their loops, the MMA issuers drain their MMAs and the
// producer its copies (bounded again), TMEM is freed and the device error word
// read by maba_device_error() is set.
#include "sa_attention.cuh"
#include "tcgen05.cuh"

#include <cudaTypedefs.h>
#include <type_traits>

namespace maba {

__device__ int g_device_error = 0;

namespace {
using namespace tc;

constexpr int QT = 64;            // query tokens per CTA
constexpr int KT = 64;            // keys per tile (= block size)
constexpr int DCX = 128;          // latent dim
constexpr int HPG = 2;            // heads per MMA tile
constexpr int ROWS = QT * HPG;    // MMA rows
constexpr int NS = 4;             // key-tile stages
constexpr int KMAX = 32;          // selected blocks per token
constexpr int UMAX = QT * KMAX;   // union capacity
// 12 warps in three warpgroups: 0-7 softmax (two groups of four), 8 TMA producer,
// 9 QK issuer, 10 PV issuer, 11 idle.  The last warpgroup gives registers to the
// softmax warpgroups (setmaxnreg): 256 x REG_SOFTMAX + 128 x REG_OTHER equals
// 384 x REG_LAUNCH, the registers the block is launched with.
constexpr int NTHR = 384;
constexpr int REG_LAUNCH = 168, REG_SOFTMAX = 224, REG_OTHER = 56;
static_assert(256 * REG_SOFTMAX + 128 * REG_OTHER <= NTHR * REG_LAUNCH, "register split exceeds the launch");
constexpr int TMEM_COLS = 512;
constexpr int COL_S = 0;
constexpr int COL_O = 128;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float RESCALE_T = 8.f;

constexpr uint32_t Q_HALF = ROWS * 128;     // 16 KB: 128 rows x 64 elements
constexpr uint32_t Q_BYTES = 2 * Q_HALF;
constexpr uint32_t KV_HALF = KT * 128;      // 8 KB: 64 rows x 64 elements
constexpr uint32_t KV_BYTES = 2 * KV_HALF;
constexpr uint32_t P_BYTES = ROWS * 128;    // 16 KB: P of one tile, 128 rows x 64 keys (16-bit)

enum { B_QFULL = 0, B_QEMPTY = 2, B_KVFULL = 4, B_KVEMPTY = B_KVFULL + NS, B_SFULL = B_KVEMPTY + NS,
       B_PFULL = B_SFULL + 2, B_ODONE = B_PFULL + 4, B_SFREE = B_ODONE + 4, B_DRAIN = B_SFREE + 2,
       B_OFREE = B_DRAIN + 2, N_BARS = B_OFREE + 1 };
static_assert(N_BARS <= 32, "barrier area holds 32 mbarriers");

struct TcLayout {
    uint32_t q, kv, p, bars, misc, umask, ulist, bitmap, wpref, scan, xch, total;
    __host__ __device__ explicit TcLayout(int nwords) {
        q = 0;
        kv = q + 2 * Q_BYTES;
        p = kv + NS * KV_BYTES;
        bars = p + 4 * P_BYTES;  // P of tile g in buffer g & 3
        misc = bars + 32 * 8;
        umask = misc + 16;
        ulist = umask + UMAX * 8;
        bitmap = ulist + UMAX * 4;
        wpref = bitmap + nwords * 4;
        scan = wpref + nwords * 4;
        // After the prologue the scan area holds: tile maxima (the running-maximum
        // kernel) or reference inputs (the bound-referenced one), both
        // [2 groups][2][128]; row sums [2 groups][3][128]; stream key-norm maxima [4]
        xch = scan;
        const uint32_t xbytes = (2 * 2 + 2 * 3) * 128 * 4 + 16, sbytes = (NTHR + 16) * 4;
        total = xch + (xbytes > sbytes ? xbytes : sbytes);
    }
};

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max of three (one instruction on sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// {d0, d1} = {a0, a1} * b + c, one packed fp32 FMA
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b, float c) {
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %4};\n\tmov.b64 rc, {%5, %5};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b), "f"(c));
}

// {a0, a1} += {b0, b1}, one packed fp32 add
__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
    asm("{\n\t.reg .b64 ra, rb;\n\t"
        "mov.b64 ra, {%0, %1};\n\tmov.b64 rb, {%2, %3};\n\t"
        "add.rn.f32x2 ra, ra, rb;\n\tmov.b64 {%0, %1}, ra;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1));
}

template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t v);
template <> __device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 unpack2<__half>(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

// EXACT = false: bound-referenced softmax (16-bit bf16 only); a CTA any of whose
// rows shows underflow in a stream's sum appends its unit to redo_list.
// EXACT = true: running-maximum softmax; with redo_list the grid covers the
// listed units only (blocks past *redo_count return at once).
template <typename T, bool EXACT>
__global__ void __launch_bounds__(NTHR, 1)
    sa_attention_tc_kernel(const SaArgs a, const __grid_constant__ CUtensorMap tm_q,
                           const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_h,
                           int nwords, const float* __restrict__ tnc, const float* __restrict__ tnh, int ntc,
                           int nth, int* __restrict__ redo_count, int* __restrict__ redo_list) {
    extern __shared__ unsigned char smem_dyn[];
    unsigned char* base =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
    const TcLayout LY(nwords);
    unsigned char* Qs = base + LY.q;
    unsigned char* KVs = base + LY.kv;
    unsigned char* Ps = base + LY.p;
    uint64_t* bars = reinterpret_cast<uint64_t*>(base + LY.bars);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + LY.misc);
    volatile int* abort_f = reinterpret_cast<volatile int*>(base + LY.misc + 4);
    volatile int* redo_f = reinterpret_cast<volatile int*>(base + LY.misc + 8);  // some row failed the bound check
    unsigned long long* umask = reinterpret_cast<unsigned long long*>(base + LY.umask);
    int* ulist = reinterpret_cast<int*>(base + LY.ulist);
    unsigned* bitmap = reinterpret_cast<unsigned*>(base + LY.bitmap);
    int* wpref = reinterpret_cast<int*>(base + LY.wpref);
    int* scan = reinterpret_cast<int*>(base + LY.scan);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int unit = blockIdx.y * gridDim.x + blockIdx.x;
    if (EXACT && redo_list != nullptr) {
        if (unit >= *redo_count) return;
        unit = redo_list[unit];
    }
    const int64_t q0 = (int64_t)(unit % gridDim.x) * QT;
    const int64_t b = unit / gridDim.x;
    const int NH = a.H / HPG;
    const int nt = (int)((a.Lq - q0) < QT ? (a.Lq - q0) : QT);
    const int64_t P0 = a.Lkv - a.Lq + q0;  // absolute position of query row 0 of the tile
    const int64_t Plast = P0 + nt - 1;
    const int64_t nb_kv = (a.Lkv + KT - 1) / KT;
    const int K = a.K;
    const int64_t* tix = a.top_idx + b * a.st[0];

    if (tid == 0) {
        for (int i = 0; i < N_BARS; ++i) {
            uint32_t cnt = 1;
            if ((i >= B_PFULL && i < B_PFULL + 4) || i == B_SFREE || i == B_SFREE + 1) cnt = 128;
            if (i == B_OFREE) cnt = 8;  // the softmax warps, once they have read a head pair's O
            if (i == B_QEMPTY || i == B_QEMPTY + 1) cnt = 1 + 8;  // the last QK's commit + 8 softmax warps
            mbar_init(&bars[i], cnt);
        }
        *abort_f = 0;
        *redo_f = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_c);
        prefetch_tmap(&tm_h);
    }
    if (warp == 9) tmem_alloc<TMEM_COLS>(tmem_slot);

    // ---------------- union of the selected blocks -------------------------
    for (int i = tid; i < nwords; i += NTHR) bitmap[i] = 0u;
    __syncthreads();
    // this thread's selected blocks (all loads in flight together; -1: none or not causal)
    constexpr int SEL_PER = (QT * KMAX + NTHR - 1) / NTHR;
    int sel[SEL_PER];
#pragma unroll
    for (int k = 0; k < SEL_PER; ++k) {
        const int e = tid + k * NTHR;
        int64_t n = -1;
        if (e < nt * K) {
            const int t = e / K, sl = e - t * K;
            n = tix[(q0 + t) * a.st[1] + sl * a.st[2]];
            if (!(n >= 0 && n < nb_kv && n * KT <= P0 + t)) n = -1;
        }
        sel[k] = (int)n;
    }
#pragma unroll
    for (int k = 0; k < SEL_PER; ++k)
        if (sel[k] >= 0) atomicOr(&bitmap[sel[k] >> 5], 1u << (sel[k] & 31));
    __syncthreads();
    {
        const int per = (nwords + NTHR - 1) / NTHR;
        const int w0 = tid * per;
        int s = 0;
        for (int i = 0; i < per; ++i)
            if (w0 + i < nwords) s += __popc(bitmap[w0 + i]);
        scan[tid] = s;
        __syncthreads();
        if (warp == 0) {
            constexpr int PL = NTHR / 32;
            int v[PL];
            int tot = 0;
#pragma unroll
            for (int i = 0; i < PL; ++i) {
                v[i] = scan[lane * PL + i];
                tot += v[i];
            }
            int inc = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            int run = inc - tot;
#pragma unroll
            for (int i = 0; i < PL; ++i) {
                scan[lane * PL + i] = run;
                run += v[i];
            }
            if (lane == 31) scan[NTHR] = inc;
        }
        __syncthreads();
        int run = scan[tid];
        for (int i = 0; i < per; ++i) {
            const int wi = w0 + i;
            if (wi < nwords) {
                wpref[wi] = run;
                unsigned bits = bitmap[wi];
                int r = run;
                while (bits) {
                    const int bit = __ffs(bits) - 1;
                    bits &= bits - 1;
                    ulist[r] = wi * 32 + bit;
                    umask[r] = 0ull;
                    ++r;
                }
                run += __popc(bitmap[wi]);
            }
        }
    }
    __syncthreads();
    const int U = scan[NTHR];
#pragma unroll
    for (int k = 0; k < SEL_PER; ++k) {
        const int n = sel[k];
        if (n >= 0) {
            const int t = (tid + k * NTHR) / K;
            const int wi = n >> 5;
            const int r = wpref[wi] + __popc(bitmap[wi] & ((1u << (n & 31)) - 1u));
            atomicOr(&umask[r], 1ull << t);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // ---------------- tile schedule (the same for every head pair) ----------
    const int64_t lo_min = P0 - a.window + 1 > 0 ? P0 - a.window + 1 : 0;
    const int64_t ws = (lo_min / KT) * KT;
    const int n_win = (int)((Plast - ws) / KT + 1);
    const bool sink_tile = ws > 0 && a.n_sinks > 0;
    const int n_local = n_win + (sink_tile ? 1 : 0);
    int64_t nhca_max = 0;
    if (Plast >= a.hca_r - 1) {
        nhca_max = (Plast + 1) / a.hca_r;
        if (nhca_max > a.NC) nhca_max = a.NC;
    }
    const int n_hca = (int)((nhca_max + KT - 1) / KT);
    const int n_tiles = n_local + U + n_hca;
    const int G = NH * n_tiles;
    constexpr bool BF = std::is_same<T, __nv_bfloat16>::value;

    if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_OTHER));
    if (warp == 8) {
        // ============================ TMA producer ============================
        // The whole warp runs the loop (warp-uniform coordinates and waits); one
        // elected lane issues the copies.
        int g = 0, nq = 0;
        bool okp = true;
        for (int hp = 0; hp < NH && okp; ++hp) {
            const int qb = hp & 1;
            if (hp >= 2) okp = mbar_wait_warp(&bars[B_QEMPTY + qb], ((hp >> 1) - 1) & 1, abort_f);
            if (!okp) break;
            if (elect_one()) {
                mbar_arrive_expect_tx(&bars[B_QFULL + qb], Q_BYTES);
                tma_load_4d(Qs + qb * Q_BYTES, &tm_q, &bars[B_QFULL + qb], 0, hp * HPG, (int)q0, (int)b);
                tma_load_4d(Qs + qb * Q_BYTES + Q_HALF, &tm_q, &bars[B_QFULL + qb], 64, hp * HPG, (int)q0, (int)b);
            }
            __syncwarp();
            ++nq;
            for (int j = 0; j < n_tiles; ++j, ++g) {
                const int st = g % NS;
                if (g >= NS) okp = mbar_wait_warp(&bars[B_KVEMPTY + st], ((g / NS) - 1) & 1, abort_f);
                if (!okp) break;
                int row0, hcat;
                if (j < n_local) {
                    hcat = 0;
                    row0 = sink_tile ? (j == 0 ? 0 : (int)ws + (j - 1) * KT) : (int)ws + j * KT;
                } else if (j < n_local + U) {
                    hcat = 0;
                    row0 = ulist[j - n_local] * KT;
                } else {
                    hcat = 1;
                    row0 = (j - n_local - U) * KT;
                }
                const CUtensorMap* m = hcat ? &tm_h : &tm_c;
                unsigned char* dst = KVs + st * KV_BYTES;
                if (elect_one()) {
                    mbar_arrive_expect_tx(&bars[B_KVFULL + st], KV_BYTES);
                    tma_load_3d(dst, m, &bars[B_KVFULL + st], 0, row0, (int)b);
                    tma_load_3d(dst + KV_HALF, m, &bars[B_KVFULL + st], 64, row0, (int)b);
                }
                __syncwarp();
            }
        }
        // every copy issued has landed before the CTA may exit
        for (int qb = 0; qb < 2 && qb < nq; ++qb) {
            const int last = ((nq - 1 - qb) / 2) * 2 + qb;
            mbar_wait_warp(&bars[B_QFULL + qb], (last >> 1) & 1, nullptr);
        }
        for (int s = 0; s < NS && s < g; ++s) {
            const int last = ((g - 1 - s) / NS) * NS + s;
            mbar_wait_warp(&bars[B_KVFULL + s], (last / NS) & 1, nullptr);
        }
    } else if (warp == 9 || warp == 10) {
        // ========================= MMA issuers ================================
        // Warp 9 issues the QK products, warp 10 the PV products, so that each
        // sleeps only on its own conditions (an MMA issue blocks its warp while the
        // tensor pipe is full).  QK(g) needs its key tile and that the group owning
        // S buffer g&1 has loaded tile g-2 out of it; PV(g) needs P(g) in shared
        // memory.  QK(g) has completed before PV(g) is issued (the softmax loaded
        // S(g)), so the PV warp's commit also frees the key tile.  The whole warp
        // runs each loop; one elected lane issues.  Descriptor bases are built once:
        // a start address moves by adding (bytes >> 4) to the descriptor.
        constexpr uint32_t ID_QK = idesc_f16(ROWS, KT, BF, false, false);
        constexpr uint32_t ID_PV = idesc_f16(ROWS, DCX, BF, false, true);
        if (warp == 9) {
            const uint64_t qd0 = sdesc_sw128(smem_addr(Qs), 16, 1024);
            const uint64_t kd0 = sdesc_sw128(smem_addr(KVs), 16, 1024);
            int jq = 0, hq = 0;
            for (int gq = 0; gq < G; ++gq) {
                const int st = gq % NS, sb = gq & 1, qb = hq & 1;
                bool okm = true;
                if (jq == 0) okm = mbar_wait_warp(&bars[B_QFULL + qb], (hq >> 1) & 1, abort_f);
                if (okm) okm = mbar_wait_warp(&bars[B_KVFULL + st], (gq / NS) & 1, abort_f);
                if (okm && gq >= 2) okm = mbar_wait_warp(&bars[B_SFREE + sb], ((gq - 2) >> 1) & 1, abort_f);
                if (!okm) break;
                tc_fence_after();
                const uint64_t qd = qd0 + (uint64_t)(qb * (Q_BYTES >> 4));
                const uint64_t kd = kd0 + (uint64_t)(st * (KV_BYTES >> 4));
#pragma unroll
                for (int k = 0; k < DCX / 16; ++k) {
                    const uint32_t off_q = (k >> 2) * (Q_HALF >> 4) + (k & 3) * 2;
                    const uint32_t off_k = (k >> 2) * (KV_HALF >> 4) + (k & 3) * 2;
                    umma_f16_ss_elect(tmem + COL_S + sb * KT, qd + off_q, kd + off_k, ID_QK, k > 0 ? 1u : 0u);
                }
                umma_commit_elect(&bars[B_SFULL + sb]);
                if (jq == n_tiles - 1) umma_commit_elect(&bars[B_QEMPTY + qb]);
                if (++jq == n_tiles) {
                    jq = 0;
                    ++hq;
                }
            }
        } else {
            const uint64_t vd0 = sdesc_sw128(smem_addr(KVs), KV_HALF, 1024);
            const uint64_t pd0 = sdesc_sw128(smem_addr(Ps), 16, 1024);
            int ij = 0;
            for (int i = 0; i < G; ++i) {
                const int st = i % NS;
                // (bound-referenced kernel) a head pair's first PV overwrites O: every softmax
                // warp has read the previous head pair's O
                if (!EXACT && ij == 0 && i > 0 && !mbar_wait_warp(&bars[B_OFREE], ((i / n_tiles) - 1) & 1, abort_f))
                    break;
                // P(i) completes phase i >> 2 of barrier i & 3: consecutive phases of one barrier
                // are four tiles apart, and P(i + 4) needs PV(i) done, so no phase is skipped
                if (!mbar_wait_warp(&bars[B_PFULL + (i & 3)], (i >> 2) & 1, abort_f)) break;
                tc_fence_after();
                const int stream = ij < n_local ? 0 : (ij < n_local + U ? 1 : 2);
                const bool first = ij == 0 || ij == n_local || ij == n_local + U;
                const uint32_t dst = tmem + COL_O + stream * DCX;
                const uint64_t vd = vd0 + (uint64_t)(st * (KV_BYTES >> 4));
                const uint64_t pd = pd0 + (uint64_t)((i & 3) * (P_BYTES >> 4));
#pragma unroll
                for (int k = 0; k < KT / 16; ++k)
                    umma_f16_ss_elect(dst, pd + (uint64_t)(k * 2), vd + (uint64_t)(k * (2048 >> 4)), ID_PV,
                                      (k > 0 || !first) ? 1u : 0u);
                umma_commit_elect(&bars[B_KVEMPTY + st]);
                umma_commit_elect(&bars[B_ODONE + (i & 3)]);  // PV(i) completes phase i >> 2 of barrier i & 3
                if (++ij == n_tiles) ij = 0;
            }
        }
        // every MMA this warp issued has completed before TMEM is freed
        const int db = B_DRAIN + (warp == 9 ? 0 : 1);
        umma_commit_elect(&bars[db]);
        mbar_wait_warp(&bars[db], 0, nullptr);
    }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_SOFTMAX));
        // ===================== softmax + epilogue (256 threads) ===============
        // Two groups of four warps, one warp per TMEM lane quarter in each.  Group wg
        // owns the key tiles whose global index has parity wg (its S buffer is wg), so
        // the two warps of a lane quarter, which share an SM sub-partition, work on
        // consecutive tiles in different phases: one runs exponentials while the other
        // loads and stores.  Each warp keeps the row sums of its own tiles; the pair
        // adds them at the end of a head pair.
        //
        // Reference maxima.  Softmax is invariant to the reference m subtracted from
        // the scores; it only has to keep every exponent in range.  Before a head
        // pair's tiles, each row gets per stream the upper bound of its scores
        // m = |q| * (max key norm of the stream's tiles): every score s has s - m <= 0,
        // so P = exp(s - m) needs no running maximum, no rescale of O and no exchange
        // between the two warps.  Underflow is checked afterwards: a stream whose row
        // sum is below e^-60 (its maximum lies more than ~60 below the bound, where
        // exponentials start to flush) sends the CTA to the running-maximum kernel, as
        // do missing key norms.  In that kernel (EXACT) the pair publishes its tiles'
        // maxima to each other (named barriers used as producer -> consumer pairs) and
        // replays the partner's, so both hold the same lazily rescaled reference at
        // every tile.  Every named-barrier call is unconditional (a wait that ran out
        // only skips TMEM work), so the two warps always make the same calls.
        const int wg = warp >> 2;
        const int q4 = warp & 3;
        const int rid = q4 * 32 + lane;
        const int t = rid >> 1, hh = rid & 1;
        const bool rvalid = t < nt;
        const int bar_mine = 1 + wg * 4 + q4, bar_other = 1 + (wg ^ 1) * 4 + q4, bar_pair = 9 + q4;
        float* xmax = reinterpret_cast<float*>(base + LY.xch);  // [2 groups][2 slots][128]
        float* xls = xmax + 2 * 2 * 128;                          // [2 groups][3 streams][128]
        float* xref = xmax;                                       // [2 groups][2][128] (bound-referenced kernel)
        float* mstr = xls + 2 * 3 * 128;                          // key-norm maxima per stream
        // positions fit in 32 bits (Lkv < 2^31 on this path)
        const int pos = (int)(P0 + t);
        const int lkv = (int)a.Lkv;
        const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
        const int lo_p = pos - a.window + 1 > 0 ? pos - a.window + 1 : 0;
        const int sink_end = a.n_sinks < lo_p ? a.n_sinks : lo_p;
        const int sp_end = pos + 1 < lkv ? pos + 1 : lkv;
        int nv_hca = 0;
        if (pos >= a.hca_r - 1) {
            nv_hca = (pos + 1) / a.hca_r;
            if (nv_hca > a.NC) nv_hca = (int)a.NC;
        }
        const unsigned long long tbit = 1ull << t;
        const T* ckv = static_cast<const T*>(a.ckv) + b * a.sc[0];
        auto clampk = [](int x) { return x < 0 ? 0 : (x > KT ? KT : x); };
        auto stream_of = [&](int j) { return j < n_local ? 0 : (j < n_local + U ? 1 : 2); };
        // valid columns of this row in tile j: [a1, b1) and the sinks [0, b2)
        auto bounds = [&](int j, int& a1, int& b1, int& b2) {
            a1 = 0;
            b1 = 0;
            b2 = 0;
            if (!rvalid) return;
            if (j < n_local) {
                const int row0 = sink_tile ? (j == 0 ? 0 : (int)ws + (j - 1) * KT) : (int)ws + j * KT;
                a1 = clampk(lo_p - row0);
                b1 = clampk(pos - row0 + 1);
                b2 = clampk(sink_end - row0);
            } else if (j < n_local + U) {
                const int u = j - n_local;
                if (umask[u] & tbit) b1 = clampk(sp_end - ulist[u] * KT);
            } else {
                b1 = clampk(nv_hca - (j - n_local - U) * KT);
            }
        };
        auto pair_sync = [&](int id) { asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory"); };
        auto all_sync = [&]() { asm volatile("bar.sync 13, 256;" ::: "memory"); };
        // ---- largest key norm of each stream's tiles (one warp; all read after a barrier)
        if (warp == 0) {
            float ml = 0.f, mu = 0.f, mh = 0.f;
            if (tnc != nullptr) {
                const float* nc = tnc + b * ntc;
                for (int j = lane; j < n_tiles; j += 32) {
                    if (j < n_local) {
                        const int row0 = sink_tile ? (j == 0 ? 0 : (int)ws + (j - 1) * KT) : (int)ws + j * KT;
                        ml = fmaxf(ml, nc[row0 / KT]);
                    } else if (j < n_local + U) {
                        mu = fmaxf(mu, nc[ulist[j - n_local]]);
                    } else {
                        mh = fmaxf(mh, tnh[b * nth + (j - n_local - U)]);
                    }
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                ml = fmaxf(ml, __shfl_xor_sync(0xffffffffu, ml, o));
                mu = fmaxf(mu, __shfl_xor_sync(0xffffffffu, mu, o));
                mh = fmaxf(mh, __shfl_xor_sync(0xffffffffu, mh, o));
            }
            if (lane == 0) {
                mstr[0] = ml;
                mstr[1] = mu;
                mstr[2] = mh;
            }
        }
        all_sync();
        const float Mloc = mstr[0], Muni = mstr[1], Mhca = mstr[2];
        // probe keys of this row: itself (local), its first attended union key, pooled entry 0
        int probe_u = -1;
        if (rvalid) {
            for (int u = 0; u < U; ++u) {
                if ((umask[u] & tbit) && ulist[u] * KT < sp_end) {
                    probe_u = ulist[u] * KT;
                    break;
                }
            }
        }
        // q . k over d_c = 128 for the query row rid of Q buffer qb (128-byte swizzled
        // rows in two 64-column halves) and a key row in global memory (k == null: |q|^2)
        auto qdot = [&](int qb, const T* k) -> float {
            const unsigned char* qrow = Qs + qb * Q_BYTES + (rid >> 3) * 1024 + (rid & 7) * 128;
            float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const uint4 qv =
                    *reinterpret_cast<const uint4*>(qrow + (c >> 3) * Q_HALF + (((c & 7) ^ (rid & 7)) << 4));
                const uint4 kv = k != nullptr ? *reinterpret_cast<const uint4*>(k + c * 8) : qv;
                const uint32_t qa[4] = {qv.x, qv.y, qv.z, qv.w}, ka[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 qf = unpack2<T>(qa[e]), kf = unpack2<T>(ka[e]);
                    acc0 = fmaf(qf.x, kf.x, acc0);
                    acc1 = fmaf(qf.y, kf.y, acc1);
                }
            }
            return acc0 + acc1;
        };
        const T* hcab = a.NC > 0 ? static_cast<const T*>(a.hca) + b * a.sh[0] : nullptr;
        bool okw = true;    // every wait of this warp completed
        bool redo = false;  // some head pair missed the range condition of the bound references
        // Reads Q of head pair hq (then releases it to the producer) and, in the
        // bound-referenced kernel, sets the row's reference maxima (log2 units) and
        // returns whether every row of the CTA meets the range condition.
        auto head_refs = [&](int hq, float& r0, float& r1, float& r2) -> bool {
            const int qb = hq & 1;
            const bool okq = mbar_wait_warp(&bars[B_QFULL + qb], (hq >> 1) & 1, abort_f);
            okw = okw && okq;
            float qq = 0.f;
            if (!EXACT && okq && rvalid && tnc != nullptr) qq = qdot(qb, nullptr);
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[B_QEMPTY + qb]);  // Q read; the QK warp commits its last QK
            if constexpr (EXACT) {
                r0 = r1 = r2 = 0.f;
                return false;
            } else {
                // the reference of each stream is the row's score bound |q| * (largest key norm
                // of the stream's tiles): no exponent can overflow, and the epilogue sends the
                // CTA to the running-maximum pass if some row's sum shows underflow
                const float qn = sqrtf(qq) * 1.0001f;
                r0 = qn * Mloc * LOG2E;
                r1 = qn * Muni * LOG2E;
                r2 = qn * Mhca * LOG2E;
                return tnc != nullptr;
            }
        };
        float rl0, rl1, rl2;
        bool fast = head_refs(0, rl0, rl1, rl2);
        for (int hp = 0; hp < NH; ++hp) {
            const int g0 = hp * n_tiles, gend = g0 + n_tiles;
            float l0 = 0.f, l1 = 0.f, l2 = 0.f;  // this warp's share of the row sums per stream
            // ---- reference maxima of this head pair (group 0: |q|^2 and the local
            // probe, group 1: the union and HCA probes)
            // gate logits of this row's head, read now and used by the epilogue
            float graw0 = 0.f, graw1 = 0.f, graw2 = 0.f;
            if (rvalid) {
                const int h = hp * HPG + hh;
                const T* gp = static_cast<const T*>(a.gate);
                const T* gr = a.gate4d ? gp + b * a.sg[0] + h * a.sg[1] + (q0 + t) * a.sg[2]
                                       : gp + b * a.sg[0] + (q0 + t) * a.sg[1];
                const int64_t gs = a.gate4d ? a.sg[3] : a.sg[2];
                graw0 = Cvt<T>::to_f(gr[0]);
                graw1 = Cvt<T>::to_f(gr[gs]);
                graw2 = Cvt<T>::to_f(gr[2 * gs]);
            }
            if constexpr (!EXACT) {
                if (!fast) redo = true;
                // ------------- bound-referenced tiles: no maximum, no rescale -------------
                const int j0 = (g0 & 1) == wg ? 0 : 1;
                int na1 = 0, nb1 = 0, nb2 = 0;
                if (j0 < n_tiles) bounds(j0, na1, nb1, nb2);
                for (int j = j0; j < n_tiles; j += 2) {
                    const int gg = g0 + j;
                    const int st = stream_of(j);
                    const int a1 = na1, b1 = nb1, b2 = nb2;
                    const bool none = b1 <= a1 && b2 == 0;
                    const bool full = a1 == 0 && b1 >= KT;
                    const bool oks = mbar_wait_warp(&bars[B_SFULL + wg], (gg >> 1) & 1, abort_f);
                    okw = okw && oks;
                    const uint32_t ts = tmem + lane_base + COL_S + wg * KT;
                    uint32_t s[KT];
                    if (oks) {
                        tc_fence_after();
                        tmem_ld32(ts, s);
                        tmem_ld32(ts + 32, s + 32);
                    }
                    // the next own tile's bounds while the loads are in flight
                    if (j + 2 < n_tiles) bounds(j + 2, na1, nb1, nb2);
                    if (oks) tmem_wait_ld_pin64(s);
                    // S is in registers: the MMA warp may compute tile gg+2 into this buffer
                    tc_fence_before();
                    mbar_arrive(&bars[B_SFREE + wg]);
                    if (oks) {
                        if (__any_sync(0xffffffffu, !none && !full)) {
                            unsigned long long vm = 0ull;
                            if (b1 > a1) vm = (b1 >= 64 ? ~0ull : ((1ull << b1) - 1ull)) & ~((1ull << a1) - 1ull);
                            if (b2 > 0) vm |= b2 >= 64 ? ~0ull : ((1ull << b2) - 1ull);
#pragma unroll
                            for (int c = 0; c < KT; ++c)
                                if (!((vm >> c) & 1ull)) s[c] = __float_as_uint(-INFINITY);
                        }
                        // rows without a valid column give p = 0 (ex2(-inf)); scores are finite
                        const float nmu = none ? -INFINITY : -(st == 0 ? rl0 : (st == 1 ? rl1 : rl2));
                        float sa0 = 0.f, sa1 = 0.f, sb0 = 0.f, sb1 = 0.f;
                        uint32_t pk[KT / 2];
#pragma unroll
                        for (int c = 0; c < KT; c += 4) {
                            float x0, x1, x2, x3;
                            fma2(x0, x1, __uint_as_float(s[c]), __uint_as_float(s[c + 1]), LOG2E, nmu);
                            fma2(x2, x3, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]), LOG2E, nmu);
                            const float p0 = ex2(x0), p1 = ex2(x1), p2 = ex2(x2), p3 = ex2(x3);
                            add2(sa0, sa1, p0, p1);
                            add2(sb0, sb1, p2, p3);
                            pk[c >> 1] = pack2<T>(p0, p1);
                            pk[(c >> 1) + 1] = pack2<T>(p2, p3);
                        }
                        const float ls = (sa0 + sa1) + (sb0 + sb1);
                        if (st == 0) l0 += ls;
                        else if (st == 1) l1 += ls;
                        else l2 += ls;
                        // P buffer gg & 3 once PV(gg-4) has read it
                        const bool okp =
                            gg < 4 || mbar_wait_warp(&bars[B_ODONE + (gg & 3)], ((gg - 4) >> 2) & 1, abort_f);
                        okw = okw && okp;
                        if (okp) {
                            unsigned char* prow = Ps + (gg & 3) * P_BYTES + (rid >> 3) * 1024 + (rid & 7) * 128;
#pragma unroll
                            for (int c = 0; c < 8; ++c)
                                *reinterpret_cast<uint4*>(prow + ((c ^ (rid & 7)) << 4)) =
                                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
                            fence_proxy_async_smem();
                        }
                    }
                    mbar_arrive(&bars[B_PFULL + (gg & 3)]);
                }
            } else {
            float m_cur = -INFINITY, l_cur = 0.f;
            int cur = -1;
            // folds the maximum mx (log2 units) of the next tile, of stream st, into the
            // running state; returns the factor of the rescale it causes (1: none)
            auto apply = [&](int st, float mx) -> float {
                if (st != cur) {
                    if (cur == 0) l0 = l_cur;
                    else if (cur == 1) l1 = l_cur;
                    m_cur = -INFINITY;
                    l_cur = 0.f;
                    cur = st;
                }
                float fac = 1.f;
                if (mx != -INFINITY) {
                    if (m_cur == -INFINITY) {
                        m_cur = mx;
                    } else if (mx > m_cur + RESCALE_T) {
                        fac = ex2(m_cur - mx);
                        m_cur = mx;
                        l_cur *= fac;
                    }
                }
                return fac;
            };
                for (int j = (g0 & 1) == wg ? 0 : 1; j < n_tiles; j += 2) {
                    const int gg = g0 + j;
                    const int st = stream_of(j);
                    int a1, b1, b2;
                    bounds(j, a1, b1, b2);
                    const bool none = b1 <= a1 && b2 == 0;
                    const bool full = a1 == 0 && b1 >= KT;
                    const bool oks = mbar_wait_warp(&bars[B_SFULL + wg], (gg >> 1) & 1, abort_f);
                    okw = okw && oks;
                    const uint32_t ts = tmem + lane_base + COL_S + wg * KT;
                    uint32_t s[KT];
                    float mt = -INFINITY;
                    if (oks) {
                        tc_fence_after();
                        tmem_ld32(ts, s);
                        tmem_ld32(ts + 32, s + 32);
                        tmem_wait_ld_pin64(s);
                    }
                    // S is in registers: the MMA warp may compute tile gg+2 into this buffer
                    tc_fence_before();
                    mbar_arrive(&bars[B_SFREE + wg]);
                    if (oks) {
                        if (__any_sync(0xffffffffu, !none && !full)) {
                            unsigned long long vm = 0ull;
                            if (b1 > a1) vm = (b1 >= 64 ? ~0ull : ((1ull << b1) - 1ull)) & ~((1ull << a1) - 1ull);
                            if (b2 > 0) vm |= b2 >= 64 ? ~0ull : ((1ull << b2) - 1ull);
    #pragma unroll
                            for (int c = 0; c < KT; ++c)
                                if (!((vm >> c) & 1ull)) s[c] = __float_as_uint(-INFINITY);
                        }
                        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    #pragma unroll
                        for (int c = 0; c < KT; c += 2)
                            m4[(c >> 1) & 3] = fmax3(m4[(c >> 1) & 3], __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
                        mt = none ? -INFINITY : fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * LOG2E;
                    }
                    // the partner's previous tile of this head pair, then this one
                    if (j >= 1) {
                        pair_sync(bar_other);
                        apply(stream_of(j - 1), xmax[((wg ^ 1) * 2 + (((gg - 1) >> 1) & 1)) * 128 + rid]);
                    }
                    xmax[(wg * 2 + ((gg >> 1) & 1)) * 128 + rid] = mt;
                    asm volatile("bar.arrive %0, 64;" ::"r"(bar_mine) : "memory");
                    const float fac = apply(st, mt);
                    if (oks) {
                        // rows without a valid column give p = 0 (ex2(-inf)); scores are finite
                        const float nmu = none ? -INFINITY : (m_cur == -INFINITY ? 0.f : -m_cur);
                        float sa0 = 0.f, sa1 = 0.f, sb0 = 0.f, sb1 = 0.f;
                        uint32_t pk[KT / 2];
    #pragma unroll
                        for (int c = 0; c < KT; c += 4) {
                            float x0, x1, x2, x3;
                            fma2(x0, x1, __uint_as_float(s[c]), __uint_as_float(s[c + 1]), LOG2E, nmu);
                            fma2(x2, x3, __uint_as_float(s[c + 2]), __uint_as_float(s[c + 3]), LOG2E, nmu);
                            const float p0 = ex2(x0), p1 = ex2(x1), p2 = ex2(x2), p3 = ex2(x3);
                            add2(sa0, sa1, p0, p1);
                            add2(sb0, sb1, p2, p3);
                            pk[c >> 1] = pack2<T>(p0, p1);
                            pk[(c >> 1) + 1] = pack2<T>(p2, p3);
                        }
                        l_cur += (sa0 + sa1) + (sb0 + sb1);
                        // P into shared-memory buffer wg (the A operand of PV, 128-byte swizzled
                        // rows) once PV(gg-2) has read the buffer
                        // P buffer gg & 3 once PV(gg-4) has read it
                        const bool okp =
                            gg < 4 || mbar_wait_warp(&bars[B_ODONE + (gg & 3)], ((gg - 4) >> 2) & 1, abort_f);
                        okw = okw && okp;
                        if (okp) {
                            unsigned char* prow = Ps + (gg & 3) * P_BYTES + (rid >> 3) * 1024 + (rid & 7) * 128;
    #pragma unroll
                            for (int c = 0; c < 8; ++c)
                                *reinterpret_cast<uint4*>(prow + ((c ^ (rid & 7)) << 4)) =
                                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
                            fence_proxy_async_smem();
                        }
                    }
                    if (__any_sync(0xffffffffu, fac != 1.f)) {
                        // every PV so far (the latest: tile gg-1, the partner's) has completed
                        const bool okr = mbar_wait_warp(&bars[B_ODONE + ((gg - 1) & 3)], ((gg - 1) >> 2) & 1, abort_f);
                        okw = okw && okr;
                        if (okr) {
                            tc_fence_after();
                            const uint32_t to = tmem + lane_base + COL_O + st * DCX;
    #pragma unroll 1
                            for (int cc = 0; cc < DCX / 32; ++cc) {
                                uint32_t o[32];
                                tmem_ld32(to + cc * 32, o);
                                tmem_wait_ld();
    #pragma unroll
                                for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * fac);
                                tmem_st32(to + cc * 32, o);
                            }
                        }
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(&bars[B_PFULL + (gg & 3)]);
                }
                // the partner's last tile, if it owns it
                if (((gend - 1) & 1) != wg) {
                    pair_sync(bar_other);
                    apply(stream_of(n_tiles - 1), xmax[((wg ^ 1) * 2 + (((gend - 1) >> 1) & 1)) * 128 + rid]);
                }
                if (cur == 0) l0 = l_cur;
                else if (cur == 1) l1 = l_cur;
                else if (cur == 2) l2 = l_cur;
            }
            // the next head pair's references (overlaps the last PVs of this one)
            float nl0 = 0.f, nl1 = 0.f, nl2 = 0.f;
            const bool nfast = hp + 1 < NH ? head_refs(hp + 1, nl0, nl1, nl2) : false;
            // ------------------------- epilogue of head pair hp ------------------
            // the last two PVs of the head pair (tiles gend-2, gend-1) have completed
            bool oke = gend < 2 || mbar_wait_warp(&bars[B_ODONE + ((gend - 2) & 3)], ((gend - 2) >> 2) & 1, abort_f);
            if (oke) oke = mbar_wait_warp(&bars[B_ODONE + ((gend - 1) & 3)], ((gend - 1) >> 2) & 1, abort_f);
            okw = okw && oke;
            xls[(wg * 3 + 0) * 128 + rid] = l0;
            xls[(wg * 3 + 1) * 128 + rid] = l1;
            xls[(wg * 3 + 2) * 128 + rid] = l2;
            pair_sync(bar_pair);
            // row sums over both warps' tiles
            const float L0 = l0 + xls[((wg ^ 1) * 3 + 0) * 128 + rid];
            const float L1 = l1 + xls[((wg ^ 1) * 3 + 1) * 128 + rid];
            const float L2 = l2 + xls[((wg ^ 1) * 3 + 2) * 128 + rid];
            if constexpr (!EXACT) {
                // a stream whose row sum fell below e^-60 (its largest score more than about 60
                // below the bound) may have lost terms to the flush of small exponentials
                constexpr float kMinL = 8.7e-27f;
                if (rvalid && (L0 < kMinL || (probe_u >= 0 && L1 < kMinL) || (nv_hca > 0 && L2 < kMinL)))
                    redo = true;
            }
            if (okw) {
                tc_fence_after();
                const int h = hp * HPG + hh;
                float g0v = graw0, g1v = graw1, g2v = graw2;
                if (rvalid) {
                    const float m = fmaxf(g0v, fmaxf(g1v, g2v));
                    const float e0 = expf(g0v - m), e1 = expf(g1v - m), e2 = expf(g2v - m);
                    const float inv = 1.f / (e0 + e1 + e2);
                    g0v = e0 * inv;
                    g1v = e1 * inv;
                    g2v = e2 * inv;
                }
                const bool u0 = L0 > 0.f, u1 = L1 > 0.f, u2 = L2 > 0.f;
                const float f0 = u0 ? g0v / L0 : 0.f, f1 = u1 ? g1v / L1 : 0.f, f2 = u2 ? g2v / L2 : 0.f;
                const bool early = rvalid && pos < a.hca_r - 1;  // HCA: mean of the latent prefix
                T* orow =
                    static_cast<T*>(a.out) + b * a.so[0] + (q0 + (rvalid ? t : 0)) * a.so[1] + (int64_t)h * a.so[2];
                const uint32_t to = tmem + lane_base + COL_O + wg * 64;
#pragma unroll 1
                for (int cc = 0; cc < 2; ++cc) {
                    const int col0 = wg * 64 + cc * 32;
                    uint32_t r0[32], r1[32], r2[32];
                    tmem_ld32(to + cc * 32, r0);
                    tmem_ld32(to + DCX + cc * 32, r1);
                    tmem_ld32(to + 2 * DCX + cc * 32, r2);
                    tmem_wait_ld();
                    float v[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        float x = u0 ? f0 * __uint_as_float(r0[e]) : 0.f;
                        x += u1 ? f1 * __uint_as_float(r1[e]) : 0.f;
                        x += u2 ? f2 * __uint_as_float(r2[e]) : 0.f;
                        v[e] = x;
                    }
                    if (early) {
                        const float w = g2v / float(pos + 1);
                        for (int jj = 0; jj <= pos; ++jj) {
                            const T* cr = ckv + (int64_t)jj * a.sc[1] + col0;
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] += w * Cvt<T>::to_f(cr[e]);
                        }
                    }
                    if (rvalid) {
#pragma unroll
                        for (int e8 = 0; e8 < 4; ++e8) {
                            uint4 w4 = make_uint4(pack2<T>(v[8 * e8 + 0], v[8 * e8 + 1]),
                                                  pack2<T>(v[8 * e8 + 2], v[8 * e8 + 3]),
                                                  pack2<T>(v[8 * e8 + 4], v[8 * e8 + 5]),
                                                  pack2<T>(v[8 * e8 + 6], v[8 * e8 + 7]));
                            *reinterpret_cast<uint4*>(orow + col0 + 8 * e8) = w4;
                        }
                    }
                }
            }
            // O has been read before the next head pair's first PV overwrites it: in the
            // running-maximum kernel both warps meet here (its named-barrier exchanges
            // stay in step), in the bound-referenced one the PV warp waits for O_FREE
            tc_fence_before();
            if constexpr (EXACT) {
                pair_sync(bar_pair);
            } else {
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars[B_OFREE]);
            }
            rl0 = nl0;
            rl1 = nl1;
            rl2 = nl2;
            fast = nfast;
        }
        if (!EXACT && redo) *redo_f = 1;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc<TMEM_COLS>(tmem);
    }
    if (!EXACT && tid == 0 && *redo_f && redo_list != nullptr) redo_list[atomicAdd(redo_count, 1)] = unit;
    if (tid == 0 && *abort_f) atomicExch(&g_device_error, 1);
}

// ------------------------------------------------------------------ host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiled>(p);
    }();
    return fn;
}

// rank-R tiled map of 16-bit elements, 128-byte swizzle; strides in elements (R-1 of them)
bool make_map(CUtensorMap* m, int dtype, const void* ptr, int rank, const int64_t* dims, const int64_t* strides,
              const uint32_t* box) {
    EncodeTiled fn = encode_fn();
    if (fn == nullptr) return false;
    cuuint64_t gd[5], gs[4];
    cuuint32_t bx[5], es[5];
    for (int i = 0; i < rank; ++i) {
        gd[i] = (cuuint64_t)dims[i];
        bx[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) gs[i] = (cuuint64_t)strides[i] * 2;
    }
    const CUresult r =
        fn(m, dtype == MABA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, (cuuint32_t)rank,
           const_cast<void*>(ptr), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

inline bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool s16(int64_t stride_elems) { return ((stride_elems * 2) % 16) == 0 && stride_elems > 0; }

// Largest L2 norm of the rows of each 64-row tile of c_kv [B, L, 128] (tiles
// 0..ntc-1) and of the pooled HCA entries [B, NC, 128] (tiles ntc..ntc+nth-1),
// scaled by 1 + 1e-3 so that |q| * norm bounds every score of the tile.
template <typename T>
__global__ void __launch_bounds__(256)
    kv_tile_norm_kernel(const T* __restrict__ c, int64_t cb, int64_t cr, int64_t L, int ntc, const T* __restrict__ h,
                        int64_t hb, int64_t hr, int64_t NC, int nth, float* __restrict__ out_c,
                        float* __restrict__ out_h, int* __restrict__ zero) {
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *zero = 0;
    __shared__ float wmax[8];
    const int64_t b = blockIdx.y;
    const int tile = blockIdx.x;
    const bool isc = tile < ntc;
    const T* base = isc ? c + b * cb : h + b * hb;
    const int64_t rs = isc ? cr : hr, n = isc ? L : NC;
    const int64_t r0 = (int64_t)(isc ? tile : tile - ntc) * KT;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float m = 0.f;
    for (int r = warp; r < KT; r += 8) {
        const int64_t row = r0 + r;
        if (row >= n) break;
        const uint2 v = *reinterpret_cast<const uint2*>(base + row * rs + lane * 4);
        const float2 x = unpack2<T>(v.x), y = unpack2<T>(v.y);
        float ss = x.x * x.x + x.y * x.y + y.x * y.x + y.y * y.y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        m = fmaxf(m, sqrtf(ss));
    }
    if (lane == 0) wmax[warp] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = 0.f;
        for (int i = 0; i < 8; ++i) mm = fmaxf(mm, wmax[i]);
        mm *= 1.001f;
        if (isc) out_c[b * ntc + tile] = mm;
        else out_h[b * nth + (tile - ntc)] = mm;
    }
}

int tc_nwords(const SaArgs& a) { return (int)(((a.Lkv + KT - 1) / KT + 31) / 32) + 1; }

}  // namespace

size_t sa_attention_tc_workspace(int64_t B, int64_t Lq, int64_t Lkv, int64_t NC) {
    // key-tile norms, the redo count (16 bytes) and the redo list (one int per unit)
    return (size_t)B * (size_t)(ceil_div(Lkv, KT) + ceil_div(NC, KT)) * sizeof(float) + 16 +
           (size_t)B * (size_t)ceil_div(Lq, QT) * sizeof(int);
}

bool sa_attention_tc_supported(const SaArgs& a, int dtype) {
    if (dtype != MABA_BF16 && dtype != MABA_F16) return false;
    if (a.pos_dev != nullptr) return false;
    if (a.DC != DCX || a.block != KT || a.K <= 0 || a.K > KMAX) return false;
    if (a.H % HPG != 0 || a.Lq < 16 || a.n_sinks > KT || a.window <= 0) return false;
    if (a.Lkv >= (int64_t(1) << 31) || a.Lq >= (int64_t(1) << 31)) return false;
    if (a.sq[3] != 1 || a.sc[2] != 1 || a.so[3] != 1 || (a.NC > 0 && a.sh[2] != 1)) return false;
    if (!s16(a.sq[2]) || !s16(a.sq[1]) || !s16(a.sq[0]) || !s16(a.sc[1]) || !s16(a.sc[0])) return false;
    if (a.NC > 0 && (!s16(a.sh[1]) || !s16(a.sh[0]) || !a16(a.hca))) return false;
    if (!a16(a.qhat) || !a16(a.ckv) || !a16(a.out) || (a.so[1] % 8) || (a.so[2] % 8)) return false;
    if (TcLayout(tc_nwords(a)).total + 1024 > 227 * 1024) return false;
    return encode_fn() != nullptr;
}

// The register split of the kernels (setmaxnreg) assumes REG_LAUNCH registers
// per thread at launch; a build with another count must not launch them (an
// increase beyond the block's registers would never complete).
template <typename T, bool EXACT> bool tc_regs_ok() {
    static const bool ok = [] {
        cudaFuncAttributes fa{};
        return cudaFuncGetAttributes(&fa, sa_attention_tc_kernel<T, EXACT>) == cudaSuccess &&
               fa.numRegs == REG_LAUNCH;
    }();
    return ok;
}

int sa_attention_tc(SaArgs& a, int64_t B, int dtype, cudaStream_t s) {
    if (dtype == MABA_BF16 ? !(tc_regs_ok<__nv_bfloat16, true>() && tc_regs_ok<__nv_bfloat16, false>())
                           : !tc_regs_ok<__half, true>())
        return sa_attention_mma(a, B, dtype, s);
    const int nwords = tc_nwords(a);
    const size_t smem = TcLayout(nwords).total + 1024;
    CUtensorMap mq, mc, mh;
    {
        const int64_t dq[4] = {a.DC, a.H, a.Lq, B};
        const int64_t sq[3] = {a.sq[2], a.sq[1], a.sq[0]};
        const uint32_t bq[4] = {64, (uint32_t)HPG, (uint32_t)QT, 1};
        const int64_t dc[3] = {a.DC, a.Lkv, B};
        const int64_t sc[2] = {a.sc[1], a.sc[0]};
        const uint32_t bc[3] = {64, (uint32_t)KT, 1};
        if (!make_map(&mq, dtype, a.qhat, 4, dq, sq, bq) || !make_map(&mc, dtype, a.ckv, 3, dc, sc, bc))
            return sa_attention_mma(a, B, dtype, s);
        if (a.NC > 0) {
            const int64_t dh[3] = {a.DC, a.NC, B};
            const int64_t sh[2] = {a.sh[1], a.sh[0]};
            if (!make_map(&mh, dtype, a.hca, 3, dh, sh, bc)) return sa_attention_mma(a, B, dtype, s);
        } else {
            mh = mc;  // no HCA tiles are scheduled
        }
    }
    // Bound-referenced pass (bf16, when the caller gave the workspace for the key
    // norms and the redo list), then the running-maximum pass over the units it
    // listed; otherwise the running-maximum pass over every unit.
    const int ntc = (int)ceil_div(a.Lkv, KT), nth = (int)ceil_div(a.NC, KT);
    const int nqt = (int)ceil_div(a.Lq, QT);
    dim3 grid((unsigned)nqt, (unsigned)B);
    float* tnc = nullptr;
    float* tnh = nullptr;
    int* redo_count = nullptr;
    int* redo_list = nullptr;
    if (dtype == MABA_BF16 && a.workspace != nullptr &&
        a.workspace_bytes >= sa_attention_tc_workspace(B, a.Lq, a.Lkv, a.NC)) {
        tnc = static_cast<float*>(a.workspace);
        tnh = tnc + B * ntc;
        redo_count = reinterpret_cast<int*>(tnh + B * nth);
        redo_list = redo_count + 4;
        using BT = __nv_bfloat16;
        kv_tile_norm_kernel<BT><<<dim3((unsigned)(ntc + nth), (unsigned)B), 256, 0, s>>>(
            static_cast<const BT*>(a.ckv), a.sc[0], a.sc[1], a.Lkv, ntc, static_cast<const BT*>(a.hca), a.sh[0],
            a.sh[1], a.NC, nth, tnc, tnh, redo_count);
        MABA_TRY(check_launch("sa_attention(key tile norms)"));
        auto fast = sa_attention_tc_kernel<BT, false>;
        cudaFuncSetAttribute(fast, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        fast<<<grid, NTHR, smem, s>>>(a, mq, mc, mh, nwords, tnc, tnh, ntc, nth, redo_count, redo_list);
        MABA_TRY(check_launch("sa_attention(tcgen05, bound references)"));
    }
    if (dtype == MABA_BF16) {
        auto kern = sa_attention_tc_kernel<__nv_bfloat16, true>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, NTHR, smem, s>>>(a, mq, mc, mh, nwords, nullptr, nullptr, ntc, nth, redo_count, redo_list);
    } else {
        auto kern = sa_attention_tc_kernel<__half, true>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, NTHR, smem, s>>>(a, mq, mc, mh, nwords, nullptr, nullptr, ntc, nth, nullptr, nullptr);
    }
    return check_launch("sa_attention(tcgen05)");
}

// One warp waits on an mbarrier that nothing ever arrives on, with the same
// bounded wait as the pipelines above; the wait runs out after ~limit cycles,
// the kernel raises the device error word (2) and returns normally.
__global__ void wait_timeout_selftest_kernel(long long limit) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const bool ok = mbar_wait_warp(&bar, 0, &abort_flag, limit);
    if (threadIdx.x == 0 && !ok) atomicExch(&g_device_error, 2);
}

int wait_timeout_selftest(long long limit, cudaStream_t s) {
    wait_timeout_selftest_kernel<<<1, 32, 0, s>>>(limit);
    return check_launch("selftest_wait_timeout");
}

int device_error_take(cudaStream_t s, int* out) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_device_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return set_error(MABA_ERR_CUDA, "device_error: %s", cudaGetErrorString(e));
    const int zero = 0;
    if (v != 0) cudaMemcpyToSymbolAsync(g_device_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    *out = v;
    return MABA_OK;
}

}  // namespace maba
