// Chunk-parallel DGDA prefill for 16-bit inputs: the state scan and the output
// pass over the chunk records written by the preparation pass (mode 3 of
// dgda_prefill_mma.cu).
//
// Same recurrence as dgda_prefill_mma.cu (reference maba_sparse/kernels/
// common.py:256-265, chunked form cpu_dgda.py:101-146) with the per-chunk WY/UT
// quantities precomputed in parallel over all chunks:
//   u  = U - W S                 (U = T w v, W = T (b k e^G))
//   o  = (q e^G) S + A u
//   S' = e^{G_end} S + (k e^{G_end - G})^T u
// so the sequential part per chunk is two 64x64x64 products (scan), and the
// output is three products per chunk, independent across chunks (out pass).
//
// Scan (grid = (B*H, segments), 8 warps): the chunk records of the next chunk
// are fetched by cp.async while the current chunk's products run; the state is
// held in fp32 accumulator registers (a 16-bit copy in shared memory feeds the
// MMAs, and is what the output pass reads as the chunk's start state).  Modes:
// 0 -- one segment from the initial state; 1 -- the affine transition [R | P]
// of each segment (the augmented state starts at [0 | I] and u = [U | 0] - W X);
// 2 -- each segment from its start state (folded from the transitions).
#include "dgda_prefill.cuh"
#include "mma_util.cuh"

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

template <int NCOL>
struct ScanSmem {
    static constexpr int LN = NCOL + 8;
    static constexpr size_t TILE = (size_t)C * LB * 2;
    static constexpr size_t REC = 3 * TILE + 64 * 4;               // W, U, KT, dend
    static constexpr size_t SB = 2 * REC;                          // [D][LN] 16-bit state
    static constexpr size_t UB = SB + (size_t)D * LN * 2;          // [C][LN] 16-bit u
    static constexpr size_t TOTAL = UB + (size_t)C * LN * 2;
};

template <typename T, typename TS, int MODE>
__global__ void __launch_bounds__(NTH, 2) dgda_scan_kernel(PrefillArgs a) {
    constexpr int NCOL = MODE == 1 ? 2 * D : D;
    using SM = ScanSmem<NCOL>;
    constexpr int LN = SM::LN;
    constexpr int NTW = NCOL / 16;
    extern __shared__ __align__(16) unsigned char sm[];
    T* SB = reinterpret_cast<T*>(sm + SM::SB);
    T* UB = reinterpret_cast<T*>(sm + SM::UB);

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

    auto fetch = [&](int64_t c, int buf) {
        unsigned char* base = sm + buf * SM::REC;
        const unsigned char* r = recs + (size_t)c * CHUNK_REC;
        fetch_tile<T>(reinterpret_cast<T*>(base), r + CH_W, tid);
        fetch_tile<T>(reinterpret_cast<T*>(base + SM::TILE), r + CH_U, tid);
        fetch_tile<T>(reinterpret_cast<T*>(base + 2 * SM::TILE), r + CH_KT, tid);
        if (tid < 16) cp_async16(base + 3 * SM::TILE + tid * 16, r + CH_DEND + tid * 16);
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
        __syncthreads();  // this chunk's record and the state copy are visible
        if (c + 1 < c_end) fetch(c + 1, buf ^ 1);
        const T* Wt = reinterpret_cast<const T*>(sm + buf * SM::REC);
        const T* Ut = reinterpret_cast<const T*>(sm + buf * SM::REC + SM::TILE);
        const T* KTt = reinterpret_cast<const T*>(sm + buf * SM::REC + 2 * SM::TILE);
        const float* dend = reinterpret_cast<const float*>(sm + buf * SM::REC + 3 * SM::TILE);
        if (MODE != 1) {
            // the chunk's start state, for the output pass
            unsigned char* dst = const_cast<unsigned char*>(recs) + (size_t)c * CHUNK_REC + CH_S;
            for (int e = tid; e < 64 * 8; e += NTH) {
                const int r = e >> 3, c8 = (e & 7) * 8;
                *reinterpret_cast<uint4*>(dst + (size_t)(r * 64 + c8) * 2) =
                    *reinterpret_cast<const uint4*>(SB + r * LN + c8);
            }
        }
        // u = [U | 0] - W S
        float racc[NTW][4] = {};
        warp_mma<T, false, true, NTW>(racc, Wt + wr * LB, LB, SB + wc, LN, D, lane);
#pragma unroll
        for (int n = 0; n < NTW; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = wr + fr + (e >> 1) * 8;
                const int col = wc + n * 8 + fc + (e & 1);
                const float u = col < D ? Cvt<T>::to_f(Ut[r * LB + col]) : 0.f;
                racc[n][e] = u - racc[n][e];
            }
        store_acc16<T, NTW>(UB + wr * LN + wc, LN, racc, lane);
        __syncthreads();
        // S = e^{G_end} S + KT^T u
#pragma unroll
        for (int n = 0; n < NTW; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) sacc[n][e] *= dend[wr + fr + (e >> 1) * 8];
        warp_mma<T, true, true, NTW>(sacc, KTt + wr, LB, UB + wc, LN, C, lane);
        store_acc16<T, NTW>(SB + wr * LN + wc, LN, sacc, lane);
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

// Output pass: o = QT S + A (U - W S) per chunk, independent across chunks.
struct OutSmem {
    static constexpr size_t TILE = (size_t)C * LB * 2;
    static constexpr size_t QT = 0, S = TILE, W = 2 * TILE, U = 3 * TILE, A = 4 * TILE, UB = 5 * TILE;
    static constexpr size_t TOTAL = 6 * TILE;
};

template <typename T>
__global__ void __launch_bounds__(NTH) dgda_out_kernel(PrefillArgs a) {
    extern __shared__ __align__(16) unsigned char sm[];
    T* QTt = reinterpret_cast<T*>(sm + OutSmem::QT);
    T* St = reinterpret_cast<T*>(sm + OutSmem::S);
    T* Wt = reinterpret_cast<T*>(sm + OutSmem::W);
    T* Ut = reinterpret_cast<T*>(sm + OutSmem::U);
    T* At = reinterpret_cast<T*>(sm + OutSmem::A);
    T* UB = reinterpret_cast<T*>(sm + OutSmem::UB);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t ci = blockIdx.x;  // chunk over (b*h, chunk)
    const int bh = (int)(ci / a.nch);
    const int64_t c = ci - (int64_t)bh * a.nch;
    const int64_t bi = bh / a.H, hi = bh % a.H;
    constexpr int NTW = D / 16;
    const int wr = (warp & 3) * 16, wc = (warp >> 2) * (D / 2);
    const int fr = lane >> 2, fc = (lane & 3) * 2;
    const unsigned char* rec = a.ws_chunk + (size_t)ci * CHUNK_REC;
    fetch_tile<T>(QTt, rec + CH_QT, tid);
    fetch_tile<T>(St, rec + CH_S, tid);
    fetch_tile<T>(Wt, rec + CH_W, tid);
    fetch_tile<T>(Ut, rec + CH_U, tid);
    fetch_tile<T>(At, rec + CH_A, tid);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
    float qacc[NTW][4] = {};
    float racc[NTW][4] = {};
    warp_mma<T, false, true, NTW>(qacc, QTt + wr * LB, LB, St + wc, LB, D, lane);
    warp_mma<T, false, true, NTW>(racc, Wt + wr * LB, LB, St + wc, LB, D, lane);
#pragma unroll
    for (int n = 0; n < NTW; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = wr + fr + (e >> 1) * 8;
            const int col = wc + n * 8 + fc + (e & 1);
            racc[n][e] = Cvt<T>::to_f(Ut[r * LB + col]) - racc[n][e];
        }
    store_acc16<T, NTW>(UB + wr * LB + wc, LB, racc, lane);
    __syncthreads();
    warp_mma<T, false, true, NTW>(qacc, At + wr * LB, LB, UB + wc, LB, C, lane);
    T* o = static_cast<T*>(a.out);
    const int64_t t0 = c * C;
#pragma unroll
    for (int n = 0; n < NTW; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int r = wr + fr + (e >> 1) * 8;
            const int col = wc + n * 8 + fc + (e & 1);
            const int64_t t = t0 + r;
            if (t < a.L && col < a.dv)
                o[bi * a.so[0] + hi * a.so[1] + t * a.so[2] + (int64_t)col * a.so[3]] = to16<T>(qacc[n][e]);
        }
}

template <typename K>
int smem_attr(K kern, size_t bytes) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return set_error(MABA_ERR_CUDA, "dgda_prefill(chunked): %s", cudaGetErrorString(e));
    return MABA_OK;
}

template <typename T, typename TS, int MODE>
int scan_one(const PrefillArgs& a, dim3 grid, cudaStream_t s) {
    constexpr size_t smem = ScanSmem<MODE == 1 ? 2 * D : D>::TOTAL;
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
int out_one(const PrefillArgs& a, int64_t BH, cudaStream_t s) {
    auto kern = dgda_out_kernel<T>;
    MABA_TRY(smem_attr(kern, OutSmem::TOTAL));
    kern<<<(unsigned)(BH * a.nch), NTH, OutSmem::TOTAL, s>>>(a);
    return check_launch("dgda_prefill(out)");
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

int dgda_out_launch(const PrefillArgs& a, int64_t BH, int dtype, cudaStream_t s) {
    if (dtype == MABA_BF16) return out_one<__nv_bfloat16>(a, BH, s);
    if (dtype == MABA_F16) return out_one<__half>(a, BH, s);
    return set_error(MABA_ERR_DTYPE, "dgda_prefill(chunked): 16-bit inputs only");
}

}  // namespace maba
