// Tensor-core MABA-SA attention for 16-bit inputs (bf16 / fp16), latent dim 128.
//
// Same math as sa_attention.cu (maba_sparse/layers/sparse_attention.py:79-219,
// 274-275 in the MLA-absorbed latent space), organised for the tensor cores:
//
// * one CTA per tile of 64 consecutive query tokens; rows of the MMA are
//   (head, token) pairs, two heads (128 rows, 8 warps x 16 rows) at a time;
// * every latent key tile (64 rows of c_kv or of the pooled HCA table) is
//   loaded once into shared memory by cp.async (double-buffered) and used as
//   both K (scores, ldmatrix) and V (values, ldmatrix.trans): keys and values
//   are never up-projected;
// * the sparse stream runs over the UNION of the blocks the 64 tokens selected
//   (built once per CTA: a shared-memory bitmap over the blocks, ranks by
//   popcount, and a 64-bit token mask per selected block); a row only sees the
//   blocks its own token selected, so rows of tokens that share blocks share
//   the key tile -- the selection is near-identical across a query block, which
//   turns ~32 gathered blocks per token into ~32 per 64 tokens;
// * S = Q K^T and O += P V are mma.sync.m16n8k16 with fp32 accumulation; one
//   online softmax (running max / sum) per (stream, row); at the end of each
//   stream the normalised output is folded into the gate-weighted result.
#include "sa_attention.cuh"

#include <cuda_pipeline_primitives.h>

namespace maba {
namespace {

constexpr int QT = 64;           // query tokens per CTA
constexpr int KT = 64;           // keys per tile
constexpr int DCX = 128;         // latent dim handled by this kernel
constexpr int LDS = DCX + 8;     // padded shared-memory row (elements): 272 B, conflict-free ldmatrix
constexpr int HPG = 2;           // heads per group (2 x 64 tokens = 128 MMA rows)
constexpr int NWARP = 8;
constexpr int NTHR = NWARP * 32;
constexpr int KMAX = 32;         // selected blocks per token handled here
constexpr int UMAX = QT * KMAX;  // union capacity
constexpr float LOG2E = 1.4426950408889634f;
constexpr int LDR = DCX + 8;     // fp32 result slab row (floats): conflict-free float2 access

struct MmaSmem {
    static size_t bytes(int nwords) {
        size_t b = 0;
        b += (size_t)HPG * QT * LDS * 2;  // Q tile
        b += (size_t)2 * KT * LDS * 2;    // two key tiles
        b += (size_t)UMAX * 8;            // union token masks
        b += (size_t)UMAX * 4;            // union block list
        b += (size_t)nwords * 4 * 2;      // bitmap + word prefix
        b += (size_t)HPG * QT * 3 * 4;    // gate weights per row
        b += (size_t)NTHR * 4 + 64;       // scan scratch
        b += (size_t)HPG * QT * LDR * 4;  // gate-weighted result (fp32), thread-private slots
        return b;
    }
};

// 2^x on the SFU (ex2.approx: relative error ~2^-22, flushes subnormals; exp2(-inf) = 0)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

template <typename T> struct MmaOp;
template <> struct MmaOp<__nv_bfloat16> {
    __device__ __forceinline__ static void run(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};
template <> struct MmaOp<__half> {
    __device__ __forceinline__ static void run(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
        __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};

// 16-byte async copy with zero fill when src_bytes == 0
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

// Loads 64 latent rows [row0, row0+64) of a [rows x 128] table (row stride ld
// elements) into a padded shared tile; rows outside [0, nrows) are zero.
template <typename T>
__device__ __forceinline__ void load_tile(T* dst, const T* base, int64_t row0, int64_t nrows, int64_t ld, int tid) {
#pragma unroll
    for (int c = tid; c < KT * (DCX / 8); c += NTHR) {
        const int r = c >> 4, ch = c & 15;
        const int64_t row = row0 + r;
        const bool ok = row >= 0 && row < nrows;
        const T* src = ok ? base + row * ld + ch * 8 : base;
        cp_async16(dst + r * LDS + ch * 8, src, ok);
    }
}

struct TileInfo {
    int stream;      // 0 local, 1 sparse, 2 hca
    int64_t row0;    // first row in the source table
    int u;           // union slot (sparse)
    bool last;       // last tile of its stream
};

template <typename T>
__global__ void __launch_bounds__(NTHR, 1) sa_attention_mma_kernel(SaArgs a, int nwords) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* Qs = reinterpret_cast<T*>(smem_raw);
    T* Ks = Qs + HPG * QT * LDS;
    unsigned long long* umask = reinterpret_cast<unsigned long long*>(Ks + 2 * KT * LDS);
    int* ulist = reinterpret_cast<int*>(umask + UMAX);
    unsigned* bitmap = reinterpret_cast<unsigned*>(ulist + UMAX);
    int* wpref = reinterpret_cast<int*>(bitmap + nwords);
    float* gsm = reinterpret_cast<float*>(wpref + nwords);
    int* scan = reinterpret_cast<int*>(gsm + HPG * QT * 3);
    float* Rs = reinterpret_cast<float*>(scan + NTHR + 16);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t b = blockIdx.y;
    const int64_t q0 = (int64_t)blockIdx.x * QT;              // first query row of the tile
    const int nt = (int)((a.Lq - q0) < QT ? (a.Lq - q0) : QT); // valid tokens
    const int64_t qpos0 = a.Lkv - a.Lq;                       // absolute position of query row 0
    const int64_t P0 = qpos0 + q0;
    const int64_t Plast = P0 + nt - 1;
    const int64_t nb_kv = (a.Lkv + a.block - 1) / a.block;
    const int K = a.K;
    const T* ckv = static_cast<const T*>(a.ckv) + b * a.sc[0];
    const T* hca = a.hca != nullptr ? static_cast<const T*>(a.hca) + b * a.sh[0] : nullptr;
    const T* qh = static_cast<const T*>(a.qhat);
    const int64_t* tix = a.top_idx + b * a.st[0];

    // ---------------- union of the selected blocks -------------------------
    for (int i = tid; i < nwords; i += NTHR) bitmap[i] = 0u;
    __syncthreads();
    for (int e = tid; e < nt * K; e += NTHR) {
        const int t = e / K, sl = e - (e / K) * K;
        const int64_t n = tix[(q0 + t) * a.st[1] + sl * a.st[2]];
        if (n >= 0 && n < nb_kv && n * a.block <= P0 + t) atomicOr(&bitmap[n >> 5], 1u << (n & 31));
    }
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
            int v[NTHR / 32];
            int tot = 0;
#pragma unroll
            for (int i = 0; i < NTHR / 32; ++i) {
                v[i] = scan[lane * (NTHR / 32) + i];
                tot += v[i];
            }
            int inc = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            int run = inc - tot;
#pragma unroll
            for (int i = 0; i < NTHR / 32; ++i) {
                scan[lane * (NTHR / 32) + i] = run;
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
    for (int e = tid; e < nt * K; e += NTHR) {
        const int t = e / K, sl = e - (e / K) * K;
        const int64_t n = tix[(q0 + t) * a.st[1] + sl * a.st[2]];
        if (n >= 0 && n < nb_kv && n * a.block <= P0 + t) {
            const int wi = (int)(n >> 5);
            const int r = wpref[wi] + __popc(bitmap[wi] & ((1u << (n & 31)) - 1u));
            atomicOr(&umask[r], 1ull << t);
        }
    }

    // ---------------- tile schedule -----------------------------------------
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

    auto tile_info = [&](int i) {
        TileInfo ti;
        if (i < n_local) {
            ti.stream = 0;
            ti.row0 = sink_tile ? (i == 0 ? 0 : ws + (int64_t)(i - 1) * KT) : ws + (int64_t)i * KT;
            ti.u = -1;
            ti.last = i == n_local - 1;
        } else if (i < n_local + U) {
            ti.stream = 1;
            ti.u = i - n_local;
            ti.row0 = (int64_t)ulist[ti.u] * a.block;
            ti.last = i == n_local + U - 1;
        } else {
            ti.stream = 2;
            ti.row0 = (int64_t)(i - n_local - U) * KT;
            ti.u = -1;
            ti.last = i == n_tiles - 1;
        }
        return ti;
    };
    auto issue_tile = [&](int i, int buf) {
        const TileInfo ti = tile_info(i);
        T* dst = Ks + buf * KT * LDS;
        if (ti.stream == 2) {
            load_tile<T>(dst, hca, ti.row0, nhca_max, a.sh[1], tid);
        } else if (ti.stream == 1) {
            // only the block's own rows: a block is `block` rows (block <= KT here)
            const int64_t end = ti.row0 + a.block < a.Lkv ? ti.row0 + a.block : a.Lkv;
            load_tile<T>(dst, ckv, ti.row0, end, a.sc[1], tid);
        } else {
            load_tile<T>(dst, ckv, ti.row0, a.Lkv, a.sc[1], tid);
        }
        cp_async_commit();
    };

    // per-thread rows: warp -> (head within group, 16 tokens); thread rows r and r+8
    const int hl = warp >> 2;
    const int tw = (warp & 3) * 16;
    const int t_r0 = tw + (lane >> 2);
    const int t_r1 = t_r0 + 8;
    const int64_t pos_r0 = P0 + t_r0, pos_r1 = P0 + t_r1;
    const bool warp_has_tokens = tw < nt;
    const int64_t pos_warp_max = P0 + (tw + 15 < nt - 1 ? tw + 15 : nt - 1);
    const int qd = (lane & 3) * 2;  // column pair offset inside an n8 fragment

    for (int h0 = 0; h0 < a.H; h0 += HPG) {
        __syncthreads();
        // Q tile (two heads x 64 tokens) and gate weights of its rows
        for (int c = tid; c < HPG * QT * (DCX / 8); c += NTHR) {
            const int row = c >> 4, ch = c & 15;
            const int h = h0 + row / QT, t = row % QT;
            const bool ok = h < a.H && t < nt;
            const T* src = ok ? qh + b * a.sq[0] + (q0 + t) * a.sq[1] + h * a.sq[2] + ch * 8 : qh;
            cp_async16(Qs + row * LDS + ch * 8, src, ok);
        }
        cp_async_commit();
        for (int row = tid; row < HPG * QT; row += NTHR) {
            const int h = h0 + row / QT, t = row % QT;
            float g0 = 0.f, g1 = 0.f, g2 = 0.f;
            if (h < a.H && t < nt) {
                const T* gp = static_cast<const T*>(a.gate);
                const T* gr = a.gate4d ? gp + b * a.sg[0] + h * a.sg[1] + (q0 + t) * a.sg[2]
                                       : gp + b * a.sg[0] + (q0 + t) * a.sg[1];
                const int64_t gs = a.gate4d ? a.sg[3] : a.sg[2];
                g0 = Cvt<T>::to_f(gr[0]);
                g1 = Cvt<T>::to_f(gr[gs]);
                g2 = Cvt<T>::to_f(gr[2 * gs]);
                const float m = fmaxf(g0, fmaxf(g1, g2));
                const float e0 = expf(g0 - m), e1 = expf(g1 - m), e2 = expf(g2 - m);
                const float inv = 1.f / (e0 + e1 + e2);
                g0 = e0 * inv;
                g1 = e1 * inv;
                g2 = e2 * inv;
            }
            gsm[row * 3 + 0] = g0;
            gsm[row * 3 + 1] = g1;
            gsm[row * 3 + 2] = g2;
        }
        const int h_my = h0 + hl;
        const bool warp_active = warp_has_tokens && h_my < a.H;

        // this thread's result slots: rows (hl,t_r0), (hl,t_r1), dims n*8+qd+{0,1}
        float* R0 = Rs + (hl * QT + t_r0) * LDR + qd;
        float* R1 = Rs + (hl * QT + t_r1) * LDR + qd;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
            *reinterpret_cast<float2*>(R0 + n * 8) = make_float2(0.f, 0.f);
            *reinterpret_cast<float2*>(R1 + n * 8) = make_float2(0.f, 0.f);
        }
        float oacc[16][4];
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

        if (n_tiles > 0) issue_tile(0, 0);
        for (int i = 0; i < n_tiles; ++i) {
            cp_async_wait_all();
            __syncthreads();
            if (i + 1 < n_tiles) issue_tile(i + 1, (i + 1) & 1);
            const TileInfo ti = tile_info(i);
            const bool first = (i == 0) || (tile_info(i - 1).stream != ti.stream);
            if (first) {
#pragma unroll
                for (int n = 0; n < 16; ++n)
#pragma unroll
                    for (int e = 0; e < 4; ++e) oacc[n][e] = 0.f;
                m0 = m1 = -INFINITY;
                l0 = l1 = 0.f;
            }
            // does any row of this warp see a key of this tile?
            bool work = warp_active;
            unsigned long long tmask = 0ull;
            if (ti.stream == 1) {
                tmask = umask[ti.u];
                work = work && (((tmask >> tw) & 0xFFFFull) != 0ull);
            } else if (ti.stream == 2) {
                work = work && ((ti.row0 + 1) * a.hca_r - 1 <= pos_warp_max);
            } else {
                work = work && (ti.row0 <= pos_warp_max);
            }
            if (work) {
                const T* kt = Ks + (i & 1) * KT * LDS;
                float s[8][4];
#pragma unroll
                for (int j = 0; j < 8; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
                const T* qbase = Qs + (hl * QT + tw) * LDS;
#pragma unroll
                for (int ks = 0; ks < DCX / 16; ++ks) {
                    uint32_t af[4];
                    {
                        const int mi = lane >> 3;
                        const int r = (mi & 1) * 8 + (lane & 7);
                        const int c = ks * 16 + (mi >> 1) * 8;
                        ldsm_x4(smem_u32(qbase + r * LDS + c), af[0], af[1], af[2], af[3]);
                    }
#pragma unroll
                    for (int jp = 0; jp < 4; ++jp) {
                        uint32_t b0, b1, b2, b3;
                        const int mi = lane >> 3;
                        const int key = jp * 16 + (mi >> 1) * 8 + (lane & 7);
                        const int c = ks * 16 + (mi & 1) * 8;
                        ldsm_x4(smem_u32(kt + key * LDS + c), b0, b1, b2, b3);
                        MmaOp<T>::run(s[2 * jp], af, b0, b1);
                        MmaOp<T>::run(s[2 * jp + 1], af, b2, b3);
                    }
                }
                // masks (per stream) and scaling to log2 units.  Each of the thread's two
                // rows is classified once per tile: every key of the tile valid, none valid,
                // or mixed (only then the per-key test runs, in 32-bit arithmetic).
                const int kb = (int)ti.row0;
                int cls[2];
#pragma unroll
                for (int rr = 0; rr < 2; ++rr) {
                    const int t = rr == 0 ? t_r0 : t_r1;
                    const int pos = (int)(rr == 0 ? pos_r0 : pos_r1);
                    const bool sel = ti.stream != 1 || ((tmask >> t) & 1ull);
                    int c;  // 0 none, 1 all, 2 mixed
                    if (t >= nt || !sel) {
                        c = 0;
                    } else if (ti.stream == 0) {
                        const bool all = kb + KT - 1 <= pos && kb + KT - 1 < a.Lkv && pos - kb < a.window;
                        const bool none = kb > pos || (pos - (kb + KT - 1) >= a.window && kb >= a.n_sinks);
                        c = all ? 1 : (none ? 0 : 2);
                    } else if (ti.stream == 1) {
                        const bool all = kb + KT - 1 <= pos && kb + KT - 1 < a.Lkv && a.block >= KT;
                        c = all ? 1 : (kb > pos ? 0 : 2);
                    } else {
                        const bool all = (kb + KT) * a.hca_r - 1 <= pos && kb + KT - 1 < a.NC;
                        c = all ? 1 : ((kb + 1) * a.hca_r - 1 > pos ? 0 : 2);
                    }
                    cls[rr] = c;
                }
                float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int rr = e >> 1;
                        bool ok = cls[rr] == 1;
                        if (cls[rr] == 2) {
                            const int key = kb + j * 8 + qd + (e & 1);
                            const int pos = (int)(rr == 0 ? pos_r0 : pos_r1);
                            if (ti.stream == 0) {
                                ok = key < a.Lkv && key <= pos && ((pos - key) < a.window || key < a.n_sinks);
                            } else if (ti.stream == 1) {
                                ok = key < a.Lkv && key <= pos && (key - kb) < a.block;
                            } else {
                                ok = key < a.NC && (key + 1) * a.hca_r - 1 <= pos;
                            }
                        }
                        const float v = ok ? s[j][e] * LOG2E : -INFINITY;
                        s[j][e] = v;
                        if (e < 2) mx0 = fmaxf(mx0, v);
                        else mx1 = fmaxf(mx1, v);
                    }
                }
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
                const float mu0 = mn0 == -INFINITY ? 0.f : mn0;
                const float mu1 = mn1 == -INFINITY ? 0.f : mn1;
                const float c0 = ex2(m0 - mu0), c1 = ex2(m1 - mu1);
                m0 = mn0;
                m1 = mn1;
                float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    s[j][0] = ex2(s[j][0] - mu0);
                    s[j][1] = ex2(s[j][1] - mu0);
                    s[j][2] = ex2(s[j][2] - mu1);
                    s[j][3] = ex2(s[j][3] - mu1);
                    ps0 += s[j][0] + s[j][1];
                    ps1 += s[j][2] + s[j][3];
                }
                l0 = l0 * c0 + ps0;
                l1 = l1 * c1 + ps1;
                if (c0 != 1.f || c1 != 1.f) {
#pragma unroll
                    for (int n = 0; n < 16; ++n) {
                        oacc[n][0] *= c0;
                        oacc[n][1] *= c0;
                        oacc[n][2] *= c1;
                        oacc[n][3] *= c1;
                    }
                }
                // O += P V  (V = the same latent tile, read transposed)
#pragma unroll
                for (int kk = 0; kk < KT / 16; ++kk) {
                    uint32_t pa[4];
                    pa[0] = MmaOp<T>::pack(s[2 * kk][0], s[2 * kk][1]);
                    pa[1] = MmaOp<T>::pack(s[2 * kk][2], s[2 * kk][3]);
                    pa[2] = MmaOp<T>::pack(s[2 * kk + 1][0], s[2 * kk + 1][1]);
                    pa[3] = MmaOp<T>::pack(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
                    for (int dp = 0; dp < DCX / 16; ++dp) {
                        uint32_t b0, b1, b2, b3;
                        const int mi = lane >> 3;
                        const int key = kk * 16 + (mi & 1) * 8 + (lane & 7);
                        const int c = dp * 16 + (mi >> 1) * 8;
                        ldsm_x4_t(smem_u32(kt + key * LDS + c), b0, b1, b2, b3);
                        MmaOp<T>::run(oacc[2 * dp], pa, b0, b1);
                        MmaOp<T>::run(oacc[2 * dp + 1], pa, b2, b3);
                    }
                }
            }
            if (ti.last) {
                // fold the finished stream into the gate-weighted result
                float L0 = l0, L1 = l1;
                L0 += __shfl_xor_sync(0xffffffffu, L0, 1);
                L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
                L1 += __shfl_xor_sync(0xffffffffu, L1, 1);
                L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
                const int row0 = hl * QT + t_r0, row1 = hl * QT + t_r1;
                const float f0 = L0 > 0.f ? gsm[row0 * 3 + ti.stream] / L0 : 0.f;
                const float f1 = L1 > 0.f ? gsm[row1 * 3 + ti.stream] / L1 : 0.f;
#pragma unroll
                for (int n = 0; n < 16; ++n) {
                    float2 x0 = *reinterpret_cast<float2*>(R0 + n * 8);
                    float2 x1 = *reinterpret_cast<float2*>(R1 + n * 8);
                    x0.x += f0 * oacc[n][0];
                    x0.y += f0 * oacc[n][1];
                    x1.x += f1 * oacc[n][2];
                    x1.y += f1 * oacc[n][3];
                    *reinterpret_cast<float2*>(R0 + n * 8) = x0;
                    *reinterpret_cast<float2*>(R1 + n * 8) = x1;
                }
            }
        }
        cp_async_wait_all();
        // HCA early path: rows with pos < r-1 take the mean of the latent prefix
        if (warp_active && P0 < a.hca_r - 1) {
            const int row0 = hl * QT + t_r0, row1 = hl * QT + t_r1;
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int64_t pos = rr == 0 ? pos_r0 : pos_r1;
                const int t = rr == 0 ? t_r0 : t_r1;
                if (t >= nt || pos >= a.hca_r - 1) continue;
                const float g2 = gsm[(rr == 0 ? row0 : row1) * 3 + 2] / float(pos + 1);
#pragma unroll
                for (int n = 0; n < 16; ++n) {
                    const int d = n * 8 + qd;
                    float s0 = 0.f, s1 = 0.f;
                    for (int64_t j = 0; j <= pos; ++j) {
                        s0 += Cvt<T>::to_f(ckv[j * a.sc[1] + d * a.sc[2]]);
                        s1 += Cvt<T>::to_f(ckv[j * a.sc[1] + (d + 1) * a.sc[2]]);
                    }
                    float* R = (rr == 0 ? R0 : R1) + n * 8;
                    R[0] += g2 * s0;
                    R[1] += g2 * s1;
                }
            }
        }
        // write the latent result of the valid rows
        if (warp_active) {
            T* out = static_cast<T*>(a.out);
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int t = rr == 0 ? t_r0 : t_r1;
                if (t >= nt) continue;
                T* orow = out + b * a.so[0] + (q0 + t) * a.so[1] + (int64_t)h_my * a.so[2];
#pragma unroll
                for (int n = 0; n < 16; ++n) {
                    const int d = n * 8 + qd;
                    const float2 x = *reinterpret_cast<const float2*>((rr == 0 ? R0 : R1) + n * 8);
                    orow[d * a.so[3]] = Cvt<T>::from_f(x.x);
                    orow[(d + 1) * a.so[3]] = Cvt<T>::from_f(x.y);
                }
            }
        }
    }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool sa_attention_mma_supported(const SaArgs& a, int dtype) {
    if (dtype != MABA_BF16 && dtype != MABA_F16) return false;
    if (a.DC != DCX || a.K > KMAX || a.K <= 0 || a.block > KT || a.block <= 0) return false;
    if (a.Lq < 16) return false;  // single-token decode: one warp per head is cheaper than 128-row tiles
    // 16-byte rows for cp.async / ldmatrix
    if (a.sq[3] != 1 || a.sc[2] != 1 || (a.NC > 0 && a.sh[2] != 1)) return false;
    if ((a.sq[2] % 8) || (a.sq[1] % 8) || (a.sc[1] % 8) || (a.NC > 0 && a.sh[1] % 8)) return false;
    if (!aligned16(a.qhat) || !aligned16(a.ckv) || (a.NC > 0 && !aligned16(a.hca))) return false;
    const int64_t nb_kv = (a.Lkv + a.block - 1) / a.block;
    if (nb_kv > 65536 * 32) return false;
    return true;
}

int sa_attention_mma(SaArgs& a, int64_t B, int dtype, cudaStream_t s) {
    const int64_t nb_kv = (a.Lkv + a.block - 1) / a.block;
    const int nwords = (int)((nb_kv + 31) / 32) + 1;
    const size_t smem = MmaSmem::bytes(nwords);
    if (smem > 227 * 1024) return sa_attention_simt(a, B, dtype, s);
    dim3 grid((unsigned)ceil_div(a.Lq, QT), (unsigned)B);
    if (dtype == MABA_BF16) {
        auto kern = sa_attention_mma_kernel<__nv_bfloat16>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, NTHR, smem, s>>>(a, nwords);
    } else {
        auto kern = sa_attention_mma_kernel<__half>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        kern<<<grid, NTHR, smem, s>>>(a, nwords);
    }
    return check_launch("sa_attention(mma)");
}

size_t sa_attention_mma_workspace(int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t H, int64_t DC, int64_t K,
                                  int32_t block) {
    (void)dtype; (void)B; (void)Lq; (void)Lkv; (void)H; (void)DC; (void)K; (void)block;
    return 0;
}

}  // namespace maba
