// Warp-level 16-bit tensor-core helpers (mma.sync.m16n8k16, fp32 accumulate)
// with ldmatrix-fed operands from padded shared-memory tiles.
//
// Fragment conventions (PTX ISA, m16n8k16): A is 16 x 16 (row = lane/4 and
// lane/4 + 8, columns 2*(lane%4)+{0,1} and +8), B is 16 x 8 (k = 2*(lane%4)+{0,1}
// and +8, n = lane/4), C/D is 16 x 8 (rows lane/4, lane/4+8; columns 2*(lane%4)+{0,1}).
#pragma once
#include "common.cuh"

namespace maba {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_addr(p)));
}
__device__ __forceinline__ void ldsm4t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_addr(p)));
}

template <typename T> struct Mma16;
template <> struct Mma16<__nv_bfloat16> {
    __device__ __forceinline__ static void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct Mma16<__half> {
    __device__ __forceinline__ static void mma(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};\n"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

// acc[NT][4] += A[16 x K] * B[K x 8*NT]   (NT even, K multiple of 16)
//  A: element (m,k) at A[m*lda + k]            (ATRANS = false)
//                   or A[k*lda + m]            (ATRANS = true: A stored k-major)
//  B: element (k,n) at B[k*ldb + n]            (BKN = true: B stored k-major)
//                   or B[n*ldb + k]            (BKN = false)
// Pointers address element (0,0) of the 16-row / 8*NT-column window.
template <typename T, bool ATRANS, bool BKN, int NT>
__device__ __forceinline__ void warp_mma(float (&acc)[NT][4], const T* A, int lda, const T* B, int ldb, int K,
                                         int lane) {
    const int mi = lane >> 3, rr = lane & 7;
    for (int k0 = 0; k0 < K; k0 += 16) {
        uint32_t a[4];
        if (!ATRANS) ldsm4(A + ((mi & 1) * 8 + rr) * lda + k0 + (mi >> 1) * 8, a[0], a[1], a[2], a[3]);
        else ldsm4t(A + (k0 + (mi >> 1) * 8 + rr) * lda + (mi & 1) * 8, a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int np = 0; np < NT; np += 2) {
            uint32_t b0, b1, b2, b3;
            if (BKN) ldsm4t(B + (k0 + (mi & 1) * 8 + rr) * ldb + np * 8 + (mi >> 1) * 8, b0, b1, b2, b3);
            else ldsm4(B + (np * 8 + (mi >> 1) * 8 + rr) * ldb + k0 + (mi & 1) * 8, b0, b1, b2, b3);
            Mma16<T>::mma(acc[np], a, b0, b1);
            Mma16<T>::mma(acc[np + 1], a, b2, b3);
        }
    }
}

template <typename T> __device__ __forceinline__ T to16(float x);
template <> __device__ __forceinline__ __nv_bfloat16 to16<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half to16<__half>(float x) { return __float2half_rn(x); }

// store a 16 x 8*NT fp32 accumulator tile as 16-bit rows (row stride ld)
template <typename T, int NT>
__device__ __forceinline__ void store_acc16(T* dst, int ld, const float (&acc)[NT][4], int lane) {
    const int r = lane >> 2, c = (lane & 3) * 2;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        dst[r * ld + n * 8 + c] = to16<T>(acc[n][0]);
        dst[r * ld + n * 8 + c + 1] = to16<T>(acc[n][1]);
        dst[(r + 8) * ld + n * 8 + c] = to16<T>(acc[n][2]);
        dst[(r + 8) * ld + n * 8 + c + 1] = to16<T>(acc[n][3]);
    }
}

}  // namespace maba
