// Internal interface shared by the DGDA prefill kernels (CUDA-core and tensor-core).
#pragma once
#include "common.cuh"

namespace maba {

struct PrefillArgs {
    const void* q; const void* k; const void* v; const void* alpha; const void* log_alpha;
    const void* b; const void* w; const void* init;
    void* out; void* fin;
    int64_t sq[4], sk[4], sv[4], sa[4], sla[4], sb[4], sw[4], si[4], so[4], sf[4];
    int64_t L;
    int H, dk, dv;
    int nseg;
    int64_t seg_len;      // tokens per segment (multiple of the chunk)
    float* ws_trans;      // [B*H][nseg][64][128]   (R | P) per segment
    float* ws_start;      // [B*H][nseg][64][64]    starting state per segment
    int vec8;             // all inputs: unit stride on d, 16-byte aligned rows (8 x 16-bit loads)
};

// Tensor-core chunk kernels for 16-bit inputs (dk, dv <= 64).
// mode 0: single pass; 1: segment transition pass; 2: segment output pass.
size_t dgda_mma_smem_bytes(int mode);
int dgda_mma_launch(const PrefillArgs& a, dim3 grid, int mode, int dtype, int state_dtype, cudaStream_t s);

}  // namespace maba
