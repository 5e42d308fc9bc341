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
    // chunk-parallel path (16-bit inputs): one record per (b*h, chunk)
    unsigned char* ws_chunk;  // [B*H][nch] records of CHUNK_REC bytes
    int64_t nch;              // chunks per (b, h)
    // preparation pass: a CTA prefetches into L2 the inputs of the CTA this many
    // places after it in launch order (one wave ahead; 0: no prefetch)
    int64_t pf_ahead;
};

// Chunk record of the chunk-parallel path: 16-bit 64x64 tiles and the chunk's
// total decay.  With T = (I + L)^{-1}, W = T (b k e^G), U = T (w v),
// KT = k e^{G_end - G}, QT = q e^G and A = tril(q . decay . k):
//   M  = KT^T W    N  = KT^T U      (state update: S' = e^{G_end} S + N - M S)
//   QW = QT - A W  AU = A U         (output: o = QW S + AU)
//   dend = e^{G_end}  (fp32 [64])
constexpr size_t CH_TILE = 64 * 64 * 2;
constexpr size_t CH_M = 0, CH_N = CH_TILE, CH_QW = 2 * CH_TILE, CH_AU = 3 * CH_TILE, CH_DEND = 4 * CH_TILE;
constexpr size_t CHUNK_REC = 4 * CH_TILE + 64 * 4;

// Tensor-core chunk kernels for 16-bit inputs (dk, dv <= 64).
// mode 0: single pass; 1: segment transition pass; 2: segment output pass.
size_t dgda_mma_smem_bytes(int mode);
int dgda_mma_launch(const PrefillArgs& a, dim3 grid, int mode, int dtype, int state_dtype, cudaStream_t s);

// Chunk-parallel path (16-bit): the state scan over chunk records, which writes
// the outputs in modes 0 and 2 (mode 0: one segment from the initial state;
// 1: segment transitions; 2: segments from their start states).
int dgda_scan_launch(const PrefillArgs& a, dim3 grid, int mode, int dtype, int state_dtype, cudaStream_t s);
int dgda_prep_launch(const PrefillArgs& a, int64_t BH, int dtype, cudaStream_t s);

}  // namespace maba
