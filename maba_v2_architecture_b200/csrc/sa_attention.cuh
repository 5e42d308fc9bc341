// Internal interface shared by the MABA-SA attention kernels.
#pragma once
#include "common.cuh"

namespace maba {

struct SaArgs {
    const void* qhat;        // [B,Lq,H,DC]
    const void* ckv;         // [B,Lkv,DC]
    const void* hca;         // [B,NC,DC]  (may be null when NC == 0)
    const int64_t* top_idx;  // [B,Lq,K]
    const void* gate;        // [B,Lq,3] or [B,H,Lq,3]
    void* out;               // [B,Lq,H,DC]
    int64_t sq[4], sc[3], sh[3], st[3], sg[4], so[4];
    int64_t Lq, Lkv, NC;
    int H, DC, K;
    int window, n_sinks, block, hca_r, gate4d;
    void* workspace;
    size_t workspace_bytes;
    const int64_t* pos_dev;  // decode at a device-held position (c_kv / hca are capacity-sized buffers)
};

int sa_attention_simt(SaArgs& a, int64_t B, int dtype, cudaStream_t s);
int sa_attention_mma(SaArgs& a, int64_t B, int dtype, cudaStream_t s);
int sa_attention_tc(SaArgs& a, int64_t B, int dtype, cudaStream_t s);
bool sa_attention_tc_supported(const SaArgs& a, int dtype);
size_t sa_attention_tc_workspace(int64_t B, int64_t Lq, int64_t Lkv, int64_t NC);
int device_error_take(cudaStream_t s, int* out);
int wait_timeout_selftest(long long limit, cudaStream_t s);
bool sa_attention_mma_supported(const SaArgs& a, int dtype);
size_t sa_attention_mma_workspace(int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t H, int64_t DC, int64_t K,
                                  int32_t block);

bool sa_attention_decode_supported(const SaArgs& a);
size_t sa_attention_decode_workspace(int64_t B, int64_t Lq, int64_t Lkv, int64_t H, int64_t DC, int64_t K,
                                     int32_t block, int32_t window, int32_t n_sinks, int32_t hca_r);
int sa_attention_decode(SaArgs& a, int64_t B, int dtype, cudaStream_t s);
size_t sa_attention_decode_at_workspace(int64_t B, int64_t Lcap, int64_t NCcap, int64_t H, int64_t DC, int64_t K,
                                        int32_t block, int32_t window, int32_t n_sinks, int32_t hca_r);

inline size_t sa_attention_workspace_bytes(int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t H, int64_t DC,
                                           int64_t K, int32_t block, int32_t window, int32_t n_sinks,
                                           int32_t hca_r) {
    size_t a = sa_attention_mma_workspace(dtype, B, Lq, Lkv, H, DC, K, block);
    size_t b = sa_attention_decode_workspace(B, Lq, Lkv, H, DC, K, block, window, n_sinks, hca_r);
    // key-tile norms of the tcgen05 kernel (pooled entries: at most ceil(Lkv / r))
    size_t c = sa_attention_tc_workspace(B, Lq, Lkv, hca_r > 0 ? (Lkv + hca_r - 1) / hca_r : 0);
    if (b > a) a = b;
    return a > c ? a : c;
}

// Single-token queries take the split-K decode kernels when the caller gave
// the workspace they need; 16-bit prefill tiles take the tcgen05 kernel (block
// 64, K <= 32, TMA-compatible strides), else the mma.sync kernel; everything
// else the exact CUDA-core kernel.
inline int sa_attention_dispatch(SaArgs& a, int64_t B, int dtype, cudaStream_t s) {
    if (dtype != MABA_F64 && sa_attention_decode_supported(a) &&
        a.workspace_bytes >= sa_attention_decode_workspace(B, a.Lq, a.Lkv, a.H, a.DC, a.K, a.block, a.window,
                                                           a.n_sinks, a.hca_r))
        return sa_attention_decode(a, B, dtype, s);
    if (sa_attention_tc_supported(a, dtype)) return sa_attention_tc(a, B, dtype, s);
    if (sa_attention_mma_supported(a, dtype)) return sa_attention_mma(a, B, dtype, s);
    return sa_attention_simt(a, B, dtype, s);
}

}  // namespace maba
