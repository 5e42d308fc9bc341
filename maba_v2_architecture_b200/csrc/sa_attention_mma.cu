// Tensor-core MABA-SA attention for 16-bit inputs (placeholder: the exact
// CUDA-core kernel serves every request until this path is enabled).
#include "sa_attention.cuh"

namespace maba {

bool sa_attention_mma_supported(const SaArgs& a, int dtype) {
    (void)a; (void)dtype;
    return false;
}

int sa_attention_mma(SaArgs& a, int64_t B, int dtype, cudaStream_t s) {
    (void)a; (void)B; (void)dtype; (void)s;
    return set_error(MABA_ERR_UNSUPPORTED, "sa_attention: tensor-core path not built");
}

size_t sa_attention_mma_workspace(int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t H, int64_t DC, int64_t K,
                                  int32_t block) {
    (void)dtype; (void)B; (void)Lq; (void)Lkv; (void)H; (void)DC; (void)K; (void)block;
    return 0;
}

}  // namespace maba
