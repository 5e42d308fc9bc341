// Stream superposition: o = g0*o_local + g1*o_sparse + g2*o_hca with
// g = softmax(gate_logits) over the last axis (or gate weights as given).
// Follows maba_sparse/kernels/common.py:406-438 and cpu_indexer.py:116-150
// (softmax in fp32).  Gate is [B,L,3] (shared by heads) or [B,H,L,3].
// One warp per (b,h,l) row: the gate is computed once per row, lanes stride
// the feature axis.  The fused MABA-SA kernel applies the same combination in
// its epilogue; this op serves direct registry callers.
#include "common.cuh"

namespace maba {
namespace {

struct SupArgs {
    const void* ol; const void* os; const void* oh; const void* gate; void* out;
    int64_t s_ol[4], s_os[4], s_oh[4], s_out[4], s_g[4];
    int64_t B, H, L, D;
    int gate4d, logits;
};

template <typename T, typename ACC>
__global__ void superposition_kernel(SupArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t warps_total = (int64_t)gridDim.x * (blockDim.x / 32);
    const int64_t rows = a.B * a.H * a.L;
    const T* ol = static_cast<const T*>(a.ol);
    const T* os = static_cast<const T*>(a.os);
    const T* oh = static_cast<const T*>(a.oh);
    const T* g = static_cast<const T*>(a.gate);
    T* out = static_cast<T*>(a.out);
    for (int64_t r = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); r < rows; r += warps_total) {
        const int64_t l = r % a.L;
        const int64_t h = (r / a.L) % a.H;
        const int64_t b = r / (a.L * a.H);
        const T* gp = a.gate4d ? g + b * a.s_g[0] + h * a.s_g[1] + l * a.s_g[2]
                               : g + b * a.s_g[0] + l * a.s_g[1];
        const int64_t gs = a.gate4d ? a.s_g[3] : a.s_g[2];
        ACC g0 = load_as<ACC>(gp), g1 = load_as<ACC>(gp + gs), g2 = load_as<ACC>(gp + 2 * gs);
        if (a.logits) {
            ACC m = g0 > g1 ? g0 : g1;
            m = m > g2 ? m : g2;
            ACC e0 = exp_acc<ACC>(g0 - m), e1 = exp_acc<ACC>(g1 - m), e2 = exp_acc<ACC>(g2 - m);
            ACC inv = ACC(1) / (e0 + e1 + e2);
            g0 = e0 * inv;
            g1 = e1 * inv;
            g2 = e2 * inv;
        }
        const int64_t bl = b * a.s_ol[0] + h * a.s_ol[1] + l * a.s_ol[2];
        const int64_t bs = b * a.s_os[0] + h * a.s_os[1] + l * a.s_os[2];
        const int64_t bh = b * a.s_oh[0] + h * a.s_oh[1] + l * a.s_oh[2];
        const int64_t bo = b * a.s_out[0] + h * a.s_out[1] + l * a.s_out[2];
        for (int64_t d = lane; d < a.D; d += 32) {
            ACC x = g0 * load_as<ACC>(ol + bl + d * a.s_ol[3]) + g1 * load_as<ACC>(os + bs + d * a.s_os[3]) +
                    g2 * load_as<ACC>(oh + bh + d * a.s_oh[3]);
            store_from<T, ACC>(out + bo + d * a.s_out[3], x);
        }
    }
}

}  // namespace
}  // namespace maba

using namespace maba;

extern "C" int maba_stream_superposition(const maba_tensor* o_local, const maba_tensor* o_sparse,
                                         const maba_tensor* o_hca, const maba_tensor* gate,
                                         int32_t gate_is_logits, const maba_tensor* out, void* stream) {
    if (!present(o_local) || o_local->ndim != 4)
        return set_error(MABA_ERR_INVALID, "stream_superposition: o_local must be [B,H,L,D]");
    const int64_t B = o_local->shape[0], H = o_local->shape[1], L = o_local->shape[2], D = o_local->shape[3];
    const int64_t s4[4] = {B, H, L, D};
    MABA_TRY(expect_shape(o_sparse, "stream_superposition: o_sparse", 4, s4));
    MABA_TRY(expect_shape(o_hca, "stream_superposition: o_hca", 4, s4));
    MABA_TRY(expect_shape(out, "stream_superposition: out", 4, s4));
    const int dt = o_local->dtype;
    MABA_TRY(expect_dtype(o_sparse, "stream_superposition: o_sparse", dt));
    MABA_TRY(expect_dtype(o_hca, "stream_superposition: o_hca", dt));
    MABA_TRY(expect_dtype(out, "stream_superposition: out", dt));
    if (!present(gate)) return set_error(MABA_ERR_INVALID, "stream_superposition: gate is required");
    MABA_TRY(expect_dtype(gate, "stream_superposition: gate", dt));
    int gate4d = 0;
    if (gate->ndim == 3) {
        const int64_t g3[3] = {B, L, 3};
        MABA_TRY(expect_shape(gate, "stream_superposition: gate", 3, g3));
    } else if (gate->ndim == 4) {
        const int64_t g4[4] = {B, H, L, 3};
        MABA_TRY(expect_shape(gate, "stream_superposition: gate", 4, g4));
        gate4d = 1;
    } else {
        return set_error(MABA_ERR_INVALID, "stream_superposition: gate tensor must be 3D or 4D, got %dD", gate->ndim);
    }
    SupArgs a{};
    a.ol = o_local->data; a.os = o_sparse->data; a.oh = o_hca->data; a.gate = gate->data; a.out = out->data;
    for (int i = 0; i < 4; ++i) {
        a.s_ol[i] = o_local->stride[i]; a.s_os[i] = o_sparse->stride[i]; a.s_oh[i] = o_hca->stride[i];
        a.s_out[i] = out->stride[i]; a.s_g[i] = i < gate->ndim ? gate->stride[i] : 0;
    }
    a.B = B; a.H = H; a.L = L; a.D = D; a.gate4d = gate4d; a.logits = gate_is_logits ? 1 : 0;
    const int64_t rows = B * H * L;
    if (rows == 0 || D == 0) return MABA_OK;
    cudaStream_t s = as_stream(stream);
    const int threads = 256;
    int64_t blocks = ceil_div(rows, threads / 32);
    const int64_t cap = (int64_t)sm_count() * 16;
    if (blocks > cap) blocks = cap;
    return MABA_DISPATCH_FLOAT(dt, "stream_superposition", [&] {
        using ACC = typename std::conditional<sizeof(T) == 8, double, float>::type;
        superposition_kernel<T, ACC><<<(unsigned)blocks, threads, 0, s>>>(a);
        return check_launch("stream_superposition");
    });
}
