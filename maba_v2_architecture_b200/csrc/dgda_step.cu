// DGDA decode step: one recurrence update per (batch, head).
//
//   Sd    = diag(alpha) S
//   delta = w*v - (b*k)^T Sd
//   S'    = Sd + k delta^T
//   o     = q^T S'
//
// Follows maba_sparse/kernels/common.py:271-309 (ref_dgda_step) and
// cpu_dgda.py:200-261 (cpu_dgda_step).  The state is a bandwidth-bound
// stream: one CTA per (b,h) pulls the dk x dv state into shared memory once
// (coalesced along dv), performs both reductions over dk from shared memory
// and writes the new state once.  Compute is fp32 (fp64 for fp64 inputs).
#include "common.cuh"

namespace maba {
namespace {

struct StepArgs {
    const void* q; const void* k; const void* v; const void* alpha; const void* log_alpha;
    const void* b; const void* w; const void* state;
    void* out; void* new_state;
    int64_t sq[3], sk[3], sv[3], sa[3], sla[3], sb[3], sw[3];
    int64_t ss[4], so[3], sns[4];
    int H, dk, dv;
};

constexpr int kStepThreads = 256;

template <typename T, typename TS, typename ACC>
__global__ void __launch_bounds__(kStepThreads) dgda_step_kernel(StepArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int dk = a.dk, dv = a.dv;
    ACC* S = reinterpret_cast<ACC*>(smem_raw);
    ACC* qv = S + dk * dv;
    ACC* kv = qv + dk;
    ACC* bkv = kv + dk;
    ACC* alv = bkv + dk;
    ACC* wvv = alv + dk;
    ACC* del = wvv + dv;
    ACC* red = del + dv;

    const int bh = blockIdx.x;
    const int64_t bi = bh / a.H, hi = bh % a.H;
    const int tid = threadIdx.x, nt = blockDim.x;

    const T* q = static_cast<const T*>(a.q);
    const T* k = static_cast<const T*>(a.k);
    const T* v = static_cast<const T*>(a.v);
    const T* bb = static_cast<const T*>(a.b);
    const T* w = static_cast<const T*>(a.w);
    for (int i = tid; i < dk; i += nt) {
        ACC qi = load_as<ACC>(q + bi * a.sq[0] + hi * a.sq[1] + i * a.sq[2]);
        ACC ki = load_as<ACC>(k + bi * a.sk[0] + hi * a.sk[1] + i * a.sk[2]);
        ACC bi_ = load_as<ACC>(bb + bi * a.sb[0] + hi * a.sb[1] + i * a.sb[2]);
        ACC al;
        if (a.alpha != nullptr) {
            al = load_as<ACC>(static_cast<const T*>(a.alpha) + bi * a.sa[0] + hi * a.sa[1] + i * a.sa[2]);
        } else {
            al = exp_acc<ACC>(load_as<ACC>(static_cast<const T*>(a.log_alpha) + bi * a.sla[0] +
                                            hi * a.sla[1] + i * a.sla[2]));
        }
        qv[i] = qi;
        kv[i] = ki;
        bkv[i] = bi_ * ki;
        alv[i] = al;
    }
    for (int j = tid; j < dv; j += nt) {
        ACC vj = load_as<ACC>(v + bi * a.sv[0] + hi * a.sv[1] + j * a.sv[2]);
        ACC wj = load_as<ACC>(w + bi * a.sw[0] + hi * a.sw[1] + j * a.sw[2]);
        wvv[j] = wj * vj;
    }
    __syncthreads();

    // decayed state
    const TS* st = static_cast<const TS*>(a.state);
    for (int e = tid; e < dk * dv; e += nt) {
        const int i = e / dv, j = e - (e / dv) * dv;
        ACC s = ACC(0);
        if (st != nullptr)
            s = load_as<ACC>(st + bi * a.ss[0] + hi * a.ss[1] + (int64_t)i * a.ss[2] + (int64_t)j * a.ss[3]);
        S[e] = alv[i] * s;
    }
    __syncthreads();

    // pred_j = sum_i bk_i Sd_ij   (row groups reduce through shared memory)
    const int nrg = (nt / dv) > 0 ? (nt / dv) : 1;
    for (int p = tid; p < dv * nrg; p += nt) {
        const int j = p % dv, g = p / dv;
        ACC acc = ACC(0);
        for (int i = g; i < dk; i += nrg) acc += bkv[i] * S[i * dv + j];
        red[g * dv + j] = acc;
    }
    __syncthreads();
    for (int j = tid; j < dv; j += nt) {
        ACC pr = ACC(0);
        for (int g = 0; g < nrg; ++g) pr += red[g * dv + j];
        del[j] = wvv[j] - pr;
    }
    __syncthreads();

    // S' = Sd + k delta^T, written once
    TS* ns = static_cast<TS*>(a.new_state);
    for (int e = tid; e < dk * dv; e += nt) {
        const int i = e / dv, j = e - (e / dv) * dv;
        ACC s = S[e] + kv[i] * del[j];
        S[e] = s;
        store_from<TS, ACC>(ns + bi * a.sns[0] + hi * a.sns[1] + (int64_t)i * a.sns[2] + (int64_t)j * a.sns[3], s);
    }
    __syncthreads();

    // o_j = sum_i q_i S'_ij
    for (int p = tid; p < dv * nrg; p += nt) {
        const int j = p % dv, g = p / dv;
        ACC acc = ACC(0);
        for (int i = g; i < dk; i += nrg) acc += qv[i] * S[i * dv + j];
        red[g * dv + j] = acc;
    }
    __syncthreads();
    T* o = static_cast<T*>(a.out);
    for (int j = tid; j < dv; j += nt) {
        ACC acc = ACC(0);
        for (int g = 0; g < nrg; ++g) acc += red[g * dv + j];
        store_from<T, ACC>(o + bi * a.so[0] + hi * a.so[1] + j * a.so[2], acc);
    }
}

// fp32 state, dk = dv = 64, unit-stride state rows: one warp per (b, h), the
// state slice held in registers (lane l owns columns 2l, 2l+1 of all 64 rows,
// read and written as float2 rows of 256 contiguous bytes per warp), so the
// only memory traffic is the state in and out once; the per-row vectors
// (decay, b*k, k, q) are broadcast from shared memory four at a time.
constexpr int kFastWarps = 4;

template <typename T>
__global__ void __launch_bounds__(kFastWarps * 32) dgda_step_fast_kernel(StepArgs a, int64_t nbh) {
    __shared__ __align__(16) float vec[kFastWarps][4][64];  // decay, b*k, k, q
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t bh = (int64_t)blockIdx.x * kFastWarps + warp;
    if (bh >= nbh) return;  // the whole warp; no block-wide barrier follows
    const int64_t bi = bh / a.H, hi = bh % a.H;
    const T* q = static_cast<const T*>(a.q);
    const T* k = static_cast<const T*>(a.k);
    const T* v = static_cast<const T*>(a.v);
    const T* bb = static_cast<const T*>(a.b);
    const T* w = static_cast<const T*>(a.w);
    const int j0 = 2 * lane;
    // the state slice first: 64 independent 8-byte loads in flight per lane
    float2 s[64];
    if (a.state != nullptr) {
        const float* st = static_cast<const float*>(a.state) + bi * a.ss[0] + hi * a.ss[1] + j0;
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] = *reinterpret_cast<const float2*>(st + (int64_t)i * a.ss[2]);
    } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] = make_float2(0.f, 0.f);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int i = lane + 32 * r;
        const float ki = load_as<float>(k + bi * a.sk[0] + hi * a.sk[1] + i * a.sk[2]);
        const float bi_ = load_as<float>(bb + bi * a.sb[0] + hi * a.sb[1] + i * a.sb[2]);
        float al;
        if (a.alpha != nullptr)
            al = load_as<float>(static_cast<const T*>(a.alpha) + bi * a.sa[0] + hi * a.sa[1] + i * a.sa[2]);
        else
            al = expf(load_as<float>(static_cast<const T*>(a.log_alpha) + bi * a.sla[0] + hi * a.sla[1] +
                                     i * a.sla[2]));
        vec[warp][0][i] = al;
        vec[warp][1][i] = bi_ * ki;
        vec[warp][2][i] = ki;
        vec[warp][3][i] = load_as<float>(q + bi * a.sq[0] + hi * a.sq[1] + i * a.sq[2]);
    }
    const float wv0 = load_as<float>(w + bi * a.sw[0] + hi * a.sw[1] + j0 * a.sw[2]) *
                      load_as<float>(v + bi * a.sv[0] + hi * a.sv[1] + j0 * a.sv[2]);
    const float wv1 = load_as<float>(w + bi * a.sw[0] + hi * a.sw[1] + (j0 + 1) * a.sw[2]) *
                      load_as<float>(v + bi * a.sv[0] + hi * a.sv[1] + (j0 + 1) * a.sv[2]);
    __syncwarp();
    // decayed state and pred_j = sum_i (b k)_i Sd_ij for this lane's two columns
    float p0 = 0.f, p1 = 0.f;
#pragma unroll
    for (int i4 = 0; i4 < 16; ++i4) {
        const float4 al = *reinterpret_cast<const float4*>(&vec[warp][0][4 * i4]);
        const float4 bk = *reinterpret_cast<const float4*>(&vec[warp][1][4 * i4]);
        const float alv[4] = {al.x, al.y, al.z, al.w}, bkv[4] = {bk.x, bk.y, bk.z, bk.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float2& x = s[4 * i4 + e];
            x.x *= alv[e];
            x.y *= alv[e];
            p0 = fmaf(bkv[e], x.x, p0);
            p1 = fmaf(bkv[e], x.y, p1);
        }
    }
    const float d0 = wv0 - p0, d1 = wv1 - p1;
    // S' = Sd + k delta^T (written once), o_j = sum_i q_i S'_ij
    float* ns = static_cast<float*>(a.new_state) + bi * a.sns[0] + hi * a.sns[1] + j0;
    float o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int i4 = 0; i4 < 16; ++i4) {
        const float4 kk = *reinterpret_cast<const float4*>(&vec[warp][2][4 * i4]);
        const float4 qq = *reinterpret_cast<const float4*>(&vec[warp][3][4 * i4]);
        const float kv[4] = {kk.x, kk.y, kk.z, kk.w}, qv[4] = {qq.x, qq.y, qq.z, qq.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int i = 4 * i4 + e;
            float2 x = s[i];
            x.x = fmaf(kv[e], d0, x.x);
            x.y = fmaf(kv[e], d1, x.y);
            *reinterpret_cast<float2*>(ns + (int64_t)i * a.sns[2]) = x;
            o0 = fmaf(qv[e], x.x, o0);
            o1 = fmaf(qv[e], x.y, o1);
        }
    }
    T* o = static_cast<T*>(a.out) + bi * a.so[0] + hi * a.so[1];
    store_from<T, float>(o + j0 * a.so[2], o0);
    store_from<T, float>(o + (j0 + 1) * a.so[2], o1);
}

bool step_fast_ok(const StepArgs& a) {
    auto al8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; };
    if (a.dk != 64 || a.dv != 64) return false;
    if (a.sns[3] != 1 || (a.sns[2] & 1) || (a.sns[1] & 1) || (a.sns[0] & 1) || !al8(a.new_state)) return false;
    if (a.state != nullptr && (a.ss[3] != 1 || (a.ss[2] & 1) || (a.ss[1] & 1) || (a.ss[0] & 1) || !al8(a.state)))
        return false;
    return true;
}

template <typename T, typename TS>
int launch_step(StepArgs& a, int64_t B, cudaStream_t stream) {
    if constexpr (std::is_same<TS, float>::value && !std::is_same<T, double>::value) {
        if (step_fast_ok(a)) {
            const int64_t nbh = B * a.H;
            if (nbh > 0) {
                dgda_step_fast_kernel<T><<<(unsigned)ceil_div(nbh, kFastWarps), kFastWarps * 32, 0, stream>>>(a, nbh);
                return check_launch("dgda_step");
            }
            return MABA_OK;
        }
    }
    using ACC = typename std::conditional<sizeof(T) == 8, double, float>::type;
    const int nrg = (kStepThreads / a.dv) > 0 ? (kStepThreads / a.dv) : 1;
    const size_t smem = sizeof(ACC) * ((size_t)a.dk * a.dv + 4 * a.dk + 2 * a.dv + (size_t)nrg * a.dv);
    if (smem > 227 * 1024)
        return set_error(MABA_ERR_UNSUPPORTED, "dgda_step: dk*dv=%d too large", a.dk * a.dv);
    auto kern = dgda_step_kernel<T, TS, ACC>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return set_error(MABA_ERR_CUDA, "dgda_step: %s", cudaGetErrorString(e));
    }
    const int64_t grid = B * a.H;
    if (grid > 0) {
        kern<<<(unsigned)grid, kStepThreads, smem, stream>>>(a);
        return check_launch("dgda_step");
    }
    return MABA_OK;
}

void copy_strides(int64_t* dst, const maba_tensor* t, int n) {
    for (int i = 0; i < n; ++i) dst[i] = present(t) ? t->stride[i] : 0;
}

}  // namespace
}  // namespace maba

using namespace maba;

extern "C" int maba_dgda_step(const maba_tensor* q, const maba_tensor* k, const maba_tensor* v,
                              const maba_tensor* alpha, const maba_tensor* log_alpha,
                              const maba_tensor* b, const maba_tensor* w, const maba_tensor* state,
                              const maba_tensor* out, const maba_tensor* new_state, void* stream) {
    if (!present(q)) return set_error(MABA_ERR_INVALID, "dgda_step: q is required");
    if (q->ndim != 3) return set_error(MABA_ERR_INVALID, "dgda_step: q must be [B,H,dk]");
    const int64_t B = q->shape[0], H = q->shape[1], dk = q->shape[2];
    if (!present(v) || v->ndim != 3) return set_error(MABA_ERR_INVALID, "dgda_step: v must be [B,H,dv]");
    const int64_t dv = v->shape[2];
    const int64_t s_dk[3] = {B, H, dk}, s_dv[3] = {B, H, dv}, s_st[4] = {B, H, dk, dv};
    MABA_TRY(expect_shape(k, "dgda_step: k", 3, s_dk));
    MABA_TRY(expect_shape(v, "dgda_step: v", 3, s_dv));
    MABA_TRY(expect_shape(b, "dgda_step: b", 3, s_dk));
    MABA_TRY(expect_shape(w, "dgda_step: w", 3, s_dv));
    MABA_TRY(expect_shape(out, "dgda_step: out", 3, s_dv));
    MABA_TRY(expect_shape(new_state, "dgda_step: new_state", 4, s_st));
    if (!present(alpha) && !present(log_alpha))
        return set_error(MABA_ERR_INVALID, "dgda_step: either alpha or log_alpha must be provided");
    if (present(alpha)) MABA_TRY(expect_shape(alpha, "dgda_step: alpha", 3, s_dk));
    if (present(log_alpha)) MABA_TRY(expect_shape(log_alpha, "dgda_step: log_alpha", 3, s_dk));
    if (present(state)) MABA_TRY(expect_shape(state, "dgda_step: state", 4, s_st));
    const int dt = q->dtype;
    const maba_tensor* same[] = {k, v, b, w, out};
    const char* names[] = {"k", "v", "b", "w", "out"};
    for (int i = 0; i < 5; ++i)
        if (same[i]->dtype != dt)
            return set_error(MABA_ERR_DTYPE, "dgda_step: %s dtype %s differs from q (%s)", names[i],
                             dtype_name(same[i]->dtype), dtype_name(dt));
    if (present(alpha) && alpha->dtype != dt) return set_error(MABA_ERR_DTYPE, "dgda_step: alpha dtype mismatch");
    if (present(log_alpha) && log_alpha->dtype != dt)
        return set_error(MABA_ERR_DTYPE, "dgda_step: log_alpha dtype mismatch");
    const int sdt = new_state->dtype;
    if (present(state) && state->dtype != sdt)
        return set_error(MABA_ERR_DTYPE, "dgda_step: state and new_state dtypes differ");
    if (sdt != dt && sdt != MABA_F32)
        return set_error(MABA_ERR_DTYPE, "dgda_step: state dtype must be q's dtype or float32");
    if (dk <= 0 || dv <= 0) return set_error(MABA_ERR_INVALID, "dgda_step: empty head dims");

    StepArgs a{};
    a.q = q->data; a.k = k->data; a.v = v->data;
    a.alpha = present(alpha) ? alpha->data : nullptr;
    a.log_alpha = present(log_alpha) ? log_alpha->data : nullptr;
    a.b = b->data; a.w = w->data;
    a.state = present(state) ? state->data : nullptr;
    a.out = out->data; a.new_state = new_state->data;
    copy_strides(a.sq, q, 3); copy_strides(a.sk, k, 3); copy_strides(a.sv, v, 3);
    copy_strides(a.sa, alpha, 3); copy_strides(a.sla, log_alpha, 3);
    copy_strides(a.sb, b, 3); copy_strides(a.sw, w, 3);
    copy_strides(a.ss, state, 4); copy_strides(a.so, out, 3); copy_strides(a.sns, new_state, 4);
    a.H = (int)H; a.dk = (int)dk; a.dv = (int)dv;
    cudaStream_t s = as_stream(stream);

    switch (dt) {
        case MABA_F32: return launch_step<float, float>(a, B, s);
        case MABA_F64:
            if (sdt != MABA_F64) return set_error(MABA_ERR_DTYPE, "dgda_step: float64 needs a float64 state");
            return launch_step<double, double>(a, B, s);
        case MABA_F16:
            return sdt == MABA_F32 ? launch_step<__half, float>(a, B, s) : launch_step<__half, __half>(a, B, s);
        case MABA_BF16:
            return sdt == MABA_F32 ? launch_step<__nv_bfloat16, float>(a, B, s)
                                   : launch_step<__nv_bfloat16, __nv_bfloat16>(a, B, s);
        default:
            return set_error(MABA_ERR_DTYPE, "dgda_step: unsupported dtype %s", dtype_name(dt));
    }
}
