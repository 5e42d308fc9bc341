/*
 * maba_b200.h -- C ABI of the B200 (sm_100a) Maba v2 hot path.
 *
 * Every entry point takes plain device pointers wrapped in `maba_tensor`
 * descriptors (pointer + dtype + shape + element strides), a caller-owned
 * CUDA stream (`void*` holding a cudaStream_t) and, where a kernel needs
 * scratch memory, a caller-owned workspace whose size the matching
 * `*_workspace_size` call reports.  Nothing here allocates device memory,
 * synchronises the device or keeps a pointer after it returns.
 *
 * Return value: MABA_OK (0) or one of the MABA_ERR_* codes; the message of
 * the last failure on the calling thread is returned by maba_last_error().
 *
 * The reference project (maba_sparse, Python) reaches this path through its
 * kernel registry; each declaration below names the reference function it
 * replaces (file:line inside the reference project).
 */
#ifndef MABA_B200_H
#define MABA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MABA_ABI_VERSION 1

/* element types */
#define MABA_F32  0
#define MABA_F16  1
#define MABA_BF16 2
#define MABA_F64  3
#define MABA_I64  4
#define MABA_I32  5

/* status codes */
#define MABA_OK               0
#define MABA_ERR_INVALID      1 /* bad shape / stride / argument            */
#define MABA_ERR_DTYPE        2 /* dtype not supported or mismatched        */
#define MABA_ERR_UNSUPPORTED  3 /* valid request outside the built kernels */
#define MABA_ERR_WORKSPACE    4 /* workspace missing or too small           */
#define MABA_ERR_CUDA         5 /* CUDA launch / runtime error              */

#define MABA_MAX_DIMS 6

#if defined(__GNUC__)
#define MABA_API __attribute__((visibility("default")))
#else
#define MABA_API
#endif

typedef struct maba_tensor {
    void*   data;                    /* device address of element [0..0]; NULL = operand absent */
    int32_t dtype;                   /* MABA_F32 ... MABA_I32 */
    int32_t ndim;                    /* valid entries in shape / stride */
    int64_t shape[MABA_MAX_DIMS];
    int64_t stride[MABA_MAX_DIMS];   /* in elements, may be any non-negative value */
} maba_tensor;

/* ---- library ---------------------------------------------------------- */

MABA_API int         maba_abi_version(void);
MABA_API const char* maba_last_error(void);

/* Reads and clears the device error word (synchronises `stream`): 0, or 1 when
 * a kernel gave up on a bounded wait (a pipeline barrier that never completed)
 * and returned early; its outputs are then not valid.  No reference
 * counterpart (the reference's kernels do not wait on barriers). */
MABA_API int maba_device_error(int32_t* out, void* stream);

/* Self-test of the bounded waits: launches one warp that waits on a barrier
 * nothing arrives on; after ~limit_cycles the wait gives up, the device error
 * word becomes 2 and the kernel returns (the context stays usable). */
MABA_API int maba_selftest_wait_timeout(int64_t limit_cycles, void* stream);

/* ---- DGDA chunked prefill ---------------------------------------------
 * Replaces the `dgda_prefill` registry op:
 *   maba_sparse/kernels/dispatcher.py:258   (dispatch_dgda_prefill)
 *   maba_sparse/kernels/common.py:229-268   (ref_dgda_prefill, sequential)
 *   maba_sparse/kernels/cpu_dgda.py:33-197  (cpu_dgda_prefill, chunked WY/UT)
 *   maba_sparse/kernels/triton_dgda.py:648  (triton_dgda_prefill)
 * q, k, b, alpha, log_alpha: [B,H,L,dk];  v, w: [B,H,L,dv];
 * initial_state (optional, NULL data = zeros): [B,H,dk,dv];
 * out: [B,H,L,dv] (dtype of q);  final_state: [B,H,dk,dv] (dtype of q or F32).
 * alpha or log_alpha may be absent (not both); when log_alpha is given it is
 * used (clamped to [-46,0]), otherwise log(clamp(alpha,1e-20,1)).
 * chunk_size is accepted for API parity; the kernels choose their own chunk
 * (the recurrence is chunk-invariant).  Workspace: see _workspace_size. */
MABA_API int maba_dgda_prefill(const maba_tensor* q, const maba_tensor* k, const maba_tensor* v,
                      const maba_tensor* alpha, const maba_tensor* log_alpha,
                      const maba_tensor* b, const maba_tensor* w,
                      const maba_tensor* initial_state,
                      const maba_tensor* out, const maba_tensor* final_state,
                      int32_t chunk_size, void* workspace, size_t workspace_bytes,
                      void* stream);
MABA_API size_t maba_dgda_prefill_workspace_size(int32_t dtype, int64_t B, int64_t H, int64_t L,
                                        int64_t dk, int64_t dv);

/* ---- DGDA segment transition -------------------------------------------
 * The affine map of a whole sequence segment on the recurrent state:
 * S_end = P S_start + R, written as trans_out [B,H,64,128] fp32 = [R | P]
 * (R: 64 x 64 padded dk x dv, P: 64 x 64 padded dk x dk).  Lets GPUs that hold
 * consecutive segments of one sequence chain their states with one small
 * all-gather (same recurrence as maba_sparse/kernels/common.py:256-265).
 * Inputs as for maba_dgda_prefill; fp32 / fp16 / bf16. */
MABA_API int maba_dgda_transition(const maba_tensor* q, const maba_tensor* k, const maba_tensor* v,
                                  const maba_tensor* alpha, const maba_tensor* log_alpha,
                                  const maba_tensor* b, const maba_tensor* w, const maba_tensor* trans_out,
                                  void* workspace, size_t workspace_bytes, void* stream);
MABA_API size_t maba_dgda_transition_workspace_size(int32_t dtype, int64_t B, int64_t H, int64_t L);

/* ---- DGDA decode step --------------------------------------------------
 * Replaces the `dgda_step` registry op:
 *   maba_sparse/kernels/dispatcher.py:330, common.py:271-309,
 *   cpu_dgda.py:200-261, triton_dgda.py:668.
 * q, k, b, alpha, log_alpha: [B,H,dk]; v, w: [B,H,dv];
 * state (optional): [B,H,dk,dv]; out: [B,H,dv]; new_state: [B,H,dk,dv].
 * alpha has priority over log_alpha (as in the reference). */
MABA_API int maba_dgda_step(const maba_tensor* q, const maba_tensor* k, const maba_tensor* v,
                   const maba_tensor* alpha, const maba_tensor* log_alpha,
                   const maba_tensor* b, const maba_tensor* w,
                   const maba_tensor* state,
                   const maba_tensor* out, const maba_tensor* new_state,
                   void* stream);

/* ---- DGDA front end ------------------------------------------------------
 * Replaces the feature path of DGDALayer between its projections and the
 * recurrence (maba_sparse/layers/dgda.py):
 *   _apply_conv :103-122 (causal depthwise conv with history + SiLU on q, k, v,
 *   called at :186-190 and :254-258), the gates :192-197 / :260-264
 *   (b = sigmoid, w = sigmoid, log alpha = max(-softplus, -14)) and the per-head
 *   k normalisation k / (||k|| + eps) at :207 / :270.
 * proj[6]: the projected inputs q, k, v, alpha, erase, write, each [B,L,C]
 *   (C = H*dk for q, k, alpha, erase; H*dv for v, write; any strides);
 * conv_w[3]: [C, K] taps of q, k, v (Conv1d weight [C,1,K] viewed 2-D);
 * hist[3] (entries with NULL data = zero history; the pointer itself may be
 *   NULL): [B, C, K-1] conv inputs before token 0, oldest first (the layer's
 *   conv_state), float32 or the feature dtype;
 * out[6]: q, k, v, log_alpha, b, w (the transforms of proj[0..5]), each
 *   [B,L,C] in the feature dtype;
 * new_hist[3] (optional, as hist; must not alias hist): the last K-1 inputs of
 *   [hist | x], the conv_state the layer returns.
 * Features float32 / float16 / bfloat16; C a multiple of 8; dk / 8 a power of
 * two <= 32; K <= 8. */
MABA_API int maba_dgda_frontend(const maba_tensor* proj, const maba_tensor* conv_w, const maba_tensor* hist,
                                const maba_tensor* out, const maba_tensor* new_hist, int32_t n_heads, float eps,
                                void* stream);

/* ---- DG-Indexer block pooling ------------------------------------------
 * Replaces `compute_centroids`: dispatcher.py:399, common.py:329-350,
 * cpu_indexer.py:16-50.  k_idx: [B,L,d] -> out: [B,ceil(L/block),d],
 * c = 0.5*(sum/block + max) with the tail block zero-padded. */
MABA_API int maba_compute_centroids(const maba_tensor* k_idx, const maba_tensor* out,
                           int32_t block_size, void* stream);

/* ---- DG-Indexer scoring + top-k ----------------------------------------
 * Replaces `index_topk`: dispatcher.py:424, common.py:353-403,
 * cpu_indexer.py:54-112, and the decode-time inline top-k of
 * maba_sparse/layers/indexer.py:101-112 (decode != 0).
 * q_idx: [B,L,d]; centroids: [B,nb,d]; idx_out: [B,L,min(top_k,nb)] int64;
 * scores_out (optional): [B,L,nb] in q_idx's dtype.
 * score[t,n] = (q_t*scale).c_n - lambda*log1p(qb(t)-n), scale = 1/sqrt(d),
 * qb(t) = t/block (prefill) or nb-1 (decode); n > qb(t) is -inf.
 * Order: score descending, ties to the lower block index; slots past the
 * number of finite candidates hold the lowest unused (future) indices in
 * ascending order.  Workspace: see _workspace_size. */
MABA_API int maba_index_topk(const maba_tensor* q_idx, const maba_tensor* centroids,
                    float lambda_dist, int32_t top_k, int32_t block_size, int32_t decode,
                    const maba_tensor* idx_out, const maba_tensor* scores_out,
                    void* workspace, size_t workspace_bytes, void* stream);
MABA_API size_t maba_index_topk_workspace_size(int64_t B, int64_t L, int64_t nb, int32_t top_k);

/* Prefill scoring for query rows that sit at absolute positions q_pos0 + t
 * (qb(t) = (q_pos0 + t) / block): the rows of one sequence segment when a
 * sequence is split across GPUs.  Same semantics as maba_index_topk with
 * decode == 0 otherwise (maba_sparse/kernels/cpu_indexer.py:54-112 on the
 * segment's rows of the full score matrix). */
MABA_API int maba_index_topk_at(const maba_tensor* q_idx, const maba_tensor* centroids,
                                float lambda_dist, int32_t top_k, int32_t block_size, int64_t q_pos0,
                                const maba_tensor* idx_out, const maba_tensor* scores_out,
                                void* workspace, size_t workspace_bytes, void* stream);
MABA_API size_t maba_index_topk_at_workspace_size(int64_t B, int64_t L, int64_t nb, int32_t top_k,
                                                  int32_t block_size, int64_t q_pos0);

/* ---- DG-Indexer scoring + top-k with no caller workspace ---------------
 * Has no counterpart in the reference: it exists for callers that cannot
 * allocate device memory -- an application whose framework owns every byte
 * of the GPU through its own pool, a latency-critical decode loop that must
 * not pay cudaMalloc's implicit device synchronisation, or a thin foreign-
 * language binding that only ever receives device pointers from elsewhere.
 * Same arguments, results and errors as maba_index_topk minus the workspace.
 * Its scratch is one file-scope device array of MABA_NOALLOC_PENALTY_MAX
 * floats (256 KiB) that every GPU which loads this library holds until the
 * process exits.  A call uses it for up to three things, in this order:
 *   1. the distance-penalty table, max(nb, ceil(L / block_size)) floats in
 *      prefill, nb in decode (always);
 *   2. the per-tile centroid norms and their prefix maxima of the pruned tile
 *      scan, 2 * B * ceil(nb / 64) floats after the table rounded up to 256
 *      bytes (prefill with scores_out absent and L >= 64);
 *   3. the partial candidate lists of the split decode scan,
 *      B * L * ceil(nb / 512) * 32 (score, index) pairs after the table
 *      (decode with scores_out absent, nb >= 2048 and B * L <= 256).
 * Requests whose penalty table alone does not fit are rejected with
 * MABA_ERR_UNSUPPORTED.  When the table fits but region 2 or 3 does not, the
 * call runs the unpruned scan or the unsplit decode scan instead: the indices
 * are the same, but such near-limit shapes can be much slower than
 * maba_index_topk with a workspace.  Each call rewrites every region it reads
 * before reading it, so nothing needs clearing between calls; calls that
 * overlap on the GPU (different streams, or different host threads) race on
 * all three regions and must be serialised by the caller.
 * The first call on a device looks the array's device address up (once per
 * device, with that device current) and keeps it for the life of the
 * process: make that first call before any stream capture, and do not use
 * this entry point across a device reset (cudaDeviceReset, or a primary-
 * context reset by the host framework), after which the kept address is
 * stale.  Allocates nothing. */
#define MABA_NOALLOC_PENALTY_MAX 65536
MABA_API int maba_index_topk_noalloc(const maba_tensor* q_idx, const maba_tensor* centroids,
                                     float lambda_dist, int32_t top_k, int32_t block_size, int32_t decode,
                                     const maba_tensor* idx_out, const maba_tensor* scores_out,
                                     void* stream);

/* ---- Stream superposition ----------------------------------------------
 * Replaces `stream_superposition`: dispatcher.py:468, common.py:406-438,
 * cpu_indexer.py:116-150.  o_*: [B,H,L,D]; gate: [B,L,3] or [B,H,L,3];
 * gate_is_logits != 0 applies a softmax over the last axis first. */
MABA_API int maba_stream_superposition(const maba_tensor* o_local, const maba_tensor* o_sparse,
                              const maba_tensor* o_hca, const maba_tensor* gate,
                              int32_t gate_is_logits, const maba_tensor* out, void* stream);

/* ---- HCA block pooling -------------------------------------------------
 * The pooled-prefix table of maba_sparse/layers/sparse_attention.py:206:
 * c_kv: [B,L,d_c] -> out: [B,L/r,d_c] (complete blocks only), mean of r rows. */
MABA_API int maba_hca_pool(const maba_tensor* c_kv, const maba_tensor* out, int32_t r, void* stream);

/* ---- MABA-SA fused three-stream attention ------------------------------
 * Replaces MabaSparseAttention._compute_local_attention,
 * _compute_sparse_attention, _compute_hca_attention and the superposition
 * call (maba_sparse/layers/sparse_attention.py:79-219, 274-275), computed in
 * the latent space of the MLA cache (keys/values never up-projected):
 *   qhat:  [B,Lq,H,d_c]   = scale * W_uk,h^T q_h   (absorbed queries)
 *   c_kv:  [B,Lkv,d_c]    latent cache, query t sits at pos = Lkv-Lq+t
 *   hca:   [B,Lkv/r,d_c]  pooled complete blocks (maba_hca_pool)
 *   top_idx: [B,Lq,K] int64 selected blocks (indices into c_kv blocks)
 *   gate:  [B,Lq,3] or [B,H,Lq,3] gate logits
 *   out:   [B,Lq,H,d_c]   sum_s softmax(gate)_s * (attention of stream s),
 *          still in latent space; the caller applies W_uv and o_proj.
 * Single-token queries (Lq == 1, decode) run split-K over the keys when the
 * workspace reported by _workspace_size is supplied. */
MABA_API int maba_sa_attention(const maba_tensor* qhat, const maba_tensor* c_kv,
                      const maba_tensor* hca, const maba_tensor* top_idx,
                      const maba_tensor* gate, const maba_tensor* out,
                      int32_t window, int32_t n_sinks, int32_t block_size, int32_t hca_r,
                      void* workspace, size_t workspace_bytes, void* stream);
MABA_API size_t maba_sa_attention_workspace_size(int32_t dtype, int64_t B, int64_t Lq, int64_t Lkv,
                                                 int64_t H, int64_t d_c, int64_t K, int32_t window,
                                                 int32_t n_sinks, int32_t block_size, int32_t hca_r);

/* ---- Decode at a device-held position ------------------------------------
 * Single-token decode over preallocated caches whose visible length lives in
 * device memory (*pos_dev = position of the new token), so that a whole decode
 * step can be captured once in a CUDA graph and replayed.  Same results as the
 * host-length entry points above (the reference's decode:
 * maba_sparse/layers/sparse_attention.py:228-261, layers/indexer.py:62-112).
 *
 * maba_decode_cache_append: writes the new latent row c_new [B,1,d_c] and
 *   index-key row k_new [B,1,d_idx] at pos into c_cache [B,Lcap,d_c] /
 *   kidx_cache [B,Lcap,d_idx], refreshes the centroid of pos's block in
 *   cent_table [B,nbcap,d_idx] (zero-padded tail, as compute_centroids) and,
 *   when pos closes an r-row group, its pooled mean in hca_table [B,NCcap,d_c]. */
MABA_API int maba_decode_cache_append(const maba_tensor* c_new, const maba_tensor* k_new,
                                      const maba_tensor* c_cache, const maba_tensor* kidx_cache,
                                      const maba_tensor* cent_table, const maba_tensor* hca_table,
                                      const int64_t* pos_dev, int32_t block_size, int32_t hca_r, void* stream);
/* Decode top-k over the first pos/block + 1 rows of cent_table; idx_out is
 * [B,1,min(top_k,nbcap)], slots past the visible blocks hold future indices. */
MABA_API int maba_index_topk_decode_at(const maba_tensor* q_idx, const maba_tensor* cent_table,
                                       float lambda_dist, int32_t top_k, int32_t block_size,
                                       const int64_t* pos_dev, const maba_tensor* idx_out,
                                       void* workspace, size_t workspace_bytes, void* stream);
MABA_API size_t maba_index_topk_decode_at_workspace_size(int64_t B, int64_t nbcap, int32_t top_k);
/* Split-K three-stream decode attention over c_cache[:, :pos+1] and the
 * complete rows of hca_table; qhat [B,1,H,d_c], top_idx [B,1,K], out [B,1,H,d_c]. */
MABA_API int maba_sa_attention_decode_at(const maba_tensor* qhat, const maba_tensor* c_cache,
                                         const maba_tensor* hca_table, const maba_tensor* top_idx,
                                         const maba_tensor* gate, const maba_tensor* out,
                                         const int64_t* pos_dev, int32_t window, int32_t n_sinks,
                                         int32_t block_size, int32_t hca_r, void* workspace,
                                         size_t workspace_bytes, void* stream);
MABA_API size_t maba_sa_attention_decode_at_workspace_size(int64_t B, int64_t Lcap, int64_t NCcap,
                                                           int64_t H, int64_t d_c, int64_t K, int32_t window,
                                                           int32_t n_sinks, int32_t block_size, int32_t hca_r);

/* ---- Model engine: the block pieces around the hot-path ops --------------
 * Used by the inference engine that runs whole models (prefill and decode)
 * from a reference state dict; each replaces torch module code of
 * maba_sparse/model.py.
 *
 * maba_rmsnorm_residual: x [N,D] float32 (updated in place when y is given):
 *   x += gate * y (gate [D] float32 = sigmoid(res_gate), y [N,D] float32 or
 *   h's dtype), then h_out = x * rsqrt(mean(x^2) + eps) * weight ([N,D], optional).
 *   model.py:18-26 (RMSNorm), :107-108 / :126-127 (the gated residual adds). */
MABA_API int maba_rmsnorm_residual(const maba_tensor* x, const maba_tensor* y, const maba_tensor* gate,
                                   const maba_tensor* weight, float eps, const maba_tensor* h_out, void* stream);

/* maba_swiglu: u [N, 2I] (gate | up projections) -> out [N, I] = silu(gate) * up;
 *   model.py:28-37 (SwiGLUFFN). */
MABA_API int maba_swiglu(const maba_tensor* u, const maba_tensor* out, void* stream);

/* maba_decode_gemv: one decode-step GEMV, out = W h, for B <= 8 rows.
 *   w: [rows, K] float32 / float16 / bfloat16, contiguous 16-byte-aligned rows, K % 8 == 0.
 *   prologue 0 (norm):   h = RMSNorm(x) * aux, x [B,K] float32, aux [K] (w's dtype), K <= 2048;
 *            1 (gather): h = aux[ids[b]], aux [V,K] embedding table, ids int64 [B];
 *            2 (vector): h = x, x [B,K] float32 or w's dtype.
 *   epilogue 0 (store):    out [B,rows] (float32 or w's dtype) = W h + bias (bias float32 [rows], optional);
 *            1 (residual): out [B,rows] float32 residual stream += gate * (W h), gate float32 [rows];
 *            2 (dgda):     out [B,rows] float32 DGDA features from the rows q|k|v|alpha|erase|write:
 *                          rows [0, n_conv) through the causal conv with taps [n_conv, Kc] and the
 *                          float32 history hist [B, n_conv, Kc-1] (updated in place) and SiLU,
 *                          rows [n_conv, alpha_end) -> max(-softplus, -14), the rest -> sigmoid
 *                          (layers/dgda.py:238-270, the step's feature path);
 *            3 (swiglu):   rows = 2I (gate rows then up rows), out [B,I] = silu(gate) * up;
 *            4 (logits):   out float32 [B,rows] logits, ids_out int64 [B] their argmax (ties to
 *                          the lower index), *pos_dev += 1 when pos_dev is not NULL; needs a
 *                          workspace of maba_decode_gemv_workspace_size(B) bytes, zeroed before
 *                          the first call (every call leaves it zeroed).
 *   The pieces of MabaBlock.step / MabaSparseForCausalLM.step (model.py:111-129, 256-276):
 *   embedding (FactorizedEmbeddings, :39-50), the norm-fused projections, the gated residual
 *   adds, SwiGLU, the tied head with greedy selection (:304-305). */
MABA_API int maba_decode_gemv(const maba_tensor* w, int32_t prologue, const maba_tensor* x,
                              const maba_tensor* aux, float eps, const maba_tensor* ids, int32_t epilogue,
                              const maba_tensor* out, const maba_tensor* bias, const maba_tensor* gate,
                              const maba_tensor* taps, const maba_tensor* hist, int32_t n_conv, int32_t alpha_end,
                              const maba_tensor* ids_out, int64_t* pos_dev, void* workspace,
                              size_t workspace_bytes, void* stream);
MABA_API size_t maba_decode_gemv_workspace_size(int64_t B);

/* maba_decode_dgda_state: the recurrence of one decode step from the features of
 *   maba_decode_gemv's dgda epilogue: feats float32 [B, 4*H*dk + 2*H*dv] (q|k|v|log
 *   alpha|b|w, k not yet normalised), state float32 [B,H,dk,dv] contiguous (updated in
 *   place), o_out float32 [B, H*dv]; k is divided by (||k_h|| + eps) first
 *   (layers/dgda.py:270), then the step of common.py:271-309.  dk <= 64, dv <= 128. */
MABA_API int maba_decode_dgda_state(const maba_tensor* feats, const maba_tensor* state, const maba_tensor* o_out,
                                    int32_t n_heads, float eps, void* stream);

/* maba_decode_dgda_mix: the DGDA mixer of one decode step up to its output projection,
 *   in one launch: the stacked input projection (w [4*H*dk + 2*H*dv, D], rows q|k|v|alpha|
 *   erase|write) of h = RMSNorm(x) * norm_w, the dgda epilogue of maba_decode_gemv (feats,
 *   taps and hist as there), then maba_decode_dgda_state's recurrence step for each head,
 *   run by the last CTA to finish that head's rows.  dk, dv multiples of 16, at most 64.
 *   workspace: maba_decode_dgda_mix_workspace_size(H) bytes, zeroed before the first call
 *   (every call leaves it zeroed).  Replaces, per DGDA block of MabaBlock.step (model.py:
 *   111-129), the layer's feature path (layers/dgda.py:238-270) and the recurrence step
 *   (common.py:271-309). */
MABA_API int maba_decode_dgda_mix(const maba_tensor* w, const maba_tensor* x, const maba_tensor* norm_w, float eps,
                                  const maba_tensor* taps, const maba_tensor* hist, const maba_tensor* feats,
                                  const maba_tensor* state, const maba_tensor* o_out, int32_t n_heads, float k_eps,
                                  void* workspace, size_t workspace_bytes, void* stream);
MABA_API size_t maba_decode_dgda_mix_workspace_size(int32_t n_heads);

#ifdef __cplusplus
}
#endif

#endif /* MABA_B200_H */
