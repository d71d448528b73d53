/*
 * C ABI of the B200 (sm_100a) routed-attention library.
 *
 * Every entry point takes raw device pointers, 64-bit sizes, a dtype code,
 * scalar parameters and a CUDA stream (as void*), and returns an int status
 * (DA_OK = 0).  Calls are stream-ordered and never synchronise the host.
 * The caller allocates every output and workspace; outputs are fully
 * overwritten unless an `accumulate` flag says otherwise.
 *
 * Each declaration names the reference interface it replaces, by
 * file:line inside the Ahnd6474/double-attention package
 * (src/double_attention/...).
 */
#ifndef DA_B200_H_
#define DA_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define DA_API __attribute__((visibility("default")))
#else
#define DA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
enum {
  DA_OK = 0,
  DA_ERR_NULL = 1,             /* a required pointer is null */
  DA_ERR_SHAPE = 2,            /* unsupported or inconsistent shape */
  DA_ERR_DTYPE = 3,            /* unsupported dtype code */
  DA_ERR_ALIGN = 4,            /* pointer or row stride not 16-byte aligned */
  DA_ERR_UNSUPPORTED = 5,      /* variant not implemented by the kernels */
  DA_ERR_DEVICE_TIMEOUT = 6,   /* a device-side bounded wait gave up */
  DA_ERR_CUDA = 7,             /* CUDA runtime/driver error: da_last_cuda_error() */
  DA_ERR_WORKSPACE = 8         /* workspace smaller than the *_workspace_size query */
};

/* ---- dtype codes ---------------------------------------------------- */
enum { DA_F16 = 0, DA_BF16 = 1, DA_F32 = 2 };

DA_API const char* da_version(void);
DA_API const char* da_status_string(int status);
/* Last CUDA error code recorded by a call on this host thread. */
DA_API int da_last_cuda_error(void);
/* Number of kernels this library has launched in this process (all devices,
 * all threads); a diagnostic for counting launches around a region. */
DA_API uint64_t da_kernel_launches(void);

/* Debug aid with no reference counterpart: pinned, device-accessible host
 * memory (8 ints per CTA) into which kernels write progress markers, or
 * null to disable.  Lets a host thread see where a kernel stands. */
DA_API int da_set_debug_trace(int* host_mapped);

/* ---- dictionary bank normalisation ----------------------------------
 * Replaces SharedDictionaryBank.normalized (modules.py:45-48: F.normalize
 * over dim 0) and the AMP cast of the normalised views (modules.py:229-231).
 * raw: [R, M] fp32 row-major.  Writes (each optional):
 *   out   [R, M] and out_t [M, R] in out_dtype (DA_F16 / DA_BF16),
 *   denom [M] fp32 = max(||raw[:, j]||, eps),
 *   max_col_norm [1] fp32 = largest 2-norm of the rounded output columns. */
DA_API int da_dict_norm_fwd(const float* raw, int64_t R, int64_t M, float eps, int out_dtype, void* out, void* out_t,
                     float* denom, float* max_col_norm, void* stream);

/* Both banks of a dictionary in one launch (the module path normalises the
 * key and value banks every forward, modules.py:45-48, :229-231): the key
 * bank as da_dict_norm_fwd in key_dtype (key, key_t, key_denom, key_max),
 * the value bank in bf16 (value, value_t, value_denom).  The raw banks are
 * [R, M] in raw_dtype (DA_F32, or the half type of a module cast to it);
 * raw_value may equal raw_key (tied dictionary in a dtype other than bf16) or
 * be null (key only).  Every output pointer may be null. */
DA_API int da_dict_norm_pair_fwd(const void* raw_key, const void* raw_value, int raw_dtype, int64_t R, int64_t M,
                                 float eps, int key_dtype, void* key, void* key_t, float* key_denom, float* key_max,
                                 void* value, void* value_t, float* value_denom, void* stream);

/* The temperatures of the path in one launch (modules.py:130-132 and
 * ops.py:160-161): beta = exp(clamp(log_beta, beta_lo, beta_hi)) and
 * gamma_s = exp(clamp(log_scales[s], scale_lo, scale_hi)), written in fp32
 * from logs held in fp32, bf16 or fp16.  Either input may be null. */
DA_API int da_temperatures(const void* log_beta, int beta_dtype, float beta_lo, float beta_hi,
                           const void* log_scales, int scales_dtype, int maps, float scale_lo, float scale_hi,
                           float* beta_out, float* scales_out, void* stream);

/* Backward of da_temperatures (autograd of exp(clamp(log, lo, hi))):
 * grad_log = g * value where lo <= log <= hi (inclusive), else 0, formed in
 * fp32 and stored once in the log's dtype, for beta and the `maps` scales in
 * one launch.  Either half is skipped when its g pointer is null (not both).
 * beta / scales are da_temperatures' outputs. */
DA_API int da_temperatures_bwd(const void* log_beta, int beta_dtype, float beta_lo, float beta_hi, const float* beta,
                               const float* g_beta, void* grad_log_beta, const void* log_scales, int scales_dtype,
                               int maps, float scale_lo, float scale_hi, const float* scales, const float* g_scales,
                               void* grad_log_scales, void* stream);

/* Backward of da_dict_norm_fwd (autograd of F.normalize, modules.py:46-47).
 * grad: [R, M] fp32 and/or grad_t: [M, R] fp32 (summed when both are given).
 * grad_raw: [R, M] fp32, overwritten (accumulate = 0) or added to. */
DA_API int da_dict_norm_bwd(const float* raw, const float* denom, const float* grad, const float* grad_t, int64_t R,
                     int64_t M, float eps, float* grad_raw, int accumulate, void* stream);

/* da_dict_norm_bwd for banks held in any dtype: raw [R, M] in raw_dtype
 * (DA_F32, or the half type of a module cast to it, read exactly), grad_raw
 * [R, M] in grad_dtype, rounded once from the fp32 result (accumulate, which
 * adds to it, needs DA_F32; DA_ERR_UNSUPPORTED otherwise).  The same fp32
 * arithmetic as converting the bank to fp32, calling da_dict_norm_bwd and
 * casting its result: bit-identical, without the two conversion launches. */
DA_API int da_dict_norm_bwd_typed(const void* raw, int raw_dtype, const float* denom, const float* grad,
                                  const float* grad_t, int64_t R, int64_t M, float eps, void* grad_raw, int grad_dtype,
                                  int accumulate, void* stream);

/* Largest column 2-norm of a [R, M] fp16/bf16 dictionary, into out[0]. */
DA_API int da_col_norm_max(const void* dict, int64_t R, int64_t M, int dtype, float* out, void* stream);

/* ---- dictionary route, forward ---------------------------------------
 * Replaces dictionary_route_triton / _DictionaryRouteFunction.forward
 * (triton_kernels.py:1984-2019, :1806-1870; math of ops.py:16-62) for the
 * identity-logit softmax route.  Input rows come from a [rows, q_cols] matrix
 * (row stride q_row_stride elements); `groups` blocks of R columns starting
 * every group_col_stride columns are routed independently (the module path
 * routes the Q and K branches of the fused projection in one call,
 * modules.py:239-241).  R in {64,128,256,512}; M a multiple of 64.
 *   dict_key_t  [M, R] normalised keys, dtype of q;
 *   dict_value  [R, M] normalised values, bf16;
 *   beta, dk_max: device fp32 scalars (dk_max = max column norm of the keys).
 * Outputs: z [groups, rows, R] (dtype of q); lse, out_norm [groups, rows] fp32
 * (log-sum-exp of the beta-scaled logits, ||softmax . Dv^T||); argmax
 * [groups, rows] int32 (optional, may be null).
 * work: int32 [2 + repair_cap], zero-filled before first use and left zeroed
 * by every call; one work buffer must not be shared by calls that run
 * concurrently. */
DA_API int da_route_fwd(const void* q, int64_t rows, int64_t q_cols, int64_t q_row_stride, int groups,
                        int64_t group_col_stride, int64_t R, int64_t M, int dtype, const void* dict_key_t,
                        const void* dict_value, const float* beta, const float* dk_max, float eps,
                        int normalize_input, int normalize_output, void* z, float* lse, float* out_norm,
                        int* argmax, int* work, int repair_cap, int* status, void* stream);

/* No counterpart in the reference.  Same computation and arguments as
 * da_route_fwd, for callers that cannot allocate device memory when they run
 * the route (for example code running under CUDA stream capture, or engines
 * that give a plugin only its inputs and outputs): the work area lives in a
 * __device__ array inside this library, so no `work` buffer is passed and
 * nothing is allocated.  At most 65536 route rows (groups * rows) per call,
 * else DA_ERR_WORKSPACE.  Every GPU that loads the library holds the array
 * (about 256 KiB) until exit; all calls on a device share it, so calls that
 * can overlap on the GPU race.  The first call on each device looks the
 * array's address up and should come before any stream capture.  The call
 * makes q's device current while it runs and restores the calling thread's
 * current device before it returns. */
DA_API int da_route_fwd_static(const void* q, int64_t rows, int64_t q_cols, int64_t q_row_stride, int groups,
                               int64_t group_col_stride, int64_t R, int64_t M, int dtype, const void* dict_key_t,
                               const void* dict_value, const float* beta, const float* dk_max, float eps,
                               int normalize_input, int normalize_output, void* z, float* lse, float* out_norm,
                               int* argmax, int* status, void* stream);

/* ---- dictionary route variants (row stages) ---------------------------
 * The variants of dictionary_route_reference (ops.py:16-62) other than
 * identity logits with softmax assignment -- SiLU logits (:39-41),
 * standardised logits (:44-53) and direct-SiLU assignment (:56-57), the
 * silu_logits / standardize_logits / direct_silu switches of
 * dictionary_route_triton (triton_kernels.py:1984-2019, kernels :215-228,
 * :417-448) -- run as the two dictionary products on da_gemm with these
 * row stages between them, one warp per route row (M <= 2048).
 * flags: OR of the DA_ROUTE_* bits below; silu_gain > 0 for direct-SiLU
 * assignment; std_scale > 0 (the reference's R^-1/2 default or its explicit
 * standardized_logit_scale) for standardised logits. */
enum {
  DA_ROUTE_SILU_LOGITS = 1, /* a = 2 silu(l) */
  DA_ROUTE_STANDARDIZE = 2, /* a' = (a - mean) rsqrt(var + eps) std_scale */
  DA_ROUTE_DIRECT_SILU = 4, /* w = (2 / gain) silu(gain a') instead of softmax(beta a') */
  DA_ROUTE_NORM_INPUT = 8   /* l = (q / max(||q||, eps)) . Dk, else q . Dk */
};

/* Forward row stage.  S [rows, M] fp32 = q . Dk (raw q); q rows (dtype,
 * row stride q_stride) for the input norm; beta (device fp32 scalar, unused
 * with direct-SiLU).  Writes W [rows, M] bf16 (the assignment weights) and
 * stats [rows, 4] fp32 = (1/||q|| or 1, mean, inverse std, log-sum-exp of
 * beta a') for the backward. */
DA_API int da_route_var_weights(const float* S, int64_t rows, int M, const void* q, int64_t q_stride, int R,
                                int dtype, int flags, float silu_gain, float std_scale, const float* beta, float eps,
                                void* W, float* stats, void* stream);

/* Output normalisation: z [rows, R] (dtype) = r / max(||r||, eps) when
 * normalize, else r; out_norm [rows] = ||r||.  r [rows, R] fp32 = W . Dv^T. */
DA_API int da_route_var_output(const float* r, int64_t rows, int R, int dtype, int normalize, float eps, void* z,
                               float* out_norm, void* stream);

/* Its backward: g [rows, R] bf16 = dL/dr from z, dz (dtype) and out_norm,
 * and delta [rows] fp32 = <g, r> (r rebuilt from z and out_norm), which is
 * the softmax backward's <W, dW> in closed form. */
DA_API int da_route_var_output_bwd(const void* z, const void* dz, const float* out_norm, int64_t rows, int R,
                                   int dtype, int normalize, float eps, void* g, float* delta, void* stream);

/* Backward row stage.  S [rows, M] fp32 = q . Dk again, dW [rows, M] fp32 =
 * g . Dv, stats from the forward, delta from da_route_var_output_bwd (or
 * null: <W, dW> is then summed from dW).  Writes dS [rows, M] (dtype) = dL/d(q . Dk)
 * (the logit gradient times 1/||q||: dDk = q^T dS, u = dS . Dk^T), W
 * [rows, M] bf16 again (dDv = g^T W) and adds the beta gradient to *dbeta
 * (softmax assignment; may be null): one partial per 8 rows goes to
 * dbeta_work (fp32, at least ceil(rows / 8) elements, else DA_ERR_WORKSPACE)
 * and a second kernel adds them in a fixed order (bit-reproducible). */
DA_API int da_route_var_weights_bwd(const float* S, const float* dW, int64_t rows, int M, const float* stats,
                                    const float* delta, int flags, float silu_gain, float std_scale,
                                    const float* beta, int dtype, void* dS, void* W, float* dbeta,
                                    float* dbeta_work, int64_t dbeta_work_elems, void* stream);

/* Input-normalisation backward: dq [rows, R] (dtype, row stride dq_stride)
 * = u - q_hat <q_hat, u> (u = dS . Dk^T [rows, R] fp32) when normalize and
 * ||q|| > eps, else u. */
DA_API int da_route_var_input_bwd(const float* u, const void* q, int64_t q_stride, const float* stats, int64_t rows,
                                  int R, int dtype, int normalize, float eps, void* dq, int64_t dq_stride,
                                  void* stream);

/* ---- dictionary route, backward --------------------------------------
 * Replaces _DictionaryRouteFunction.backward (triton_kernels.py:1873-1981)
 * with its row-normalisation and scaled-softmax backward kernels
 * (:1410-1501) for the identity-logit softmax route; the two
 * dictionary-gradient GEMMs it leaves to cuBLAS (:1939, :1961) run on
 * da_gemm_splitk over the rows this call stores.  Same q addressing, R, M,
 * dtype, eps and flags as the forward call; R in {128, 256, 512}, M a
 * multiple of 128.  dict_key_t [M, R] (dtype), dict_value_t [M, R] bf16;
 * z / dz [groups, rows, R] (forward output and its gradient, dtype); lse /
 * out_norm from the forward.  Outputs: dq in the layout of q (dtype,
 * overwritten at the routed columns); p_out [groups, rows, M] bf16 = the
 * assignment weights; dl_out [groups, rows, M] dtype = the logit gradient
 * divided by the input norm (dDk = sum_groups q_g^T dl_out_g); g_out
 * [groups, rows, R] bf16 = gradient of the reconstruction (dDv = g_out^T
 * p_out); p_out and dl_out may both be null (then only dq and g_out are
 * written, as da_route_bwd_fused's row pass does); dbeta (may be null) is
 * accumulated (+=): with dbeta_work (fp32, at least 8 * groups *
 * ceil(rows / 128) elements, else DA_ERR_WORKSPACE) from per-warp partials
 * added in a fixed order (bit-reproducible), without it by fp32 atomics. */
DA_API int da_route_bwd(const void* q, int64_t rows, int64_t q_cols, int64_t q_row_stride, int groups,
                        int64_t group_col_stride, int64_t R, int64_t M, int dtype, const void* dict_key_t,
                        const void* dict_value_t, const float* beta, float eps, int normalize_input,
                        int normalize_output, const void* z, const void* dz, const float* lse, const float* out_norm,
                        void* dq, void* p_out, void* dl_out, void* g_out, float* dbeta, float* dbeta_work,
                        int64_t dbeta_work_elems, int* status, void* stream);

/* The whole route backward with deterministic dictionary gradients: replaces
 * _DictionaryRouteFunction.backward (triton_kernels.py:1873-1981) including
 * the two dictionary-gradient GEMMs it leaves to cuBLAS (:1706-1707 fused
 * path, :1938-1961 multi-kernel path) and its per-row beta gradient
 * (:1447-1501).  Arguments as da_route_bwd; R in {128, 256}, M a multiple of
 * 128, q_cols and group_col_stride multiples of 64, rows >= 128 (R = 128) or
 * >= 64 (R = 256); other shapes return DA_ERR_UNSUPPORTED (use da_route_bwd).
 * Outputs: dq as da_route_bwd; d_key, d_value [R, M] fp32 = dDk, dDv summed
 * over every routed row of every group (overwritten; either may be null);
 * dbeta [1] fp32 (overwritten; may be null).  No [rows, M] tensor is written:
 * an atom-parallel kernel recomputes the scores and dP per 128-atom tile with
 * the tile's dictionary rows resident in shared memory, keeps dDk / dDv in
 * TMEM over a chunk of rows and stores per-chunk partial sums, which a second
 * kernel adds in a fixed order, so the results are bit-identical from run to
 * run.  workspace: device memory of at least da_route_bwd_workspace_size()
 * bytes (16-byte aligned), else DA_ERR_WORKSPACE; its contents need no
 * initialisation. */
DA_API int64_t da_route_bwd_workspace_size(int64_t rows, int groups, int64_t R, int64_t M);
DA_API int da_route_bwd_fused(const void* q, int64_t rows, int64_t q_cols, int64_t q_row_stride, int groups,
                              int64_t group_col_stride, int64_t R, int64_t M, int dtype, const void* dict_key_t,
                              const void* dict_value_t, const float* beta, float eps, int normalize_input,
                              int normalize_output, const void* z, const void* dz, const float* lse,
                              const float* out_norm, void* dq, float* d_key, float* d_value, float* dbeta,
                              void* workspace, int64_t workspace_bytes, int* status, void* stream);

/* ---- outer routed attention with the map mix, forward -------------------
 * Replaces routed_attention_triton / _routed_attention_triton_forward
 * (triton_kernels.py:2290-2305, :2022-2090; math of ops.py:65-93) together
 * with score-map assembly (ops.py:96-139, as addressing) and the alpha mix
 * (modules.py:265-272):  Y = sum_s alpha_s softmax(gamma_s Q_s K_s^T) V.
 * Q/K rows: row(b, branch, t) = base + b*sb + branch*sbr + t inside [rows, R]
 * matrices of dtype `dtype`; map s concatenates `group` branches starting at
 * branch0[s] (host array of `maps` ints) and scales the dot product by
 * gamma_s / sqrt(group).  v: [B, T, D] bf16, D in {128, 256, 512};
 * maps <= 4 and maps*group*R <= 512.  weights: [maps] alpha (may be null when
 * maps == 1).  key_norm_max: [B*maps] upper bounds of ||k|| per (b, map), or
 * null to use key_norm_bound for all.  Outputs y [B, T, D] (dtype) and lse
 * [B, maps, T] fp32 (natural-log normaliser of every map's softmax). */
DA_API int da_attn_fwd(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr, const void* k,
                       int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr, const void* v, int B, int T,
                       int R, int D, int maps, int group, const int* branch0, int causal, int dtype,
                       const float* scales, const float* weights, const float* key_norm_max, float key_norm_bound,
                       void* y, float* lse, int* status, void* stream);

/* Bytes of device workspace da_attn_fwd_ws uses for these sizes: 0 when it
 * runs exactly as da_attn_fwd, -1 for invalid sizes.  With several maps and
 * few query tiles (their CTAs, two per pair, fit on the SMs of the current
 * device at once) the key range of every query tile is split over two pairs:
 * a first launch writes each share's per-map row sums, a second forms the
 * probabilities from the combined sums and each share's fp32 output, a third
 * adds the shares' outputs (in share order, so results repeat bit for bit). */
DA_API int64_t da_attn_fwd_workspace_size(int B, int T, int maps, int D);

/* da_attn_fwd with a caller-owned device workspace (16-byte aligned, at least
 * da_attn_fwd_workspace_size bytes, DA_ERR_WORKSPACE otherwise; ignored when
 * that size is 0).  Same reference interface and results as da_attn_fwd. */
DA_API int da_attn_fwd_ws(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr, const void* k,
                          int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr, const void* v, int B, int T,
                          int R, int D, int maps, int group, const int* branch0, int causal, int dtype,
                          const float* scales, const float* weights, const float* key_norm_max,
                          float key_norm_bound, void* y, float* lse, void* workspace, int64_t workspace_bytes,
                          int* status, void* stream);

/* ---- outer routed attention, backward -----------------------------------
 * Replaces the preprocess kernel of _routed_attention_triton_backward
 * (triton_kernels.py:2093-2160): delta[r] = <dy[r, :], y[r, :]> over `rows`
 * rows of D (D a multiple of 256; dtype bf16 or fp16), y the output of one map
 * (the forward output when there is one map).  The products of the backward
 * are da_attn_bwd_mixed below. */
DA_API int da_attn_bwd_delta(const void* dy, const void* y, int64_t rows, int D, int dtype, float* delta,
                             void* stream);

/* The whole backward of a (mixed) attention in one call, all maps at once
 * Replaces the dq, dk and dv kernels and the atomic d-scale of
 * _routed_attention_triton_backward (triton_kernels.py:2093-2263), plus the
 * gradient of the alpha mix (modules.py:265-272):
 * dP = dy.V^T is formed once per tile for every map and dV once from the
 * mixed probabilities.  Arguments as da_attn_fwd (branch0: host array of
 * `maps` ints), v / dy [B*T, D] in `dtype`, lse [B, maps, T] from the
 * forward.  delta [B, maps, T]: read when delta_given (one map: from
 * da_attn_bwd_delta on the saved output), else computed exactly by a first
 * sweep and written.  Accumulates (+=) into fp32 dq / dk (Q / K rows; may be
 * one buffer), dv [B*T, D], dscale [maps] (d gamma_s) and, when delta is
 * computed, dweight [maps] (d alpha_s); any output may be null.
 * D in {256, 512}; group*R in {128, 256, 512}; maps*group*R <= 512.
 * dscale and dweight are sums over every query row: the dQ kernel stores
 * one partial per (CTA, warp) in `workspace` (device memory of at least
 * da_attn_bwd_workspace_size(B, T, maps) bytes, 16-byte aligned; needed when
 * dscale or a computed dweight is requested, else DA_ERR_WORKSPACE) and a
 * second kernel adds them in a fixed order, so every output of this call is
 * bit-identical from run to run. */
DA_API int64_t da_attn_bwd_workspace_size(int B, int T, int maps);

/* Bytes of workspace with which da_attn_bwd_mixed and da_attn_bwd_mixed_ow run
 * their split form at these sizes on the current device: 0 when they never
 * split here, -1 for invalid sizes.  With several maps and few query tiles
 * (the split launches' CTAs, four per pair, fit on the SMs at once) every
 * pair's long row -- the keys of a query tile (delta, dQ), the queries of a
 * key tile (dK, dV) -- is split over two CTA pairs writing fp32 partial rows
 * into the workspace, which a combine adds in share order and stores (so
 * results repeat bit for bit; they differ from the unsplit form's only by
 * fp32 reassociation).  Without a given delta the delta sweep runs first, on
 * its own.  A call splits when the maps' branch ranges do not overlap and
 * `workspace_bytes` is at least this size; with less (but at least
 * da_attn_bwd_workspace_size) it runs unsplit.  A split call takes a given
 * delta as the exact row sums (as this entry's own sweep writes them) and
 * does not correct d gamma towards its own. */
DA_API int64_t da_attn_bwd_split_workspace_size(int B, int T, int R, int D, int maps, int group);
DA_API int da_attn_bwd_mixed(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr,
                             const void* k, int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr,
                             const void* v, const void* dy, int B, int T, int R, int D, int maps, int group,
                             const int* branch0, int causal, int dtype, const float* scales, const float* weights,
                             const float* lse, float* delta, int delta_given, float* dq, float* dk, float* dv,
                             float* dscale, float* dweight, void* workspace, int64_t workspace_bytes,
                             int* status, void* stream);

/* da_attn_bwd_mixed writing dq, dk and dv once each instead of adding to fp32
 * buffers: every gradient row the op produces is stored in the input dtype
 * (dq, dk: [rows, R]; dv: [B*T, D]), rows it does not produce are left as they
 * are; dscale and dweight are stored (=) rather than added to.  Needs maps
 * whose branch ranges do not overlap (each row then has one writer;
 * DA_ERR_UNSUPPORTED otherwise).  Same reference interface as
 * da_attn_bwd_mixed, without the zero-filled fp32 buffers and the casts the
 * module path otherwise runs around it. */
DA_API int da_attn_bwd_mixed_ow(const void* q, int64_t q_rows, int64_t q_base, int64_t q_sb, int64_t q_sbr,
                                const void* k, int64_t k_rows, int64_t k_base, int64_t k_sb, int64_t k_sbr,
                                const void* v, const void* dy, int B, int T, int R, int D, int maps, int group,
                                const int* branch0, int causal, int dtype, const float* scales, const float* weights,
                                const float* lse, float* delta, int delta_given, void* dq, void* dk, void* dv,
                                float* dscale, float* dweight, void* workspace, int64_t workspace_bytes,
                                int* status, void* stream);
/* ---- dense GEMM (fused Q/K projection and its backward) -----------------
 * Replaces the cuBLAS GEMM of _project_query_key (modules.py:143-157,
 * F.linear(x, cat(W_q, W_k))) and its autograd backward.
 * C[M, N] (+)= sum_k A(m, k) B(n, k), fp16/bf16 operands, fp32 accumulation.
 * A is [M, K] row-major (a_mn_major = 0) or [K, M] (= 1), leading dimension
 * lda; B is [N, K] (b_mn_major = 0) or [K, N] (= 1).  C is [M, N] with
 * leading dimension ldc, in the operand dtype or fp32 (out_f32); accumulate
 * (fp32 only) adds to C.  N must be a multiple of 128; lda/ldb/ldc multiples
 * of 8 elements. */
DA_API int da_gemm(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major, void* C,
                   int64_t ldc, int64_t M, int64_t N, int64_t K, int dtype, int out_f32, int accumulate, int* status,
                   void* stream);

/* The GEMM with an epilogue and an optional second K segment, for the
 * Linear layers around the routed attention (no reference counterpart of its
 * own: it replaces the cuBLAS calls and the eager GELU of the value-projection
 * backward, the output projection (modules.py:272) and the feed-forward
 * branch (modules.py:339-346)):
 *   C[M, N] = act(sum_k A(m, k) B(n, k) [+ sum_k A2(m, k) B2(n, k)] + bias[n])
 * in the operand dtype (fp32 accumulation).  A [M, K] row-major (K-major);
 * B [N, K] (b_mn_major = 0) or [K, N] (= 1); A2 [M, K2] / B2 likewise (both
 * null for one segment; with two, K is a multiple of 64).  bias [N] in the
 * operand dtype or null.  act 0: none; 1: GELU (erf form), with the
 * pre-activation also stored in aux [M, N] (row stride ldaux) when aux is
 * not null; 2: times GELU'(aux[m, n]) (the backward of act 1 through the
 * next product).  N a multiple of 128; strides multiples of 8 elements. */
DA_API int da_gemm_ex(const void* A, int64_t lda, const void* B, int64_t ldb, int b_mn_major, int64_t K,
                      const void* A2, int64_t lda2, const void* B2, int64_t ldb2, int64_t K2, void* C, int64_t ldc,
                      int64_t M, int64_t N, int dtype, const void* bias, int act, void* aux, int64_t ldaux,
                      int* status, void* stream);

/* Several projections of one input in one launch: C_s = A . B_s^T (+ bias_s)
 * for nseg <= 3 weight matrices B_s [N_s, K] (row stride ldb[s]) sharing A
 * [M, K] (row stride lda); C_s [M, N_s] with row stride ldc[s] in out_dtype[s]
 * (DA_F16 / DA_BF16 / DA_F32); bias_s [N_s] in the operand dtype, or null.
 * Replaces F.linear(x, cat(W_q, W_k)) (modules.py:143-157) together with the
 * value projection, writing V in the bf16 the attention consumes.  Every N_s
 * a multiple of 128.  B, ldb, N, C, ldc, out_dtype, bias are host arrays. */
DA_API int da_gemm_segments(const void* A, int64_t lda, int64_t M, int64_t K, int dtype, int nseg,
                            const void* const* B, const int64_t* ldb, const int64_t* N, void* const* C,
                            const int64_t* ldc, const int* out_dtype, const void* const* bias, int* status,
                            void* stream);

/* Split-K variant for reductions over many rows (the dictionary gradients
 * dDk = q^T dL and dDv = g^T P, triton_kernels.py:1939, :1961):
 * C[M, N] += sum_k A(m, k) B(n, k) in fp32, the K range split over `splits`
 * CTAs per output tile (0 = pick from the SM count), so C must hold its
 * initial value (e.g. zeros).  M and N multiples of 128.  With a workspace
 * (fp32, at least da_gemm_splitk_workspace_elems(M, N, K, splits) elements,
 * 16-byte aligned, else DA_ERR_WORKSPACE) every split stores its partial sum
 * there and a second kernel adds them to C in split order: the result is
 * bit-identical from run to run.  With workspace = null the partial sums are
 * added with fp32 atomics, whose order (and so the last bits) varies. */
DA_API int64_t da_gemm_splitk_workspace_elems(int64_t M, int64_t N, int64_t K, int splits);
DA_API int da_gemm_splitk(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major,
                          float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int dtype, int splits,
                          float* workspace, int64_t workspace_elems, int* status, void* stream);

/* da_gemm_splitk storing C once instead of adding to it: C = A.B^T in fp32
 * (c_dtype DA_F32) or in the operand dtype (c_dtype = dtype; DA_ERR_DTYPE
 * otherwise), the splits' partial sums (workspace required, else
 * DA_ERR_WORKSPACE) added in split order and rounded once.  For weight
 * gradients stored in the parameters' dtype without a zero-filled fp32 buffer
 * and a cast. */
DA_API int da_gemm_splitk_store(const void* A, int64_t lda, int a_mn_major, const void* B, int64_t ldb, int b_mn_major,
                                void* C, int64_t ldc, int c_dtype, int64_t M, int64_t N, int64_t K, int dtype,
                                int splits, float* workspace, int64_t workspace_elems, int* status, void* stream);

/* The same sum over several groups at once: C [M, N] fp32 += sum over g < groups and k < K_group of
 * A(m, g, k) B(n, g, k) with A MN-major, its group g starting a_group_cols columns to the right
 * (A(m, g, k) = A[k * lda + g * a_group_cols + m]), and B MN-major with the groups stacked along K
 * (B(n, g, k) = B[(g * K_group + k) * ldb + n]).  This is the key-dictionary gradient of the route
 * backward, dDk = sum_groups q_g^T dL'_g (triton_kernels.py:1939), in one launch instead of one per
 * group.  K_group a multiple of 64, M and N multiples of 128, a_group_cols a multiple of 8.  Workspace as
 * da_gemm_splitk with K = K_group * groups. */
DA_API int da_gemm_splitk_grouped(const void* A, int64_t lda, int64_t a_group_cols, const void* B, int64_t ldb,
                                  float* C, int64_t ldc, int64_t M, int64_t N, int64_t K_group, int groups, int dtype,
                                  int splits, float* workspace, int64_t workspace_elems, int* status, void* stream);

/* Bias gradient of a Linear layer: out[c] = sum over rows of d[r, c] in fp32
 * (d: [rows, cols] bf16 / fp16 with row stride ld; cols and ld multiples of 8,
 * d 16-byte aligned).  Replaces the autograd column sum of nn.Linear's bias
 * gradient in the block layers (reference modules.py:212, :272, :339-346).
 * Partial sums per row chunk go to `workspace` (fp32, at least
 * da_col_sum_workspace_elems(rows, cols) elements; DA_ERR_WORKSPACE otherwise)
 * and are added in a fixed order, so the result is bit-reproducible. */
DA_API int64_t da_col_sum_workspace_elems(int64_t rows, int64_t cols);
DA_API int da_col_sum(const void* d, int64_t rows, int64_t cols, int64_t ld, int dtype, float* out,
                      float* workspace, int64_t workspace_elems, void* stream);

/* ---- residual add + LayerNorm around the block -----------------------
 * Replaces x + branch followed by nn.LayerNorm in DoubleAttentionBlock.forward
 * (modules.py:294-356) and the final norm of DoubleAttentionLM (modules.py:415-460).
 * Forward: x_out = x + branch (fp32 [rows, D]; branch in branch_dtype, or null,
 * then x_out is not written and x itself is normalised), y = LayerNorm(x_out) *
 * gamma + beta written in y_dtype, per-row mean and rstd (fp32 [rows]).
 * D in {256, 512, 768, 1024}; every pointer 16-byte aligned. */
DA_API int da_add_layernorm_fwd(const float* x, const void* branch, int branch_dtype, const float* gamma,
                                const float* beta, int64_t rows, int64_t D, float eps, float* x_out, void* y,
                                int y_dtype, float* mean, float* rstd, void* stream);
/* Backward: dx = d_res (fp32, or null for 0) + LayerNorm backward of dy (in
 * dy_dtype); d_branch (optional, branch_dtype) = dx; dgamma, dbeta (fp32 [D],
 * optional) written from per-block partial sums in `partial`, a caller-provided
 * fp32 buffer of [partial_blocks, 2, D] with partial_blocks =
 * da_layernorm_bwd_blocks(rows) (DA_ERR_WORKSPACE otherwise). */
DA_API int da_layernorm_bwd_blocks(int64_t rows);
DA_API int da_add_layernorm_bwd(const void* dy, int dy_dtype, const float* d_res, const float* x_out,
                                const float* mean, const float* rstd, const float* gamma, int64_t rows, int64_t D,
                                float* dx, void* d_branch, int branch_dtype, float* partial, int partial_blocks,
                                float* dgamma, float* dbeta, void* stream);

/* ---- building-block check -------------------------------------------
 * No reference counterpart: D[128, n] = A[128, k] * B^T computed by one
 * tcgen05 tile (cta_group 1 or 2) for testing the descriptor layouts.
 * A: [128, k] bf16; B: [n, k] bf16 (b_mn_major = 0) or [k, n] (= 1). */
/* No reference counterpart: the failure-detection path of every kernel wait.
 * One CTA waits on a barrier that nothing signals, bounded by timeout_ns
 * (at most 0.1 s); when the limit runs out the wait records DA_DEV_TIMEOUT
 * in status[0] and `site` in status[1] (status: int32 [2] on the device,
 * zeroed by the caller) and a second waiter of the same CTA leaves on the
 * CTA's abort flag.  The kernel then returns normally and the context stays
 * usable.  elapsed_ns (device uint64 [2], may be null) receives how long each
 * waiter waited. */
DA_API int da_selftest_wait_timeout(int64_t timeout_ns, int site, int* status, uint64_t* elapsed_ns, void* stream);

DA_API int da_selftest_mma(int cta_group, int n, int b_mn_major, int k, const void* A, const void* B, float* D,
                    int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DA_B200_H_ */
