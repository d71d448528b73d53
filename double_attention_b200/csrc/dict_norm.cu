// Column normalisation of a dictionary bank and its backward.
//
// Forward (reference: src/double_attention/modules.py:45-48, F.normalize over
// dim 0, then the AMP cast at modules.py:229-231):
//   denom_j = max(||raw[:, j]||_2, eps),  D[:, j] = raw[:, j] / denom_j,
// written in the compute dtype, optionally also transposed ([M, R]), plus the
// largest 2-norm over the ROUNDED output columns (an upper bound the routing
// kernels use for their fixed softmax offset).
//
// Backward: y = raw / denom,
//   d raw[:, j] = (g[:, j] - y[:, j] <g[:, j], y[:, j]>) / denom_j   if ||raw[:, j]|| > eps
//               = g[:, j] / eps                                     otherwise.
// The layout is memory-bound and tiny (R*M <= 1.5 M elements): one thread
// per column, coalesced across columns.
#include "common.cuh"
#include "host_util.h"

namespace da {
namespace {

// One CTA per 32 columns: the [R, 32] tile is staged in shared memory with
// coalesced row reads, column norms are reduced across 8 row groups, and both
// the [R, M] and the transposed [M, R] outputs are written coalesced.
template <typename T>
__global__ void __launch_bounds__(256) dict_norm_fwd_kernel(const float* __restrict__ raw, int R, int M, float eps,
                                                            T* __restrict__ out, T* __restrict__ out_t,
                                                            float* __restrict__ denom_out,
                                                            float* __restrict__ max_norm) {
  extern __shared__ float tile[];          // [R][33] (padded)
  grid_dependency_wait();
  grid_launch_dependents();
  __shared__ float part[8][33], part2[8][33], inv[32];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int j0 = blockIdx.x * 32, j = j0 + tx;
  float ss = 0.f;
  for (int r = ty; r < R; r += 8) {
    const float v = j < M ? raw[(size_t)r * M + j] : 0.f;
    tile[r * 33 + tx] = v;
    ss = fmaf(v, v, ss);
  }
  part[ty][tx] = ss;
  __syncthreads();
  if (ty == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += part[i][tx];
    const float denom = fmaxf(sqrtf(t), eps);
    inv[tx] = denom;
    if (denom_out && j < M) denom_out[j] = denom;
  }
  __syncthreads();
  const float denom = inv[tx];
  float rs = 0.f;
  for (int r = ty; r < R; r += 8) {
    const T y = from_f32<T>(tile[r * 33 + tx] / denom);
    const float yr = static_cast<float>(y);
    rs = fmaf(yr, yr, rs);
    tile[r * 33 + tx] = yr;
    if (out && j < M) out[(size_t)r * M + j] = y;
  }
  part2[ty][tx] = rs;
  __syncthreads();
  if (max_norm && ty == 0 && j < M) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += part2[i][tx];
    atomicMax(reinterpret_cast<int*>(max_norm), __float_as_int(sqrtf(t)));
  }
  if (out_t) {
    // column c of the tile becomes row (j0 + c) of out_t: consecutive threads
    // write consecutive elements of that row.
    for (int c = ty; c < 32; c += 8) {
      if (j0 + c >= M) break;
      T* dst = out_t + (size_t)(j0 + c) * R;
      for (int r = tx; r < R; r += 32) dst[r] = from_f32<T>(tile[r * 33 + c]);
    }
  }
}

// Key and value banks in one launch (grid.y = 0: key in the compute dtype,
// 1: value in bf16), eight columns per CTA so that even a 512-atom bank
// spreads over 128 CTAs.  Each thread keeps its column's rows in shared
// memory between the norm and the write passes.
template <typename TR, typename TK>
__global__ void __launch_bounds__(256) dict_norm_pair_kernel(const TR* __restrict__ raw_key,
                                                             const TR* __restrict__ raw_value, int R, int M,
                                                             float eps, TK* __restrict__ key, TK* __restrict__ key_t,
                                                             float* __restrict__ key_denom,
                                                             float* __restrict__ key_max,
                                                             __nv_bfloat16* __restrict__ value,
                                                             __nv_bfloat16* __restrict__ value_t,
                                                             float* __restrict__ value_denom) {
  extern __shared__ float tile8[];  // [R][9]
  grid_dependency_wait();
  grid_launch_dependents();
  __shared__ float part[32][9], colden[8];
  const bool is_key = blockIdx.y == 0;
  const TR* raw = is_key ? raw_key : raw_value;
  const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;
  const int j0 = blockIdx.x * 8, j = j0 + tx;
  const bool col = j < M;
  float ss = 0.f;
#pragma unroll 8
  for (int r = ty; r < R; r += 32) {
    const float v = col ? static_cast<float>(raw[(size_t)r * M + j]) : 0.f;
    tile8[r * 9 + tx] = v;
    ss = fmaf(v, v, ss);
  }
  part[ty][tx] = ss;
  __syncthreads();
  if (ty == 0) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) t += part[i][tx];
    const float d = fmaxf(sqrtf(t), eps);
    colden[tx] = d;
    float* dout = is_key ? key_denom : value_denom;
    if (dout && col) dout[j] = d;
  }
  __syncthreads();
  const float inv = 1.f / colden[tx];
  float rs = 0.f;
#pragma unroll 8
  for (int r = ty; r < R; r += 32) {
    const float x = tile8[r * 9 + tx] * inv;
    float yr;
    if (is_key) {
      const TK y = from_f32<TK>(x);
      yr = static_cast<float>(y);
      if (key && col) key[(size_t)r * M + j] = y;
    } else {
      const __nv_bfloat16 y = __float2bfloat16_rn(x);
      yr = __bfloat162float(y);
      if (value && col) value[(size_t)r * M + j] = y;
    }
    rs = fmaf(yr, yr, rs);
    tile8[r * 9 + tx] = yr;
  }
  part[ty][tx] = rs;
  __syncthreads();
  if (is_key && key_max && ty == 0 && col) {
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) t += part[i][tx];
    atomicMax(reinterpret_cast<int*>(key_max), __float_as_int(sqrtf(t)));
  }
  // transposed rows j0 .. j0+7, R elements each, written by all 256 threads
  for (int c = 0; c < 8 && j0 + c < M; ++c) {
    if (is_key) {
      if (!key_t) break;
      TK* dst = key_t + (size_t)(j0 + c) * R;
      for (int r = threadIdx.x; r < R; r += 256) dst[r] = from_f32<TK>(tile8[r * 9 + c]);
    } else {
      if (!value_t) break;
      __nv_bfloat16* dst = value_t + (size_t)(j0 + c) * R;
      for (int r = threadIdx.x; r < R; r += 256) dst[r] = __float2bfloat16_rn(tile8[r * 9 + c]);
    }
  }
}

// grad (and grad_t, the same gradient given in [M, R] layout) are summed.
// One CTA per 32 columns, both operands staged in shared memory.
// raw banks of type TR (fp32, or the half type of a module cast to it; read exactly as fp32), the gradient
// stored as TG (fp32, added to when `accumulate`, else rounded once to TG)
template <typename TR, typename TG>
__global__ void __launch_bounds__(256) dict_norm_bwd_kernel(const TR* __restrict__ raw,
                                                            const float* __restrict__ denom,
                                                            const float* __restrict__ grad,
                                                            const float* __restrict__ grad_t, int R, int M, float eps,
                                                            TG* __restrict__ grad_raw, int accumulate) {
  extern __shared__ float smem_f[];
  grid_dependency_wait();
  grid_launch_dependents();
  float* tx_ = smem_f;              // [R][33] raw
  float* tg = smem_f + R * 33;      // [R][33] gradient
  __shared__ float part_ss[8][33], part_dot[8][33], colv[2][32];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int j0 = blockIdx.x * 32, j = j0 + tx;
  for (int r = ty; r < R; r += 8) {
    tx_[r * 33 + tx] = j < M ? static_cast<float>(raw[(size_t)r * M + j]) : 0.f;
    tg[r * 33 + tx] = (grad && j < M) ? grad[(size_t)r * M + j] : 0.f;
  }
  __syncthreads();
  if (grad_t) {
    for (int c = ty; c < 32; c += 8) {
      if (j0 + c >= M) break;
      const float* src = grad_t + (size_t)(j0 + c) * R;
      for (int r = tx; r < R; r += 32) tg[r * 33 + c] += src[r];
    }
    __syncthreads();
  }
  const float d = j < M ? denom[j] : 1.f;
  float ss = 0.f, dot = 0.f;
  for (int r = ty; r < R; r += 8) {
    const float x = tx_[r * 33 + tx], g = tg[r * 33 + tx];
    ss = fmaf(x, x, ss);
    dot = fmaf(g, x / d, dot);
  }
  part_ss[ty][tx] = ss;
  part_dot[ty][tx] = dot;
  __syncthreads();
  if (ty == 0) {
    float a = 0.f, b = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a += part_ss[i][tx];
      b += part_dot[i][tx];
    }
    colv[0][tx] = a;
    colv[1][tx] = b;
  }
  __syncthreads();
  const bool clamped = !(sqrtf(colv[0][tx]) > eps);
  const float cdot = colv[1][tx];
  if (j < M) {
    for (int r = ty; r < R; r += 8) {
      const float x = tx_[r * 33 + tx], g = tg[r * 33 + tx];
      const float dx = clamped ? g / eps : (g - (x / d) * cdot) / d;
      TG* dst = grad_raw + (size_t)r * M + j;
      if constexpr (std::is_same<TG, float>::value) *dst = accumulate ? *dst + dx : dx;
      else *dst = static_cast<TG>(dx);
    }
  }
}

}  // namespace
}  // namespace da

extern "C" int da_dict_norm_fwd(const float* raw, int64_t R, int64_t M, float eps, int out_dtype, void* out,
                                void* out_t, float* denom, float* max_col_norm, void* stream) {
  using namespace da;
  if (!raw) return DA_ERR_NULL;
  if (int rc = bind_device(raw)) return rc;
  if (R <= 0 || M <= 0 || R > 1536 || M > (1 << 24)) return DA_ERR_SHAPE;
  if (out_dtype != DA_BF16 && out_dtype != DA_F16) return DA_ERR_DTYPE;
  if (out_t && (reinterpret_cast<uintptr_t>(out_t) & 15)) return DA_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (max_col_norm && cudaMemsetAsync(max_col_norm, 0, sizeof(float), st) != cudaSuccess) return record_cuda_error();
  const dim3 grid((unsigned)((M + 31) / 32)), block(256);
  const size_t smem = (size_t)R * 33 * sizeof(float);
  if (smem > 200 * 1024) return DA_ERR_SHAPE;
  if (out_dtype == DA_BF16) {
    auto k = dict_norm_fwd_kernel<__nv_bfloat16>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return record_cuda_error();
    if (int rc = launch_kernel(k, grid, block, smem, st, false, raw, (int)R, (int)M, eps, (__nv_bfloat16*)out,
                               (__nv_bfloat16*)out_t, denom, max_col_norm))
      return rc;
  } else {
    auto k = dict_norm_fwd_kernel<__half>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return record_cuda_error();
    if (int rc = launch_kernel(k, grid, block, smem, st, false, raw, (int)R, (int)M, eps, (__half*)out,
                               (__half*)out_t, denom, max_col_norm))
      return rc;
  }
  return DA_OK;
}

namespace {

template <typename TR, typename TG>
int launch_norm_bwd(const void* raw, const float* denom, const float* grad, const float* grad_t, int64_t R, int64_t M,
                    float eps, void* grad_raw, int accumulate, cudaStream_t st) {
  using namespace da;
  const size_t smem = 2 * (size_t)R * 33 * sizeof(float);
  auto k = dict_norm_bwd_kernel<TR, TG>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return record_cuda_error();
  return launch_kernel(k, dim3((unsigned)((M + 31) / 32)), dim3(256), smem, st, false, static_cast<const TR*>(raw),
                       denom, grad, grad_t, (int)R, (int)M, eps, static_cast<TG*>(grad_raw), accumulate);
}

template <typename TR>
int launch_norm_bwd_to(int grad_dtype, const void* raw, const float* denom, const float* grad, const float* grad_t,
                       int64_t R, int64_t M, float eps, void* grad_raw, int accumulate, cudaStream_t st) {
  if (grad_dtype == DA_F32)
    return launch_norm_bwd<TR, float>(raw, denom, grad, grad_t, R, M, eps, grad_raw, accumulate, st);
  if (grad_dtype == DA_BF16)
    return launch_norm_bwd<TR, __nv_bfloat16>(raw, denom, grad, grad_t, R, M, eps, grad_raw, 0, st);
  return launch_norm_bwd<TR, __half>(raw, denom, grad, grad_t, R, M, eps, grad_raw, 0, st);
}

}  // namespace

extern "C" int da_dict_norm_bwd_typed(const void* raw, int raw_dtype, const float* denom, const float* grad,
                                      const float* grad_t, int64_t R, int64_t M, float eps, void* grad_raw,
                                      int grad_dtype, int accumulate, void* stream) {
  using namespace da;
  if (!raw || !denom || !grad_raw || (!grad && !grad_t)) return DA_ERR_NULL;
  if (int rc = bind_device(raw)) return rc;
  if (R <= 0 || M <= 0 || R > (1 << 16) || M > (1 << 24)) return DA_ERR_SHAPE;
  for (int d : {raw_dtype, grad_dtype})
    if (d != DA_F32 && d != DA_BF16 && d != DA_F16) return DA_ERR_DTYPE;
  if (accumulate && grad_dtype != DA_F32) return DA_ERR_UNSUPPORTED;
  if (2 * (size_t)R * 33 * sizeof(float) > 200 * 1024) return DA_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (raw_dtype == DA_F32)
    return launch_norm_bwd_to<float>(grad_dtype, raw, denom, grad, grad_t, R, M, eps, grad_raw, accumulate, st);
  if (raw_dtype == DA_BF16)
    return launch_norm_bwd_to<__nv_bfloat16>(grad_dtype, raw, denom, grad, grad_t, R, M, eps, grad_raw, accumulate,
                                             st);
  return launch_norm_bwd_to<__half>(grad_dtype, raw, denom, grad, grad_t, R, M, eps, grad_raw, accumulate, st);
}

extern "C" int da_dict_norm_bwd(const float* raw, const float* denom, const float* grad, const float* grad_t,
                                int64_t R, int64_t M, float eps, float* grad_raw, int accumulate, void* stream) {
  return da_dict_norm_bwd_typed(raw, DA_F32, denom, grad, grad_t, R, M, eps, grad_raw, DA_F32, accumulate, stream);
}

// Largest column 2-norm of a [R, M] dictionary in fp16/bf16 (for callers that
// pass their own normalised dictionaries to the routing kernels).
namespace da {
namespace {
template <typename T>
__global__ void col_norm_max_kernel(const T* __restrict__ d, int R, int M, float* __restrict__ out) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= M) return;
  float ss = 0.f;
  for (int r = 0; r < R; ++r) {
    const float v = static_cast<float>(d[(size_t)r * M + j]);
    ss = fmaf(v, v, ss);
  }
  atomicMax(reinterpret_cast<int*>(out), __float_as_int(sqrtf(ss)));
}
}  // namespace
}  // namespace da

extern "C" int da_col_norm_max(const void* dict, int64_t R, int64_t M, int dtype, float* out, void* stream) {
  using namespace da;
  if (!dict || !out) return DA_ERR_NULL;
  if (int rc = bind_device(dict)) return rc;
  if (R <= 0 || M <= 0) return DA_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(out, 0, sizeof(float), st) != cudaSuccess) return record_cuda_error();
  const dim3 grid((unsigned)((M + 127) / 128)), block(128);
  if (dtype == DA_BF16)
    return launch_kernel(col_norm_max_kernel<__nv_bfloat16>, grid, block, 0, st, false,
                         (const __nv_bfloat16*)dict, (int)R, (int)M, out);
  if (dtype == DA_F16)
    return launch_kernel(col_norm_max_kernel<__half>, grid, block, 0, st, false, (const __half*)dict, (int)R,
                         (int)M, out);
  return DA_ERR_DTYPE;
}

extern "C" int da_dict_norm_pair_fwd(const void* raw_key, const void* raw_value, int raw_dtype, int64_t R,
                                     int64_t M, float eps, int key_dtype, void* key, void* key_t, float* key_denom,
                                     float* key_max, void* value, void* value_t, float* value_denom, void* stream) {
  using namespace da;
  if (!raw_key) return DA_ERR_NULL;
  if (int rc = bind_device(raw_key)) return rc;
  if (R <= 0 || M <= 0 || R > 1536 || M > (1 << 24)) return DA_ERR_SHAPE;
  if (key_dtype != DA_BF16 && key_dtype != DA_F16) return DA_ERR_DTYPE;
  if (raw_dtype != DA_F32 && raw_dtype != DA_BF16 && raw_dtype != DA_F16) return DA_ERR_DTYPE;
  const bool with_value = raw_value && (value || value_t || value_denom);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (key_max && cudaMemsetAsync(key_max, 0, sizeof(float), st) != cudaSuccess) return record_cuda_error();
  const dim3 grid((unsigned)((M + 7) / 8), with_value ? 2u : 1u), block(256);
  const size_t smem = (size_t)R * 9 * sizeof(float);
  auto run = [&](auto kern, auto raw_tag, auto key_tag) -> int {
    using TR = decltype(raw_tag);
    using TK = decltype(key_tag);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return record_cuda_error();
    return launch_kernel(kern, grid, block, smem, st, false, static_cast<const TR*>(raw_key),
                         static_cast<const TR*>(raw_value), (int)R, (int)M, eps, static_cast<TK*>(key),
                         static_cast<TK*>(key_t), key_denom, key_max, static_cast<__nv_bfloat16*>(value),
                         static_cast<__nv_bfloat16*>(value_t), value_denom);
  };
  const bool kb = key_dtype == DA_BF16;
  if (raw_dtype == DA_F32)
    return kb ? run(dict_norm_pair_kernel<float, __nv_bfloat16>, float{}, __nv_bfloat16{})
              : run(dict_norm_pair_kernel<float, __half>, float{}, __half{});
  if (raw_dtype == DA_BF16)
    return kb ? run(dict_norm_pair_kernel<__nv_bfloat16, __nv_bfloat16>, __nv_bfloat16{}, __nv_bfloat16{})
              : run(dict_norm_pair_kernel<__nv_bfloat16, __half>, __nv_bfloat16{}, __half{});
  return kb ? run(dict_norm_pair_kernel<__half, __nv_bfloat16>, __half{}, __nv_bfloat16{})
            : run(dict_norm_pair_kernel<__half, __half>, __half{}, __half{});
}

// ---- temperatures: beta = exp(clamp(log_beta)), gamma_s = exp(clamp(log_gamma_s)) in fp32
namespace da {
namespace {
template <typename T>
DA_DEV float load_as_float(const void* p, int i) {
  return static_cast<float>(static_cast<const T*>(p)[i]);
}
DA_DEV float load_any(const void* p, int dtype, int i) {
  if (dtype == DA_F32) return static_cast<const float*>(p)[i];
  if (dtype == DA_BF16) return load_as_float<__nv_bfloat16>(p, i);
  return load_as_float<__half>(p, i);
}
__global__ void temperatures_kernel(const void* log_beta, int beta_dtype, float beta_lo, float beta_hi,
                                    const void* log_scales, int scales_dtype, int maps, float scale_lo,
                                    float scale_hi, float* beta_out, float* scales_out) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int i = threadIdx.x;
  if (i == 0 && log_beta) beta_out[0] = expf(fminf(fmaxf(load_any(log_beta, beta_dtype, 0), beta_lo), beta_hi));
  if (i < maps && log_scales)
    scales_out[i] = expf(fminf(fmaxf(load_any(log_scales, scales_dtype, i), scale_lo), scale_hi));
}
// Backward of exp(clamp(log, lo, hi)): g * value where lo <= log <= hi, else 0, in fp32, rounded once to
// the log's dtype.
DA_DEV void store_any(void* p, int dtype, int i, float v) {
  if (dtype == DA_F32) static_cast<float*>(p)[i] = v;
  else if (dtype == DA_BF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<__half*>(p)[i] = __float2half_rn(v);
}
__global__ void temperatures_bwd_kernel(const void* log_beta, int beta_dtype, float beta_lo, float beta_hi,
                                        const float* beta, const float* g_beta, void* grad_log_beta,
                                        const void* log_scales, int scales_dtype, int maps, float scale_lo,
                                        float scale_hi, const float* scales, const float* g_scales,
                                        void* grad_log_scales) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int i = threadIdx.x;
  if (i == 0 && g_beta) {
    const float x = load_any(log_beta, beta_dtype, 0);
    store_any(grad_log_beta, beta_dtype, 0, g_beta[0] * beta[0] * ((x >= beta_lo && x <= beta_hi) ? 1.f : 0.f));
  }
  if (i < maps && g_scales) {
    const float x = load_any(log_scales, scales_dtype, i);
    store_any(grad_log_scales, scales_dtype, i,
              g_scales[i] * scales[i] * ((x >= scale_lo && x <= scale_hi) ? 1.f : 0.f));
  }
}
}  // namespace
}  // namespace da

extern "C" int da_temperatures_bwd(const void* log_beta, int beta_dtype, float beta_lo, float beta_hi,
                                   const float* beta, const float* g_beta, void* grad_log_beta,
                                   const void* log_scales, int scales_dtype, int maps, float scale_lo, float scale_hi,
                                   const float* scales, const float* g_scales, void* grad_log_scales, void* stream) {
  using namespace da;
  if (!g_beta && !g_scales) return DA_ERR_NULL;
  if (g_beta && (!log_beta || !beta || !grad_log_beta)) return DA_ERR_NULL;
  if (g_scales && (!log_scales || !scales || !grad_log_scales)) return DA_ERR_NULL;
  if (int rc = bind_device(g_beta ? (const void*)g_beta : (const void*)g_scales)) return rc;
  if (maps < 0 || maps > 32) return DA_ERR_SHAPE;
  for (int d : {beta_dtype, scales_dtype})
    if (d != DA_F32 && d != DA_BF16 && d != DA_F16) return DA_ERR_DTYPE;
  return launch_kernel(temperatures_bwd_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), false,
                       log_beta, beta_dtype, beta_lo, beta_hi, beta, g_beta, grad_log_beta, log_scales, scales_dtype,
                       maps, scale_lo, scale_hi, scales, g_scales, grad_log_scales);
}

extern "C" int da_temperatures(const void* log_beta, int beta_dtype, float beta_lo, float beta_hi,
                               const void* log_scales, int scales_dtype, int maps, float scale_lo, float scale_hi,
                               float* beta_out, float* scales_out, void* stream) {
  using namespace da;
  if ((log_beta && !beta_out) || (log_scales && !scales_out) || (!log_beta && !log_scales)) return DA_ERR_NULL;
  if (int rc = bind_device(log_beta ? log_beta : log_scales)) return rc;
  if (maps < 0 || maps > 32) return DA_ERR_SHAPE;
  for (int d : {beta_dtype, scales_dtype})
    if (d != DA_F32 && d != DA_BF16 && d != DA_F16) return DA_ERR_DTYPE;
  return launch_kernel(temperatures_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), false, log_beta,
                       beta_dtype, beta_lo, beta_hi, log_scales, scales_dtype, maps, scale_lo, scale_hi, beta_out,
                       scales_out);
}
