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

template <typename T>
__global__ void dict_norm_fwd_kernel(const float* __restrict__ raw, int R, int M, float eps, T* __restrict__ out,
                                     T* __restrict__ out_t, float* __restrict__ denom_out,
                                     float* __restrict__ max_norm) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= M) return;
  float ss = 0.f;
  for (int r = 0; r < R; ++r) {
    const float v = raw[(size_t)r * M + j];
    ss = fmaf(v, v, ss);
  }
  const float denom = fmaxf(sqrtf(ss), eps);
  if (denom_out) denom_out[j] = denom;
  float rounded_ss = 0.f;
  for (int r0 = 0; r0 < R; r0 += 8) {
    T vals[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = r0 + i;
      const float y = r < R ? raw[(size_t)r * M + j] / denom : 0.f;
      vals[i] = from_f32<T>(y);
      const float yr = static_cast<float>(vals[i]);
      rounded_ss = fmaf(yr, yr, rounded_ss);
      if (out && r < R) out[(size_t)r * M + j] = vals[i];
    }
    if (out_t) {
      T* dst = out_t + (size_t)j * R + r0;
      if (r0 + 8 <= R && (R % 8) == 0) {
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<uint4*>(vals);
      } else {
        for (int i = 0; i < 8 && r0 + i < R; ++i) dst[i] = vals[i];
      }
    }
  }
  if (max_norm) atomicMax(reinterpret_cast<int*>(max_norm), __float_as_int(sqrtf(rounded_ss)));
}

// grad (and grad_t, the same gradient given in [M, R] layout) are summed.
__global__ void dict_norm_bwd_kernel(const float* __restrict__ raw, const float* __restrict__ denom, const float* __restrict__ grad,
                                     const float* __restrict__ grad_t, int R, int M, float eps,
                                     float* __restrict__ grad_raw, int accumulate) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= M) return;
  const float d = denom[j];
  float ss = 0.f, dot = 0.f;
  for (int r = 0; r < R; ++r) {
    const float x = raw[(size_t)r * M + j];
    float g = grad ? grad[(size_t)r * M + j] : 0.f;
    if (grad_t) g += grad_t[(size_t)j * R + r];
    ss = fmaf(x, x, ss);
    dot = fmaf(g, x / d, dot);
  }
  const bool clamped = !(sqrtf(ss) > eps);
  for (int r = 0; r < R; ++r) {
    const float x = raw[(size_t)r * M + j];
    float g = grad ? grad[(size_t)r * M + j] : 0.f;
    if (grad_t) g += grad_t[(size_t)j * R + r];
    const float dx = clamped ? g / eps : (g - (x / d) * dot) / d;
    float* dst = grad_raw + (size_t)r * M + j;
    *dst = accumulate ? *dst + dx : dx;
  }
}

}  // namespace
}  // namespace da

extern "C" int da_dict_norm_fwd(const float* raw, int64_t R, int64_t M, float eps, int out_dtype, void* out,
                                void* out_t, float* denom, float* max_col_norm, void* stream) {
  using namespace da;
  if (!raw) return DA_ERR_NULL;
  if (int rc = bind_device(raw)) return rc;
  if (R <= 0 || M <= 0 || R > (1 << 16) || M > (1 << 24)) return DA_ERR_SHAPE;
  if (out_dtype != DA_BF16 && out_dtype != DA_F16) return DA_ERR_DTYPE;
  if (out_t && (reinterpret_cast<uintptr_t>(out_t) & 15)) return DA_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (max_col_norm && cudaMemsetAsync(max_col_norm, 0, sizeof(float), st) != cudaSuccess) return record_cuda_error();
  const dim3 grid((unsigned)((M + 127) / 128)), block(128);
  if (out_dtype == DA_BF16)
    dict_norm_fwd_kernel<__nv_bfloat16><<<grid, block, 0, st>>>(raw, (int)R, (int)M, eps, (__nv_bfloat16*)out,
                                                                (__nv_bfloat16*)out_t, denom, max_col_norm);
  else
    dict_norm_fwd_kernel<__half><<<grid, block, 0, st>>>(raw, (int)R, (int)M, eps, (__half*)out, (__half*)out_t,
                                                         denom, max_col_norm);
  if (cudaPeekAtLastError() != cudaSuccess) return record_cuda_error();
  return DA_OK;
}

extern "C" int da_dict_norm_bwd(const float* raw, const float* denom, const float* grad, const float* grad_t,
                                int64_t R, int64_t M, float eps, float* grad_raw, int accumulate, void* stream) {
  using namespace da;
  if (!raw || !denom || !grad_raw || (!grad && !grad_t)) return DA_ERR_NULL;
  if (int rc = bind_device(raw)) return rc;
  if (R <= 0 || M <= 0 || R > (1 << 16) || M > (1 << 24)) return DA_ERR_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dict_norm_bwd_kernel<<<dim3((unsigned)((M + 127) / 128)), dim3(128), 0, st>>>(raw, denom, grad, grad_t, (int)R,
                                                                                 (int)M, eps, grad_raw, accumulate);
  if (cudaPeekAtLastError() != cudaSuccess) return record_cuda_error();
  return DA_OK;
}

// Largest column 2-norm of a [R, M] dictionary in fp16/bf16 (for callers that
// pass their own normalised dictionaries to the routing kernels).
namespace da {
namespace {
template <typename T>
__global__ void col_norm_max_kernel(const T* __restrict__ d, int R, int M, float* __restrict__ out) {
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
    col_norm_max_kernel<__nv_bfloat16><<<grid, block, 0, st>>>((const __nv_bfloat16*)dict, (int)R, (int)M, out);
  else if (dtype == DA_F16)
    col_norm_max_kernel<__half><<<grid, block, 0, st>>>((const __half*)dict, (int)R, (int)M, out);
  else
    return DA_ERR_DTYPE;
  if (cudaPeekAtLastError() != cudaSuccess) return record_cuda_error();
  return DA_OK;
}
