// Route variants: SiLU logits, standardised logits and direct-SiLU assignment.
//
// Reference: dictionary_route_reference (src/double_attention/ops.py:16-62),
// with the variant switches of the Triton path (triton_kernels.py:215-228,
// :417-448, :1984-2019):
//
//   l  = q_hat . Dk                       (q_hat = q / max(||q||, eps) or q)
//   a  = l               | 2 silu(l)                       (activation)
//   a' = a               | (a - mean) rsqrt(var + eps) c   (standardize, c = R^-1/2 or given)
//   w  = softmax(beta a')| (2/g) silu(g a')                (assignment)
//   r  = w . Dv^T,  z = r / max(||r||, eps) or r
//
// Standardisation needs statistics of the whole row of M logits before any
// weight exists, and its backward two more row reductions, so these
// variants run as the two dictionary products on the tcgen05 GEMM with the
// row stages below between them (one warp per route row, the row's M
// values in registers).  Identity logits with softmax assignment keep the
// fused tile kernel.
#include <math.h>

#include "common.cuh"
#include "host_util.h"

namespace da {
namespace route_var {

constexpr int kWarps = 8;  // rows per CTA

template <typename T> DA_DEV float to_f(T v);
template <> DA_DEV float to_f<__half>(__half v) { return __half2float(v); }
template <> DA_DEV float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> DA_DEV T from_f(float v);
template <> DA_DEV __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> DA_DEV __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

DA_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
DA_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
DA_DEV float sigmoid(float x) { return 1.f / (1.f + expf(-x)); }

// ||q||^-1 of one row (or 1 without input normalisation), lanes striding R.
template <typename T>
DA_DEV float inverse_norm(const T* q, int R, bool normalize, float eps, int lane) {
  if (!normalize) return 1.f;
  float s = 0.f;
  for (int c = lane; c < R; c += 32) {
    const float v = to_f<T>(q[c]);
    s = fmaf(v, v, s);
  }
  return 1.f / fmaxf(sqrtf(warp_sum(s)), eps);
}

struct RowCfg {
  int M, flags;
  float gain, std_scale, eps;
  const float* beta;
};

// Activation and standardisation of one row held as v[i] = S[lane + 32 i]
// (raw q.Dk); returns a' in place and the statistics (mean, inverse std).
template <int NPL>
DA_DEV void activate_row(float (&v)[NPL], const RowCfg& c, float invn, int lane, float& mean, float& istd) {
  const bool silu = c.flags & DA_ROUTE_SILU_LOGITS;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const bool live = lane + 32 * i < c.M;
    float l = v[i] * invn;
    if (silu) l = 2.f * l * sigmoid(l);
    v[i] = live ? l : 0.f;
    s += v[i];
  }
  mean = 0.f;
  istd = 1.f;
  if (c.flags & DA_ROUTE_STANDARDIZE) {
    mean = warp_sum(s) / (float)c.M;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (lane + 32 * i < c.M) {
        const float d = v[i] - mean;
        ss = fmaf(d, d, ss);
      }
    istd = rsqrtf(warp_sum(ss) / (float)c.M + c.eps);
#pragma unroll
    for (int i = 0; i < NPL; ++i) v[i] = (v[i] - mean) * istd * c.std_scale;
  }
}

template <typename T, int NPL>
__global__ void __launch_bounds__(32 * kWarps) weights_kernel(const float* __restrict__ S, int64_t rows,
                                                             const T* __restrict__ q, int64_t q_stride, int R,
                                                             RowCfg c, __nv_bfloat16* __restrict__ W,
                                                             float4* __restrict__ stats) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  const float invn = inverse_norm<T>(q + row * q_stride, R, c.flags & DA_ROUTE_NORM_INPUT, c.eps, lane);
  const float* srow = S + row * c.M;
  float v[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) v[i] = lane + 32 * i < c.M ? srow[lane + 32 * i] : 0.f;
  float mean, istd;
  activate_row<NPL>(v, c, invn, lane, mean, istd);
  float lse = 0.f;
  __nv_bfloat16* wrow = W + row * c.M;
  if (c.flags & DA_ROUTE_DIRECT_SILU) {
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (lane + 32 * i < c.M) {
        const float y = c.gain * v[i];
        wrow[lane + 32 * i] = __float2bfloat16_rn((2.f / c.gain) * y * sigmoid(y));
      }
  } else {
    const float beta = *c.beta;
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (lane + 32 * i < c.M) mx = fmaxf(mx, beta * v[i]);
    mx = warp_max(mx);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      v[i] = lane + 32 * i < c.M ? expf(beta * v[i] - mx) : 0.f;
      s += v[i];
    }
    s = warp_sum(s);
    const float inv = 1.f / s;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (lane + 32 * i < c.M) wrow[lane + 32 * i] = __float2bfloat16_rn(v[i] * inv);
    lse = mx + logf(s);
  }
  if (lane == 0) stats[row] = make_float4(invn, mean, istd, lse);
}

// z = r / max(||r||, eps) (or r) and ||r||.
template <typename T>
__global__ void __launch_bounds__(32 * kWarps) output_kernel(const float* __restrict__ r, int64_t rows, int R,
                                                            int normalize, float eps, T* __restrict__ z,
                                                            float* __restrict__ onorm) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  const float* rr = r + row * R;
  float s = 0.f;
  for (int c = lane; c < R; c += 32) s = fmaf(rr[c], rr[c], s);
  const float n = sqrtf(warp_sum(s));
  const float f = normalize ? 1.f / fmaxf(n, eps) : 1.f;
  for (int c = lane; c < R; c += 32) z[row * R + c] = from_f<T>(rr[c] * f);
  if (lane == 0) onorm[row] = n;
}

// g = dL/dr from dz: the output-normalisation backward (or dz), in bf16,
// and delta = <g, r> with r = z max(||r||, eps) (or z) in fp32: the softmax
// backward's <W, dW> in closed form (W . Dv^T = r), free of g's rounding.
template <typename T>
__global__ void __launch_bounds__(32 * kWarps) output_bwd_kernel(const T* __restrict__ z, const T* __restrict__ dz,
                                                                const float* __restrict__ onorm, int64_t rows, int R,
                                                                int normalize, float eps,
                                                                __nv_bfloat16* __restrict__ g,
                                                                float* __restrict__ delta) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  const T* zr = z + row * R;
  const T* dzr = dz + row * R;
  float d = 0.f, zz = 0.f;
  for (int c = lane; c < R; c += 32) {
    const float zc = to_f<T>(zr[c]);
    d = fmaf(zc, to_f<T>(dzr[c]), d);
    zz = fmaf(zc, zc, zz);
  }
  d = warp_sum(d);
  zz = warp_sum(zz);
  if (!normalize) {
    for (int c = lane; c < R; c += 32) g[row * R + c] = __float2bfloat16_rn(to_f<T>(dzr[c]));
    if (lane == 0) delta[row] = d;
    return;
  }
  const float n = onorm[row];
  // z = r / n for n > eps (d z/d r = (I - z z^T) / n); r / eps below it
  const bool big = n > eps;
  const float inv = 1.f / fmaxf(n, eps);
  for (int c = lane; c < R; c += 32) {
    const float dzc = to_f<T>(dzr[c]);
    g[row * R + c] = __float2bfloat16_rn((big ? dzc - to_f<T>(zr[c]) * d : dzc) * inv);
  }
  if (lane == 0) delta[row] = big ? d * (1.f - zz) : d;
}

// Backward of the row stage: dS = d loss / d (q.Dk) in the compute dtype,
// the weights W again (bf16, for dDv = g^T W) and the beta gradient.
template <typename T, int NPL>
__global__ void __launch_bounds__(32 * kWarps) weights_bwd_kernel(const float* __restrict__ S,
                                                                 const float* __restrict__ dW, int64_t rows,
                                                                 const float4* __restrict__ stats,
                                                                 const float* __restrict__ delta, RowCfg c,
                                                                 T* __restrict__ dS, __nv_bfloat16* __restrict__ W,
                                                                 float* __restrict__ dbeta_part) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * kWarps + threadIdx.x / 32;
  float db = 0.f;
  if (row < rows) {
    const float4 st = stats[row];
    const float invn = st.x, mean = st.y, istd = st.z, lse = st.w;
    const bool silu = c.flags & DA_ROUTE_SILU_LOGITS, stdz = c.flags & DA_ROUTE_STANDARDIZE;
    const float* srow = S + row * c.M;
    const float* dwrow = dW + row * c.M;
    float l[NPL], a[NPL], d[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const bool live = lane + 32 * i < c.M;
      l[i] = live ? srow[lane + 32 * i] * invn : 0.f;
      const float act = silu ? 2.f * l[i] * sigmoid(l[i]) : l[i];
      a[i] = live ? (stdz ? (act - mean) * istd * c.std_scale : act) : 0.f;
      d[i] = live ? dwrow[lane + 32 * i] : 0.f;
    }
    __nv_bfloat16* wrow = W + row * c.M;
    // assignment backward: d[i] <- dL/da'_i
    if (c.flags & DA_ROUTE_DIRECT_SILU) {
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const float y = c.gain * a[i], sg = sigmoid(y);
        if (lane + 32 * i < c.M) wrow[lane + 32 * i] = __float2bfloat16_rn((2.f / c.gain) * y * sg);
        d[i] *= 2.f * sg * (1.f + y * (1.f - sg));
      }
    } else {
      const float beta = *c.beta;
      float w[NPL], dot = 0.f;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        w[i] = lane + 32 * i < c.M ? expf(beta * a[i] - lse) : 0.f;
        dot = fmaf(w[i], d[i], dot);
        if (lane + 32 * i < c.M) wrow[lane + 32 * i] = __float2bfloat16_rn(w[i]);
      }
      dot = delta ? delta[row] : warp_sum(dot);  // <W, dW> = <g, r>
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const float dx = w[i] * (d[i] - dot);  // d loss / d (beta a')
        db = fmaf(dx, a[i], db);
        d[i] = beta * dx;
      }
    }
    // standardisation backward: h = (act - mean) istd, a' = c h
    if (stdz) {
      float sd = 0.f, sdh = 0.f;
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        d[i] *= c.std_scale;  // dL/dh
        const float h = a[i] / c.std_scale;
        sd += d[i];
        sdh = fmaf(d[i], h, sdh);
      }
      const float md = warp_sum(sd) / (float)c.M, mdh = warp_sum(sdh) / (float)c.M;
#pragma unroll
      for (int i = 0; i < NPL; ++i) d[i] = istd * (d[i] - md - (a[i] / c.std_scale) * mdh);
    }
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      if (silu) {
        const float sg = sigmoid(l[i]);
        d[i] *= 2.f * sg * (1.f + l[i] * (1.f - sg));
      }
      if (lane + 32 * i < c.M) dS[row * c.M + lane + 32 * i] = from_f<T>(d[i] * invn);
    }
  }
  if (dbeta_part && !(c.flags & DA_ROUTE_DIRECT_SILU)) {  // this block's beta-gradient partial (fixed order)
    __shared__ float part[kWarps];
    db = warp_sum(db);
    if (lane == 0) part[threadIdx.x / 32] = db;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int i = 0; i < kWarps; ++i) t += part[i];
      dbeta_part[blockIdx.x] = t;
    }
  }
}

// *dbeta += the sum of n per-block partials: strided in index order per thread, then a fixed tree.
__global__ void __launch_bounds__(256) dbeta_reduce_kernel(const float* part, int n, float* dbeta) {
  __shared__ float red[256];
  grid_dependency_wait();
  grid_launch_dependents();
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += 256) s += part[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w; w >>= 1) {
    if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) *dbeta += red[0];
}

// Input-normalisation backward: dq = u - q_hat <q_hat, u> with u = dS . Dk^T
// (= dq_hat / ||q||), or u without input normalisation.
template <typename T>
__global__ void __launch_bounds__(32 * kWarps) input_bwd_kernel(const float* __restrict__ u, const T* __restrict__ q,
                                                               int64_t q_stride, const float4* __restrict__ stats,
                                                               int64_t rows, int R, int normalize, float eps,
                                                               T* __restrict__ dq, int64_t dq_stride) {
  grid_dependency_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x % 32;
  const int64_t row = (int64_t)blockIdx.x * kWarps + threadIdx.x / 32;
  if (row >= rows) return;
  const float* ur = u + row * R;
  const T* qr = q + row * q_stride;
  T* out = dq + row * dq_stride;
  const float invn = stats[row].x;
  // q_hat = q / max(||q||, eps); the projection removes the q_hat component only when ||q|| > eps
  const bool big = normalize && invn < 1.f / eps;
  float d = 0.f;
  if (big)
    for (int c = lane; c < R; c += 32) d = fmaf(to_f<T>(qr[c]) * invn, ur[c], d);
  d = warp_sum(d);
  for (int c = lane; c < R; c += 32) out[c] = from_f<T>(big ? ur[c] - to_f<T>(qr[c]) * invn * d : ur[c]);
}

template <typename T, int NPL>
int launch_weights(const float* S, int64_t rows, const void* q, int64_t q_stride, int R, const RowCfg& c, void* W,
                   float* stats, cudaStream_t st) {
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
  return launch_kernel(weights_kernel<T, NPL>, grid, dim3(32 * kWarps), 0, st, false, S, rows,
                       static_cast<const T*>(q), q_stride, R, c, static_cast<__nv_bfloat16*>(W),
                       reinterpret_cast<float4*>(stats));
}

template <typename T, int NPL>
int launch_weights_bwd(const float* S, const float* dW, int64_t rows, const float* stats, const float* delta,
                       const RowCfg& c, void* dS, void* W, float* dbeta, float* dbeta_part, cudaStream_t st) {
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
  const bool want_beta = dbeta && !(c.flags & DA_ROUTE_DIRECT_SILU);
  if (int rc = launch_kernel(weights_bwd_kernel<T, NPL>, grid, dim3(32 * kWarps), 0, st, false, S, dW, rows,
                             reinterpret_cast<const float4*>(stats), delta, c, static_cast<T*>(dS),
                             static_cast<__nv_bfloat16*>(W), want_beta ? dbeta_part : (float*)nullptr))
    return rc;
  if (!want_beta) return DA_OK;
  return launch_kernel(dbeta_reduce_kernel, dim3(1), dim3(256), 0, st, false, (const float*)dbeta_part,
                       (int)grid.x, dbeta);
}

// Values per lane for a row of M (M <= 2048).
inline int npl_for(int M) { return M <= 512 ? 16 : M <= 1024 ? 32 : M <= 1536 ? 48 : 64; }

inline int check_cfg(int64_t rows, int M, int flags, float gain, float std_scale) {
  if (rows <= 0 || M <= 0 || M > 2048) return DA_ERR_SHAPE;
  if (flags & ~(DA_ROUTE_SILU_LOGITS | DA_ROUTE_STANDARDIZE | DA_ROUTE_DIRECT_SILU | DA_ROUTE_NORM_INPUT))
    return DA_ERR_UNSUPPORTED;
  if ((flags & DA_ROUTE_DIRECT_SILU) && !(gain > 0.f)) return DA_ERR_SHAPE;
  if ((flags & DA_ROUTE_STANDARDIZE) && !(std_scale > 0.f)) return DA_ERR_SHAPE;
  return DA_OK;
}

}  // namespace route_var
}  // namespace da

extern "C" int da_route_var_weights(const float* S, int64_t rows, int M, const void* q, int64_t q_stride, int R,
                                    int dtype, int flags, float silu_gain, float std_scale, const float* beta,
                                    float eps, void* W, float* stats, void* stream) {
  using namespace da;
  using namespace da::route_var;
  if (!S || !q || !W || !stats || (!beta && !(flags & DA_ROUTE_DIRECT_SILU))) return DA_ERR_NULL;
  if (int rc = check_cfg(rows, M, flags, silu_gain, std_scale)) return rc;
  if (R <= 0 || q_stride < R) return DA_ERR_SHAPE;
  if (dtype != DA_F16 && dtype != DA_BF16) return DA_ERR_DTYPE;
  if (int rc = bind_device(S)) return rc;
  const RowCfg c{M, flags, silu_gain, std_scale, eps, beta};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int npl = npl_for(M);
#define DA_RV_W(TT)                                                                          \
  switch (npl) {                                                                             \
    case 16: return launch_weights<TT, 16>(S, rows, q, q_stride, R, c, W, stats, st);        \
    case 32: return launch_weights<TT, 32>(S, rows, q, q_stride, R, c, W, stats, st);        \
    case 48: return launch_weights<TT, 48>(S, rows, q, q_stride, R, c, W, stats, st);        \
    default: return launch_weights<TT, 64>(S, rows, q, q_stride, R, c, W, stats, st);        \
  }
  if (dtype == DA_BF16) { DA_RV_W(__nv_bfloat16) }
  DA_RV_W(__half)
#undef DA_RV_W
}

extern "C" int da_route_var_output(const float* r, int64_t rows, int R, int dtype, int normalize, float eps, void* z,
                                   float* onorm, void* stream) {
  using namespace da;
  using namespace da::route_var;
  if (!r || !z || !onorm) return DA_ERR_NULL;
  if (rows <= 0 || R <= 0) return DA_ERR_SHAPE;
  if (dtype != DA_F16 && dtype != DA_BF16) return DA_ERR_DTYPE;
  if (int rc = bind_device(r)) return rc;
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DA_BF16)
    return launch_kernel(output_kernel<__nv_bfloat16>, grid, dim3(32 * kWarps), 0, st, false, r, rows, R, normalize,
                         eps, static_cast<__nv_bfloat16*>(z), onorm);
  return launch_kernel(output_kernel<__half>, grid, dim3(32 * kWarps), 0, st, false, r, rows, R, normalize, eps,
                       static_cast<__half*>(z), onorm);
}

extern "C" int da_route_var_output_bwd(const void* z, const void* dz, const float* onorm, int64_t rows, int R,
                                       int dtype, int normalize, float eps, void* g, float* delta, void* stream) {
  using namespace da;
  using namespace da::route_var;
  if (!z || !dz || !onorm || !g || !delta) return DA_ERR_NULL;
  if (rows <= 0 || R <= 0) return DA_ERR_SHAPE;
  if (dtype != DA_F16 && dtype != DA_BF16) return DA_ERR_DTYPE;
  if (int rc = bind_device(z)) return rc;
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == DA_BF16)
    return launch_kernel(output_bwd_kernel<__nv_bfloat16>, grid, dim3(32 * kWarps), 0, st, false,
                         static_cast<const __nv_bfloat16*>(z), static_cast<const __nv_bfloat16*>(dz), onorm, rows, R,
                         normalize, eps, static_cast<__nv_bfloat16*>(g), delta);
  return launch_kernel(output_bwd_kernel<__half>, grid, dim3(32 * kWarps), 0, st, false, static_cast<const __half*>(z),
                       static_cast<const __half*>(dz), onorm, rows, R, normalize, eps,
                       static_cast<__nv_bfloat16*>(g), delta);
}

extern "C" int da_route_var_weights_bwd(const float* S, const float* dW, int64_t rows, int M, const float* stats,
                                        const float* delta, int flags, float silu_gain, float std_scale,
                                        const float* beta, int dtype, void* dS, void* W, float* dbeta,
                                        float* dbeta_work, int64_t dbeta_work_elems, void* stream) {
  using namespace da;
  using namespace da::route_var;
  if (!S || !dW || !stats || !dS || !W || (!beta && !(flags & DA_ROUTE_DIRECT_SILU))) return DA_ERR_NULL;
  if (int rc = check_cfg(rows, M, flags, silu_gain, std_scale)) return rc;
  if (dbeta && !(flags & DA_ROUTE_DIRECT_SILU) && (!dbeta_work || dbeta_work_elems < (rows + kWarps - 1) / kWarps))
    return DA_ERR_WORKSPACE;
  if (dtype != DA_F16 && dtype != DA_BF16) return DA_ERR_DTYPE;
  if (int rc = bind_device(S)) return rc;
  const RowCfg c{M, flags, silu_gain, std_scale, 0.f, beta};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int npl = npl_for(M);
#define DA_RV_B(TT)                                                                                  \
  switch (npl) {                                                                                     \
    case 16: return launch_weights_bwd<TT, 16>(S, dW, rows, stats, delta, c, dS, W, dbeta, dbeta_work, st);             \
    case 32: return launch_weights_bwd<TT, 32>(S, dW, rows, stats, delta, c, dS, W, dbeta, dbeta_work, st);             \
    case 48: return launch_weights_bwd<TT, 48>(S, dW, rows, stats, delta, c, dS, W, dbeta, dbeta_work, st);             \
    default: return launch_weights_bwd<TT, 64>(S, dW, rows, stats, delta, c, dS, W, dbeta, dbeta_work, st);             \
  }
  if (dtype == DA_BF16) { DA_RV_B(__nv_bfloat16) }
  DA_RV_B(__half)
#undef DA_RV_B
}

extern "C" int da_route_var_input_bwd(const float* u, const void* q, int64_t q_stride, const float* stats,
                                      int64_t rows, int R, int dtype, int normalize, float eps, void* dq,
                                      int64_t dq_stride, void* stream) {
  using namespace da;
  using namespace da::route_var;
  if (!u || !q || !stats || !dq) return DA_ERR_NULL;
  if (rows <= 0 || R <= 0 || q_stride < R || dq_stride < R) return DA_ERR_SHAPE;
  if (dtype != DA_F16 && dtype != DA_BF16) return DA_ERR_DTYPE;
  if (int rc = bind_device(u)) return rc;
  const dim3 grid((unsigned)((rows + kWarps - 1) / kWarps));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float4* s4 = reinterpret_cast<const float4*>(stats);
  if (dtype == DA_BF16)
    return launch_kernel(input_bwd_kernel<__nv_bfloat16>, grid, dim3(32 * kWarps), 0, st, false, u,
                         static_cast<const __nv_bfloat16*>(q), q_stride, s4, rows, R, normalize, eps,
                         static_cast<__nv_bfloat16*>(dq), dq_stride);
  return launch_kernel(input_bwd_kernel<__half>, grid, dim3(32 * kWarps), 0, st, false, u,
                       static_cast<const __half*>(q), q_stride, s4, rows, R, normalize, eps,
                       static_cast<__half*>(dq), dq_stride);
}
